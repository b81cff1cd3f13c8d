.version 8.0
.target sm_89
.address_size 64

.visible .entry softmax_mid(
	.param .u64 p_x,
	.param .u64 p_y
)
.maxntid 64, 1, 1
{
	.reg .pred %p<5>;
	.reg .b32 %r<25>;
	.reg .f32 %f<15>;
	.reg .b64 %rd<7>;
	ld.param.u64 %rd1, [p_x];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_y];
	cvta.to.global.u64 %rd2, %rd2;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	setp.lt.s32 %p1, %r4, 64;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 16;
	mul.lo.s32 %r8, %r7, 16;
	sub.s32 %r9, %r4, %r8;
	mov.b32 %f1, 0fFF800000;
	mov.s32 %r10, 0;
L3_top:
	setp.ge.s32 %p2, %r10, 32;
	@%p2 bra L2_lend;
	mad.lo.s32 %r12, %r7, 32, %r10;
	mad.lo.s32 %r14, %r12, 16, %r9;
	mad.wide.s32 %rd3, %r14, 4, %rd1;
	ld.global.f32 %f2, [%rd3];
	max.f32 %f1, %f1, %f2;
	add.s32 %r10, %r10, 1;
	bra L3_top;
L2_lend:
	mov.b32 %f3, 0f00000000;
	mov.s32 %r15, 0;
L5_top:
	setp.ge.s32 %p3, %r15, 32;
	@%p3 bra L4_lend;
	mad.lo.s32 %r17, %r7, 32, %r15;
	mad.lo.s32 %r19, %r17, 16, %r9;
	mad.wide.s32 %rd4, %r19, 4, %rd1;
	ld.global.f32 %f4, [%rd4];
	sub.f32 %f5, %f4, %f1;
	mov.b32 %f6, 0f3FB8AA3B;
	mul.f32 %f7, %f5, %f6;
	ex2.approx.f32 %f8, %f7;
	add.f32 %f3, %f3, %f8;
	add.s32 %r15, %r15, 1;
	bra L5_top;
L4_lend:
	mov.s32 %r20, 0;
L7_top:
	setp.ge.s32 %p4, %r20, 32;
	@%p4 bra L6_lend;
	mad.lo.s32 %r22, %r7, 32, %r20;
	mad.lo.s32 %r24, %r22, 16, %r9;
	mad.wide.s32 %rd5, %r24, 4, %rd1;
	ld.global.f32 %f9, [%rd5];
	sub.f32 %f10, %f9, %f1;
	mov.b32 %f11, 0f3FB8AA3B;
	mul.f32 %f12, %f10, %f11;
	ex2.approx.f32 %f13, %f12;
	div.rn.f32 %f14, %f13, %f3;
	mad.wide.s32 %rd6, %r24, 4, %rd2;
	st.global.f32 [%rd6], %f14;
	add.s32 %r20, %r20, 1;
	bra L7_top;
L6_lend:
L1_end:
	ret;
}
