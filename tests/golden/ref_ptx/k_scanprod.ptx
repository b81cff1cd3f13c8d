.version 8.0
.target sm_89
.address_size 64

.visible .entry scan_max_prod(
	.param .u64 p_x,
	.param .u64 p_cm,
	.param .u64 p_pr
)
.maxntid 32, 1, 1
{
	.reg .pred %p<11>;
	.reg .b32 %r<26>;
	.reg .f32 %f<15>;
	.reg .b64 %rd<8>;
	ld.param.u64 %rd1, [p_x];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_cm];
	cvta.to.global.u64 %rd2, %rd2;
	ld.param.u64 %rd3, [p_pr];
	cvta.to.global.u64 %rd3, %rd3;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	setp.lt.s32 %p1, %r4, 128;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 32;
	mul.lo.s32 %r8, %r7, 32;
	sub.s32 %r9, %r4, %r8;
	setp.eq.s32 %p2, %r9, 0;
	@!%p2 bra L2_else;
	mov.b32 %f1, 0fFF800000;
	mov.s32 %r10, 0;
L5_top:
	setp.ge.s32 %p3, %r10, 64;
	@%p3 bra L4_lend;
	mad.lo.s32 %r12, %r7, 64, %r10;
	mad.wide.s32 %rd4, %r12, 4, %rd1;
	ld.global.f32 %f2, [%rd4];
	max.f32 %f1, %f1, %f2;
	mad.wide.s32 %rd5, %r12, 4, %rd2;
	st.global.f32 [%rd5], %f1;
	add.s32 %r10, %r10, 1;
	bra L5_top;
L4_lend:
L2_else:
	mov.b32 %f3, 0f3F800000;
	mov.s32 %r13, %r9;
L6_top:
	setp.ge.s32 %p4, %r13, 64;
	@%p4 bra L7_lend;
	mad.lo.s32 %r15, %r7, 64, %r13;
	mad.wide.s32 %rd6, %r15, 4, %rd1;
	ld.global.f32 %f4, [%rd6];
	mul.f32 %f3, %f3, %f4;
	add.s32 %r13, %r13, 32;
	bra L6_top;
L7_lend:
	mov.b32 %r16, %f3;
	shfl.sync.bfly.b32 %r17|%p5, %r16, 16, 0x1f, 0xffffffff;
	mov.b32 %f5, %r17;
	mul.f32 %f6, %f3, %f5;
	mov.b32 %r18, %f6;
	shfl.sync.bfly.b32 %r19|%p6, %r18, 8, 0x1f, 0xffffffff;
	mov.b32 %f7, %r19;
	mul.f32 %f8, %f6, %f7;
	mov.b32 %r20, %f8;
	shfl.sync.bfly.b32 %r21|%p7, %r20, 4, 0x1f, 0xffffffff;
	mov.b32 %f9, %r21;
	mul.f32 %f10, %f8, %f9;
	mov.b32 %r22, %f10;
	shfl.sync.bfly.b32 %r23|%p8, %r22, 2, 0x1f, 0xffffffff;
	mov.b32 %f11, %r23;
	mul.f32 %f12, %f10, %f11;
	mov.b32 %r24, %f12;
	shfl.sync.bfly.b32 %r25|%p9, %r24, 1, 0x1f, 0xffffffff;
	mov.b32 %f13, %r25;
	mul.f32 %f14, %f12, %f13;
	setp.eq.s32 %p10, %r9, 0;
	@!%p10 bra L8_else;
	mad.wide.s32 %rd7, %r7, 4, %rd3;
	st.global.f32 [%rd7], %f14;
L8_else:
L1_end:
	ret;
}
