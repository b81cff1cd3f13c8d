.version 8.0
.target sm_89
.address_size 64

.visible .entry bmm_naive(
	.param .u64 p_A,
	.param .u64 p_B,
	.param .u64 p_C
)
.maxntid 256, 1, 1
{
	.reg .pred %p<3>;
	.reg .b32 %r<26>;
	.reg .f32 %f<5>;
	.reg .b64 %rd<7>;
	.reg .b16 %rs<3>;
	ld.param.u64 %rd1, [p_A];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_B];
	cvta.to.global.u64 %rd2, %rd2;
	ld.param.u64 %rd3, [p_C];
	cvta.to.global.u64 %rd3, %rd3;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	setp.lt.s32 %p1, %r4, 2048;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 1024;
	mul.lo.s32 %r8, %r7, 1024;
	sub.s32 %r9, %r4, %r8;
	div.s32 %r10, %r9, 32;
	mul.lo.s32 %r11, %r10, 32;
	sub.s32 %r12, %r9, %r11;
	mov.b32 %f1, 0f00000000;
	mov.s32 %r13, 0;
	mad.lo.s32 %r15, %r7, 32, %r10;
L3_top:
	setp.ge.s32 %p2, %r13, 64;
	@%p2 bra L2_lend;
	mad.lo.s32 %r17, %r15, 64, %r13;
	mad.wide.s32 %rd4, %r17, 2, %rd1;
	ld.global.b16 %rs1, [%rd4];
	cvt.f32.bf16 %f2, %rs1;
	mad.lo.s32 %r19, %r7, 64, %r13;
	mad.lo.s32 %r21, %r19, 32, %r12;
	mad.wide.s32 %rd5, %r21, 2, %rd2;
	ld.global.b16 %rs2, [%rd5];
	cvt.f32.bf16 %f3, %rs2;
	mul.f32 %f4, %f2, %f3;
	add.f32 %f1, %f1, %f4;
	add.s32 %r13, %r13, 1;
	bra L3_top;
L2_lend:
	mad.lo.s32 %r23, %r7, 32, %r10;
	mad.lo.s32 %r25, %r23, 32, %r12;
	mad.wide.s32 %rd6, %r25, 4, %rd3;
	st.global.f32 [%rd6], %f1;
L1_end:
	ret;
}
