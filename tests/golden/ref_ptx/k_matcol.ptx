.version 8.0
.target sm_89
.address_size 64

.visible .entry matmul_odd(
	.param .u64 p_A,
	.param .u64 p_B,
	.param .u64 p_C
)
.maxntid 128, 1, 1
{
	.reg .pred %p<3>;
	.reg .b32 %r<11>;
	.reg .f32 %f<5>;
	.reg .b64 %rd<7>;
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
	setp.lt.s32 %p1, %r4, 256;
	@!%p1 bra L1_end;
	sub.s32 %r7, %r4, %r4;
	mov.b32 %f1, 0f00000000;
	mov.s32 %r8, 0;
L3_top:
	setp.ge.s32 %p2, %r8, 256;
	@%p2 bra L2_lend;
	mad.lo.s32 %r10, %r4, 256, %r8;
	mad.wide.s32 %rd4, %r10, 4, %rd1;
	ld.global.f32 %f2, [%rd4];
	mad.wide.s32 %rd5, %r8, 4, %rd2;
	ld.global.f32 %f3, [%rd5];
	mul.f32 %f4, %f2, %f3;
	add.f32 %f1, %f1, %f4;
	add.s32 %r8, %r8, 1;
	bra L3_top;
L2_lend:
	mad.wide.s32 %rd6, %r4, 4, %rd3;
	st.global.f32 [%rd6], %f1;
L1_end:
	ret;
}
