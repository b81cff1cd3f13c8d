.version 8.0
.target sm_89
.address_size 64

.visible .entry f64_affine(
	.param .u64 p_x,
	.param .u64 p_y
)
.maxntid 64, 1, 1
{
	.reg .pred %p<2>;
	.reg .b32 %r<11>;
	.reg .f32 %f<6>;
	.reg .b64 %rd<5>;
	.reg .b64 %fd<3>;
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
	div.s32 %r7, %r4, 32;
	mul.lo.s32 %r8, %r7, 32;
	sub.s32 %r9, %r4, %r8;
	add.s32 %r10, %r8, %r9;
	mad.wide.s32 %rd3, %r10, 8, %rd1;
	ld.global.f64 %fd1, [%rd3];
	cvt.rn.f32.f64 %f1, %fd1;
	mov.b32 %f2, 0f40200000;
	mul.f32 %f3, %f1, %f2;
	mov.b32 %f4, 0f3F800000;
	add.f32 %f5, %f3, %f4;
	mad.wide.s32 %rd4, %r10, 8, %rd2;
	cvt.f64.f32 %fd2, %f5;
	st.global.f64 [%rd4], %fd2;
L1_end:
	ret;
}
