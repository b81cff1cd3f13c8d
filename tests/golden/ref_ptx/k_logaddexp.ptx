.version 8.0
.target sm_89
.address_size 64

.visible .entry log_add_exp(
	.param .u64 p_a,
	.param .u64 p_b,
	.param .u64 p_y
)
.maxntid 128, 1, 1
{
	.reg .pred %p<2>;
	.reg .b32 %r<7>;
	.reg .f32 %f<16>;
	.reg .b64 %rd<7>;
	ld.param.u64 %rd1, [p_a];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_b];
	cvta.to.global.u64 %rd2, %rd2;
	ld.param.u64 %rd3, [p_y];
	cvta.to.global.u64 %rd3, %rd3;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	setp.lt.s32 %p1, %r4, 1000;
	@!%p1 bra L1_end;
	mad.wide.s32 %rd4, %r4, 4, %rd1;
	ld.global.f32 %f1, [%rd4];
	mad.wide.s32 %rd5, %r4, 4, %rd2;
	ld.global.f32 %f2, [%rd5];
	max.f32 %f3, %f1, %f2;
	sub.f32 %f4, %f1, %f2;
	abs.f32 %f5, %f4;
	neg.f32 %f6, %f5;
	mov.b32 %f7, 0f3FB8AA3B;
	mul.f32 %f8, %f6, %f7;
	ex2.approx.f32 %f9, %f8;
	mov.b32 %f10, 0f3F800000;
	add.f32 %f11, %f9, %f10;
	lg2.approx.f32 %f12, %f11;
	mov.b32 %f13, 0f3F317218;
	mul.f32 %f14, %f12, %f13;
	add.f32 %f15, %f3, %f14;
	mad.wide.s32 %rd6, %r4, 4, %rd3;
	st.global.f32 [%rd6], %f15;
L1_end:
	ret;
}
