.version 8.0
.target sm_89
.address_size 64

.visible .entry elu_selu(
	.param .u64 p_x,
	.param .u64 p_elu,
	.param .u64 p_selu
)
.maxntid 64, 1, 1
{
	.reg .pred %p<6>;
	.reg .b32 %r<8>;
	.reg .f32 %f<53>;
	.reg .b64 %rd<7>;
	ld.param.u64 %rd1, [p_x];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_elu];
	cvta.to.global.u64 %rd2, %rd2;
	ld.param.u64 %rd3, [p_selu];
	cvta.to.global.u64 %rd3, %rd3;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	setp.lt.s32 %p1, %r4, 160;
	@!%p1 bra L1_end;
	mul.lo.s32 %r7, %r4, 4;
	mad.wide.s32 %rd4, %r7, 4, %rd1;
	ld.global.v4.f32 {%f1, %f2, %f3, %f4}, [%rd4];
	mov.b32 %f5, 0f00000000;
	setp.gt.f32 %p2, %f1, %f5;
	mov.b32 %f6, 0f3FB8AA3B;
	mul.f32 %f7, %f1, %f6;
	ex2.approx.f32 %f8, %f7;
	mov.b32 %f9, 0f3F800000;
	sub.f32 %f10, %f8, %f9;
	selp.b32 %f11, %f1, %f10, %p2;
	mov.b32 %f12, 0f3FD62D7D;
	mul.f32 %f13, %f10, %f12;
	selp.b32 %f14, %f1, %f13, %p2;
	mov.b32 %f15, 0f3F867D5F;
	mul.f32 %f16, %f14, %f15;
	mov.b32 %f17, 0f00000000;
	setp.gt.f32 %p3, %f2, %f17;
	mov.b32 %f18, 0f3FB8AA3B;
	mul.f32 %f19, %f2, %f18;
	ex2.approx.f32 %f20, %f19;
	mov.b32 %f21, 0f3F800000;
	sub.f32 %f22, %f20, %f21;
	selp.b32 %f23, %f2, %f22, %p3;
	mov.b32 %f24, 0f3FD62D7D;
	mul.f32 %f25, %f22, %f24;
	selp.b32 %f26, %f2, %f25, %p3;
	mov.b32 %f27, 0f3F867D5F;
	mul.f32 %f28, %f26, %f27;
	mov.b32 %f29, 0f00000000;
	setp.gt.f32 %p4, %f3, %f29;
	mov.b32 %f30, 0f3FB8AA3B;
	mul.f32 %f31, %f3, %f30;
	ex2.approx.f32 %f32, %f31;
	mov.b32 %f33, 0f3F800000;
	sub.f32 %f34, %f32, %f33;
	selp.b32 %f35, %f3, %f34, %p4;
	mov.b32 %f36, 0f3FD62D7D;
	mul.f32 %f37, %f34, %f36;
	selp.b32 %f38, %f3, %f37, %p4;
	mov.b32 %f39, 0f3F867D5F;
	mul.f32 %f40, %f38, %f39;
	mov.b32 %f41, 0f00000000;
	setp.gt.f32 %p5, %f4, %f41;
	mov.b32 %f42, 0f3FB8AA3B;
	mul.f32 %f43, %f4, %f42;
	ex2.approx.f32 %f44, %f43;
	mov.b32 %f45, 0f3F800000;
	sub.f32 %f46, %f44, %f45;
	selp.b32 %f47, %f4, %f46, %p5;
	mov.b32 %f48, 0f3FD62D7D;
	mul.f32 %f49, %f46, %f48;
	selp.b32 %f50, %f4, %f49, %p5;
	mov.b32 %f51, 0f3F867D5F;
	mul.f32 %f52, %f50, %f51;
	mad.wide.s32 %rd5, %r7, 4, %rd2;
	st.global.v4.f32 [%rd5], {%f11, %f23, %f35, %f47};
	mad.wide.s32 %rd6, %r7, 4, %rd3;
	st.global.v4.f32 [%rd6], {%f16, %f28, %f40, %f52};
L1_end:
	ret;
}
