.version 8.0
.target sm_89
.address_size 64

.visible .entry expr_forms(
	.param .u64 p_x,
	.param .u64 p_y
)
.maxntid 128, 1, 1
{
	.reg .pred %p<7>;
	.reg .b32 %r<11>;
	.reg .f32 %f<15>;
	.reg .b64 %rd<5>;
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
	setp.lt.s32 %p1, %r4, 512;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 64;
	mul.lo.s32 %r8, %r7, 64;
	sub.s32 %r9, %r4, %r8;
	add.s32 %r10, %r8, %r9;
	mad.wide.s32 %rd3, %r10, 4, %rd1;
	ld.global.f32 %f1, [%rd3];
	cvt.rn.f32.s32 %f2, %r10;
	mov.b32 %f3, 0f3C23D70A;
	mul.f32 %f4, %f2, %f3;
	setp.lt.s32 %p2, %r9, 32;
	mov.b32 %f5, 0f00000000;
	selp.f32 %f6, %f1, %f5, %p2;
	add.f32 %f7, %f6, %f4;
	mov.b32 %f8, 0f3FB8AA3B;
	mul.f32 %f9, %f1, %f8;
	ex2.approx.f32 %f10, %f9;
	mov.b32 %f11, 0f3F000000;
	mul.f32 %f12, %f10, %f11;
	mov.b32 %f13, 0f00000000;
	setp.gt.f32 %p3, %f1, %f13;
	setp.lt.s32 %p4, %r9, 48;
	and.pred %p5, %p3, %p4;
	not.pred %p6, %p5;
	selp.b32 %f14, %f12, %f7, %p6;
	mad.wide.s32 %rd4, %r10, 4, %rd2;
	st.global.f32 [%rd4], %f14;
L1_end:
	ret;
}
