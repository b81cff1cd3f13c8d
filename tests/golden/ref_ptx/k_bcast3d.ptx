.version 8.0
.target sm_89
.address_size 64

.visible .entry bcast3d(
	.param .u64 p_x,
	.param .u64 p_w,
	.param .u64 p_bias,
	.param .u64 p_y
)
.maxntid 64, 1, 1
{
	.reg .pred %p<2>;
	.reg .b32 %r<17>;
	.reg .f32 %f<8>;
	.reg .b64 %rd<9>;
	.reg .b16 %rs<2>;
	ld.param.u64 %rd1, [p_x];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_w];
	cvta.to.global.u64 %rd2, %rd2;
	ld.param.u64 %rd3, [p_bias];
	cvta.to.global.u64 %rd3, %rd3;
	ld.param.u64 %rd4, [p_y];
	cvta.to.global.u64 %rd4, %rd4;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	setp.lt.s32 %p1, %r4, 555;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 185;
	mul.lo.s32 %r8, %r7, 185;
	sub.s32 %r9, %r4, %r8;
	div.s32 %r10, %r9, 37;
	mul.lo.s32 %r11, %r10, 37;
	sub.s32 %r12, %r9, %r11;
	mad.lo.s32 %r14, %r7, 5, %r10;
	mad.lo.s32 %r16, %r14, 37, %r12;
	mad.wide.s32 %rd5, %r16, 4, %rd1;
	ld.global.f32 %f1, [%rd5];
	mad.wide.s32 %rd6, %r7, 4, %rd2;
	ld.global.f32 %f2, [%rd6];
	mad.wide.s32 %rd7, %r12, 4, %rd3;
	ld.global.f32 %f3, [%rd7];
	mul.f32 %f4, %f1, %f2;
	add.f32 %f5, %f4, %f3;
	mov.b32 %f6, 0f00000000;
	max.f32 %f7, %f5, %f6;
	mad.wide.s32 %rd8, %r16, 2, %rd4;
	cvt.rn.bf16.f32 %rs1, %f7;
	st.global.b16 [%rd8], %rs1;
L1_end:
	ret;
}
