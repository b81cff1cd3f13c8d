.version 8.0
.target sm_89
.address_size 64

.visible .entry attention_causal(
	.param .u64 p_Q,
	.param .u64 p_K,
	.param .u64 p_V,
	.param .u64 p_O
)
.maxntid 128, 1, 1
{
	.reg .pred %p<9>;
	.reg .b32 %r<49>;
	.reg .f32 %f<62>;
	.reg .b64 %rd<21>;
	.reg .b16 %rs<17>;
	ld.param.u64 %rd1, [p_Q];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_K];
	cvta.to.global.u64 %rd2, %rd2;
	ld.param.u64 %rd3, [p_V];
	cvta.to.global.u64 %rd3, %rd3;
	ld.param.u64 %rd4, [p_O];
	cvta.to.global.u64 %rd4, %rd4;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	setp.lt.s32 %p1, %r4, 33554432;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 4194304;
	mul.lo.s32 %r8, %r7, 4194304;
	sub.s32 %r9, %r4, %r8;
	div.s32 %r10, %r9, 131072;
	mul.lo.s32 %r11, %r10, 131072;
	sub.s32 %r12, %r9, %r11;
	div.s32 %r13, %r12, 32;
	mul.lo.s32 %r14, %r13, 32;
	sub.s32 %r15, %r12, %r14;
	mul.lo.s32 %r16, %r15, 4;
	mad.lo.s32 %r18, %r7, 32, %r10;
	mul.lo.s32 %r19, %r18, 4096;
	add.s32 %r20, %r19, %r13;
	mad.lo.s32 %r22, %r20, 128, %r16;
	mad.wide.s32 %rd5, %r22, 2, %rd1;
	ld.global.b16 %rs1, [%rd5];
	cvt.f32.bf16 %f1, %rs1;
	add.s64 %rd6, %rd5, 2;
	ld.global.b16 %rs2, [%rd6];
	cvt.f32.bf16 %f2, %rs2;
	add.s64 %rd7, %rd5, 4;
	ld.global.b16 %rs3, [%rd7];
	cvt.f32.bf16 %f3, %rs3;
	add.s64 %rd8, %rd5, 6;
	ld.global.b16 %rs4, [%rd8];
	cvt.f32.bf16 %f4, %rs4;
	mov.b32 %f5, 0fFF800000;
	mov.b32 %f6, 0f00000000;
	mov.b32 %f7, 0f00000000;
	mov.b32 %f8, 0f00000000;
	mov.b32 %f9, 0f00000000;
	mov.b32 %f10, 0f00000000;
	mov.s32 %r23, 0;
	mad.lo.s32 %r38, %r7, 32, %r10;
L2_top:
	setp.ge.s32 %p2, %r23, 4096;
	@%p2 bra L3_lend;
	add.s32 %r24, %r19, %r23;
	mad.lo.s32 %r26, %r24, 128, %r16;
	mad.wide.s32 %rd9, %r26, 2, %rd2;
	ld.global.b16 %rs5, [%rd9];
	cvt.f32.bf16 %f11, %rs5;
	add.s64 %rd10, %rd9, 2;
	ld.global.b16 %rs6, [%rd10];
	cvt.f32.bf16 %f12, %rs6;
	add.s64 %rd11, %rd9, 4;
	ld.global.b16 %rs7, [%rd11];
	cvt.f32.bf16 %f13, %rs7;
	add.s64 %rd12, %rd9, 6;
	ld.global.b16 %rs8, [%rd12];
	cvt.f32.bf16 %f14, %rs8;
	mul.f32 %f15, %f1, %f11;
	mul.f32 %f16, %f2, %f12;
	mul.f32 %f17, %f3, %f13;
	mul.f32 %f18, %f4, %f14;
	add.f32 %f19, %f15, %f16;
	add.f32 %f20, %f17, %f18;
	add.f32 %f21, %f19, %f20;
	mov.b32 %r27, %f21;
	shfl.sync.bfly.b32 %r28|%p3, %r27, 16, 0x1f, 0xffffffff;
	mov.b32 %f22, %r28;
	add.f32 %f23, %f21, %f22;
	mov.b32 %r29, %f23;
	shfl.sync.bfly.b32 %r30|%p4, %r29, 8, 0x1f, 0xffffffff;
	mov.b32 %f24, %r30;
	add.f32 %f25, %f23, %f24;
	mov.b32 %r31, %f25;
	shfl.sync.bfly.b32 %r32|%p5, %r31, 4, 0x1f, 0xffffffff;
	mov.b32 %f26, %r32;
	add.f32 %f27, %f25, %f26;
	mov.b32 %r33, %f27;
	shfl.sync.bfly.b32 %r34|%p6, %r33, 2, 0x1f, 0xffffffff;
	mov.b32 %f28, %r34;
	add.f32 %f29, %f27, %f28;
	mov.b32 %r35, %f29;
	shfl.sync.bfly.b32 %r36|%p7, %r35, 1, 0x1f, 0xffffffff;
	mov.b32 %f30, %r36;
	add.f32 %f31, %f29, %f30;
	mov.b32 %f32, 0f3DB504F3;
	mul.f32 %f33, %f31, %f32;
	setp.gt.s32 %p8, %r23, %r13;
	@!%p8 bra L6_selnext;
	mov.b32 %f34, 0fFF800000;
	mov.b32 %f35, %f34;
	bra L4_selend;
L6_selnext:
	mov.b32 %f35, %f33;
L4_selend:
	max.f32 %f36, %f5, %f35;
	sub.f32 %f37, %f5, %f36;
	mov.b32 %f38, 0f3FB8AA3B;
	mul.f32 %f39, %f37, %f38;
	ex2.approx.f32 %f40, %f39;
	sub.f32 %f41, %f35, %f36;
	mov.b32 %f42, 0f3FB8AA3B;
	mul.f32 %f43, %f41, %f42;
	ex2.approx.f32 %f44, %f43;
	mul.f32 %f45, %f6, %f40;
	add.f32 %f6, %f45, %f44;
	mad.lo.s32 %r40, %r38, 4096, %r23;
	mad.lo.s32 %r42, %r40, 128, %r16;
	mad.wide.s32 %rd13, %r42, 2, %rd3;
	ld.global.b16 %rs9, [%rd13];
	cvt.f32.bf16 %f46, %rs9;
	add.s64 %rd14, %rd13, 2;
	ld.global.b16 %rs10, [%rd14];
	cvt.f32.bf16 %f47, %rs10;
	add.s64 %rd15, %rd13, 4;
	ld.global.b16 %rs11, [%rd15];
	cvt.f32.bf16 %f48, %rs11;
	add.s64 %rd16, %rd13, 6;
	ld.global.b16 %rs12, [%rd16];
	cvt.f32.bf16 %f49, %rs12;
	mul.f32 %f50, %f7, %f40;
	mul.f32 %f51, %f8, %f40;
	mul.f32 %f52, %f9, %f40;
	mul.f32 %f53, %f10, %f40;
	mul.f32 %f54, %f44, %f46;
	mul.f32 %f55, %f44, %f47;
	mul.f32 %f56, %f44, %f48;
	mul.f32 %f57, %f44, %f49;
	add.f32 %f7, %f50, %f54;
	add.f32 %f8, %f51, %f55;
	add.f32 %f9, %f52, %f56;
	add.f32 %f10, %f53, %f57;
	max.f32 %f5, %f5, %f35;
	add.s32 %r23, %r23, 1;
	bra L2_top;
L3_lend:
	div.rn.f32 %f58, %f7, %f6;
	div.rn.f32 %f59, %f8, %f6;
	div.rn.f32 %f60, %f9, %f6;
	div.rn.f32 %f61, %f10, %f6;
	mad.lo.s32 %r44, %r7, 32, %r10;
	mad.lo.s32 %r46, %r44, 4096, %r13;
	mad.lo.s32 %r48, %r46, 128, %r16;
	mad.wide.s32 %rd17, %r48, 2, %rd4;
	cvt.rn.bf16.f32 %rs13, %f58;
	st.global.b16 [%rd17], %rs13;
	add.s64 %rd18, %rd17, 2;
	cvt.rn.bf16.f32 %rs14, %f59;
	st.global.b16 [%rd18], %rs14;
	add.s64 %rd19, %rd17, 4;
	cvt.rn.bf16.f32 %rs15, %f60;
	st.global.b16 [%rd19], %rs15;
	add.s64 %rd20, %rd17, 6;
	cvt.rn.bf16.f32 %rs16, %f61;
	st.global.b16 [%rd20], %rs16;
L1_end:
	ret;
}
