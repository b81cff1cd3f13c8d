.version 8.0
.target sm_89
.address_size 64

.visible .entry attention(
	.param .u64 p_Q,
	.param .u64 p_K,
	.param .u64 p_V,
	.param .u64 p_O
)
.maxntid 128, 1, 1
{
	.reg .pred %p<8>;
	.reg .b32 %r<49>;
	.reg .f32 %f<43>;
	.reg .b64 %rd<13>;
	.reg .b16 %rs<9>;
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
	setp.lt.s32 %p1, %r4, 16384;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 16384;
	mul.lo.s32 %r8, %r7, 16384;
	sub.s32 %r9, %r4, %r8;
	div.s32 %r10, %r9, 4096;
	mul.lo.s32 %r11, %r10, 4096;
	sub.s32 %r12, %r9, %r11;
	div.s32 %r13, %r12, 32;
	mul.lo.s32 %r14, %r13, 32;
	sub.s32 %r15, %r12, %r14;
	mul.lo.s32 %r16, %r15, 2;
	mad.lo.s32 %r18, %r7, 4, %r10;
	mul.lo.s32 %r19, %r18, 128;
	add.s32 %r20, %r19, %r13;
	mad.lo.s32 %r22, %r20, 64, %r16;
	mad.wide.s32 %rd5, %r22, 2, %rd1;
	ld.global.b16 %rs1, [%rd5];
	cvt.f32.bf16 %f1, %rs1;
	add.s64 %rd6, %rd5, 2;
	ld.global.b16 %rs2, [%rd6];
	cvt.f32.bf16 %f2, %rs2;
	mov.b32 %f3, 0fFF800000;
	mov.b32 %f4, 0f00000000;
	mov.b32 %f5, 0f00000000;
	mov.b32 %f6, 0f00000000;
	mov.s32 %r23, 0;
	mad.lo.s32 %r38, %r7, 4, %r10;
L2_top:
	setp.ge.s32 %p2, %r23, 128;
	@%p2 bra L3_lend;
	add.s32 %r24, %r19, %r23;
	mad.lo.s32 %r26, %r24, 64, %r16;
	mad.wide.s32 %rd7, %r26, 2, %rd2;
	ld.global.b16 %rs3, [%rd7];
	cvt.f32.bf16 %f7, %rs3;
	add.s64 %rd8, %rd7, 2;
	ld.global.b16 %rs4, [%rd8];
	cvt.f32.bf16 %f8, %rs4;
	mul.f32 %f9, %f1, %f7;
	mul.f32 %f10, %f2, %f8;
	add.f32 %f11, %f9, %f10;
	mov.b32 %r27, %f11;
	shfl.sync.bfly.b32 %r28|%p3, %r27, 16, 0x1f, 0xffffffff;
	mov.b32 %f12, %r28;
	add.f32 %f13, %f11, %f12;
	mov.b32 %r29, %f13;
	shfl.sync.bfly.b32 %r30|%p4, %r29, 8, 0x1f, 0xffffffff;
	mov.b32 %f14, %r30;
	add.f32 %f15, %f13, %f14;
	mov.b32 %r31, %f15;
	shfl.sync.bfly.b32 %r32|%p5, %r31, 4, 0x1f, 0xffffffff;
	mov.b32 %f16, %r32;
	add.f32 %f17, %f15, %f16;
	mov.b32 %r33, %f17;
	shfl.sync.bfly.b32 %r34|%p6, %r33, 2, 0x1f, 0xffffffff;
	mov.b32 %f18, %r34;
	add.f32 %f19, %f17, %f18;
	mov.b32 %r35, %f19;
	shfl.sync.bfly.b32 %r36|%p7, %r35, 1, 0x1f, 0xffffffff;
	mov.b32 %f20, %r36;
	add.f32 %f21, %f19, %f20;
	mov.b32 %f22, 0f3E000000;
	mul.f32 %f23, %f21, %f22;
	mov.b32 %f24, %f23;
L4_selend:
	max.f32 %f25, %f3, %f24;
	sub.f32 %f26, %f3, %f25;
	mov.b32 %f27, 0f3FB8AA3B;
	mul.f32 %f28, %f26, %f27;
	ex2.approx.f32 %f29, %f28;
	sub.f32 %f30, %f24, %f25;
	mov.b32 %f31, 0f3FB8AA3B;
	mul.f32 %f32, %f30, %f31;
	ex2.approx.f32 %f33, %f32;
	mul.f32 %f34, %f4, %f29;
	add.f32 %f4, %f34, %f33;
	mad.lo.s32 %r40, %r38, 128, %r23;
	mad.lo.s32 %r42, %r40, 64, %r16;
	mad.wide.s32 %rd9, %r42, 2, %rd3;
	ld.global.b16 %rs5, [%rd9];
	cvt.f32.bf16 %f35, %rs5;
	add.s64 %rd10, %rd9, 2;
	ld.global.b16 %rs6, [%rd10];
	cvt.f32.bf16 %f36, %rs6;
	mul.f32 %f37, %f5, %f29;
	mul.f32 %f38, %f6, %f29;
	mul.f32 %f39, %f33, %f35;
	mul.f32 %f40, %f33, %f36;
	add.f32 %f5, %f37, %f39;
	add.f32 %f6, %f38, %f40;
	max.f32 %f3, %f3, %f24;
	add.s32 %r23, %r23, 1;
	bra L2_top;
L3_lend:
	div.rn.f32 %f41, %f5, %f4;
	div.rn.f32 %f42, %f6, %f4;
	mad.lo.s32 %r44, %r7, 4, %r10;
	mad.lo.s32 %r46, %r44, 128, %r13;
	mad.lo.s32 %r48, %r46, 64, %r16;
	mad.wide.s32 %rd11, %r48, 2, %rd4;
	cvt.rn.bf16.f32 %rs7, %f41;
	st.global.b16 [%rd11], %rs7;
	add.s64 %rd12, %rd11, 2;
	cvt.rn.bf16.f32 %rs8, %f42;
	st.global.b16 [%rd12], %rs8;
L1_end:
	ret;
}
