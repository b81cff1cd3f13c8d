.version 8.0
.target sm_89
.address_size 64

.visible .entry attention(
	.param .u64 p_Q,
	.param .u64 p_K,
	.param .u64 p_V,
	.param .u64 p_M,
	.param .u64 p_O
)
.maxntid 128, 1, 1
{
	.reg .pred %p<10>;
	.reg .b32 %r<51>;
	.reg .f32 %f<38>;
	.reg .b64 %rd<11>;
	.reg .b16 %rs<5>;
	ld.param.u64 %rd1, [p_Q];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_K];
	cvta.to.global.u64 %rd2, %rd2;
	ld.param.u64 %rd3, [p_V];
	cvta.to.global.u64 %rd3, %rd3;
	ld.param.u64 %rd4, [p_M];
	cvta.to.global.u64 %rd4, %rd4;
	ld.param.u64 %rd5, [p_O];
	cvta.to.global.u64 %rd5, %rd5;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	setp.lt.s32 %p1, %r4, 1024;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 1024;
	mul.lo.s32 %r8, %r7, 1024;
	sub.s32 %r9, %r4, %r8;
	div.s32 %r10, %r9, 512;
	mul.lo.s32 %r11, %r10, 512;
	sub.s32 %r12, %r9, %r11;
	div.s32 %r13, %r12, 32;
	mul.lo.s32 %r14, %r13, 32;
	sub.s32 %r15, %r12, %r14;
	mad.lo.s32 %r17, %r7, 2, %r10;
	mul.lo.s32 %r18, %r17, 16;
	add.s32 %r19, %r18, %r13;
	mad.lo.s32 %r21, %r19, 32, %r15;
	mad.wide.s32 %rd6, %r21, 2, %rd1;
	ld.global.b16 %rs1, [%rd6];
	cvt.f32.bf16 %f1, %rs1;
	mov.b32 %f2, 0fFF800000;
	mov.b32 %f3, 0f00000000;
	mov.b32 %f4, 0f00000000;
	mov.s32 %r22, 0;
	mad.lo.s32 %r40, %r7, 2, %r10;
L2_top:
	setp.ge.s32 %p2, %r22, 16;
	@%p2 bra L3_lend;
	add.s32 %r23, %r18, %r22;
	mad.lo.s32 %r25, %r23, 32, %r15;
	mad.wide.s32 %rd7, %r25, 2, %rd2;
	ld.global.b16 %rs2, [%rd7];
	cvt.f32.bf16 %f5, %rs2;
	mad.lo.s32 %r27, %r13, 16, %r22;
	mad.wide.s32 %rd8, %r27, 1, %rd4;
	ld.global.u8 %r28, [%rd8];
	mul.f32 %f6, %f1, %f5;
	mov.b32 %r29, %f6;
	shfl.sync.bfly.b32 %r30|%p3, %r29, 16, 0x1f, 0xffffffff;
	mov.b32 %f7, %r30;
	add.f32 %f8, %f6, %f7;
	mov.b32 %r31, %f8;
	shfl.sync.bfly.b32 %r32|%p4, %r31, 8, 0x1f, 0xffffffff;
	mov.b32 %f9, %r32;
	add.f32 %f10, %f8, %f9;
	mov.b32 %r33, %f10;
	shfl.sync.bfly.b32 %r34|%p5, %r33, 4, 0x1f, 0xffffffff;
	mov.b32 %f11, %r34;
	add.f32 %f12, %f10, %f11;
	mov.b32 %r35, %f12;
	shfl.sync.bfly.b32 %r36|%p6, %r35, 2, 0x1f, 0xffffffff;
	mov.b32 %f13, %r36;
	add.f32 %f14, %f12, %f13;
	mov.b32 %r37, %f14;
	shfl.sync.bfly.b32 %r38|%p7, %r37, 1, 0x1f, 0xffffffff;
	mov.b32 %f15, %r38;
	add.f32 %f16, %f14, %f15;
	mov.b32 %f17, 0f3E3504F3;
	mul.f32 %f18, %f16, %f17;
	setp.eq.s32 %p8, %r28, 0;
	@!%p8 bra L6_selnext;
	mov.b32 %f19, 0fFF800000;
	mov.b32 %f20, %f19;
	bra L4_selend;
L6_selnext:
	mov.b32 %f20, %f18;
L4_selend:
	max.f32 %f21, %f2, %f20;
	mov.b32 %f22, 0fFF800000;
	setp.eq.f32 %p9, %f21, %f22;
	@!%p9 bra L9_selnext;
	mov.b32 %f23, 0f00000000;
	mov.b32 %f24, %f23;
	bra L7_selend;
L9_selnext:
	mov.b32 %f24, %f21;
L7_selend:
	sub.f32 %f25, %f2, %f24;
	mov.b32 %f26, 0f3FB8AA3B;
	mul.f32 %f27, %f25, %f26;
	ex2.approx.f32 %f28, %f27;
	sub.f32 %f29, %f20, %f24;
	mov.b32 %f30, 0f3FB8AA3B;
	mul.f32 %f31, %f29, %f30;
	ex2.approx.f32 %f32, %f31;
	mul.f32 %f33, %f3, %f28;
	add.f32 %f3, %f33, %f32;
	mad.lo.s32 %r42, %r40, 16, %r22;
	mad.lo.s32 %r44, %r42, 32, %r15;
	mad.wide.s32 %rd9, %r44, 2, %rd3;
	ld.global.b16 %rs3, [%rd9];
	cvt.f32.bf16 %f34, %rs3;
	mul.f32 %f35, %f4, %f28;
	mul.f32 %f36, %f32, %f34;
	add.f32 %f4, %f35, %f36;
	max.f32 %f2, %f2, %f20;
	add.s32 %r22, %r22, 1;
	bra L2_top;
L3_lend:
	div.rn.f32 %f37, %f4, %f3;
	mad.lo.s32 %r46, %r7, 2, %r10;
	mad.lo.s32 %r48, %r46, 16, %r13;
	mad.lo.s32 %r50, %r48, 32, %r15;
	mad.wide.s32 %rd10, %r50, 2, %rd5;
	cvt.rn.bf16.f32 %rs4, %f37;
	st.global.b16 [%rd10], %rs4;
L1_end:
	ret;
}
