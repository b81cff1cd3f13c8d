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
	.reg .b32 %r<48>;
	.reg .f32 %f<34>;
	.reg .b64 %rd<9>;
	.reg .b16 %rs<5>;
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
	setp.lt.s32 %p1, %r4, 6144;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 6144;
	mul.lo.s32 %r8, %r7, 6144;
	sub.s32 %r9, %r4, %r8;
	div.s32 %r10, %r9, 1536;
	mul.lo.s32 %r11, %r10, 1536;
	sub.s32 %r12, %r9, %r11;
	div.s32 %r13, %r12, 32;
	mul.lo.s32 %r14, %r13, 32;
	sub.s32 %r15, %r12, %r14;
	mad.lo.s32 %r17, %r7, 4, %r10;
	mul.lo.s32 %r18, %r17, 48;
	add.s32 %r19, %r18, %r13;
	mad.lo.s32 %r21, %r19, 32, %r15;
	mad.wide.s32 %rd5, %r21, 2, %rd1;
	ld.global.b16 %rs1, [%rd5];
	cvt.f32.bf16 %f1, %rs1;
	mov.b32 %f2, 0fFF800000;
	mov.b32 %f3, 0f00000000;
	mov.b32 %f4, 0f00000000;
	mov.s32 %r22, 0;
	mad.lo.s32 %r37, %r7, 4, %r10;
L2_top:
	setp.ge.s32 %p2, %r22, 48;
	@%p2 bra L3_lend;
	add.s32 %r23, %r18, %r22;
	mad.lo.s32 %r25, %r23, 32, %r15;
	mad.wide.s32 %rd6, %r25, 2, %rd2;
	ld.global.b16 %rs2, [%rd6];
	cvt.f32.bf16 %f5, %rs2;
	mul.f32 %f6, %f1, %f5;
	mov.b32 %r26, %f6;
	shfl.sync.bfly.b32 %r27|%p3, %r26, 16, 0x1f, 0xffffffff;
	mov.b32 %f7, %r27;
	add.f32 %f8, %f6, %f7;
	mov.b32 %r28, %f8;
	shfl.sync.bfly.b32 %r29|%p4, %r28, 8, 0x1f, 0xffffffff;
	mov.b32 %f9, %r29;
	add.f32 %f10, %f8, %f9;
	mov.b32 %r30, %f10;
	shfl.sync.bfly.b32 %r31|%p5, %r30, 4, 0x1f, 0xffffffff;
	mov.b32 %f11, %r31;
	add.f32 %f12, %f10, %f11;
	mov.b32 %r32, %f12;
	shfl.sync.bfly.b32 %r33|%p6, %r32, 2, 0x1f, 0xffffffff;
	mov.b32 %f13, %r33;
	add.f32 %f14, %f12, %f13;
	mov.b32 %r34, %f14;
	shfl.sync.bfly.b32 %r35|%p7, %r34, 1, 0x1f, 0xffffffff;
	mov.b32 %f15, %r35;
	add.f32 %f16, %f14, %f15;
	mov.b32 %f17, 0f3E4CCCCD;
	mul.f32 %f18, %f16, %f17;
	mov.b32 %f19, %f18;
L4_selend:
	max.f32 %f20, %f2, %f19;
	sub.f32 %f21, %f2, %f20;
	mov.b32 %f22, 0f3FB8AA3B;
	mul.f32 %f23, %f21, %f22;
	ex2.approx.f32 %f24, %f23;
	sub.f32 %f25, %f19, %f20;
	mov.b32 %f26, 0f3FB8AA3B;
	mul.f32 %f27, %f25, %f26;
	ex2.approx.f32 %f28, %f27;
	mul.f32 %f29, %f3, %f24;
	add.f32 %f3, %f29, %f28;
	mad.lo.s32 %r39, %r37, 48, %r22;
	mad.lo.s32 %r41, %r39, 32, %r15;
	mad.wide.s32 %rd7, %r41, 2, %rd3;
	ld.global.b16 %rs3, [%rd7];
	cvt.f32.bf16 %f30, %rs3;
	mul.f32 %f31, %f4, %f24;
	mul.f32 %f32, %f28, %f30;
	add.f32 %f4, %f31, %f32;
	max.f32 %f2, %f2, %f19;
	add.s32 %r22, %r22, 1;
	bra L2_top;
L3_lend:
	div.rn.f32 %f33, %f4, %f3;
	mad.lo.s32 %r43, %r7, 4, %r10;
	mad.lo.s32 %r45, %r43, 48, %r13;
	mad.lo.s32 %r47, %r45, 32, %r15;
	mad.wide.s32 %rd8, %r47, 2, %rd4;
	cvt.rn.bf16.f32 %rs4, %f33;
	st.global.b16 [%rd8], %rs4;
L1_end:
	ret;
}
