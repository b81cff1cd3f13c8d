.version 8.0
.target sm_89
.address_size 64

.shared .align 16 .f32 red_s[2];
.shared .align 16 .f32 red_q[2];

.visible .entry group_norm(
	.param .u64 p_x,
	.param .u64 p_y
)
.maxntid 64, 1, 1
{
	.reg .pred %p<16>;
	.reg .b32 %r<71>;
	.reg .f32 %f<45>;
	.reg .b64 %rd<6>;
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
	mov.u32 %r7, red_s;
	mov.u32 %r8, red_q;
	setp.lt.s32 %p1, %r4, 128;
	@!%p1 bra L1_end;
	div.s32 %r9, %r4, 128;
	mul.lo.s32 %r10, %r9, 128;
	sub.s32 %r11, %r4, %r10;
	div.s32 %r12, %r11, 64;
	mul.lo.s32 %r13, %r12, 64;
	sub.s32 %r14, %r11, %r13;
	mov.b32 %f1, 0f00000000;
	mov.b32 %f2, 0f00000000;
	mov.s32 %r15, %r14;
L2_top:
	setp.ge.s32 %p2, %r15, 256;
	@%p2 bra L3_lend;
	div.s32 %r18, %r15, 128;
	mad.lo.s32 %r19, %r12, 2, %r18;
	mad.lo.s32 %r20, %r9, 4, %r19;
	rem.s32 %r22, %r15, 128;
	div.s32 %r23, %r22, 16;
	mad.lo.s32 %r24, %r20, 8, %r23;
	rem.s32 %r26, %r15, 16;
	mad.lo.s32 %r27, %r24, 16, %r26;
	mad.wide.s32 %rd3, %r27, 4, %rd1;
	ld.global.f32 %f3, [%rd3];
	add.f32 %f1, %f1, %f3;
	mul.f32 %f4, %f3, %f3;
	add.f32 %f2, %f2, %f4;
	add.s32 %r15, %r15, 64;
	bra L2_top;
L3_lend:
	mov.b32 %r28, %f1;
	shfl.sync.bfly.b32 %r29|%p3, %r28, 16, 0x1f, 0xffffffff;
	mov.b32 %f5, %r29;
	mov.b32 %r30, %f2;
	shfl.sync.bfly.b32 %r31|%p4, %r30, 16, 0x1f, 0xffffffff;
	mov.b32 %f6, %r31;
	add.f32 %f7, %f1, %f5;
	add.f32 %f8, %f2, %f6;
	mov.b32 %r32, %f7;
	shfl.sync.bfly.b32 %r33|%p5, %r32, 8, 0x1f, 0xffffffff;
	mov.b32 %f9, %r33;
	mov.b32 %r34, %f8;
	shfl.sync.bfly.b32 %r35|%p6, %r34, 8, 0x1f, 0xffffffff;
	mov.b32 %f10, %r35;
	add.f32 %f11, %f7, %f9;
	add.f32 %f12, %f8, %f10;
	mov.b32 %r36, %f11;
	shfl.sync.bfly.b32 %r37|%p7, %r36, 4, 0x1f, 0xffffffff;
	mov.b32 %f13, %r37;
	mov.b32 %r38, %f12;
	shfl.sync.bfly.b32 %r39|%p8, %r38, 4, 0x1f, 0xffffffff;
	mov.b32 %f14, %r39;
	add.f32 %f15, %f11, %f13;
	add.f32 %f16, %f12, %f14;
	mov.b32 %r40, %f15;
	shfl.sync.bfly.b32 %r41|%p9, %r40, 2, 0x1f, 0xffffffff;
	mov.b32 %f17, %r41;
	mov.b32 %r42, %f16;
	shfl.sync.bfly.b32 %r43|%p10, %r42, 2, 0x1f, 0xffffffff;
	mov.b32 %f18, %r43;
	add.f32 %f19, %f15, %f17;
	add.f32 %f20, %f16, %f18;
	mov.b32 %r44, %f19;
	shfl.sync.bfly.b32 %r45|%p11, %r44, 1, 0x1f, 0xffffffff;
	mov.b32 %f21, %r45;
	mov.b32 %r46, %f20;
	shfl.sync.bfly.b32 %r47|%p12, %r46, 1, 0x1f, 0xffffffff;
	mov.b32 %f22, %r47;
	add.f32 %f23, %f19, %f21;
	add.f32 %f24, %f20, %f22;
	setp.eq.s32 %p13, %r5, 0;
	@!%p13 bra L4_else;
	mul.lo.s32 %r48, %r6, 4;
	add.s32 %r49, %r7, %r48;
	st.shared.f32 [%r49], %f23;
	add.s32 %r50, %r8, %r48;
	st.shared.f32 [%r50], %f24;
L4_else:
	bar.sync 0;
	setp.lt.s32 %p14, %r14, 1;
	@!%p14 bra L6_tskip;
	mul.lo.s32 %r51, %r14, 4;
	add.s32 %r52, %r7, %r51;
	add.s32 %r53, %r14, 1;
	mul.lo.s32 %r54, %r53, 4;
	add.s32 %r55, %r7, %r54;
	ld.shared.f32 %f25, [%r52];
	ld.shared.f32 %f26, [%r55];
	add.s32 %r56, %r8, %r51;
	add.s32 %r57, %r8, %r54;
	ld.shared.f32 %f27, [%r56];
	ld.shared.f32 %f28, [%r57];
	add.f32 %f29, %f25, %f26;
	add.f32 %f30, %f27, %f28;
	st.shared.f32 [%r52], %f29;
	st.shared.f32 [%r56], %f30;
L6_tskip:
	bar.sync 0;
	ld.shared.f32 %f31, [%r7];
	ld.shared.f32 %f32, [%r8];
	mov.b32 %f33, 0f3B800000;
	mul.f32 %f34, %f31, %f33;
	mov.b32 %f35, 0f3B800000;
	mul.f32 %f36, %f32, %f35;
	mul.f32 %f37, %f34, %f34;
	sub.f32 %f38, %f36, %f37;
	mov.b32 %f39, 0f3727C5AC;
	add.f32 %f40, %f38, %f39;
	rsqrt.approx.f32 %f41, %f40;
	mov.s32 %r58, %r14;
L7_top:
	setp.ge.s32 %p15, %r58, 256;
	@%p15 bra L8_lend;
	div.s32 %r61, %r58, 128;
	mad.lo.s32 %r62, %r12, 2, %r61;
	mad.lo.s32 %r63, %r9, 4, %r62;
	rem.s32 %r65, %r58, 128;
	div.s32 %r66, %r65, 16;
	mad.lo.s32 %r67, %r63, 8, %r66;
	rem.s32 %r69, %r58, 16;
	mad.lo.s32 %r70, %r67, 16, %r69;
	mad.wide.s32 %rd4, %r70, 4, %rd1;
	ld.global.f32 %f42, [%rd4];
	sub.f32 %f43, %f42, %f34;
	mul.f32 %f44, %f43, %f41;
	mad.wide.s32 %rd5, %r70, 4, %rd2;
	st.global.f32 [%rd5], %f44;
	add.s32 %r58, %r58, 64;
	bra L7_top;
L8_lend:
L1_end:
	ret;
}
