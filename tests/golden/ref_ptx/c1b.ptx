.version 8.0
.target sm_89
.address_size 64

.shared .align 16 .f32 red_m[2];
.shared .align 16 .f32 red_s[2];

.visible .entry row_softmax(
	.param .u64 p_x,
	.param .u64 p_y
)
.maxntid 64, 1, 1
{
	.reg .pred %p<16>;
	.reg .b32 %r<51>;
	.reg .f32 %f<59>;
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
	mov.u32 %r7, red_m;
	mov.u32 %r8, red_s;
	setp.lt.s32 %p1, %r4, 2112;
	@!%p1 bra L1_end;
	div.s32 %r9, %r4, 64;
	mul.lo.s32 %r10, %r9, 64;
	sub.s32 %r11, %r4, %r10;
	mul.lo.s32 %r12, %r11, 4;
	mad.lo.s32 %r14, %r9, 256, %r12;
	mad.wide.s32 %rd3, %r14, 4, %rd1;
	ld.global.v4.f32 {%f1, %f2, %f3, %f4}, [%rd3];
	max.f32 %f5, %f1, %f2;
	max.f32 %f6, %f3, %f4;
	max.f32 %f7, %f5, %f6;
	mov.b32 %r15, %f7;
	shfl.sync.bfly.b32 %r16|%p2, %r15, 16, 0x1f, 0xffffffff;
	mov.b32 %f8, %r16;
	max.f32 %f9, %f7, %f8;
	mov.b32 %r17, %f9;
	shfl.sync.bfly.b32 %r18|%p3, %r17, 8, 0x1f, 0xffffffff;
	mov.b32 %f10, %r18;
	max.f32 %f11, %f9, %f10;
	mov.b32 %r19, %f11;
	shfl.sync.bfly.b32 %r20|%p4, %r19, 4, 0x1f, 0xffffffff;
	mov.b32 %f12, %r20;
	max.f32 %f13, %f11, %f12;
	mov.b32 %r21, %f13;
	shfl.sync.bfly.b32 %r22|%p5, %r21, 2, 0x1f, 0xffffffff;
	mov.b32 %f14, %r22;
	max.f32 %f15, %f13, %f14;
	mov.b32 %r23, %f15;
	shfl.sync.bfly.b32 %r24|%p6, %r23, 1, 0x1f, 0xffffffff;
	mov.b32 %f16, %r24;
	max.f32 %f17, %f15, %f16;
	setp.eq.s32 %p7, %r5, 0;
	@!%p7 bra L2_else;
	mad.lo.s32 %r26, %r6, 4, %r7;
	st.shared.f32 [%r26], %f17;
L2_else:
	bar.sync 0;
	setp.lt.s32 %p8, %r11, 1;
	@!%p8 bra L4_tskip;
	mad.lo.s32 %r28, %r11, 4, %r7;
	add.s32 %r29, %r11, 1;
	mad.lo.s32 %r31, %r29, 4, %r7;
	ld.shared.f32 %f18, [%r28];
	ld.shared.f32 %f19, [%r31];
	max.f32 %f20, %f18, %f19;
	st.shared.f32 [%r28], %f20;
L4_tskip:
	bar.sync 0;
	ld.shared.f32 %f21, [%r7];
	sub.f32 %f22, %f1, %f21;
	sub.f32 %f23, %f2, %f21;
	sub.f32 %f24, %f3, %f21;
	sub.f32 %f25, %f4, %f21;
	mov.b32 %f26, 0f3FB8AA3B;
	mul.f32 %f27, %f22, %f26;
	ex2.approx.f32 %f28, %f27;
	mov.b32 %f29, 0f3FB8AA3B;
	mul.f32 %f30, %f23, %f29;
	ex2.approx.f32 %f31, %f30;
	mov.b32 %f32, 0f3FB8AA3B;
	mul.f32 %f33, %f24, %f32;
	ex2.approx.f32 %f34, %f33;
	mov.b32 %f35, 0f3FB8AA3B;
	mul.f32 %f36, %f25, %f35;
	ex2.approx.f32 %f37, %f36;
	add.f32 %f38, %f28, %f31;
	add.f32 %f39, %f34, %f37;
	add.f32 %f40, %f38, %f39;
	mov.b32 %r32, %f40;
	shfl.sync.bfly.b32 %r33|%p9, %r32, 16, 0x1f, 0xffffffff;
	mov.b32 %f41, %r33;
	add.f32 %f42, %f40, %f41;
	mov.b32 %r34, %f42;
	shfl.sync.bfly.b32 %r35|%p10, %r34, 8, 0x1f, 0xffffffff;
	mov.b32 %f43, %r35;
	add.f32 %f44, %f42, %f43;
	mov.b32 %r36, %f44;
	shfl.sync.bfly.b32 %r37|%p11, %r36, 4, 0x1f, 0xffffffff;
	mov.b32 %f45, %r37;
	add.f32 %f46, %f44, %f45;
	mov.b32 %r38, %f46;
	shfl.sync.bfly.b32 %r39|%p12, %r38, 2, 0x1f, 0xffffffff;
	mov.b32 %f47, %r39;
	add.f32 %f48, %f46, %f47;
	mov.b32 %r40, %f48;
	shfl.sync.bfly.b32 %r41|%p13, %r40, 1, 0x1f, 0xffffffff;
	mov.b32 %f49, %r41;
	add.f32 %f50, %f48, %f49;
	setp.eq.s32 %p14, %r5, 0;
	@!%p14 bra L5_else;
	mad.lo.s32 %r43, %r6, 4, %r8;
	st.shared.f32 [%r43], %f50;
L5_else:
	bar.sync 0;
	setp.lt.s32 %p15, %r11, 1;
	@!%p15 bra L7_tskip;
	mad.lo.s32 %r45, %r11, 4, %r8;
	add.s32 %r46, %r11, 1;
	mad.lo.s32 %r48, %r46, 4, %r8;
	ld.shared.f32 %f51, [%r45];
	ld.shared.f32 %f52, [%r48];
	add.f32 %f53, %f51, %f52;
	st.shared.f32 [%r45], %f53;
L7_tskip:
	bar.sync 0;
	ld.shared.f32 %f54, [%r8];
	div.rn.f32 %f55, %f28, %f54;
	div.rn.f32 %f56, %f31, %f54;
	div.rn.f32 %f57, %f34, %f54;
	div.rn.f32 %f58, %f37, %f54;
	mad.lo.s32 %r50, %r9, 256, %r12;
	mad.wide.s32 %rd4, %r50, 4, %rd2;
	st.global.v4.f32 [%rd4], {%f55, %f56, %f57, %f58};
L1_end:
	ret;
}
