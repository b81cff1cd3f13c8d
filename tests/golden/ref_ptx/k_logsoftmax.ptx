.version 8.0
.target sm_89
.address_size 64

.shared .align 16 .f32 red_m[4];
.shared .align 16 .f32 red_s[4];

.visible .entry log_softmax(
	.param .u64 p_x,
	.param .u64 p_y
)
.maxntid 128, 1, 1
{
	.reg .pred %p<21>;
	.reg .b32 %r<61>;
	.reg .f32 %f<49>;
	.reg .b64 %rd<7>;
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
	setp.lt.s32 %p1, %r4, 1024;
	@!%p1 bra L1_end;
	div.s32 %r9, %r4, 128;
	mul.lo.s32 %r10, %r9, 128;
	sub.s32 %r11, %r4, %r10;
	mov.b32 %f1, 0fFF800000;
	mov.s32 %r12, %r11;
L2_top:
	setp.ge.s32 %p2, %r12, 512;
	@%p2 bra L3_lend;
	mad.lo.s32 %r14, %r9, 512, %r12;
	mad.wide.s32 %rd3, %r14, 4, %rd1;
	ld.global.f32 %f2, [%rd3];
	max.f32 %f1, %f1, %f2;
	add.s32 %r12, %r12, 128;
	bra L2_top;
L3_lend:
	mov.b32 %r15, %f1;
	shfl.sync.bfly.b32 %r16|%p3, %r15, 16, 0x1f, 0xffffffff;
	mov.b32 %f3, %r16;
	max.f32 %f4, %f1, %f3;
	mov.b32 %r17, %f4;
	shfl.sync.bfly.b32 %r18|%p4, %r17, 8, 0x1f, 0xffffffff;
	mov.b32 %f5, %r18;
	max.f32 %f6, %f4, %f5;
	mov.b32 %r19, %f6;
	shfl.sync.bfly.b32 %r20|%p5, %r19, 4, 0x1f, 0xffffffff;
	mov.b32 %f7, %r20;
	max.f32 %f8, %f6, %f7;
	mov.b32 %r21, %f8;
	shfl.sync.bfly.b32 %r22|%p6, %r21, 2, 0x1f, 0xffffffff;
	mov.b32 %f9, %r22;
	max.f32 %f10, %f8, %f9;
	mov.b32 %r23, %f10;
	shfl.sync.bfly.b32 %r24|%p7, %r23, 1, 0x1f, 0xffffffff;
	mov.b32 %f11, %r24;
	max.f32 %f12, %f10, %f11;
	setp.eq.s32 %p8, %r5, 0;
	@!%p8 bra L4_else;
	mad.lo.s32 %r26, %r6, 4, %r7;
	st.shared.f32 [%r26], %f12;
L4_else:
	bar.sync 0;
	setp.lt.s32 %p9, %r11, 2;
	@!%p9 bra L6_tskip;
	mad.lo.s32 %r28, %r11, 4, %r7;
	add.s32 %r29, %r11, 2;
	mad.lo.s32 %r31, %r29, 4, %r7;
	ld.shared.f32 %f13, [%r28];
	ld.shared.f32 %f14, [%r31];
	max.f32 %f15, %f13, %f14;
	st.shared.f32 [%r28], %f15;
L6_tskip:
	bar.sync 0;
	setp.lt.s32 %p10, %r11, 1;
	@!%p10 bra L7_tskip;
	add.s32 %r32, %r11, 1;
	mad.lo.s32 %r34, %r32, 4, %r7;
	ld.shared.f32 %f16, [%r28];
	ld.shared.f32 %f17, [%r34];
	max.f32 %f18, %f16, %f17;
	st.shared.f32 [%r28], %f18;
L7_tskip:
	bar.sync 0;
	ld.shared.f32 %f19, [%r7];
	mov.b32 %f20, 0f00000000;
	mov.s32 %r35, %r11;
L8_top:
	setp.ge.s32 %p11, %r35, 512;
	@%p11 bra L9_lend;
	mad.lo.s32 %r37, %r9, 512, %r35;
	mad.wide.s32 %rd4, %r37, 4, %rd1;
	ld.global.f32 %f21, [%rd4];
	sub.f32 %f22, %f21, %f19;
	mov.b32 %f23, 0f3FB8AA3B;
	mul.f32 %f24, %f22, %f23;
	ex2.approx.f32 %f25, %f24;
	add.f32 %f20, %f20, %f25;
	add.s32 %r35, %r35, 128;
	bra L8_top;
L9_lend:
	mov.b32 %r38, %f20;
	shfl.sync.bfly.b32 %r39|%p12, %r38, 16, 0x1f, 0xffffffff;
	mov.b32 %f26, %r39;
	add.f32 %f27, %f20, %f26;
	mov.b32 %r40, %f27;
	shfl.sync.bfly.b32 %r41|%p13, %r40, 8, 0x1f, 0xffffffff;
	mov.b32 %f28, %r41;
	add.f32 %f29, %f27, %f28;
	mov.b32 %r42, %f29;
	shfl.sync.bfly.b32 %r43|%p14, %r42, 4, 0x1f, 0xffffffff;
	mov.b32 %f30, %r43;
	add.f32 %f31, %f29, %f30;
	mov.b32 %r44, %f31;
	shfl.sync.bfly.b32 %r45|%p15, %r44, 2, 0x1f, 0xffffffff;
	mov.b32 %f32, %r45;
	add.f32 %f33, %f31, %f32;
	mov.b32 %r46, %f33;
	shfl.sync.bfly.b32 %r47|%p16, %r46, 1, 0x1f, 0xffffffff;
	mov.b32 %f34, %r47;
	add.f32 %f35, %f33, %f34;
	setp.eq.s32 %p17, %r5, 0;
	@!%p17 bra L10_else;
	mad.lo.s32 %r49, %r6, 4, %r8;
	st.shared.f32 [%r49], %f35;
L10_else:
	bar.sync 0;
	setp.lt.s32 %p18, %r11, 2;
	@!%p18 bra L12_tskip;
	mad.lo.s32 %r51, %r11, 4, %r8;
	add.s32 %r52, %r11, 2;
	mad.lo.s32 %r54, %r52, 4, %r8;
	ld.shared.f32 %f36, [%r51];
	ld.shared.f32 %f37, [%r54];
	add.f32 %f38, %f36, %f37;
	st.shared.f32 [%r51], %f38;
L12_tskip:
	bar.sync 0;
	setp.lt.s32 %p19, %r11, 1;
	@!%p19 bra L13_tskip;
	add.s32 %r55, %r11, 1;
	mad.lo.s32 %r57, %r55, 4, %r8;
	ld.shared.f32 %f39, [%r51];
	ld.shared.f32 %f40, [%r57];
	add.f32 %f41, %f39, %f40;
	st.shared.f32 [%r51], %f41;
L13_tskip:
	bar.sync 0;
	ld.shared.f32 %f42, [%r8];
	lg2.approx.f32 %f43, %f42;
	mov.b32 %f44, 0f3F317218;
	mul.f32 %f45, %f43, %f44;
	mov.s32 %r58, %r11;
L14_top:
	setp.ge.s32 %p20, %r58, 512;
	@%p20 bra L15_lend;
	mad.lo.s32 %r60, %r9, 512, %r58;
	mad.wide.s32 %rd5, %r60, 4, %rd1;
	ld.global.f32 %f46, [%rd5];
	sub.f32 %f47, %f46, %f19;
	sub.f32 %f48, %f47, %f45;
	mad.wide.s32 %rd6, %r60, 4, %rd2;
	st.global.f32 [%rd6], %f48;
	add.s32 %r58, %r58, 128;
	bra L14_top;
L15_lend:
L1_end:
	ret;
}
