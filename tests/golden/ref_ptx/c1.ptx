.version 8.0
.target sm_89
.address_size 64

.shared .align 16 .f32 red_m[8];
.shared .align 16 .f32 red_s[8];

.visible .entry row_softmax(
	.param .u64 p_x,
	.param .u64 p_y
)
.maxntid 256, 1, 1
{
	.reg .pred %p<20>;
	.reg .b32 %r<63>;
	.reg .f32 %f<71>;
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
	setp.lt.s32 %p1, %r4, 16384;
	@!%p1 bra L1_end;
	div.s32 %r9, %r4, 256;
	mul.lo.s32 %r10, %r9, 256;
	sub.s32 %r11, %r4, %r10;
	mul.lo.s32 %r12, %r11, 4;
	mad.lo.s32 %r14, %r9, 1024, %r12;
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
	setp.lt.s32 %p8, %r11, 4;
	@!%p8 bra L4_tskip;
	mad.lo.s32 %r28, %r11, 4, %r7;
	add.s32 %r29, %r11, 4;
	mad.lo.s32 %r31, %r29, 4, %r7;
	ld.shared.f32 %f18, [%r28];
	ld.shared.f32 %f19, [%r31];
	max.f32 %f20, %f18, %f19;
	st.shared.f32 [%r28], %f20;
L4_tskip:
	bar.sync 0;
	setp.lt.s32 %p9, %r11, 2;
	@!%p9 bra L5_tskip;
	add.s32 %r32, %r11, 2;
	mad.lo.s32 %r34, %r32, 4, %r7;
	ld.shared.f32 %f21, [%r28];
	ld.shared.f32 %f22, [%r34];
	max.f32 %f23, %f21, %f22;
	st.shared.f32 [%r28], %f23;
L5_tskip:
	bar.sync 0;
	setp.lt.s32 %p10, %r11, 1;
	@!%p10 bra L6_tskip;
	add.s32 %r35, %r11, 1;
	mad.lo.s32 %r37, %r35, 4, %r7;
	ld.shared.f32 %f24, [%r28];
	ld.shared.f32 %f25, [%r37];
	max.f32 %f26, %f24, %f25;
	st.shared.f32 [%r28], %f26;
L6_tskip:
	bar.sync 0;
	ld.shared.f32 %f27, [%r7];
	sub.f32 %f28, %f1, %f27;
	sub.f32 %f29, %f2, %f27;
	sub.f32 %f30, %f3, %f27;
	sub.f32 %f31, %f4, %f27;
	mov.b32 %f32, 0f3FB8AA3B;
	mul.f32 %f33, %f28, %f32;
	ex2.approx.f32 %f34, %f33;
	mov.b32 %f35, 0f3FB8AA3B;
	mul.f32 %f36, %f29, %f35;
	ex2.approx.f32 %f37, %f36;
	mov.b32 %f38, 0f3FB8AA3B;
	mul.f32 %f39, %f30, %f38;
	ex2.approx.f32 %f40, %f39;
	mov.b32 %f41, 0f3FB8AA3B;
	mul.f32 %f42, %f31, %f41;
	ex2.approx.f32 %f43, %f42;
	add.f32 %f44, %f34, %f37;
	add.f32 %f45, %f40, %f43;
	add.f32 %f46, %f44, %f45;
	mov.b32 %r38, %f46;
	shfl.sync.bfly.b32 %r39|%p11, %r38, 16, 0x1f, 0xffffffff;
	mov.b32 %f47, %r39;
	add.f32 %f48, %f46, %f47;
	mov.b32 %r40, %f48;
	shfl.sync.bfly.b32 %r41|%p12, %r40, 8, 0x1f, 0xffffffff;
	mov.b32 %f49, %r41;
	add.f32 %f50, %f48, %f49;
	mov.b32 %r42, %f50;
	shfl.sync.bfly.b32 %r43|%p13, %r42, 4, 0x1f, 0xffffffff;
	mov.b32 %f51, %r43;
	add.f32 %f52, %f50, %f51;
	mov.b32 %r44, %f52;
	shfl.sync.bfly.b32 %r45|%p14, %r44, 2, 0x1f, 0xffffffff;
	mov.b32 %f53, %r45;
	add.f32 %f54, %f52, %f53;
	mov.b32 %r46, %f54;
	shfl.sync.bfly.b32 %r47|%p15, %r46, 1, 0x1f, 0xffffffff;
	mov.b32 %f55, %r47;
	add.f32 %f56, %f54, %f55;
	setp.eq.s32 %p16, %r5, 0;
	@!%p16 bra L7_else;
	mad.lo.s32 %r49, %r6, 4, %r8;
	st.shared.f32 [%r49], %f56;
L7_else:
	bar.sync 0;
	setp.lt.s32 %p17, %r11, 4;
	@!%p17 bra L9_tskip;
	mad.lo.s32 %r51, %r11, 4, %r8;
	add.s32 %r52, %r11, 4;
	mad.lo.s32 %r54, %r52, 4, %r8;
	ld.shared.f32 %f57, [%r51];
	ld.shared.f32 %f58, [%r54];
	add.f32 %f59, %f57, %f58;
	st.shared.f32 [%r51], %f59;
L9_tskip:
	bar.sync 0;
	setp.lt.s32 %p18, %r11, 2;
	@!%p18 bra L10_tskip;
	add.s32 %r55, %r11, 2;
	mad.lo.s32 %r57, %r55, 4, %r8;
	ld.shared.f32 %f60, [%r51];
	ld.shared.f32 %f61, [%r57];
	add.f32 %f62, %f60, %f61;
	st.shared.f32 [%r51], %f62;
L10_tskip:
	bar.sync 0;
	setp.lt.s32 %p19, %r11, 1;
	@!%p19 bra L11_tskip;
	add.s32 %r58, %r11, 1;
	mad.lo.s32 %r60, %r58, 4, %r8;
	ld.shared.f32 %f63, [%r51];
	ld.shared.f32 %f64, [%r60];
	add.f32 %f65, %f63, %f64;
	st.shared.f32 [%r51], %f65;
L11_tskip:
	bar.sync 0;
	ld.shared.f32 %f66, [%r8];
	div.rn.f32 %f67, %f34, %f66;
	div.rn.f32 %f68, %f37, %f66;
	div.rn.f32 %f69, %f40, %f66;
	div.rn.f32 %f70, %f43, %f66;
	mad.lo.s32 %r62, %r9, 1024, %r12;
	mad.wide.s32 %rd4, %r62, 4, %rd2;
	st.global.v4.f32 [%rd4], {%f67, %f68, %f69, %f70};
L1_end:
	ret;
}
