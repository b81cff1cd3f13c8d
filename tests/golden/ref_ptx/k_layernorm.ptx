.version 8.0
.target sm_89
.address_size 64

.shared .align 16 .f32 red_s[2];
.shared .align 16 .f32 red_q[2];

.visible .entry layer_norm(
	.param .u64 p_x,
	.param .u64 p_g,
	.param .u64 p_b,
	.param .u64 p_y
)
.maxntid 64, 1, 1
{
	.reg .pred %p<16>;
	.reg .b32 %r<48>;
	.reg .f32 %f<49>;
	.reg .b64 %rd<10>;
	ld.param.u64 %rd1, [p_x];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_g];
	cvta.to.global.u64 %rd2, %rd2;
	ld.param.u64 %rd3, [p_b];
	cvta.to.global.u64 %rd3, %rd3;
	ld.param.u64 %rd4, [p_y];
	cvta.to.global.u64 %rd4, %rd4;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	mov.u32 %r7, red_s;
	mov.u32 %r8, red_q;
	setp.lt.s32 %p1, %r4, 1024;
	@!%p1 bra L1_end;
	div.s32 %r9, %r4, 64;
	mul.lo.s32 %r10, %r9, 64;
	sub.s32 %r11, %r4, %r10;
	mov.b32 %f1, 0f00000000;
	mov.b32 %f2, 0f00000000;
	mov.s32 %r12, %r11;
L2_top:
	setp.ge.s32 %p2, %r12, 256;
	@%p2 bra L3_lend;
	mad.lo.s32 %r14, %r9, 256, %r12;
	mad.wide.s32 %rd5, %r14, 4, %rd1;
	ld.global.f32 %f3, [%rd5];
	add.f32 %f1, %f1, %f3;
	mul.f32 %f4, %f3, %f3;
	add.f32 %f2, %f2, %f4;
	add.s32 %r12, %r12, 64;
	bra L2_top;
L3_lend:
	mov.b32 %r15, %f1;
	shfl.sync.bfly.b32 %r16|%p3, %r15, 16, 0x1f, 0xffffffff;
	mov.b32 %f5, %r16;
	mov.b32 %r17, %f2;
	shfl.sync.bfly.b32 %r18|%p4, %r17, 16, 0x1f, 0xffffffff;
	mov.b32 %f6, %r18;
	add.f32 %f7, %f1, %f5;
	add.f32 %f8, %f2, %f6;
	mov.b32 %r19, %f7;
	shfl.sync.bfly.b32 %r20|%p5, %r19, 8, 0x1f, 0xffffffff;
	mov.b32 %f9, %r20;
	mov.b32 %r21, %f8;
	shfl.sync.bfly.b32 %r22|%p6, %r21, 8, 0x1f, 0xffffffff;
	mov.b32 %f10, %r22;
	add.f32 %f11, %f7, %f9;
	add.f32 %f12, %f8, %f10;
	mov.b32 %r23, %f11;
	shfl.sync.bfly.b32 %r24|%p7, %r23, 4, 0x1f, 0xffffffff;
	mov.b32 %f13, %r24;
	mov.b32 %r25, %f12;
	shfl.sync.bfly.b32 %r26|%p8, %r25, 4, 0x1f, 0xffffffff;
	mov.b32 %f14, %r26;
	add.f32 %f15, %f11, %f13;
	add.f32 %f16, %f12, %f14;
	mov.b32 %r27, %f15;
	shfl.sync.bfly.b32 %r28|%p9, %r27, 2, 0x1f, 0xffffffff;
	mov.b32 %f17, %r28;
	mov.b32 %r29, %f16;
	shfl.sync.bfly.b32 %r30|%p10, %r29, 2, 0x1f, 0xffffffff;
	mov.b32 %f18, %r30;
	add.f32 %f19, %f15, %f17;
	add.f32 %f20, %f16, %f18;
	mov.b32 %r31, %f19;
	shfl.sync.bfly.b32 %r32|%p11, %r31, 1, 0x1f, 0xffffffff;
	mov.b32 %f21, %r32;
	mov.b32 %r33, %f20;
	shfl.sync.bfly.b32 %r34|%p12, %r33, 1, 0x1f, 0xffffffff;
	mov.b32 %f22, %r34;
	add.f32 %f23, %f19, %f21;
	add.f32 %f24, %f20, %f22;
	setp.eq.s32 %p13, %r5, 0;
	@!%p13 bra L4_else;
	mul.lo.s32 %r35, %r6, 4;
	add.s32 %r36, %r7, %r35;
	st.shared.f32 [%r36], %f23;
	add.s32 %r37, %r8, %r35;
	st.shared.f32 [%r37], %f24;
L4_else:
	bar.sync 0;
	setp.lt.s32 %p14, %r11, 1;
	@!%p14 bra L6_tskip;
	mul.lo.s32 %r38, %r11, 4;
	add.s32 %r39, %r7, %r38;
	add.s32 %r40, %r11, 1;
	mul.lo.s32 %r41, %r40, 4;
	add.s32 %r42, %r7, %r41;
	ld.shared.f32 %f25, [%r39];
	ld.shared.f32 %f26, [%r42];
	add.s32 %r43, %r8, %r38;
	add.s32 %r44, %r8, %r41;
	ld.shared.f32 %f27, [%r43];
	ld.shared.f32 %f28, [%r44];
	add.f32 %f29, %f25, %f26;
	add.f32 %f30, %f27, %f28;
	st.shared.f32 [%r39], %f29;
	st.shared.f32 [%r43], %f30;
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
	sqrt.rn.f32 %f41, %f40;
	mov.s32 %r45, %r11;
L7_top:
	setp.ge.s32 %p15, %r45, 256;
	@%p15 bra L8_lend;
	mad.lo.s32 %r47, %r9, 256, %r45;
	mad.wide.s32 %rd6, %r47, 4, %rd1;
	ld.global.f32 %f42, [%rd6];
	mad.wide.s32 %rd7, %r45, 4, %rd2;
	ld.global.f32 %f43, [%rd7];
	mad.wide.s32 %rd8, %r45, 4, %rd3;
	ld.global.f32 %f44, [%rd8];
	sub.f32 %f45, %f42, %f34;
	div.rn.f32 %f46, %f45, %f41;
	mul.f32 %f47, %f46, %f43;
	add.f32 %f48, %f47, %f44;
	mad.wide.s32 %rd9, %r47, 4, %rd4;
	st.global.f32 [%rd9], %f48;
	add.s32 %r45, %r45, 64;
	bra L7_top;
L8_lend:
L1_end:
	ret;
}
