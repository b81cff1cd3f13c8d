.version 8.0
.target sm_89
.address_size 64

.shared .align 16 .f32 red[16];

.visible .entry array_sum_f32(
	.param .u64 p_x,
	.param .u64 p_out
)
.maxntid 512, 1, 1
{
	.reg .pred %p<14>;
	.reg .b32 %r<36>;
	.reg .f32 %f<29>;
	.reg .b64 %rd<4>;
	ld.param.u64 %rd1, [p_x];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_out];
	cvta.to.global.u64 %rd2, %rd2;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	mov.u32 %r7, red;
	setp.lt.s32 %p1, %r4, 303104;
	@!%p1 bra L1_end;
	mov.b32 %f1, 0f00000000;
	mov.s32 %r8, %r4;
L2_top:
	setp.ge.s32 %p2, %r8, 67108864;
	@%p2 bra L3_lend;
	mul.lo.s32 %r9, %r8, 4;
	mad.wide.s32 %rd3, %r9, 4, %rd1;
	ld.global.v4.f32 {%f2, %f3, %f4, %f5}, [%rd3];
	add.f32 %f1, %f1, %f2;
	add.f32 %f1, %f1, %f3;
	add.f32 %f1, %f1, %f4;
	add.f32 %f1, %f1, %f5;
	add.s32 %r8, %r8, 303104;
	bra L2_top;
L3_lend:
	mov.b32 %r10, %f1;
	shfl.sync.bfly.b32 %r11|%p3, %r10, 16, 0x1f, 0xffffffff;
	mov.b32 %f6, %r11;
	add.f32 %f7, %f1, %f6;
	mov.b32 %r12, %f7;
	shfl.sync.bfly.b32 %r13|%p4, %r12, 8, 0x1f, 0xffffffff;
	mov.b32 %f8, %r13;
	add.f32 %f9, %f7, %f8;
	mov.b32 %r14, %f9;
	shfl.sync.bfly.b32 %r15|%p5, %r14, 4, 0x1f, 0xffffffff;
	mov.b32 %f10, %r15;
	add.f32 %f11, %f9, %f10;
	mov.b32 %r16, %f11;
	shfl.sync.bfly.b32 %r17|%p6, %r16, 2, 0x1f, 0xffffffff;
	mov.b32 %f12, %r17;
	add.f32 %f13, %f11, %f12;
	mov.b32 %r18, %f13;
	shfl.sync.bfly.b32 %r19|%p7, %r18, 1, 0x1f, 0xffffffff;
	mov.b32 %f14, %r19;
	add.f32 %f15, %f13, %f14;
	setp.eq.s32 %p8, %r5, 0;
	@!%p8 bra L4_else;
	mad.lo.s32 %r21, %r6, 4, %r7;
	st.shared.f32 [%r21], %f15;
L4_else:
	bar.sync 0;
	setp.lt.s32 %p9, %r1, 8;
	@!%p9 bra L6_tskip;
	mad.lo.s32 %r23, %r1, 4, %r7;
	add.s32 %r24, %r1, 8;
	mad.lo.s32 %r26, %r24, 4, %r7;
	ld.shared.f32 %f16, [%r23];
	ld.shared.f32 %f17, [%r26];
	add.f32 %f18, %f16, %f17;
	st.shared.f32 [%r23], %f18;
L6_tskip:
	bar.sync 0;
	setp.lt.s32 %p10, %r1, 4;
	@!%p10 bra L7_tskip;
	add.s32 %r27, %r1, 4;
	mad.lo.s32 %r29, %r27, 4, %r7;
	ld.shared.f32 %f19, [%r23];
	ld.shared.f32 %f20, [%r29];
	add.f32 %f21, %f19, %f20;
	st.shared.f32 [%r23], %f21;
L7_tskip:
	bar.sync 0;
	setp.lt.s32 %p11, %r1, 2;
	@!%p11 bra L8_tskip;
	add.s32 %r30, %r1, 2;
	mad.lo.s32 %r32, %r30, 4, %r7;
	ld.shared.f32 %f22, [%r23];
	ld.shared.f32 %f23, [%r32];
	add.f32 %f24, %f22, %f23;
	st.shared.f32 [%r23], %f24;
L8_tskip:
	bar.sync 0;
	setp.lt.s32 %p12, %r1, 1;
	@!%p12 bra L9_tskip;
	add.s32 %r33, %r1, 1;
	mad.lo.s32 %r35, %r33, 4, %r7;
	ld.shared.f32 %f25, [%r23];
	ld.shared.f32 %f26, [%r35];
	add.f32 %f27, %f25, %f26;
	st.shared.f32 [%r23], %f27;
L9_tskip:
	bar.sync 0;
	ld.shared.f32 %f28, [%r7];
	setp.eq.s32 %p13, %r1, 0;
	@!%p13 bra L10_else;
	red.global.add.f32 [%rd2], %f28;
L10_else:
L1_end:
	ret;
}
