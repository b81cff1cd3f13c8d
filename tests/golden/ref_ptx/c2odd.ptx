.version 8.0
.target sm_89
.address_size 64

.shared .align 16 .f32 red[4];

.visible .entry array_sum_f32(
	.param .u64 p_x,
	.param .u64 p_out
)
.maxntid 128, 1, 1
{
	.reg .pred %p<13>;
	.reg .b32 %r<32>;
	.reg .f32 %f<24>;
	.reg .b64 %rd<5>;
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
	setp.lt.s32 %p1, %r4, 256;
	@!%p1 bra L1_end;
	mov.b32 %f1, 0f00000000;
	mov.s32 %r8, %r4;
L2_top:
	setp.ge.s32 %p2, %r8, 249;
	@%p2 bra L3_lend;
	mul.lo.s32 %r9, %r8, 4;
	mad.wide.s32 %rd3, %r9, 4, %rd1;
	ld.global.v4.f32 {%f2, %f3, %f4, %f5}, [%rd3];
	add.f32 %f1, %f1, %f2;
	add.f32 %f1, %f1, %f3;
	add.f32 %f1, %f1, %f4;
	add.f32 %f1, %f1, %f5;
	add.s32 %r8, %r8, 256;
	bra L2_top;
L3_lend:
	add.s32 %r10, %r4, 996;
	mov.s32 %r11, %r10;
L4_top:
	setp.ge.s32 %p3, %r11, 997;
	@%p3 bra L5_lend;
	mad.wide.s32 %rd4, %r11, 4, %rd1;
	ld.global.f32 %f6, [%rd4];
	add.f32 %f1, %f1, %f6;
	add.s32 %r11, %r11, 256;
	bra L4_top;
L5_lend:
	mov.b32 %r12, %f1;
	shfl.sync.bfly.b32 %r13|%p4, %r12, 16, 0x1f, 0xffffffff;
	mov.b32 %f7, %r13;
	add.f32 %f8, %f1, %f7;
	mov.b32 %r14, %f8;
	shfl.sync.bfly.b32 %r15|%p5, %r14, 8, 0x1f, 0xffffffff;
	mov.b32 %f9, %r15;
	add.f32 %f10, %f8, %f9;
	mov.b32 %r16, %f10;
	shfl.sync.bfly.b32 %r17|%p6, %r16, 4, 0x1f, 0xffffffff;
	mov.b32 %f11, %r17;
	add.f32 %f12, %f10, %f11;
	mov.b32 %r18, %f12;
	shfl.sync.bfly.b32 %r19|%p7, %r18, 2, 0x1f, 0xffffffff;
	mov.b32 %f13, %r19;
	add.f32 %f14, %f12, %f13;
	mov.b32 %r20, %f14;
	shfl.sync.bfly.b32 %r21|%p8, %r20, 1, 0x1f, 0xffffffff;
	mov.b32 %f15, %r21;
	add.f32 %f16, %f14, %f15;
	setp.eq.s32 %p9, %r5, 0;
	@!%p9 bra L6_else;
	mad.lo.s32 %r23, %r6, 4, %r7;
	st.shared.f32 [%r23], %f16;
L6_else:
	bar.sync 0;
	setp.lt.s32 %p10, %r1, 2;
	@!%p10 bra L8_tskip;
	mad.lo.s32 %r25, %r1, 4, %r7;
	add.s32 %r26, %r1, 2;
	mad.lo.s32 %r28, %r26, 4, %r7;
	ld.shared.f32 %f17, [%r25];
	ld.shared.f32 %f18, [%r28];
	add.f32 %f19, %f17, %f18;
	st.shared.f32 [%r25], %f19;
L8_tskip:
	bar.sync 0;
	setp.lt.s32 %p11, %r1, 1;
	@!%p11 bra L9_tskip;
	add.s32 %r29, %r1, 1;
	mad.lo.s32 %r31, %r29, 4, %r7;
	ld.shared.f32 %f20, [%r25];
	ld.shared.f32 %f21, [%r31];
	add.f32 %f22, %f20, %f21;
	st.shared.f32 [%r25], %f22;
L9_tskip:
	bar.sync 0;
	ld.shared.f32 %f23, [%r7];
	setp.eq.s32 %p12, %r1, 0;
	@!%p12 bra L10_else;
	red.global.add.f32 [%rd2], %f23;
L10_else:
L1_end:
	ret;
}
