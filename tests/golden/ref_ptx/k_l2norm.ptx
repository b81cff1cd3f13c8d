.version 8.0
.target sm_89
.address_size 64

.shared .align 16 .f32 red[2];

.visible .entry l2_normalize(
	.param .u64 p_x,
	.param .u64 p_y
)
.maxntid 64, 1, 1
{
	.reg .pred %p<11>;
	.reg .b32 %r<34>;
	.reg .f32 %f<23>;
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
	mov.u32 %r7, red;
	setp.lt.s32 %p1, %r4, 4096;
	@!%p1 bra L1_end;
	div.s32 %r8, %r4, 64;
	mul.lo.s32 %r9, %r8, 64;
	sub.s32 %r10, %r4, %r9;
	mov.b32 %f1, 0f00000000;
	mov.s32 %r11, %r10;
L2_top:
	setp.ge.s32 %p2, %r11, 256;
	@%p2 bra L3_lend;
	mad.lo.s32 %r13, %r8, 256, %r11;
	mad.wide.s32 %rd3, %r13, 4, %rd1;
	ld.global.f32 %f2, [%rd3];
	mul.f32 %f3, %f2, %f2;
	add.f32 %f1, %f1, %f3;
	add.s32 %r11, %r11, 64;
	bra L2_top;
L3_lend:
	mov.b32 %r14, %f1;
	shfl.sync.bfly.b32 %r15|%p3, %r14, 16, 0x1f, 0xffffffff;
	mov.b32 %f4, %r15;
	add.f32 %f5, %f1, %f4;
	mov.b32 %r16, %f5;
	shfl.sync.bfly.b32 %r17|%p4, %r16, 8, 0x1f, 0xffffffff;
	mov.b32 %f6, %r17;
	add.f32 %f7, %f5, %f6;
	mov.b32 %r18, %f7;
	shfl.sync.bfly.b32 %r19|%p5, %r18, 4, 0x1f, 0xffffffff;
	mov.b32 %f8, %r19;
	add.f32 %f9, %f7, %f8;
	mov.b32 %r20, %f9;
	shfl.sync.bfly.b32 %r21|%p6, %r20, 2, 0x1f, 0xffffffff;
	mov.b32 %f10, %r21;
	add.f32 %f11, %f9, %f10;
	mov.b32 %r22, %f11;
	shfl.sync.bfly.b32 %r23|%p7, %r22, 1, 0x1f, 0xffffffff;
	mov.b32 %f12, %r23;
	add.f32 %f13, %f11, %f12;
	setp.eq.s32 %p8, %r5, 0;
	@!%p8 bra L4_else;
	mad.lo.s32 %r25, %r6, 4, %r7;
	st.shared.f32 [%r25], %f13;
L4_else:
	bar.sync 0;
	setp.lt.s32 %p9, %r10, 1;
	@!%p9 bra L6_tskip;
	mad.lo.s32 %r27, %r10, 4, %r7;
	add.s32 %r28, %r10, 1;
	mad.lo.s32 %r30, %r28, 4, %r7;
	ld.shared.f32 %f14, [%r27];
	ld.shared.f32 %f15, [%r30];
	add.f32 %f16, %f14, %f15;
	st.shared.f32 [%r27], %f16;
L6_tskip:
	bar.sync 0;
	ld.shared.f32 %f17, [%r7];
	sqrt.rn.f32 %f18, %f17;
	mov.b32 %f19, 0f2B8CBCCC;
	max.f32 %f20, %f18, %f19;
	mov.s32 %r31, %r10;
L7_top:
	setp.ge.s32 %p10, %r31, 256;
	@%p10 bra L8_lend;
	mad.lo.s32 %r33, %r8, 256, %r31;
	mad.wide.s32 %rd4, %r33, 4, %rd1;
	ld.global.f32 %f21, [%rd4];
	div.rn.f32 %f22, %f21, %f20;
	mad.wide.s32 %rd5, %r33, 4, %rd2;
	st.global.f32 [%rd5], %f22;
	add.s32 %r31, %r31, 64;
	bra L7_top;
L8_lend:
L1_end:
	ret;
}
