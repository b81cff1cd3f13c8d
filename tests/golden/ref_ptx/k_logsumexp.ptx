.version 8.0
.target sm_89
.address_size 64

.visible .entry log_sum_exp(
	.param .u64 p_x,
	.param .u64 p_y
)
.maxntid 128, 1, 1
{
	.reg .pred %p<15>;
	.reg .b32 %r<45>;
	.reg .f32 %f<33>;
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
	setp.lt.s32 %p1, %r4, 2048;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 1024;
	mul.lo.s32 %r8, %r7, 1024;
	sub.s32 %r9, %r4, %r8;
	div.s32 %r10, %r9, 32;
	mul.lo.s32 %r11, %r10, 32;
	sub.s32 %r12, %r9, %r11;
	mov.b32 %f1, 0fFF800000;
	mov.s32 %r13, %r12;
	mad.lo.s32 %r15, %r7, 32, %r10;
L2_top:
	setp.ge.s32 %p2, %r13, 64;
	@%p2 bra L3_lend;
	mad.lo.s32 %r17, %r15, 64, %r13;
	mad.wide.s32 %rd3, %r17, 4, %rd1;
	ld.global.f32 %f2, [%rd3];
	max.f32 %f1, %f1, %f2;
	add.s32 %r13, %r13, 32;
	bra L2_top;
L3_lend:
	mov.b32 %r18, %f1;
	shfl.sync.bfly.b32 %r19|%p3, %r18, 16, 0x1f, 0xffffffff;
	mov.b32 %f3, %r19;
	max.f32 %f4, %f1, %f3;
	mov.b32 %r20, %f4;
	shfl.sync.bfly.b32 %r21|%p4, %r20, 8, 0x1f, 0xffffffff;
	mov.b32 %f5, %r21;
	max.f32 %f6, %f4, %f5;
	mov.b32 %r22, %f6;
	shfl.sync.bfly.b32 %r23|%p5, %r22, 4, 0x1f, 0xffffffff;
	mov.b32 %f7, %r23;
	max.f32 %f8, %f6, %f7;
	mov.b32 %r24, %f8;
	shfl.sync.bfly.b32 %r25|%p6, %r24, 2, 0x1f, 0xffffffff;
	mov.b32 %f9, %r25;
	max.f32 %f10, %f8, %f9;
	mov.b32 %r26, %f10;
	shfl.sync.bfly.b32 %r27|%p7, %r26, 1, 0x1f, 0xffffffff;
	mov.b32 %f11, %r27;
	max.f32 %f12, %f10, %f11;
	mov.b32 %f13, 0f00000000;
	mov.s32 %r28, %r12;
	mad.lo.s32 %r30, %r7, 32, %r10;
L4_top:
	setp.ge.s32 %p8, %r28, 64;
	@%p8 bra L5_lend;
	mad.lo.s32 %r32, %r30, 64, %r28;
	mad.wide.s32 %rd4, %r32, 4, %rd1;
	ld.global.f32 %f14, [%rd4];
	sub.f32 %f15, %f14, %f12;
	mov.b32 %f16, 0f3FB8AA3B;
	mul.f32 %f17, %f15, %f16;
	ex2.approx.f32 %f18, %f17;
	add.f32 %f13, %f13, %f18;
	add.s32 %r28, %r28, 32;
	bra L4_top;
L5_lend:
	mov.b32 %r33, %f13;
	shfl.sync.bfly.b32 %r34|%p9, %r33, 16, 0x1f, 0xffffffff;
	mov.b32 %f19, %r34;
	add.f32 %f20, %f13, %f19;
	mov.b32 %r35, %f20;
	shfl.sync.bfly.b32 %r36|%p10, %r35, 8, 0x1f, 0xffffffff;
	mov.b32 %f21, %r36;
	add.f32 %f22, %f20, %f21;
	mov.b32 %r37, %f22;
	shfl.sync.bfly.b32 %r38|%p11, %r37, 4, 0x1f, 0xffffffff;
	mov.b32 %f23, %r38;
	add.f32 %f24, %f22, %f23;
	mov.b32 %r39, %f24;
	shfl.sync.bfly.b32 %r40|%p12, %r39, 2, 0x1f, 0xffffffff;
	mov.b32 %f25, %r40;
	add.f32 %f26, %f24, %f25;
	mov.b32 %r41, %f26;
	shfl.sync.bfly.b32 %r42|%p13, %r41, 1, 0x1f, 0xffffffff;
	mov.b32 %f27, %r42;
	add.f32 %f28, %f26, %f27;
	lg2.approx.f32 %f29, %f28;
	mov.b32 %f30, 0f3F317218;
	mul.f32 %f31, %f29, %f30;
	add.f32 %f32, %f12, %f31;
	setp.eq.s32 %p14, %r12, 0;
	@!%p14 bra L6_else;
	mad.lo.s32 %r44, %r7, 32, %r10;
	mad.wide.s32 %rd5, %r44, 4, %rd2;
	st.global.f32 [%rd5], %f32;
L6_else:
L1_end:
	ret;
}
