.version 8.0
.target sm_89
.address_size 64

.visible .entry row_var_std(
	.param .u64 p_x,
	.param .u64 p_var,
	.param .u64 p_std
)
.maxntid 32, 1, 1
{
	.reg .pred %p<15>;
	.reg .b32 %r<36>;
	.reg .f32 %f<32>;
	.reg .b64 %rd<8>;
	ld.param.u64 %rd1, [p_x];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_var];
	cvta.to.global.u64 %rd2, %rd2;
	ld.param.u64 %rd3, [p_std];
	cvta.to.global.u64 %rd3, %rd3;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	setp.lt.s32 %p1, %r4, 128;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 32;
	mul.lo.s32 %r8, %r7, 32;
	sub.s32 %r9, %r4, %r8;
	mov.b32 %f1, 0f00000000;
	mov.s32 %r10, %r9;
L2_top:
	setp.ge.s32 %p2, %r10, 128;
	@%p2 bra L3_lend;
	mad.lo.s32 %r12, %r7, 128, %r10;
	mad.wide.s32 %rd4, %r12, 4, %rd1;
	ld.global.f32 %f2, [%rd4];
	add.f32 %f1, %f1, %f2;
	add.s32 %r10, %r10, 32;
	bra L2_top;
L3_lend:
	mov.b32 %r13, %f1;
	shfl.sync.bfly.b32 %r14|%p3, %r13, 16, 0x1f, 0xffffffff;
	mov.b32 %f3, %r14;
	add.f32 %f4, %f1, %f3;
	mov.b32 %r15, %f4;
	shfl.sync.bfly.b32 %r16|%p4, %r15, 8, 0x1f, 0xffffffff;
	mov.b32 %f5, %r16;
	add.f32 %f6, %f4, %f5;
	mov.b32 %r17, %f6;
	shfl.sync.bfly.b32 %r18|%p5, %r17, 4, 0x1f, 0xffffffff;
	mov.b32 %f7, %r18;
	add.f32 %f8, %f6, %f7;
	mov.b32 %r19, %f8;
	shfl.sync.bfly.b32 %r20|%p6, %r19, 2, 0x1f, 0xffffffff;
	mov.b32 %f9, %r20;
	add.f32 %f10, %f8, %f9;
	mov.b32 %r21, %f10;
	shfl.sync.bfly.b32 %r22|%p7, %r21, 1, 0x1f, 0xffffffff;
	mov.b32 %f11, %r22;
	add.f32 %f12, %f10, %f11;
	mov.b32 %f13, 0f43000000;
	div.rn.f32 %f14, %f12, %f13;
	mov.b32 %f15, 0f00000000;
	mov.s32 %r23, %r9;
L4_top:
	setp.ge.s32 %p8, %r23, 128;
	@%p8 bra L5_lend;
	mad.lo.s32 %r25, %r7, 128, %r23;
	mad.wide.s32 %rd5, %r25, 4, %rd1;
	ld.global.f32 %f16, [%rd5];
	sub.f32 %f17, %f16, %f14;
	mul.f32 %f18, %f17, %f17;
	add.f32 %f15, %f15, %f18;
	add.s32 %r23, %r23, 32;
	bra L4_top;
L5_lend:
	mov.b32 %r26, %f15;
	shfl.sync.bfly.b32 %r27|%p9, %r26, 16, 0x1f, 0xffffffff;
	mov.b32 %f19, %r27;
	add.f32 %f20, %f15, %f19;
	mov.b32 %r28, %f20;
	shfl.sync.bfly.b32 %r29|%p10, %r28, 8, 0x1f, 0xffffffff;
	mov.b32 %f21, %r29;
	add.f32 %f22, %f20, %f21;
	mov.b32 %r30, %f22;
	shfl.sync.bfly.b32 %r31|%p11, %r30, 4, 0x1f, 0xffffffff;
	mov.b32 %f23, %r31;
	add.f32 %f24, %f22, %f23;
	mov.b32 %r32, %f24;
	shfl.sync.bfly.b32 %r33|%p12, %r32, 2, 0x1f, 0xffffffff;
	mov.b32 %f25, %r33;
	add.f32 %f26, %f24, %f25;
	mov.b32 %r34, %f26;
	shfl.sync.bfly.b32 %r35|%p13, %r34, 1, 0x1f, 0xffffffff;
	mov.b32 %f27, %r35;
	add.f32 %f28, %f26, %f27;
	mov.b32 %f29, 0f42FE0000;
	div.rn.f32 %f30, %f28, %f29;
	sqrt.rn.f32 %f31, %f30;
	setp.eq.s32 %p14, %r9, 0;
	@!%p14 bra L6_else;
	mad.wide.s32 %rd6, %r7, 4, %rd2;
	st.global.f32 [%rd6], %f30;
	mad.wide.s32 %rd7, %r7, 4, %rd3;
	st.global.f32 [%rd7], %f31;
L6_else:
L1_end:
	ret;
}
