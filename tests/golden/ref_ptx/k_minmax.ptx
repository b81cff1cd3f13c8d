.version 8.0
.target sm_89
.address_size 64

.visible .entry row_minmax(
	.param .u64 p_x,
	.param .u64 p_mx,
	.param .u64 p_mn
)
.maxntid 32, 1, 1
{
	.reg .pred %p<14>;
	.reg .b32 %r<33>;
	.reg .f32 %f<24>;
	.reg .b64 %rd<7>;
	ld.param.u64 %rd1, [p_x];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_mx];
	cvta.to.global.u64 %rd2, %rd2;
	ld.param.u64 %rd3, [p_mn];
	cvta.to.global.u64 %rd3, %rd3;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	setp.lt.s32 %p1, %r4, 608;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 32;
	mul.lo.s32 %r8, %r7, 32;
	sub.s32 %r9, %r4, %r8;
	mov.b32 %f1, 0fFF800000;
	mov.b32 %f2, 0f7F800000;
	mov.s32 %r10, %r9;
L2_top:
	setp.ge.s32 %p2, %r10, 777;
	@%p2 bra L3_lend;
	mad.lo.s32 %r12, %r7, 777, %r10;
	mad.wide.s32 %rd4, %r12, 4, %rd1;
	ld.global.f32 %f3, [%rd4];
	max.f32 %f1, %f1, %f3;
	min.f32 %f2, %f2, %f3;
	add.s32 %r10, %r10, 32;
	bra L2_top;
L3_lend:
	mov.b32 %r13, %f1;
	shfl.sync.bfly.b32 %r14|%p3, %r13, 16, 0x1f, 0xffffffff;
	mov.b32 %f4, %r14;
	mov.b32 %r15, %f2;
	shfl.sync.bfly.b32 %r16|%p4, %r15, 16, 0x1f, 0xffffffff;
	mov.b32 %f5, %r16;
	max.f32 %f6, %f1, %f4;
	min.f32 %f7, %f2, %f5;
	mov.b32 %r17, %f6;
	shfl.sync.bfly.b32 %r18|%p5, %r17, 8, 0x1f, 0xffffffff;
	mov.b32 %f8, %r18;
	mov.b32 %r19, %f7;
	shfl.sync.bfly.b32 %r20|%p6, %r19, 8, 0x1f, 0xffffffff;
	mov.b32 %f9, %r20;
	max.f32 %f10, %f6, %f8;
	min.f32 %f11, %f7, %f9;
	mov.b32 %r21, %f10;
	shfl.sync.bfly.b32 %r22|%p7, %r21, 4, 0x1f, 0xffffffff;
	mov.b32 %f12, %r22;
	mov.b32 %r23, %f11;
	shfl.sync.bfly.b32 %r24|%p8, %r23, 4, 0x1f, 0xffffffff;
	mov.b32 %f13, %r24;
	max.f32 %f14, %f10, %f12;
	min.f32 %f15, %f11, %f13;
	mov.b32 %r25, %f14;
	shfl.sync.bfly.b32 %r26|%p9, %r25, 2, 0x1f, 0xffffffff;
	mov.b32 %f16, %r26;
	mov.b32 %r27, %f15;
	shfl.sync.bfly.b32 %r28|%p10, %r27, 2, 0x1f, 0xffffffff;
	mov.b32 %f17, %r28;
	max.f32 %f18, %f14, %f16;
	min.f32 %f19, %f15, %f17;
	mov.b32 %r29, %f18;
	shfl.sync.bfly.b32 %r30|%p11, %r29, 1, 0x1f, 0xffffffff;
	mov.b32 %f20, %r30;
	mov.b32 %r31, %f19;
	shfl.sync.bfly.b32 %r32|%p12, %r31, 1, 0x1f, 0xffffffff;
	mov.b32 %f21, %r32;
	max.f32 %f22, %f18, %f20;
	min.f32 %f23, %f19, %f21;
	setp.eq.s32 %p13, %r9, 0;
	@!%p13 bra L4_else;
	mad.wide.s32 %rd5, %r7, 4, %rd2;
	st.global.f32 [%rd5], %f22;
	mad.wide.s32 %rd6, %r7, 4, %rd3;
	st.global.f32 [%rd6], %f23;
L4_else:
L1_end:
	ret;
}
