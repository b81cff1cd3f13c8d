.version 8.0
.target sm_89
.address_size 64

.visible .entry cumsum_rows(
	.param .u64 p_x,
	.param .u64 p_y
)
.maxntid 32, 1, 1
{
	.reg .pred %p<13>;
	.reg .b32 %r<36>;
	.reg .f32 %f<26>;
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
	setp.lt.s32 %p1, %r4, 128;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 32;
	mul.lo.s32 %r8, %r7, 32;
	sub.s32 %r9, %r4, %r8;
	mul.lo.s32 %r10, %r7, 64;
	add.s32 %r11, %r10, %r9;
	mad.wide.s32 %rd3, %r11, 4, %rd1;
	ld.global.f32 %f1, [%rd3];
	add.s32 %r12, %r9, 32;
	add.s32 %r13, %r10, %r12;
	mad.wide.s32 %rd4, %r13, 4, %rd1;
	ld.global.f32 %f2, [%rd4];
	mov.b32 %r14, %f1;
	shfl.sync.up.b32 %r15|%p2, %r14, 1, 0x0, 0xffffffff;
	selp.b32 %f3, %r15, 0f00000000, %p2;
	add.f32 %f4, %f1, %f3;
	mov.b32 %r16, %f4;
	shfl.sync.up.b32 %r17|%p3, %r16, 2, 0x0, 0xffffffff;
	selp.b32 %f5, %r17, 0f00000000, %p3;
	add.f32 %f6, %f4, %f5;
	mov.b32 %r18, %f6;
	shfl.sync.up.b32 %r19|%p4, %r18, 4, 0x0, 0xffffffff;
	selp.b32 %f7, %r19, 0f00000000, %p4;
	add.f32 %f8, %f6, %f7;
	mov.b32 %r20, %f8;
	shfl.sync.up.b32 %r21|%p5, %r20, 8, 0x0, 0xffffffff;
	selp.b32 %f9, %r21, 0f00000000, %p5;
	add.f32 %f10, %f8, %f9;
	mov.b32 %r22, %f10;
	shfl.sync.up.b32 %r23|%p6, %r22, 16, 0x0, 0xffffffff;
	selp.b32 %f11, %r23, 0f00000000, %p6;
	add.f32 %f12, %f10, %f11;
	mov.b32 %r24, %f2;
	shfl.sync.up.b32 %r25|%p7, %r24, 1, 0x0, 0xffffffff;
	selp.b32 %f13, %r25, 0f00000000, %p7;
	add.f32 %f14, %f2, %f13;
	mov.b32 %r26, %f14;
	shfl.sync.up.b32 %r27|%p8, %r26, 2, 0x0, 0xffffffff;
	selp.b32 %f15, %r27, 0f00000000, %p8;
	add.f32 %f16, %f14, %f15;
	mov.b32 %r28, %f16;
	shfl.sync.up.b32 %r29|%p9, %r28, 4, 0x0, 0xffffffff;
	selp.b32 %f17, %r29, 0f00000000, %p9;
	add.f32 %f18, %f16, %f17;
	mov.b32 %r30, %f18;
	shfl.sync.up.b32 %r31|%p10, %r30, 8, 0x0, 0xffffffff;
	selp.b32 %f19, %r31, 0f00000000, %p10;
	add.f32 %f20, %f18, %f19;
	mov.b32 %r32, %f20;
	shfl.sync.up.b32 %r33|%p11, %r32, 16, 0x0, 0xffffffff;
	selp.b32 %f21, %r33, 0f00000000, %p11;
	add.f32 %f22, %f20, %f21;
	mov.b32 %f23, %f12;
	mov.b32 %r34, %f23;
	shfl.sync.idx.b32 %r35|%p12, %r34, 31, 31, 0xffffffff;
	mov.b32 %f24, %r35;
	add.f32 %f25, %f22, %f24;
	mad.wide.s32 %rd5, %r11, 4, %rd2;
	st.global.f32 [%rd5], %f12;
	mad.wide.s32 %rd6, %r13, 4, %rd2;
	st.global.f32 [%rd6], %f25;
L1_end:
	ret;
}
