.version 8.0
.target sm_89
.address_size 64

.visible .entry cumsum_1d(
	.param .u64 p_x,
	.param .u64 p_y
)
.maxntid 32, 1, 1
{
	.reg .pred %p<9>;
	.reg .b32 %r<27>;
	.reg .f32 %f<16>;
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
	setp.lt.s32 %p1, %r4, 32;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 32;
	mul.lo.s32 %r8, %r7, 32;
	sub.s32 %r9, %r4, %r8;
	mov.b32 %f1, 0f00000000;
	mov.s32 %r10, 0;
L3_top:
	setp.ge.s32 %p2, %r10, 4;
	@%p2 bra L2_lend;
	mad.lo.s32 %r12, %r10, 32, %r9;
	mad.lo.s32 %r14, %r7, 128, %r12;
	mad.wide.s32 %rd3, %r14, 4, %rd1;
	ld.global.f32 %f2, [%rd3];
	mov.b32 %r15, %f2;
	shfl.sync.up.b32 %r16|%p3, %r15, 1, 0x0, 0xffffffff;
	selp.b32 %f3, %r16, 0f00000000, %p3;
	add.f32 %f4, %f2, %f3;
	mov.b32 %r17, %f4;
	shfl.sync.up.b32 %r18|%p4, %r17, 2, 0x0, 0xffffffff;
	selp.b32 %f5, %r18, 0f00000000, %p4;
	add.f32 %f6, %f4, %f5;
	mov.b32 %r19, %f6;
	shfl.sync.up.b32 %r20|%p5, %r19, 4, 0x0, 0xffffffff;
	selp.b32 %f7, %r20, 0f00000000, %p5;
	add.f32 %f8, %f6, %f7;
	mov.b32 %r21, %f8;
	shfl.sync.up.b32 %r22|%p6, %r21, 8, 0x0, 0xffffffff;
	selp.b32 %f9, %r22, 0f00000000, %p6;
	add.f32 %f10, %f8, %f9;
	mov.b32 %r23, %f10;
	shfl.sync.up.b32 %r24|%p7, %r23, 16, 0x0, 0xffffffff;
	selp.b32 %f11, %r24, 0f00000000, %p7;
	add.f32 %f12, %f10, %f11;
	add.f32 %f13, %f12, %f1;
	mad.wide.s32 %rd4, %r14, 4, %rd2;
	st.global.f32 [%rd4], %f13;
	mov.b32 %f14, %f12;
	mov.b32 %r25, %f14;
	shfl.sync.idx.b32 %r26|%p8, %r25, 31, 31, 0xffffffff;
	mov.b32 %f15, %r26;
	add.f32 %f1, %f1, %f15;
	add.s32 %r10, %r10, 1;
	bra L3_top;
L2_lend:
L1_end:
	ret;
}
