.version 8.0
.target sm_89
.address_size 64

.visible .entry zero_kernel(
	.param .u64 p_x,
	.param .u64 p_hist
)
.maxntid 64, 1, 1
{
	.reg .pred %p<2>;
	.reg .b32 %r<34>;
	.reg .b64 %rd<5>;
	ld.param.u64 %rd1, [p_x];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_hist];
	cvta.to.global.u64 %rd2, %rd2;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	mov.u32 %r7, %ntid.x;
	mov.u32 %r8, %ntid.y;
	mov.u32 %r9, %ntid.z;
	mov.u32 %r10, %tid.x;
	mov.u32 %r11, %tid.y;
	mov.u32 %r12, %tid.z;
	mov.u32 %r13, %ctaid.x;
	mov.u32 %r14, %ctaid.y;
	mov.u32 %r15, %ctaid.z;
	mov.u32 %r16, %nctaid.x;
	mov.u32 %r17, %nctaid.y;
	mov.u32 %r18, %nctaid.z;
	mul.lo.s32 %r19, %r7, %r8;
	mul.lo.s32 %r20, %r19, %r9;
	mul.lo.s32 %r21, %r8, %r12;
	add.s32 %r22, %r11, %r21;
	mul.lo.s32 %r23, %r7, %r22;
	add.s32 %r24, %r10, %r23;
	mul.lo.s32 %r25, %r17, %r15;
	add.s32 %r26, %r14, %r25;
	mul.lo.s32 %r27, %r16, %r26;
	add.s32 %r28, %r13, %r27;
	mul.lo.s32 %r29, %r17, %r18;
	mul.lo.s32 %r30, %r16, %r29;
	mul.lo.s32 %r31, %r20, %r30;
	mul.lo.s32 %r32, %r28, %r20;
	add.s32 %r33, %r32, %r24;
L1_zptop:
	setp.ge.u32 %p1, %r33, 16;
	@%p1 bra L2_zpend;
	mul.wide.u32 %rd3, %r33, 4;
	add.s64 %rd4, %rd2, %rd3;
	st.global.u32 [%rd4], 0;
	add.u32 %r33, %r33, %r31;
	bra L1_zptop;
L2_zpend:
	ret;
}

.visible .entry hist_kernel(
	.param .u64 p_x,
	.param .u64 p_hist
)
.maxntid 128, 1, 1
{
	.reg .pred %p<2>;
	.reg .b32 %r<9>;
	.reg .b64 %rd<5>;
	ld.param.u64 %rd1, [p_x];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_hist];
	cvta.to.global.u64 %rd2, %rd2;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	setp.lt.s32 %p1, %r4, 4096;
	@!%p1 bra L1_end;
	mad.wide.s32 %rd3, %r4, 4, %rd1;
	ld.global.s32 %r7, [%rd3];
	rem.s32 %r8, %r7, 16;
	mad.wide.s32 %rd4, %r8, 4, %rd2;
	red.global.add.s32 [%rd4], 1;
L1_end:
	ret;
}
