.version 8.0
.target sm_89
.address_size 64

.shared .align 16 .s32 red[16];

.visible .entry array_sum_i32(
	.param .u64 p_x,
	.param .u64 p_out
)
.maxntid 512, 1, 1
{
	.reg .pred %p<14>;
	.reg .b32 %r<64>;
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
	mov.s32 %r8, 0;
	mov.s32 %r9, %r4;
L2_top:
	setp.ge.s32 %p2, %r9, 67108864;
	@%p2 bra L3_lend;
	mul.lo.s32 %r10, %r9, 4;
	mad.wide.s32 %rd3, %r10, 4, %rd1;
	ld.global.v4.s32 {%r11, %r12, %r13, %r14}, [%rd3];
	add.s32 %r8, %r8, %r11;
	add.s32 %r8, %r8, %r12;
	add.s32 %r8, %r8, %r13;
	add.s32 %r8, %r8, %r14;
	add.s32 %r9, %r9, 303104;
	bra L2_top;
L3_lend:
	mov.b32 %r15, %r8;
	shfl.sync.bfly.b32 %r16|%p3, %r15, 16, 0x1f, 0xffffffff;
	mov.b32 %r17, %r16;
	add.s32 %r18, %r8, %r17;
	mov.b32 %r19, %r18;
	shfl.sync.bfly.b32 %r20|%p4, %r19, 8, 0x1f, 0xffffffff;
	mov.b32 %r21, %r20;
	add.s32 %r22, %r18, %r21;
	mov.b32 %r23, %r22;
	shfl.sync.bfly.b32 %r24|%p5, %r23, 4, 0x1f, 0xffffffff;
	mov.b32 %r25, %r24;
	add.s32 %r26, %r22, %r25;
	mov.b32 %r27, %r26;
	shfl.sync.bfly.b32 %r28|%p6, %r27, 2, 0x1f, 0xffffffff;
	mov.b32 %r29, %r28;
	add.s32 %r30, %r26, %r29;
	mov.b32 %r31, %r30;
	shfl.sync.bfly.b32 %r32|%p7, %r31, 1, 0x1f, 0xffffffff;
	mov.b32 %r33, %r32;
	add.s32 %r34, %r30, %r33;
	setp.eq.s32 %p8, %r5, 0;
	@!%p8 bra L4_else;
	mad.lo.s32 %r36, %r6, 4, %r7;
	st.shared.s32 [%r36], %r34;
L4_else:
	bar.sync 0;
	setp.lt.s32 %p9, %r1, 8;
	@!%p9 bra L6_tskip;
	mad.lo.s32 %r38, %r1, 4, %r7;
	add.s32 %r39, %r1, 8;
	mad.lo.s32 %r41, %r39, 4, %r7;
	ld.shared.s32 %r42, [%r38];
	ld.shared.s32 %r43, [%r41];
	add.s32 %r44, %r42, %r43;
	st.shared.s32 [%r38], %r44;
L6_tskip:
	bar.sync 0;
	setp.lt.s32 %p10, %r1, 4;
	@!%p10 bra L7_tskip;
	add.s32 %r45, %r1, 4;
	mad.lo.s32 %r47, %r45, 4, %r7;
	ld.shared.s32 %r48, [%r38];
	ld.shared.s32 %r49, [%r47];
	add.s32 %r50, %r48, %r49;
	st.shared.s32 [%r38], %r50;
L7_tskip:
	bar.sync 0;
	setp.lt.s32 %p11, %r1, 2;
	@!%p11 bra L8_tskip;
	add.s32 %r51, %r1, 2;
	mad.lo.s32 %r53, %r51, 4, %r7;
	ld.shared.s32 %r54, [%r38];
	ld.shared.s32 %r55, [%r53];
	add.s32 %r56, %r54, %r55;
	st.shared.s32 [%r38], %r56;
L8_tskip:
	bar.sync 0;
	setp.lt.s32 %p12, %r1, 1;
	@!%p12 bra L9_tskip;
	add.s32 %r57, %r1, 1;
	mad.lo.s32 %r59, %r57, 4, %r7;
	ld.shared.s32 %r60, [%r38];
	ld.shared.s32 %r61, [%r59];
	add.s32 %r62, %r60, %r61;
	st.shared.s32 [%r38], %r62;
L9_tskip:
	bar.sync 0;
	ld.shared.s32 %r63, [%r7];
	setp.eq.s32 %p13, %r1, 0;
	@!%p13 bra L10_else;
	red.global.add.s32 [%rd2], %r63;
L10_else:
L1_end:
	ret;
}
