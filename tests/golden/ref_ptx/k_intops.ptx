.version 8.0
.target sm_89
.address_size 64

.visible .entry int_ops(
	.param .u64 p_x,
	.param .u64 p_y,
	.param .u64 p_z,
	.param .u64 p_s,
	.param .u64 p_w,
	.param .u64 p_bd
)
.maxntid 128, 1, 1
{
	.reg .pred %p<7>;
	.reg .b32 %r<20>;
	.reg .b64 %rd<13>;
	ld.param.u64 %rd1, [p_x];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_y];
	cvta.to.global.u64 %rd2, %rd2;
	ld.param.u64 %rd3, [p_z];
	cvta.to.global.u64 %rd3, %rd3;
	ld.param.u64 %rd4, [p_s];
	cvta.to.global.u64 %rd4, %rd4;
	ld.param.u64 %rd5, [p_w];
	cvta.to.global.u64 %rd5, %rd5;
	ld.param.u64 %rd6, [p_bd];
	cvta.to.global.u64 %rd6, %rd6;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	setp.lt.s32 %p1, %r4, 1000;
	@!%p1 bra L1_end;
	mad.wide.s32 %rd7, %r4, 4, %rd1;
	ld.global.s32 %r7, [%rd7];
	mad.wide.s32 %rd8, %r4, 4, %rd2;
	ld.global.s32 %r8, [%rd8];
	and.b32 %r9, %r7, %r8;
	or.b32 %r10, %r7, %r8;
	sub.s32 %r11, %r10, 3;
	setp.gt.s32 %p2, %r7, 4;
	@!%p2 bra L4_selnext;
	mov.b32 %r12, %r9;
	bra L2_selend;
L4_selnext:
	mov.b32 %r12, %r11;
L2_selend:
	setp.lt.s32 %p3, %r7, 0;
	@!%p3 bra L7_selnext;
	mov.b32 %r13, -1;
	bra L5_selend;
L7_selnext:
	setp.eq.s32 %p4, %r7, 0;
	@!%p4 bra L8_selnext;
	mov.b32 %r13, 0;
	bra L5_selend;
L8_selnext:
	mov.b32 %r13, 1;
L5_selend:
	setp.gt.s32 %p5, %r7, 10;
	@!%p5 bra L11_selnext;
	mov.b32 %r14, 2;
	bra L9_selend;
L11_selnext:
	setp.gt.s32 %p6, %r7, 0;
	@!%p6 bra L12_selnext;
	mov.b32 %r14, 1;
	bra L9_selend;
L12_selnext:
	mov.b32 %r14, 0;
L9_selend:
	div.s32 %r15, %r7, 3;
	rem.s32 %r16, %r7, 3;
	shl.b32 %r17, %r8, 2;
	max.s32 %r18, %r15, %r16;
	add.s32 %r19, %r18, %r17;
	mad.wide.s32 %rd9, %r4, 4, %rd3;
	st.global.s32 [%rd9], %r12;
	mad.wide.s32 %rd10, %r4, 4, %rd4;
	st.global.s32 [%rd10], %r13;
	mad.wide.s32 %rd11, %r4, 4, %rd5;
	st.global.s32 [%rd11], %r19;
	mad.wide.s32 %rd12, %r4, 4, %rd6;
	st.global.s32 [%rd12], %r14;
L1_end:
	ret;
}
