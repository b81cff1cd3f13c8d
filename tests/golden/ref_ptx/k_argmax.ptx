.version 8.0
.target sm_89
.address_size 64

.visible .entry row_argmax(
	.param .u64 p_x,
	.param .u64 p_idx,
	.param .u64 p_cnt
)
.maxntid 32, 1, 1
{
	.reg .pred %p<22>;
	.reg .b32 %r<70>;
	.reg .f32 %f<15>;
	.reg .b64 %rd<8>;
	ld.param.u64 %rd1, [p_x];
	cvta.to.global.u64 %rd1, %rd1;
	ld.param.u64 %rd2, [p_idx];
	cvta.to.global.u64 %rd2, %rd2;
	ld.param.u64 %rd3, [p_cnt];
	cvta.to.global.u64 %rd3, %rd3;
	mov.u32 %r1, %tid.x;
	mov.u32 %r2, %ctaid.x;
	mov.u32 %r3, %ntid.x;
	mad.lo.s32 %r4, %r2, %r3, %r1;
	and.b32 %r5, %r1, 31;
	shr.u32 %r6, %r1, 5;
	setp.lt.s32 %p1, %r4, 1184;
	@!%p1 bra L1_end;
	div.s32 %r7, %r4, 32;
	mul.lo.s32 %r8, %r7, 32;
	sub.s32 %r9, %r4, %r8;
	mov.b32 %f1, 0fFF800000;
	mov.s32 %r10, 0;
	mov.s32 %r11, %r9;
L2_top:
	setp.ge.s32 %p2, %r11, 333;
	@%p2 bra L3_lend;
	mad.lo.s32 %r13, %r7, 333, %r11;
	mad.wide.s32 %rd4, %r13, 4, %rd1;
	ld.global.f32 %f2, [%rd4];
	max.f32 %f1, %f1, %f2;
	mov.b32 %f3, 0f40000000;
	setp.gt.f32 %p3, %f2, %f3;
	@!%p3 bra L6_selnext;
	mov.b32 %r14, 1;
	bra L4_selend;
L6_selnext:
	mov.b32 %r14, 0;
L4_selend:
	add.s32 %r10, %r10, %r14;
	add.s32 %r11, %r11, 32;
	bra L2_top;
L3_lend:
	mov.b32 %r15, %f1;
	shfl.sync.bfly.b32 %r16|%p4, %r15, 16, 0x1f, 0xffffffff;
	mov.b32 %f4, %r16;
	mov.b32 %r17, %r10;
	shfl.sync.bfly.b32 %r18|%p5, %r17, 16, 0x1f, 0xffffffff;
	mov.b32 %r19, %r18;
	max.f32 %f5, %f1, %f4;
	add.s32 %r20, %r10, %r19;
	mov.b32 %r21, %f5;
	shfl.sync.bfly.b32 %r22|%p6, %r21, 8, 0x1f, 0xffffffff;
	mov.b32 %f6, %r22;
	mov.b32 %r23, %r20;
	shfl.sync.bfly.b32 %r24|%p7, %r23, 8, 0x1f, 0xffffffff;
	mov.b32 %r25, %r24;
	max.f32 %f7, %f5, %f6;
	add.s32 %r26, %r20, %r25;
	mov.b32 %r27, %f7;
	shfl.sync.bfly.b32 %r28|%p8, %r27, 4, 0x1f, 0xffffffff;
	mov.b32 %f8, %r28;
	mov.b32 %r29, %r26;
	shfl.sync.bfly.b32 %r30|%p9, %r29, 4, 0x1f, 0xffffffff;
	mov.b32 %r31, %r30;
	max.f32 %f9, %f7, %f8;
	add.s32 %r32, %r26, %r31;
	mov.b32 %r33, %f9;
	shfl.sync.bfly.b32 %r34|%p10, %r33, 2, 0x1f, 0xffffffff;
	mov.b32 %f10, %r34;
	mov.b32 %r35, %r32;
	shfl.sync.bfly.b32 %r36|%p11, %r35, 2, 0x1f, 0xffffffff;
	mov.b32 %r37, %r36;
	max.f32 %f11, %f9, %f10;
	add.s32 %r38, %r32, %r37;
	mov.b32 %r39, %f11;
	shfl.sync.bfly.b32 %r40|%p12, %r39, 1, 0x1f, 0xffffffff;
	mov.b32 %f12, %r40;
	mov.b32 %r41, %r38;
	shfl.sync.bfly.b32 %r42|%p13, %r41, 1, 0x1f, 0xffffffff;
	mov.b32 %r43, %r42;
	max.f32 %f13, %f11, %f12;
	add.s32 %r44, %r38, %r43;
	mov.s32 %r45, 2147483647;
	mov.s32 %r46, %r9;
L7_top:
	setp.ge.s32 %p14, %r46, 333;
	@%p14 bra L8_lend;
	mad.lo.s32 %r48, %r7, 333, %r46;
	mad.wide.s32 %rd5, %r48, 4, %rd1;
	ld.global.f32 %f14, [%rd5];
	setp.eq.f32 %p15, %f14, %f13;
	@!%p15 bra L11_selnext;
	mov.b32 %r49, %r46;
	bra L9_selend;
L11_selnext:
	mov.b32 %r49, 333;
L9_selend:
	min.s32 %r45, %r45, %r49;
	add.s32 %r46, %r46, 32;
	bra L7_top;
L8_lend:
	mov.b32 %r50, %r45;
	shfl.sync.bfly.b32 %r51|%p16, %r50, 16, 0x1f, 0xffffffff;
	mov.b32 %r52, %r51;
	min.s32 %r53, %r45, %r52;
	mov.b32 %r54, %r53;
	shfl.sync.bfly.b32 %r55|%p17, %r54, 8, 0x1f, 0xffffffff;
	mov.b32 %r56, %r55;
	min.s32 %r57, %r53, %r56;
	mov.b32 %r58, %r57;
	shfl.sync.bfly.b32 %r59|%p18, %r58, 4, 0x1f, 0xffffffff;
	mov.b32 %r60, %r59;
	min.s32 %r61, %r57, %r60;
	mov.b32 %r62, %r61;
	shfl.sync.bfly.b32 %r63|%p19, %r62, 2, 0x1f, 0xffffffff;
	mov.b32 %r64, %r63;
	min.s32 %r65, %r61, %r64;
	mov.b32 %r66, %r65;
	shfl.sync.bfly.b32 %r67|%p20, %r66, 1, 0x1f, 0xffffffff;
	mov.b32 %r68, %r67;
	min.s32 %r69, %r65, %r68;
	setp.eq.s32 %p21, %r9, 0;
	@!%p21 bra L12_else;
	mad.wide.s32 %rd6, %r7, 4, %rd2;
	st.global.s32 [%rd6], %r69;
	mad.wide.s32 %rd7, %r7, 4, %rd3;
	st.global.s32 [%rd7], %r44;
L12_else:
L1_end:
	ret;
}
