.version 8.0
.target sm_89
.address_size 64

.visible .entry col_sum(
	.param .u64 p_x,
	.param .u64 p_out
)
.maxntid 64, 1, 1
{
	.reg .pred %p<3>;
	.reg .b32 %r<10>;
	.reg .f32 %f<3>;
	.reg .b64 %rd<5>;
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
	setp.lt.s32 %p1, %r4, 96;
	@!%p1 bra L1_end;
	mov.b32 %f1, 0f00000000;
	mov.s32 %r7, 0;
L3_top:
	setp.ge.s32 %p2, %r7, 100;
	@%p2 bra L2_lend;
	mad.lo.s32 %r9, %r7, 96, %r4;
	mad.wide.s32 %rd3, %r9, 4, %rd1;
	ld.global.f32 %f2, [%rd3];
	add.f32 %f1, %f1, %f2;
	add.s32 %r7, %r7, 1;
	bra L3_top;
L2_lend:
	mad.wide.s32 %rd4, %r4, 4, %rd2;
	st.global.f32 [%rd4], %f1;
L1_end:
	ret;
}
