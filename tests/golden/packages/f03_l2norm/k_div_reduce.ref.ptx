.version 8.0
.target sm_89
.address_size 64

.shared .align 4 .b8 s_acc0_smem[16];

.visible .entry k_div_reduce(
	.param .u64 param_x,
	.param .u64 param_div
)
{
	.reg .pred %p<7>;
	.reg .b32 %r<24>;
	.reg .b64 %rd<9>;
	.reg .b32 %v__gid, %v_a0, %v_a1_co, %v_a1, %v_lane, %v_warp, %v_a2;
	.reg .b64 %g_x, %g_div;
	.reg .f32 %v_acc0, %v_in0, %v_v0, %v_acc0__o, %v_v1, %v_v2, %v_in1, %v_v3;

	mov.u32 %v_lane, %tid.x;
	and.b32 %v_lane, %v_lane, 31;
	mov.u32 %v_warp, %tid.x;
	shr.u32 %v_warp, %v_warp, 5;
	ld.param.u64 %rd1, [param_x];
	cvta.to.global.u64 %g_x, %rd1;
	ld.param.u64 %rd2, [param_div];
	cvta.to.global.u64 %g_div, %rd2;
	// Tile[a0, a1_co] (N=8192)
	mov.u32 %r1, %ctaid.x;
	mov.u32 %r2, %ntid.x;
	mov.u32 %r3, %tid.x;
	mad.lo.u32 %v__gid, %r1, %r2, %r3;
	setp.ge.u32 %p1, %v__gid, 8192;
	@%p1 bra TILE_END_1;
	// START: decoding each axis index
	div.u32 %v_a0, %v__gid, 128;
	rem.u32 %v_a1_co, %v__gid, 128;
	// END: decoding each axis index
	// StridedLoop(axis=Axis(name=a1, extent=Dim(value=512)), start=a1_co)
	mov.f32 %v_acc0, 0f00000000;
	mov.s32 %v_a1, %v_a1_co;
LOOP_2:
	setp.ge.s32 %p2, %v_a1, 512;
	@%p2 bra LOOP_END_3;
	// Load(names=in0, input=x)
	mad.lo.s32 %r4, %v_a0, 512, %v_a1;
	mul.wide.s32 %rd3, %r4, 4;
	add.s64 %rd4, %g_x, %rd3;
	ld.global.f32 %v_in0, [%rd4];
	// Assign(name=v0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v0, %v_in0, %v_in0;
	// Accum(name=acc0, value=v0)
	add.rn.f32 %v_acc0, %v_acc0, %v_v0;
	add.s32 %v_a1, %v_a1, 128;
	bra LOOP_2;
LOOP_END_3:
	// WarpShuffle(state=acc0, state_b=acc0__o)
	activemask.b32 %r5;
	// butterfly step: exchange with lane ^ 16
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 16, 0x1f, %r5;
	// Assign(name=acc0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__o;
	// butterfly step: exchange with lane ^ 8
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 8, 0x1f, %r5;
	// Assign(name=acc0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__o;
	// butterfly step: exchange with lane ^ 4
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 4, 0x1f, %r5;
	// Assign(name=acc0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__o;
	// butterfly step: exchange with lane ^ 2
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 2, 0x1f, %r5;
	// Assign(name=acc0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__o;
	// butterfly step: exchange with lane ^ 1
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 1, 0x1f, %r5;
	// Assign(name=acc0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__o;
	// Smem(name=acc0_smem, extents=4)
	// if (lane == 0)
	setp.eq.s32 %p3, %v_lane, 0;
	@!%p3 bra IF_END_4;
	// Write(output=acc0_smem, index=warp)
	mov.u32 %r6, s_acc0_smem;
	mad.lo.s32 %r7, %v_warp, 4, %r6;
	st.shared.f32 [%r7], %v_acc0;
IF_END_4:
	// Sync(barrier_id=0, count=None)
	bar.sync 0;
	// TreeHalve(bufs=acc0_smem, state=acc0)
	// tree step: warp < 2 folds slot warp + 2
	setp.lt.s32 %p4, %v_warp, 2;
	@!%p4 bra TREE_SKIP_5;
	mov.u32 %r8, s_acc0_smem;
	mad.lo.s32 %r9, %v_warp, 4, %r8;
	ld.shared.f32 %v_acc0, [%r9];
	add.s32 %r10, %v_warp, 2;
	mov.u32 %r11, s_acc0_smem;
	mad.lo.s32 %r12, %r10, 4, %r11;
	ld.shared.f32 %v_acc0__o, [%r12];
	// Assign(name=acc0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__o;
	mov.u32 %r13, s_acc0_smem;
	mad.lo.s32 %r14, %v_warp, 4, %r13;
	st.shared.f32 [%r14], %v_acc0;
TREE_SKIP_5:
	// Sync(barrier_id=0, count=None)
	bar.sync 0;
	// tree step: warp < 1 folds slot warp + 1
	setp.lt.s32 %p5, %v_warp, 1;
	@!%p5 bra TREE_SKIP_6;
	mov.u32 %r15, s_acc0_smem;
	mad.lo.s32 %r16, %v_warp, 4, %r15;
	ld.shared.f32 %v_acc0, [%r16];
	add.s32 %r17, %v_warp, 1;
	mov.u32 %r18, s_acc0_smem;
	mad.lo.s32 %r19, %r17, 4, %r18;
	ld.shared.f32 %v_acc0__o, [%r19];
	// Assign(name=acc0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__o;
	mov.u32 %r20, s_acc0_smem;
	mad.lo.s32 %r21, %v_warp, 4, %r20;
	st.shared.f32 [%r21], %v_acc0;
TREE_SKIP_6:
	// Sync(barrier_id=0, count=None)
	bar.sync 0;
	ld.shared.f32 %v_acc0, [s_acc0_smem];
	// Assign(name=v1, op=ElementwiseImpl('sqrt'))
	sqrt.rn.f32 %v_v1, %v_acc0;
	// Assign(name=v2, op=ElementwiseImpl('reciprocal'))
	rcp.rn.f32 %v_v2, %v_v1;
	// StridedLoop(axis=Axis(name=a2, extent=Dim(value=512)), start=a1_co)
	mov.s32 %v_a2, %v_a1_co;
LOOP_7:
	setp.ge.s32 %p6, %v_a2, 512;
	@%p6 bra LOOP_END_8;
	// Load(names=in1, input=x)
	mad.lo.s32 %r22, %v_a0, 512, %v_a2;
	mul.wide.s32 %rd5, %r22, 4;
	add.s64 %rd6, %g_x, %rd5;
	ld.global.f32 %v_in1, [%rd6];
	// Assign(name=v3, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v3, %v_in1, %v_v2;
	// Write(output=div, index=a0, a2)
	mad.lo.s32 %r23, %v_a0, 512, %v_a2;
	mul.wide.s32 %rd7, %r23, 4;
	add.s64 %rd8, %g_div, %rd7;
	st.global.f32 [%rd8], %v_v3;
	add.s32 %v_a2, %v_a2, 128;
	bra LOOP_7;
LOOP_END_8:
TILE_END_1:
	ret;
}
