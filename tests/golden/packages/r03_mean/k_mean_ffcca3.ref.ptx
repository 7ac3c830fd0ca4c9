.version 8.0
.target sm_89
.address_size 64

.shared .align 4 .b8 s_acc0_smem[16];

.visible .entry k_mean_ffcca3(
	.param .u64 param_x,
	.param .u64 param_mean_keepdim_count,
	.param .u64 param_mean
)
{
	.reg .pred %p<7>;
	.reg .b32 %r<21>;
	.reg .b64 %rd<8>;
	.reg .b32 %v__gid, %v_a0_co, %v_a0, %v_lane, %v_warp;
	.reg .b64 %g_x, %g_mean_keepdim_count, %g_mean;
	.reg .f32 %v_acc0, %v_in0, %v_acc0__o, %v_in1, %v_v0;

	mov.u32 %v_lane, %tid.x;
	and.b32 %v_lane, %v_lane, 31;
	mov.u32 %v_warp, %tid.x;
	shr.u32 %v_warp, %v_warp, 5;
	ld.param.u64 %rd1, [param_x];
	cvta.to.global.u64 %g_x, %rd1;
	ld.param.u64 %rd2, [param_mean_keepdim_count];
	cvta.to.global.u64 %g_mean_keepdim_count, %rd2;
	ld.param.u64 %rd3, [param_mean];
	cvta.to.global.u64 %g_mean, %rd3;
	// Tile[a0_co] (N=128)
	mov.u32 %r1, %ctaid.x;
	mov.u32 %r2, %ntid.x;
	mov.u32 %r3, %tid.x;
	mad.lo.u32 %v__gid, %r1, %r2, %r3;
	setp.ge.u32 %p1, %v__gid, 128;
	@%p1 bra TILE_END_1;
	// START: decoding each axis index
	mov.u32 %v_a0_co, %v__gid;
	// END: decoding each axis index
	// StridedLoop(axis=Axis(name=a0, extent=Dim(value=32768)), start=a0_co)
	mov.f32 %v_acc0, 0f00000000;
	mov.s32 %v_a0, %v_a0_co;
LOOP_2:
	setp.ge.s32 %p2, %v_a0, 32768;
	@%p2 bra LOOP_END_3;
	// Load(names=in0, input=x)
	mul.wide.s32 %rd4, %v_a0, 4;
	add.s64 %rd5, %g_x, %rd4;
	ld.global.f32 %v_in0, [%rd5];
	// Accum(name=acc0, value=in0)
	add.rn.f32 %v_acc0, %v_acc0, %v_in0;
	add.s32 %v_a0, %v_a0, 128;
	bra LOOP_2;
LOOP_END_3:
	// WarpShuffle(state=acc0, state_b=acc0__o)
	activemask.b32 %r4;
	// butterfly step: exchange with lane ^ 16
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 16, 0x1f, %r4;
	// Assign(name=acc0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__o;
	// butterfly step: exchange with lane ^ 8
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 8, 0x1f, %r4;
	// Assign(name=acc0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__o;
	// butterfly step: exchange with lane ^ 4
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 4, 0x1f, %r4;
	// Assign(name=acc0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__o;
	// butterfly step: exchange with lane ^ 2
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 2, 0x1f, %r4;
	// Assign(name=acc0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__o;
	// butterfly step: exchange with lane ^ 1
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 1, 0x1f, %r4;
	// Assign(name=acc0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__o;
	// Smem(name=acc0_smem, extents=4)
	// if (lane == 0)
	setp.eq.s32 %p3, %v_lane, 0;
	@!%p3 bra IF_END_4;
	// Write(output=acc0_smem, index=warp)
	mov.u32 %r5, s_acc0_smem;
	mad.lo.s32 %r6, %v_warp, 4, %r5;
	st.shared.f32 [%r6], %v_acc0;
IF_END_4:
	// Sync(barrier_id=0, count=None)
	bar.sync 0;
	// TreeHalve(bufs=acc0_smem, state=acc0)
	// tree step: warp < 2 folds slot warp + 2
	setp.lt.s32 %p4, %v_warp, 2;
	@!%p4 bra TREE_SKIP_5;
	mov.u32 %r7, s_acc0_smem;
	mad.lo.s32 %r8, %v_warp, 4, %r7;
	ld.shared.f32 %v_acc0, [%r8];
	add.s32 %r9, %v_warp, 2;
	mov.u32 %r10, s_acc0_smem;
	mad.lo.s32 %r11, %r9, 4, %r10;
	ld.shared.f32 %v_acc0__o, [%r11];
	// Assign(name=acc0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__o;
	mov.u32 %r12, s_acc0_smem;
	mad.lo.s32 %r13, %v_warp, 4, %r12;
	st.shared.f32 [%r13], %v_acc0;
TREE_SKIP_5:
	// Sync(barrier_id=0, count=None)
	bar.sync 0;
	// tree step: warp < 1 folds slot warp + 1
	setp.lt.s32 %p5, %v_warp, 1;
	@!%p5 bra TREE_SKIP_6;
	mov.u32 %r14, s_acc0_smem;
	mad.lo.s32 %r15, %v_warp, 4, %r14;
	ld.shared.f32 %v_acc0, [%r15];
	add.s32 %r16, %v_warp, 1;
	mov.u32 %r17, s_acc0_smem;
	mad.lo.s32 %r18, %r16, 4, %r17;
	ld.shared.f32 %v_acc0__o, [%r18];
	// Assign(name=acc0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__o;
	mov.u32 %r19, s_acc0_smem;
	mad.lo.s32 %r20, %v_warp, 4, %r19;
	st.shared.f32 [%r20], %v_acc0;
TREE_SKIP_6:
	// Sync(barrier_id=0, count=None)
	bar.sync 0;
	ld.shared.f32 %v_acc0, [s_acc0_smem];
	// if (a0_co == 0)
	setp.eq.s32 %p6, %v_a0_co, 0;
	@!%p6 bra IF_END_7;
	// Load(names=in1, input=mean_keepdim_count)
	mov.b64 %rd6, 0;
	add.s64 %rd7, %g_mean_keepdim_count, %rd6;
	ld.global.f32 %v_in1, [%rd7];
	// Assign(name=v0, op=ElementwiseImpl('divide'))
	div.rn.f32 %v_v0, %v_acc0, %v_in1;
	// Write(output=mean, index=)
	st.global.f32 [%g_mean], %v_v0;
IF_END_7:
TILE_END_1:
	ret;
}
