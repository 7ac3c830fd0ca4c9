.version 8.0
.target sm_89
.address_size 64

.shared .align 4 .b8 s_acc0_smem[16];
.shared .align 4 .b8 s_acc1_smem[16];

.visible .entry k_softmax_05263d(
	.param .u64 param_x,
	.param .u64 param_softmax
)
{
	.reg .pred %p<7>;
	.reg .b32 %r<40>;
	.reg .b64 %rd<9>;
	.reg .f32 %f<18>;
	.reg .b32 %v__gid, %v_a0, %v_a1_co, %v_a1, %v_lane, %v_warp, %v_a3;
	.reg .b64 %g_x, %g_softmax;
	.reg .f32 %v_acc1, %v_acc0, %v_one, %v_in0, %v_in0__gn, %v_in0__dg, %v_in0__alpha, %v_in0__dg_o, %v_in0__beta, %v_in0__acc1_sa, %v_in0__acc1_sb, %v_acc0__o, %v_acc1__o, %v_acc0__o__gn, %v_acc0__o__dg, %v_acc0__o__alpha, %v_acc0__o__dg_o, %v_acc0__o__beta, %v_acc0__o__acc1_sa, %v_acc0__o__acc1_sb, %v_v2, %v_in2, %v_v3, %v_v4, %v_v5;

	mov.u32 %v_lane, %tid.x;
	and.b32 %v_lane, %v_lane, 31;
	mov.u32 %v_warp, %tid.x;
	shr.u32 %v_warp, %v_warp, 5;
	ld.param.u64 %rd1, [param_x];
	cvta.to.global.u64 %g_x, %rd1;
	ld.param.u64 %rd2, [param_softmax];
	cvta.to.global.u64 %g_softmax, %rd2;
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
	// StridedLoop(axis=Axis(name=a1, extent=Dim(value=256)), start=a1_co)
	mov.f32 %v_acc1, 0f00000000;
	mov.f32 %v_acc0, 0fF149F2CA;
	mov.s32 %v_a1, %v_a1_co;
LOOP_2:
	setp.ge.s32 %p2, %v_a1, 256;
	@%p2 bra LOOP_END_3;
	// Let(name=one, value=1.0)
	mov.f32 %v_one, 0f3F800000;
	// Load(names=in0, input=x)
	mad.lo.s32 %r4, %v_a0, 256, %v_a1;
	mul.wide.s32 %rd3, %r4, 4;
	add.s64 %rd4, %g_x, %rd3;
	ld.global.f32 %v_in0, [%rd4];
	// Assign(name=in0__gn, op=ElementwiseImpl('maximum'))
	max.f32 %v_in0__gn, %v_acc0, %v_in0;
	// Assign(name=in0__dg, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_in0__dg, %v_acc0, %v_in0__gn;
	// Assign(name=in0__alpha, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f1, %v_in0__dg, 0f3FB8AA3B;
	ex2.approx.f32 %v_in0__alpha, %f1;
	// Assign(name=in0__dg_o, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_in0__dg_o, %v_in0, %v_in0__gn;
	// Assign(name=in0__beta, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f2, %v_in0__dg_o, 0f3FB8AA3B;
	ex2.approx.f32 %v_in0__beta, %f2;
	// Assign(name=in0__acc1_sa, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_in0__acc1_sa, %v_acc1, %v_in0__alpha;
	// Assign(name=in0__acc1_sb, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_in0__acc1_sb, %v_in0__beta, %v_one;
	// Accum(name=acc1, value=in0__acc1_sb)
	add.rn.f32 %v_acc1, %v_in0__acc1_sa, %v_in0__acc1_sb;
	// Accum(name=acc0, value=in0)
	max.f32 %v_acc0, %v_acc0, %v_in0;
	add.s32 %v_a1, %v_a1, 128;
	bra LOOP_2;
LOOP_END_3:
	// WarpShuffle(state=acc0, acc1, state_b=acc0__o, acc1__o)
	activemask.b32 %r5;
	// butterfly step: exchange with lane ^ 16
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 16, 0x1f, %r5;
	shfl.sync.bfly.b32 %v_acc1__o, %v_acc1, 16, 0x1f, %r5;
	// Assign(name=acc0__o__gn, op=ElementwiseImpl('maximum'))
	max.f32 %v_acc0__o__gn, %v_acc0, %v_acc0__o;
	// Assign(name=acc0__o__dg, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_acc0__o__dg, %v_acc0, %v_acc0__o__gn;
	// Assign(name=acc0__o__alpha, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f3, %v_acc0__o__dg, 0f3FB8AA3B;
	ex2.approx.f32 %v_acc0__o__alpha, %f3;
	// Assign(name=acc0__o__dg_o, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_acc0__o__dg_o, %v_acc0__o, %v_acc0__o__gn;
	// Assign(name=acc0__o__beta, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f4, %v_acc0__o__dg_o, 0f3FB8AA3B;
	ex2.approx.f32 %v_acc0__o__beta, %f4;
	// Assign(name=acc0__o__acc1_sa, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__o__acc1_sa, %v_acc0__o__alpha, %v_acc1;
	// Assign(name=acc0__o__acc1_sb, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__o__acc1_sb, %v_acc0__o__beta, %v_acc1__o;
	// Assign(name=acc1, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc1, %v_acc0__o__acc1_sa, %v_acc0__o__acc1_sb;
	// Assign(name=acc0, op=ElementwiseImpl('copy'))
	mov.f32 %v_acc0, %v_acc0__o__gn;
	// butterfly step: exchange with lane ^ 8
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 8, 0x1f, %r5;
	shfl.sync.bfly.b32 %v_acc1__o, %v_acc1, 8, 0x1f, %r5;
	// Assign(name=acc0__o__gn, op=ElementwiseImpl('maximum'))
	max.f32 %v_acc0__o__gn, %v_acc0, %v_acc0__o;
	// Assign(name=acc0__o__dg, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_acc0__o__dg, %v_acc0, %v_acc0__o__gn;
	// Assign(name=acc0__o__alpha, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f5, %v_acc0__o__dg, 0f3FB8AA3B;
	ex2.approx.f32 %v_acc0__o__alpha, %f5;
	// Assign(name=acc0__o__dg_o, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_acc0__o__dg_o, %v_acc0__o, %v_acc0__o__gn;
	// Assign(name=acc0__o__beta, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f6, %v_acc0__o__dg_o, 0f3FB8AA3B;
	ex2.approx.f32 %v_acc0__o__beta, %f6;
	// Assign(name=acc0__o__acc1_sa, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__o__acc1_sa, %v_acc0__o__alpha, %v_acc1;
	// Assign(name=acc0__o__acc1_sb, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__o__acc1_sb, %v_acc0__o__beta, %v_acc1__o;
	// Assign(name=acc1, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc1, %v_acc0__o__acc1_sa, %v_acc0__o__acc1_sb;
	// Assign(name=acc0, op=ElementwiseImpl('copy'))
	mov.f32 %v_acc0, %v_acc0__o__gn;
	// butterfly step: exchange with lane ^ 4
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 4, 0x1f, %r5;
	shfl.sync.bfly.b32 %v_acc1__o, %v_acc1, 4, 0x1f, %r5;
	// Assign(name=acc0__o__gn, op=ElementwiseImpl('maximum'))
	max.f32 %v_acc0__o__gn, %v_acc0, %v_acc0__o;
	// Assign(name=acc0__o__dg, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_acc0__o__dg, %v_acc0, %v_acc0__o__gn;
	// Assign(name=acc0__o__alpha, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f7, %v_acc0__o__dg, 0f3FB8AA3B;
	ex2.approx.f32 %v_acc0__o__alpha, %f7;
	// Assign(name=acc0__o__dg_o, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_acc0__o__dg_o, %v_acc0__o, %v_acc0__o__gn;
	// Assign(name=acc0__o__beta, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f8, %v_acc0__o__dg_o, 0f3FB8AA3B;
	ex2.approx.f32 %v_acc0__o__beta, %f8;
	// Assign(name=acc0__o__acc1_sa, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__o__acc1_sa, %v_acc0__o__alpha, %v_acc1;
	// Assign(name=acc0__o__acc1_sb, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__o__acc1_sb, %v_acc0__o__beta, %v_acc1__o;
	// Assign(name=acc1, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc1, %v_acc0__o__acc1_sa, %v_acc0__o__acc1_sb;
	// Assign(name=acc0, op=ElementwiseImpl('copy'))
	mov.f32 %v_acc0, %v_acc0__o__gn;
	// butterfly step: exchange with lane ^ 2
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 2, 0x1f, %r5;
	shfl.sync.bfly.b32 %v_acc1__o, %v_acc1, 2, 0x1f, %r5;
	// Assign(name=acc0__o__gn, op=ElementwiseImpl('maximum'))
	max.f32 %v_acc0__o__gn, %v_acc0, %v_acc0__o;
	// Assign(name=acc0__o__dg, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_acc0__o__dg, %v_acc0, %v_acc0__o__gn;
	// Assign(name=acc0__o__alpha, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f9, %v_acc0__o__dg, 0f3FB8AA3B;
	ex2.approx.f32 %v_acc0__o__alpha, %f9;
	// Assign(name=acc0__o__dg_o, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_acc0__o__dg_o, %v_acc0__o, %v_acc0__o__gn;
	// Assign(name=acc0__o__beta, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f10, %v_acc0__o__dg_o, 0f3FB8AA3B;
	ex2.approx.f32 %v_acc0__o__beta, %f10;
	// Assign(name=acc0__o__acc1_sa, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__o__acc1_sa, %v_acc0__o__alpha, %v_acc1;
	// Assign(name=acc0__o__acc1_sb, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__o__acc1_sb, %v_acc0__o__beta, %v_acc1__o;
	// Assign(name=acc1, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc1, %v_acc0__o__acc1_sa, %v_acc0__o__acc1_sb;
	// Assign(name=acc0, op=ElementwiseImpl('copy'))
	mov.f32 %v_acc0, %v_acc0__o__gn;
	// butterfly step: exchange with lane ^ 1
	shfl.sync.bfly.b32 %v_acc0__o, %v_acc0, 1, 0x1f, %r5;
	shfl.sync.bfly.b32 %v_acc1__o, %v_acc1, 1, 0x1f, %r5;
	// Assign(name=acc0__o__gn, op=ElementwiseImpl('maximum'))
	max.f32 %v_acc0__o__gn, %v_acc0, %v_acc0__o;
	// Assign(name=acc0__o__dg, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_acc0__o__dg, %v_acc0, %v_acc0__o__gn;
	// Assign(name=acc0__o__alpha, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f11, %v_acc0__o__dg, 0f3FB8AA3B;
	ex2.approx.f32 %v_acc0__o__alpha, %f11;
	// Assign(name=acc0__o__dg_o, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_acc0__o__dg_o, %v_acc0__o, %v_acc0__o__gn;
	// Assign(name=acc0__o__beta, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f12, %v_acc0__o__dg_o, 0f3FB8AA3B;
	ex2.approx.f32 %v_acc0__o__beta, %f12;
	// Assign(name=acc0__o__acc1_sa, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__o__acc1_sa, %v_acc0__o__alpha, %v_acc1;
	// Assign(name=acc0__o__acc1_sb, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__o__acc1_sb, %v_acc0__o__beta, %v_acc1__o;
	// Assign(name=acc1, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc1, %v_acc0__o__acc1_sa, %v_acc0__o__acc1_sb;
	// Assign(name=acc0, op=ElementwiseImpl('copy'))
	mov.f32 %v_acc0, %v_acc0__o__gn;
	// Smem(name=acc0_smem, extents=4)
	// Smem(name=acc1_smem, extents=4)
	// if (lane == 0)
	setp.eq.s32 %p3, %v_lane, 0;
	@!%p3 bra IF_END_4;
	// Write(output=acc0_smem, index=warp)
	mov.u32 %r6, s_acc0_smem;
	mad.lo.s32 %r7, %v_warp, 4, %r6;
	st.shared.f32 [%r7], %v_acc0;
	// Write(output=acc1_smem, index=warp)
	mov.u32 %r8, s_acc1_smem;
	mad.lo.s32 %r9, %v_warp, 4, %r8;
	st.shared.f32 [%r9], %v_acc1;
IF_END_4:
	// Sync(barrier_id=0, count=None)
	bar.sync 0;
	// TreeHalve(bufs=acc0_smem, acc1_smem, state=acc0, acc1)
	// tree step: warp < 2 folds slot warp + 2
	setp.lt.s32 %p4, %v_warp, 2;
	@!%p4 bra TREE_SKIP_5;
	mov.u32 %r10, s_acc0_smem;
	mad.lo.s32 %r11, %v_warp, 4, %r10;
	ld.shared.f32 %v_acc0, [%r11];
	add.s32 %r12, %v_warp, 2;
	mov.u32 %r13, s_acc0_smem;
	mad.lo.s32 %r14, %r12, 4, %r13;
	ld.shared.f32 %v_acc0__o, [%r14];
	mov.u32 %r15, s_acc1_smem;
	mad.lo.s32 %r16, %v_warp, 4, %r15;
	ld.shared.f32 %v_acc1, [%r16];
	add.s32 %r17, %v_warp, 2;
	mov.u32 %r18, s_acc1_smem;
	mad.lo.s32 %r19, %r17, 4, %r18;
	ld.shared.f32 %v_acc1__o, [%r19];
	// Assign(name=acc0__o__gn, op=ElementwiseImpl('maximum'))
	max.f32 %v_acc0__o__gn, %v_acc0, %v_acc0__o;
	// Assign(name=acc0__o__dg, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_acc0__o__dg, %v_acc0, %v_acc0__o__gn;
	// Assign(name=acc0__o__alpha, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f13, %v_acc0__o__dg, 0f3FB8AA3B;
	ex2.approx.f32 %v_acc0__o__alpha, %f13;
	// Assign(name=acc0__o__dg_o, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_acc0__o__dg_o, %v_acc0__o, %v_acc0__o__gn;
	// Assign(name=acc0__o__beta, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f14, %v_acc0__o__dg_o, 0f3FB8AA3B;
	ex2.approx.f32 %v_acc0__o__beta, %f14;
	// Assign(name=acc0__o__acc1_sa, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__o__acc1_sa, %v_acc0__o__alpha, %v_acc1;
	// Assign(name=acc0__o__acc1_sb, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__o__acc1_sb, %v_acc0__o__beta, %v_acc1__o;
	// Assign(name=acc1, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc1, %v_acc0__o__acc1_sa, %v_acc0__o__acc1_sb;
	// Assign(name=acc0, op=ElementwiseImpl('copy'))
	mov.f32 %v_acc0, %v_acc0__o__gn;
	mov.u32 %r20, s_acc0_smem;
	mad.lo.s32 %r21, %v_warp, 4, %r20;
	st.shared.f32 [%r21], %v_acc0;
	mov.u32 %r22, s_acc1_smem;
	mad.lo.s32 %r23, %v_warp, 4, %r22;
	st.shared.f32 [%r23], %v_acc1;
TREE_SKIP_5:
	// Sync(barrier_id=0, count=None)
	bar.sync 0;
	// tree step: warp < 1 folds slot warp + 1
	setp.lt.s32 %p5, %v_warp, 1;
	@!%p5 bra TREE_SKIP_6;
	mov.u32 %r24, s_acc0_smem;
	mad.lo.s32 %r25, %v_warp, 4, %r24;
	ld.shared.f32 %v_acc0, [%r25];
	add.s32 %r26, %v_warp, 1;
	mov.u32 %r27, s_acc0_smem;
	mad.lo.s32 %r28, %r26, 4, %r27;
	ld.shared.f32 %v_acc0__o, [%r28];
	mov.u32 %r29, s_acc1_smem;
	mad.lo.s32 %r30, %v_warp, 4, %r29;
	ld.shared.f32 %v_acc1, [%r30];
	add.s32 %r31, %v_warp, 1;
	mov.u32 %r32, s_acc1_smem;
	mad.lo.s32 %r33, %r31, 4, %r32;
	ld.shared.f32 %v_acc1__o, [%r33];
	// Assign(name=acc0__o__gn, op=ElementwiseImpl('maximum'))
	max.f32 %v_acc0__o__gn, %v_acc0, %v_acc0__o;
	// Assign(name=acc0__o__dg, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_acc0__o__dg, %v_acc0, %v_acc0__o__gn;
	// Assign(name=acc0__o__alpha, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f15, %v_acc0__o__dg, 0f3FB8AA3B;
	ex2.approx.f32 %v_acc0__o__alpha, %f15;
	// Assign(name=acc0__o__dg_o, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_acc0__o__dg_o, %v_acc0__o, %v_acc0__o__gn;
	// Assign(name=acc0__o__beta, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f16, %v_acc0__o__dg_o, 0f3FB8AA3B;
	ex2.approx.f32 %v_acc0__o__beta, %f16;
	// Assign(name=acc0__o__acc1_sa, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__o__acc1_sa, %v_acc0__o__alpha, %v_acc1;
	// Assign(name=acc0__o__acc1_sb, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__o__acc1_sb, %v_acc0__o__beta, %v_acc1__o;
	// Assign(name=acc1, op=ElementwiseImpl('add'))
	add.rn.f32 %v_acc1, %v_acc0__o__acc1_sa, %v_acc0__o__acc1_sb;
	// Assign(name=acc0, op=ElementwiseImpl('copy'))
	mov.f32 %v_acc0, %v_acc0__o__gn;
	mov.u32 %r34, s_acc0_smem;
	mad.lo.s32 %r35, %v_warp, 4, %r34;
	st.shared.f32 [%r35], %v_acc0;
	mov.u32 %r36, s_acc1_smem;
	mad.lo.s32 %r37, %v_warp, 4, %r36;
	st.shared.f32 [%r37], %v_acc1;
TREE_SKIP_6:
	// Sync(barrier_id=0, count=None)
	bar.sync 0;
	ld.shared.f32 %v_acc0, [s_acc0_smem];
	ld.shared.f32 %v_acc1, [s_acc1_smem];
	// Assign(name=v2, op=ElementwiseImpl('reciprocal'))
	rcp.rn.f32 %v_v2, %v_acc1;
	// StridedLoop(axis=Axis(name=a3, extent=Dim(value=256)), start=a1_co)
	mov.s32 %v_a3, %v_a1_co;
LOOP_7:
	setp.ge.s32 %p6, %v_a3, 256;
	@%p6 bra LOOP_END_8;
	// Load(names=in2, input=x)
	mad.lo.s32 %r38, %v_a0, 256, %v_a3;
	mul.wide.s32 %rd5, %r38, 4;
	add.s64 %rd6, %g_x, %rd5;
	ld.global.f32 %v_in2, [%rd6];
	// Assign(name=v3, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v3, %v_in2, %v_acc0;
	// Assign(name=v4, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f17, %v_v3, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4, %f17;
	// Assign(name=v5, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v5, %v_v2, %v_v4;
	// Write(output=softmax, index=a0, a3)
	mad.lo.s32 %r39, %v_a0, 256, %v_a3;
	mul.wide.s32 %rd7, %r39, 4;
	add.s64 %rd8, %g_softmax, %rd7;
	st.global.f32 [%rd8], %v_v5;
	add.s32 %v_a3, %v_a3, 128;
	bra LOOP_7;
LOOP_END_8:
TILE_END_1:
	ret;
}
