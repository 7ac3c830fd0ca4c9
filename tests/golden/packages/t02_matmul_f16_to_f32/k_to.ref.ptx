.version 8.0
.target sm_89
.address_size 64


.visible .entry k_to(
	.param .u64 param_to__partial,
	.param .u64 param_to
)
{
	.reg .pred %p<3>;
	.reg .b32 %r<7>;
	.reg .b64 %rd<7>;
	.reg .b16 %v_v1;
	.reg .b32 %v__gid, %v_a0, %v_a1, %v__a2_ks;
	.reg .b64 %g_to__partial, %g_to;
	.reg .f32 %v_acc0, %v_acc0__p, %v_v2;

	ld.param.u64 %rd1, [param_to__partial];
	cvta.to.global.u64 %g_to__partial, %rd1;
	ld.param.u64 %rd2, [param_to];
	cvta.to.global.u64 %g_to, %rd2;
	// Tile[a0, a1] (N=8192)
	mov.u32 %r1, %ctaid.x;
	mov.u32 %r2, %ntid.x;
	mov.u32 %r3, %tid.x;
	mad.lo.u32 %v__gid, %r1, %r2, %r3;
	setp.ge.u32 %p1, %v__gid, 8192;
	@%p1 bra TILE_END_1;
	// START: decoding each axis index
	div.u32 %v_a0, %v__gid, 64;
	rem.u32 %v_a1, %v__gid, 64;
	// END: decoding each axis index
	// Loop(axis=Axis(name=_a2_ks, extent=Dim(value=2)))
	mov.f32 %v_acc0, 0f00000000;
	mov.s32 %v__a2_ks, 0;
LOOP_2:
	setp.ge.s32 %p2, %v__a2_ks, 2;
	@%p2 bra LOOP_END_3;
	// Load(names=acc0__p, input=to__partial)
	mad.lo.s32 %r4, %v__a2_ks, 128, %v_a0;
	mad.lo.s32 %r5, %r4, 64, %v_a1;
	mul.wide.s32 %rd3, %r5, 4;
	add.s64 %rd4, %g_to__partial, %rd3;
	ld.global.f32 %v_acc0__p, [%rd4];
	// Accum(name=acc0, value=acc0__p)
	add.rn.f32 %v_acc0, %v_acc0, %v_acc0__p;
	add.s32 %v__a2_ks, %v__a2_ks, 1;
	bra LOOP_2;
LOOP_END_3:
	// Assign(name=v1, op=ElementwiseImpl('copy'))
	cvt.rn.f16.f32 %v_v1, %v_acc0;
	// Assign(name=v2, op=ElementwiseImpl('copy'))
	cvt.f32.f16 %v_v2, %v_v1;
	// Write(output=to, index=a0, a1)
	mad.lo.s32 %r6, %v_a0, 64, %v_a1;
	mul.wide.s32 %rd5, %r6, 4;
	add.s64 %rd6, %g_to, %rd5;
	st.global.f32 [%rd6], %v_v2;
TILE_END_1:
	ret;
}
