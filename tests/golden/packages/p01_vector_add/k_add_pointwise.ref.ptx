.version 8.0
.target sm_89
.address_size 64


.visible .entry k_add_pointwise(
	.param .u64 param_x0,
	.param .u64 param_x1,
	.param .u64 param_add
)
{
	.reg .pred %p<2>;
	.reg .b32 %r<14>;
	.reg .b64 %rd<14>;
	.reg .b32 %v__gid, %v_a0;
	.reg .b64 %g_x0, %g_x1, %g_add;
	.reg .f32 %v_in0__u0, %v_in1__u0, %v_v0__u0, %v_in0__u1, %v_in1__u1, %v_v0__u1;

	ld.param.u64 %rd1, [param_x0];
	cvta.to.global.u64 %g_x0, %rd1;
	ld.param.u64 %rd2, [param_x1];
	cvta.to.global.u64 %g_x1, %rd2;
	ld.param.u64 %rd3, [param_add];
	cvta.to.global.u64 %g_add, %rd3;
	// Tile[a0] (N=512)
	mov.u32 %r1, %ctaid.x;
	mov.u32 %r2, %ntid.x;
	mov.u32 %r3, %tid.x;
	mad.lo.u32 %v__gid, %r1, %r2, %r3;
	setp.ge.u32 %p1, %v__gid, 512;
	@%p1 bra TILE_END_1;
	// START: decoding each axis index
	mov.u32 %v_a0, %v__gid;
	// END: decoding each axis index
	// Load(names=in0__u0, input=x0)
	mul.lo.s32 %r4, %v_a0, 2;
	add.s32 %r5, %r4, 0;
	mul.wide.s32 %rd4, %r5, 4;
	add.s64 %rd5, %g_x0, %rd4;
	ld.global.f32 %v_in0__u0, [%rd5];
	// Load(names=in1__u0, input=x1)
	mul.lo.s32 %r6, %v_a0, 2;
	add.s32 %r7, %r6, 0;
	mul.wide.s32 %rd6, %r7, 4;
	add.s64 %rd7, %g_x1, %rd6;
	ld.global.f32 %v_in1__u0, [%rd7];
	// Assign(name=v0__u0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_v0__u0, %v_in0__u0, %v_in1__u0;
	// Load(names=in0__u1, input=x0)
	mul.lo.s32 %r8, %v_a0, 2;
	add.s32 %r9, %r8, 1;
	mul.wide.s32 %rd8, %r9, 4;
	add.s64 %rd9, %g_x0, %rd8;
	ld.global.f32 %v_in0__u1, [%rd9];
	// Load(names=in1__u1, input=x1)
	mul.lo.s32 %r10, %v_a0, 2;
	add.s32 %r11, %r10, 1;
	mul.wide.s32 %rd10, %r11, 4;
	add.s64 %rd11, %g_x1, %rd10;
	ld.global.f32 %v_in1__u1, [%rd11];
	// Assign(name=v0__u1, op=ElementwiseImpl('add'))
	add.rn.f32 %v_v0__u1, %v_in0__u1, %v_in1__u1;
	// Write(output=add, index=((a0 * 2) + 0))
	mul.lo.s32 %r12, %v_a0, 2;
	add.s32 %r13, %r12, 0;
	mul.wide.s32 %rd12, %r13, 4;
	add.s64 %rd13, %g_add, %rd12;
	st.global.v2.f32 [%rd13], {%v_v0__u0, %v_v0__u1};
TILE_END_1:
	ret;
}
