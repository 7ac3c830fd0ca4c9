.version 8.0
.target sm_89
.address_size 64


.visible .entry k_add_pointwise(
	.param .u64 param_mul_c1,
	.param .u64 param_add_c1,
	.param .u64 param_x,
	.param .u64 param_add
)
{
	.reg .pred %p<2>;
	.reg .b32 %r<14>;
	.reg .b64 %rd<31>;
	.reg .b32 %v__gid, %v_a0;
	.reg .b64 %g_mul_c1, %g_add_c1, %g_x, %g_add;
	.reg .f32 %v_in1__u0, %v_in2__u0, %v_v0__u0, %v_in0__u0, %v_v1__u0, %v_in1__u1, %v_in2__u1, %v_v0__u1, %v_in0__u1, %v_v1__u1, %v_in1__u2, %v_in2__u2, %v_v0__u2, %v_in0__u2, %v_v1__u2, %v_in1__u3, %v_in2__u3, %v_v0__u3, %v_in0__u3, %v_v1__u3;

	ld.param.u64 %rd1, [param_mul_c1];
	cvta.to.global.u64 %g_mul_c1, %rd1;
	ld.param.u64 %rd2, [param_add_c1];
	cvta.to.global.u64 %g_add_c1, %rd2;
	ld.param.u64 %rd3, [param_x];
	cvta.to.global.u64 %g_x, %rd3;
	ld.param.u64 %rd4, [param_add];
	cvta.to.global.u64 %g_add, %rd4;
	// Tile[a0] (N=1024)
	mov.u32 %r1, %ctaid.x;
	mov.u32 %r2, %ntid.x;
	mov.u32 %r3, %tid.x;
	mad.lo.u32 %v__gid, %r1, %r2, %r3;
	setp.ge.u32 %p1, %v__gid, 1024;
	@%p1 bra TILE_END_1;
	// START: decoding each axis index
	mov.u32 %v_a0, %v__gid;
	// END: decoding each axis index
	// Load(names=in1__u0, input=mul_c1)
	mov.b64 %rd5, 0;
	add.s64 %rd6, %g_mul_c1, %rd5;
	ld.global.f32 %v_in1__u0, [%rd6];
	// Load(names=in2__u0, input=x)
	mul.lo.s32 %r4, %v_a0, 4;
	add.s32 %r5, %r4, 0;
	mul.wide.s32 %rd7, %r5, 4;
	add.s64 %rd8, %g_x, %rd7;
	ld.global.f32 %v_in2__u0, [%rd8];
	// Assign(name=v0__u0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v0__u0, %v_in1__u0, %v_in2__u0;
	// Load(names=in0__u0, input=add_c1)
	mov.b64 %rd9, 0;
	add.s64 %rd10, %g_add_c1, %rd9;
	ld.global.f32 %v_in0__u0, [%rd10];
	// Assign(name=v1__u0, op=ElementwiseImpl('add'))
	add.rn.f32 %v_v1__u0, %v_in0__u0, %v_v0__u0;
	// Load(names=in1__u1, input=mul_c1)
	mov.b64 %rd11, 0;
	add.s64 %rd12, %g_mul_c1, %rd11;
	ld.global.f32 %v_in1__u1, [%rd12];
	// Load(names=in2__u1, input=x)
	mul.lo.s32 %r6, %v_a0, 4;
	add.s32 %r7, %r6, 1;
	mul.wide.s32 %rd13, %r7, 4;
	add.s64 %rd14, %g_x, %rd13;
	ld.global.f32 %v_in2__u1, [%rd14];
	// Assign(name=v0__u1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v0__u1, %v_in1__u1, %v_in2__u1;
	// Load(names=in0__u1, input=add_c1)
	mov.b64 %rd15, 0;
	add.s64 %rd16, %g_add_c1, %rd15;
	ld.global.f32 %v_in0__u1, [%rd16];
	// Assign(name=v1__u1, op=ElementwiseImpl('add'))
	add.rn.f32 %v_v1__u1, %v_in0__u1, %v_v0__u1;
	// Load(names=in1__u2, input=mul_c1)
	mov.b64 %rd17, 0;
	add.s64 %rd18, %g_mul_c1, %rd17;
	ld.global.f32 %v_in1__u2, [%rd18];
	// Load(names=in2__u2, input=x)
	mul.lo.s32 %r8, %v_a0, 4;
	add.s32 %r9, %r8, 2;
	mul.wide.s32 %rd19, %r9, 4;
	add.s64 %rd20, %g_x, %rd19;
	ld.global.f32 %v_in2__u2, [%rd20];
	// Assign(name=v0__u2, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v0__u2, %v_in1__u2, %v_in2__u2;
	// Load(names=in0__u2, input=add_c1)
	mov.b64 %rd21, 0;
	add.s64 %rd22, %g_add_c1, %rd21;
	ld.global.f32 %v_in0__u2, [%rd22];
	// Assign(name=v1__u2, op=ElementwiseImpl('add'))
	add.rn.f32 %v_v1__u2, %v_in0__u2, %v_v0__u2;
	// Load(names=in1__u3, input=mul_c1)
	mov.b64 %rd23, 0;
	add.s64 %rd24, %g_mul_c1, %rd23;
	ld.global.f32 %v_in1__u3, [%rd24];
	// Load(names=in2__u3, input=x)
	mul.lo.s32 %r10, %v_a0, 4;
	add.s32 %r11, %r10, 3;
	mul.wide.s32 %rd25, %r11, 4;
	add.s64 %rd26, %g_x, %rd25;
	ld.global.f32 %v_in2__u3, [%rd26];
	// Assign(name=v0__u3, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v0__u3, %v_in1__u3, %v_in2__u3;
	// Load(names=in0__u3, input=add_c1)
	mov.b64 %rd27, 0;
	add.s64 %rd28, %g_add_c1, %rd27;
	ld.global.f32 %v_in0__u3, [%rd28];
	// Assign(name=v1__u3, op=ElementwiseImpl('add'))
	add.rn.f32 %v_v1__u3, %v_in0__u3, %v_v0__u3;
	// Write(output=add, index=((a0 * 4) + 0))
	mul.lo.s32 %r12, %v_a0, 4;
	add.s32 %r13, %r12, 0;
	mul.wide.s32 %rd29, %r13, 4;
	add.s64 %rd30, %g_add, %rd29;
	st.global.v4.f32 [%rd30], {%v_v1__u0, %v_v1__u1, %v_v1__u2, %v_v1__u3};
TILE_END_1:
	ret;
}
