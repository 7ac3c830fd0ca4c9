.version 8.0
.target sm_89
.address_size 64


.visible .entry k_mul_pointwise(
	.param .u64 param_x,
	.param .u64 param_y,
	.param .u64 param_mul
)
{
	.reg .pred %p<2>;
	.reg .b32 %r<22>;
	.reg .b64 %rd<22>;
	.reg .b32 %v__gid, %v_a0;
	.reg .b64 %g_x, %g_y, %g_mul;
	.reg .f32 %v_in0__u0, %v_v0__u0, %v_in1__u0, %v_v1__u0, %v_in0__u1, %v_v0__u1, %v_in1__u1, %v_v1__u1, %v_in0__u2, %v_v0__u2, %v_in1__u2, %v_v1__u2, %v_in0__u3, %v_v0__u3, %v_in1__u3, %v_v1__u3;

	ld.param.u64 %rd1, [param_x];
	cvta.to.global.u64 %g_x, %rd1;
	ld.param.u64 %rd2, [param_y];
	cvta.to.global.u64 %g_y, %rd2;
	ld.param.u64 %rd3, [param_mul];
	cvta.to.global.u64 %g_mul, %rd3;
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
	// Load(names=in0__u0, input=x)
	mul.lo.s32 %r4, %v_a0, 4;
	add.s32 %r5, %r4, 0;
	mul.wide.s32 %rd4, %r5, 4;
	add.s64 %rd5, %g_x, %rd4;
	ld.global.f32 %v_in0__u0, [%rd5];
	// Assign(name=v0__u0, op=ElementwiseImpl('relu'))
	max.f32 %v_v0__u0, %v_in0__u0, 0f00000000;
	// Load(names=in1__u0, input=y)
	mul.lo.s32 %r6, %v_a0, 4;
	add.s32 %r7, %r6, 0;
	mul.wide.s32 %rd6, %r7, 4;
	add.s64 %rd7, %g_y, %rd6;
	ld.global.f32 %v_in1__u0, [%rd7];
	// Assign(name=v1__u0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v1__u0, %v_in1__u0, %v_v0__u0;
	// Load(names=in0__u1, input=x)
	mul.lo.s32 %r8, %v_a0, 4;
	add.s32 %r9, %r8, 1;
	mul.wide.s32 %rd8, %r9, 4;
	add.s64 %rd9, %g_x, %rd8;
	ld.global.f32 %v_in0__u1, [%rd9];
	// Assign(name=v0__u1, op=ElementwiseImpl('relu'))
	max.f32 %v_v0__u1, %v_in0__u1, 0f00000000;
	// Load(names=in1__u1, input=y)
	mul.lo.s32 %r10, %v_a0, 4;
	add.s32 %r11, %r10, 1;
	mul.wide.s32 %rd10, %r11, 4;
	add.s64 %rd11, %g_y, %rd10;
	ld.global.f32 %v_in1__u1, [%rd11];
	// Assign(name=v1__u1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v1__u1, %v_in1__u1, %v_v0__u1;
	// Load(names=in0__u2, input=x)
	mul.lo.s32 %r12, %v_a0, 4;
	add.s32 %r13, %r12, 2;
	mul.wide.s32 %rd12, %r13, 4;
	add.s64 %rd13, %g_x, %rd12;
	ld.global.f32 %v_in0__u2, [%rd13];
	// Assign(name=v0__u2, op=ElementwiseImpl('relu'))
	max.f32 %v_v0__u2, %v_in0__u2, 0f00000000;
	// Load(names=in1__u2, input=y)
	mul.lo.s32 %r14, %v_a0, 4;
	add.s32 %r15, %r14, 2;
	mul.wide.s32 %rd14, %r15, 4;
	add.s64 %rd15, %g_y, %rd14;
	ld.global.f32 %v_in1__u2, [%rd15];
	// Assign(name=v1__u2, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v1__u2, %v_in1__u2, %v_v0__u2;
	// Load(names=in0__u3, input=x)
	mul.lo.s32 %r16, %v_a0, 4;
	add.s32 %r17, %r16, 3;
	mul.wide.s32 %rd16, %r17, 4;
	add.s64 %rd17, %g_x, %rd16;
	ld.global.f32 %v_in0__u3, [%rd17];
	// Assign(name=v0__u3, op=ElementwiseImpl('relu'))
	max.f32 %v_v0__u3, %v_in0__u3, 0f00000000;
	// Load(names=in1__u3, input=y)
	mul.lo.s32 %r18, %v_a0, 4;
	add.s32 %r19, %r18, 3;
	mul.wide.s32 %rd18, %r19, 4;
	add.s64 %rd19, %g_y, %rd18;
	ld.global.f32 %v_in1__u3, [%rd19];
	// Assign(name=v1__u3, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v1__u3, %v_in1__u3, %v_v0__u3;
	// Write(output=mul, index=((a0 * 4) + 0))
	mul.lo.s32 %r20, %v_a0, 4;
	add.s32 %r21, %r20, 0;
	mul.wide.s32 %rd20, %r21, 4;
	add.s64 %rd21, %g_mul, %rd20;
	st.global.v4.f32 [%rd21], {%v_v1__u0, %v_v1__u1, %v_v1__u2, %v_v1__u3};
TILE_END_1:
	ret;
}
