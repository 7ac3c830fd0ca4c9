.version 8.0
.target sm_89
.address_size 64


.visible .entry k_div_pointwise(
	.param .u64 param_add_c1,
	.param .u64 param_x,
	.param .u64 param_y,
	.param .u64 param_div
)
{
	.reg .pred %p<2>;
	.reg .b32 %r<28>;
	.reg .b64 %rd<37>;
	.reg .b32 %v__gid, %v_a0;
	.reg .b64 %g_add_c1, %g_x, %g_y, %g_div;
	.reg .f64 %v_in1__u0, %v_v0__u0, %v_in0__u0, %v_v1__u0, %v_v2__u0, %v_in2__u0, %v_v3__u0, %v_in1__u1, %v_v0__u1, %v_in0__u1, %v_v1__u1, %v_v2__u1, %v_in2__u1, %v_v3__u1, %v_in1__u2, %v_v0__u2, %v_in0__u2, %v_v1__u2, %v_v2__u2, %v_in2__u2, %v_v3__u2, %v_in1__u3, %v_v0__u3, %v_in0__u3, %v_v1__u3, %v_v2__u3, %v_in2__u3, %v_v3__u3;

	ld.param.u64 %rd1, [param_add_c1];
	cvta.to.global.u64 %g_add_c1, %rd1;
	ld.param.u64 %rd2, [param_x];
	cvta.to.global.u64 %g_x, %rd2;
	ld.param.u64 %rd3, [param_y];
	cvta.to.global.u64 %g_y, %rd3;
	ld.param.u64 %rd4, [param_div];
	cvta.to.global.u64 %g_div, %rd4;
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
	// Load(names=in1__u0, input=x)
	mul.lo.s32 %r4, %v_a0, 4;
	add.s32 %r5, %r4, 0;
	mul.wide.s32 %rd5, %r5, 8;
	add.s64 %rd6, %g_x, %rd5;
	ld.global.f64 %v_in1__u0, [%rd6];
	// Assign(name=v0__u0, op=ElementwiseImpl('multiply'))
	mul.rn.f64 %v_v0__u0, %v_in1__u0, %v_in1__u0;
	// Load(names=in0__u0, input=add_c1)
	mov.b64 %rd7, 0;
	add.s64 %rd8, %g_add_c1, %rd7;
	ld.global.f64 %v_in0__u0, [%rd8];
	// Assign(name=v1__u0, op=ElementwiseImpl('add'))
	add.rn.f64 %v_v1__u0, %v_in0__u0, %v_v0__u0;
	// Assign(name=v2__u0, op=ElementwiseImpl('sqrt'))
	sqrt.rn.f64 %v_v2__u0, %v_v1__u0;
	// Load(names=in2__u0, input=y)
	mul.lo.s32 %r6, %v_a0, 4;
	add.s32 %r7, %r6, 0;
	mul.wide.s32 %rd9, %r7, 8;
	add.s64 %rd10, %g_y, %rd9;
	ld.global.f64 %v_in2__u0, [%rd10];
	// Assign(name=v3__u0, op=ElementwiseImpl('divide'))
	div.rn.f64 %v_v3__u0, %v_v2__u0, %v_in2__u0;
	// Load(names=in1__u1, input=x)
	mul.lo.s32 %r8, %v_a0, 4;
	add.s32 %r9, %r8, 1;
	mul.wide.s32 %rd11, %r9, 8;
	add.s64 %rd12, %g_x, %rd11;
	ld.global.f64 %v_in1__u1, [%rd12];
	// Assign(name=v0__u1, op=ElementwiseImpl('multiply'))
	mul.rn.f64 %v_v0__u1, %v_in1__u1, %v_in1__u1;
	// Load(names=in0__u1, input=add_c1)
	mov.b64 %rd13, 0;
	add.s64 %rd14, %g_add_c1, %rd13;
	ld.global.f64 %v_in0__u1, [%rd14];
	// Assign(name=v1__u1, op=ElementwiseImpl('add'))
	add.rn.f64 %v_v1__u1, %v_in0__u1, %v_v0__u1;
	// Assign(name=v2__u1, op=ElementwiseImpl('sqrt'))
	sqrt.rn.f64 %v_v2__u1, %v_v1__u1;
	// Load(names=in2__u1, input=y)
	mul.lo.s32 %r10, %v_a0, 4;
	add.s32 %r11, %r10, 1;
	mul.wide.s32 %rd15, %r11, 8;
	add.s64 %rd16, %g_y, %rd15;
	ld.global.f64 %v_in2__u1, [%rd16];
	// Assign(name=v3__u1, op=ElementwiseImpl('divide'))
	div.rn.f64 %v_v3__u1, %v_v2__u1, %v_in2__u1;
	// Load(names=in1__u2, input=x)
	mul.lo.s32 %r12, %v_a0, 4;
	add.s32 %r13, %r12, 2;
	mul.wide.s32 %rd17, %r13, 8;
	add.s64 %rd18, %g_x, %rd17;
	ld.global.f64 %v_in1__u2, [%rd18];
	// Assign(name=v0__u2, op=ElementwiseImpl('multiply'))
	mul.rn.f64 %v_v0__u2, %v_in1__u2, %v_in1__u2;
	// Load(names=in0__u2, input=add_c1)
	mov.b64 %rd19, 0;
	add.s64 %rd20, %g_add_c1, %rd19;
	ld.global.f64 %v_in0__u2, [%rd20];
	// Assign(name=v1__u2, op=ElementwiseImpl('add'))
	add.rn.f64 %v_v1__u2, %v_in0__u2, %v_v0__u2;
	// Assign(name=v2__u2, op=ElementwiseImpl('sqrt'))
	sqrt.rn.f64 %v_v2__u2, %v_v1__u2;
	// Load(names=in2__u2, input=y)
	mul.lo.s32 %r14, %v_a0, 4;
	add.s32 %r15, %r14, 2;
	mul.wide.s32 %rd21, %r15, 8;
	add.s64 %rd22, %g_y, %rd21;
	ld.global.f64 %v_in2__u2, [%rd22];
	// Assign(name=v3__u2, op=ElementwiseImpl('divide'))
	div.rn.f64 %v_v3__u2, %v_v2__u2, %v_in2__u2;
	// Load(names=in1__u3, input=x)
	mul.lo.s32 %r16, %v_a0, 4;
	add.s32 %r17, %r16, 3;
	mul.wide.s32 %rd23, %r17, 8;
	add.s64 %rd24, %g_x, %rd23;
	ld.global.f64 %v_in1__u3, [%rd24];
	// Assign(name=v0__u3, op=ElementwiseImpl('multiply'))
	mul.rn.f64 %v_v0__u3, %v_in1__u3, %v_in1__u3;
	// Load(names=in0__u3, input=add_c1)
	mov.b64 %rd25, 0;
	add.s64 %rd26, %g_add_c1, %rd25;
	ld.global.f64 %v_in0__u3, [%rd26];
	// Assign(name=v1__u3, op=ElementwiseImpl('add'))
	add.rn.f64 %v_v1__u3, %v_in0__u3, %v_v0__u3;
	// Assign(name=v2__u3, op=ElementwiseImpl('sqrt'))
	sqrt.rn.f64 %v_v2__u3, %v_v1__u3;
	// Load(names=in2__u3, input=y)
	mul.lo.s32 %r18, %v_a0, 4;
	add.s32 %r19, %r18, 3;
	mul.wide.s32 %rd27, %r19, 8;
	add.s64 %rd28, %g_y, %rd27;
	ld.global.f64 %v_in2__u3, [%rd28];
	// Assign(name=v3__u3, op=ElementwiseImpl('divide'))
	div.rn.f64 %v_v3__u3, %v_v2__u3, %v_in2__u3;
	// Write(output=div, index=((a0 * 4) + 0))
	mul.lo.s32 %r20, %v_a0, 4;
	add.s32 %r21, %r20, 0;
	mul.wide.s32 %rd29, %r21, 8;
	add.s64 %rd30, %g_div, %rd29;
	st.global.f64 [%rd30], %v_v3__u0;
	// Write(output=div, index=((a0 * 4) + 1))
	mul.lo.s32 %r22, %v_a0, 4;
	add.s32 %r23, %r22, 1;
	mul.wide.s32 %rd31, %r23, 8;
	add.s64 %rd32, %g_div, %rd31;
	st.global.f64 [%rd32], %v_v3__u1;
	// Write(output=div, index=((a0 * 4) + 2))
	mul.lo.s32 %r24, %v_a0, 4;
	add.s32 %r25, %r24, 2;
	mul.wide.s32 %rd33, %r25, 8;
	add.s64 %rd34, %g_div, %rd33;
	st.global.f64 [%rd34], %v_v3__u2;
	// Write(output=div, index=((a0 * 4) + 3))
	mul.lo.s32 %r26, %v_a0, 4;
	add.s32 %r27, %r26, 3;
	mul.wide.s32 %rd35, %r27, 8;
	add.s64 %rd36, %g_div, %rd35;
	st.global.f64 [%rd36], %v_v3__u3;
TILE_END_1:
	ret;
}
