.version 8.0
.target sm_89
.address_size 64


.visible .entry k_matmul_softmax_reduce_b55365(
	.param .u64 param_div_c1,
	.param .u64 param_q,
	.param .u64 param_kt,
	.param .u64 param_v,
	.param .u64 param_matmul_1
)
{
	.reg .pred %p<7>;
	.reg .b32 %r<107>;
	.reg .b64 %rd<42>;
	.reg .f32 %f<17>;
	.reg .b32 %v__gid, %v_a0_b, %v_a5_b, %v_a0_u, %v_a5_u, %v_a1, %v_a2;
	.reg .b64 %g_div_c1, %g_q, %g_kt, %g_v, %g_matmul_1;
	.reg .f32 %v_in0, %v_v1, %v_acc3__c0_0, %v_acc5__sum__c0_0, %v_acc1__c0_0, %v_acc3__c0_1, %v_acc5__sum__c0_1, %v_acc1__c0_1, %v_acc3__c1_0, %v_acc5__sum__c1_0, %v_acc1__c1_0, %v_acc3__c1_1, %v_acc5__sum__c1_1, %v_acc1__c1_1, %v_acc3__c2_0, %v_acc5__sum__c2_0, %v_acc1__c2_0, %v_acc3__c2_1, %v_acc5__sum__c2_1, %v_acc1__c2_1, %v_acc3__c3_0, %v_acc5__sum__c3_0, %v_acc1__c3_0, %v_acc3__c3_1, %v_acc5__sum__c3_1, %v_acc1__c3_1, %v_acc0__ar0, %v_in2__ar0, %v_in1__ar0, %v_v3__ar0, %v_acc0__ar1, %v_in2__ar1, %v_in1__ar1, %v_v3__ar1, %v_acc0__ar2, %v_in2__ar2, %v_in1__ar2, %v_v3__ar2, %v_acc0__ar3, %v_in2__ar3, %v_in1__ar3, %v_v3__ar3, %v_v4__c0_0, %v_one__c0_0, %v_v4__gn__c0_0, %v_v4__dg__c0_0, %v_v4__alpha__c0_0, %v_v4__dg_o__c0_0, %v_v4__beta__c0_0, %v_v4__acc3_sa__c0_0, %v_v4__acc3_sb__c0_0, %v_v4__acc5__sum_sa__c0_0, %v_in7__bc0, %v_in7__bc1, %v_v4__acc5__sum_sb__c0_0, %v_v4__c0_1, %v_one__c0_1, %v_v4__gn__c0_1, %v_v4__dg__c0_1, %v_v4__alpha__c0_1, %v_v4__dg_o__c0_1, %v_v4__beta__c0_1, %v_v4__acc3_sa__c0_1, %v_v4__acc3_sb__c0_1, %v_v4__acc5__sum_sa__c0_1, %v_v4__acc5__sum_sb__c0_1, %v_v4__c1_0, %v_one__c1_0, %v_v4__gn__c1_0, %v_v4__dg__c1_0, %v_v4__alpha__c1_0, %v_v4__dg_o__c1_0, %v_v4__beta__c1_0, %v_v4__acc3_sa__c1_0, %v_v4__acc3_sb__c1_0, %v_v4__acc5__sum_sa__c1_0, %v_v4__acc5__sum_sb__c1_0, %v_v4__c1_1, %v_one__c1_1, %v_v4__gn__c1_1, %v_v4__dg__c1_1, %v_v4__alpha__c1_1, %v_v4__dg_o__c1_1, %v_v4__beta__c1_1, %v_v4__acc3_sa__c1_1, %v_v4__acc3_sb__c1_1, %v_v4__acc5__sum_sa__c1_1, %v_v4__acc5__sum_sb__c1_1, %v_v4__c2_0, %v_one__c2_0, %v_v4__gn__c2_0, %v_v4__dg__c2_0, %v_v4__alpha__c2_0, %v_v4__dg_o__c2_0, %v_v4__beta__c2_0, %v_v4__acc3_sa__c2_0, %v_v4__acc3_sb__c2_0, %v_v4__acc5__sum_sa__c2_0, %v_v4__acc5__sum_sb__c2_0, %v_v4__c2_1, %v_one__c2_1, %v_v4__gn__c2_1, %v_v4__dg__c2_1, %v_v4__alpha__c2_1, %v_v4__dg_o__c2_1, %v_v4__beta__c2_1, %v_v4__acc3_sa__c2_1, %v_v4__acc3_sb__c2_1, %v_v4__acc5__sum_sa__c2_1, %v_v4__acc5__sum_sb__c2_1, %v_v4__c3_0, %v_one__c3_0, %v_v4__gn__c3_0, %v_v4__dg__c3_0, %v_v4__alpha__c3_0, %v_v4__dg_o__c3_0, %v_v4__beta__c3_0, %v_v4__acc3_sa__c3_0, %v_v4__acc3_sb__c3_0, %v_v4__acc5__sum_sa__c3_0, %v_v4__acc5__sum_sb__c3_0, %v_v4__c3_1, %v_one__c3_1, %v_v4__gn__c3_1, %v_v4__dg__c3_1, %v_v4__alpha__c3_1, %v_v4__dg_o__c3_1, %v_v4__beta__c3_1, %v_v4__acc3_sa__c3_1, %v_v4__acc3_sb__c3_1, %v_v4__acc5__sum_sa__c3_1, %v_v4__acc5__sum_sb__c3_1, %v_v9__c0_0, %v_acc5__c0_0, %v_v9__c0_1, %v_acc5__c0_1, %v_v9__c1_0, %v_acc5__c1_0, %v_v9__c1_1, %v_acc5__c1_1, %v_v9__c2_0, %v_acc5__c2_0, %v_v9__c2_1, %v_acc5__c2_1, %v_v9__c3_0, %v_acc5__c3_0, %v_v9__c3_1, %v_acc5__c3_1;

	ld.param.u64 %rd1, [param_div_c1];
	cvta.to.global.u64 %g_div_c1, %rd1;
	ld.param.u64 %rd2, [param_q];
	cvta.to.global.u64 %g_q, %rd2;
	ld.param.u64 %rd3, [param_kt];
	cvta.to.global.u64 %g_kt, %rd3;
	ld.param.u64 %rd4, [param_v];
	cvta.to.global.u64 %g_v, %rd4;
	ld.param.u64 %rd5, [param_matmul_1];
	cvta.to.global.u64 %g_matmul_1, %rd5;
	// Tile[a0_b, a5_b, a0_u, a5_u] (N=512)
	mov.u32 %r1, %ctaid.x;
	mov.u32 %r2, %ntid.x;
	mov.u32 %r3, %tid.x;
	mad.lo.u32 %v__gid, %r1, %r2, %r3;
	setp.ge.u32 %p1, %v__gid, 512;
	@%p1 bra TILE_END_1;
	// START: decoding each axis index
	div.u32 %v_a0_b, %v__gid, 256;
	div.u32 %r4, %v__gid, 128;
	rem.u32 %v_a5_b, %r4, 2;
	div.u32 %r5, %v__gid, 16;
	rem.u32 %v_a0_u, %r5, 8;
	rem.u32 %v_a5_u, %v__gid, 16;
	// END: decoding each axis index
	// Load(names=in0, input=div_c1)
	mov.b64 %rd6, 0;
	add.s64 %rd7, %g_div_c1, %rd6;
	ld.global.f32 %v_in0, [%rd7];
	// Assign(name=v1, op=ElementwiseImpl('reciprocal'))
	rcp.rn.f32 %v_v1, %v_in0;
	// Loop(axis=Axis(name=a1, extent=Dim(value=64)))
	mov.f32 %v_acc3__c0_0, 0f00000000;
	mov.f32 %v_acc5__sum__c0_0, 0f00000000;
	mov.f32 %v_acc1__c0_0, 0fF149F2CA;
	mov.f32 %v_acc3__c0_1, 0f00000000;
	mov.f32 %v_acc5__sum__c0_1, 0f00000000;
	mov.f32 %v_acc1__c0_1, 0fF149F2CA;
	mov.f32 %v_acc3__c1_0, 0f00000000;
	mov.f32 %v_acc5__sum__c1_0, 0f00000000;
	mov.f32 %v_acc1__c1_0, 0fF149F2CA;
	mov.f32 %v_acc3__c1_1, 0f00000000;
	mov.f32 %v_acc5__sum__c1_1, 0f00000000;
	mov.f32 %v_acc1__c1_1, 0fF149F2CA;
	mov.f32 %v_acc3__c2_0, 0f00000000;
	mov.f32 %v_acc5__sum__c2_0, 0f00000000;
	mov.f32 %v_acc1__c2_0, 0fF149F2CA;
	mov.f32 %v_acc3__c2_1, 0f00000000;
	mov.f32 %v_acc5__sum__c2_1, 0f00000000;
	mov.f32 %v_acc1__c2_1, 0fF149F2CA;
	mov.f32 %v_acc3__c3_0, 0f00000000;
	mov.f32 %v_acc5__sum__c3_0, 0f00000000;
	mov.f32 %v_acc1__c3_0, 0fF149F2CA;
	mov.f32 %v_acc3__c3_1, 0f00000000;
	mov.f32 %v_acc5__sum__c3_1, 0f00000000;
	mov.f32 %v_acc1__c3_1, 0fF149F2CA;
	mov.s32 %v_a1, 0;
LOOP_2:
	setp.ge.s32 %p2, %v_a1, 64;
	@%p2 bra LOOP_END_3;
	// Loop(axis=Axis(name=a2, extent=Dim(value=64)))
	mov.f32 %v_acc0__ar0, 0f00000000;
	mov.s32 %v_a2, 0;
LOOP_4:
	setp.ge.s32 %p3, %v_a2, 64;
	@%p3 bra LOOP_END_5;
	// Load(names=in2__ar0, input=q)
	mul.lo.s32 %r6, %v_a0_b, 32;
	mul.lo.s32 %r7, %v_a0_u, 4;
	add.s32 %r8, %r6, %r7;
	add.s32 %r9, %r8, 0;
	mad.lo.s32 %r10, %r9, 64, %v_a2;
	mul.wide.s32 %rd8, %r10, 4;
	add.s64 %rd9, %g_q, %rd8;
	ld.global.f32 %v_in2__ar0, [%rd9];
	// Load(names=in1__ar0, input=kt)
	mad.lo.s32 %r11, %v_a2, 64, %v_a1;
	mul.wide.s32 %rd10, %r11, 4;
	add.s64 %rd11, %g_kt, %rd10;
	ld.global.f32 %v_in1__ar0, [%rd11];
	// Assign(name=v3__ar0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v3__ar0, %v_in1__ar0, %v_in2__ar0;
	// Accum(name=acc0__ar0, value=v3__ar0)
	add.rn.f32 %v_acc0__ar0, %v_acc0__ar0, %v_v3__ar0;
	add.s32 %v_a2, %v_a2, 1;
	bra LOOP_4;
LOOP_END_5:
	// Loop(axis=Axis(name=a2, extent=Dim(value=64)))
	mov.f32 %v_acc0__ar1, 0f00000000;
	mov.s32 %v_a2, 0;
LOOP_6:
	setp.ge.s32 %p4, %v_a2, 64;
	@%p4 bra LOOP_END_7;
	// Load(names=in2__ar1, input=q)
	mul.lo.s32 %r12, %v_a0_b, 32;
	mul.lo.s32 %r13, %v_a0_u, 4;
	add.s32 %r14, %r12, %r13;
	add.s32 %r15, %r14, 1;
	mad.lo.s32 %r16, %r15, 64, %v_a2;
	mul.wide.s32 %rd12, %r16, 4;
	add.s64 %rd13, %g_q, %rd12;
	ld.global.f32 %v_in2__ar1, [%rd13];
	// Load(names=in1__ar1, input=kt)
	mad.lo.s32 %r17, %v_a2, 64, %v_a1;
	mul.wide.s32 %rd14, %r17, 4;
	add.s64 %rd15, %g_kt, %rd14;
	ld.global.f32 %v_in1__ar1, [%rd15];
	// Assign(name=v3__ar1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v3__ar1, %v_in1__ar1, %v_in2__ar1;
	// Accum(name=acc0__ar1, value=v3__ar1)
	add.rn.f32 %v_acc0__ar1, %v_acc0__ar1, %v_v3__ar1;
	add.s32 %v_a2, %v_a2, 1;
	bra LOOP_6;
LOOP_END_7:
	// Loop(axis=Axis(name=a2, extent=Dim(value=64)))
	mov.f32 %v_acc0__ar2, 0f00000000;
	mov.s32 %v_a2, 0;
LOOP_8:
	setp.ge.s32 %p5, %v_a2, 64;
	@%p5 bra LOOP_END_9;
	// Load(names=in2__ar2, input=q)
	mul.lo.s32 %r18, %v_a0_b, 32;
	mul.lo.s32 %r19, %v_a0_u, 4;
	add.s32 %r20, %r18, %r19;
	add.s32 %r21, %r20, 2;
	mad.lo.s32 %r22, %r21, 64, %v_a2;
	mul.wide.s32 %rd16, %r22, 4;
	add.s64 %rd17, %g_q, %rd16;
	ld.global.f32 %v_in2__ar2, [%rd17];
	// Load(names=in1__ar2, input=kt)
	mad.lo.s32 %r23, %v_a2, 64, %v_a1;
	mul.wide.s32 %rd18, %r23, 4;
	add.s64 %rd19, %g_kt, %rd18;
	ld.global.f32 %v_in1__ar2, [%rd19];
	// Assign(name=v3__ar2, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v3__ar2, %v_in1__ar2, %v_in2__ar2;
	// Accum(name=acc0__ar2, value=v3__ar2)
	add.rn.f32 %v_acc0__ar2, %v_acc0__ar2, %v_v3__ar2;
	add.s32 %v_a2, %v_a2, 1;
	bra LOOP_8;
LOOP_END_9:
	// Loop(axis=Axis(name=a2, extent=Dim(value=64)))
	mov.f32 %v_acc0__ar3, 0f00000000;
	mov.s32 %v_a2, 0;
LOOP_10:
	setp.ge.s32 %p6, %v_a2, 64;
	@%p6 bra LOOP_END_11;
	// Load(names=in2__ar3, input=q)
	mul.lo.s32 %r24, %v_a0_b, 32;
	mul.lo.s32 %r25, %v_a0_u, 4;
	add.s32 %r26, %r24, %r25;
	add.s32 %r27, %r26, 3;
	mad.lo.s32 %r28, %r27, 64, %v_a2;
	mul.wide.s32 %rd20, %r28, 4;
	add.s64 %rd21, %g_q, %rd20;
	ld.global.f32 %v_in2__ar3, [%rd21];
	// Load(names=in1__ar3, input=kt)
	mad.lo.s32 %r29, %v_a2, 64, %v_a1;
	mul.wide.s32 %rd22, %r29, 4;
	add.s64 %rd23, %g_kt, %rd22;
	ld.global.f32 %v_in1__ar3, [%rd23];
	// Assign(name=v3__ar3, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v3__ar3, %v_in1__ar3, %v_in2__ar3;
	// Accum(name=acc0__ar3, value=v3__ar3)
	add.rn.f32 %v_acc0__ar3, %v_acc0__ar3, %v_v3__ar3;
	add.s32 %v_a2, %v_a2, 1;
	bra LOOP_10;
LOOP_END_11:
	// Assign(name=v4__c0_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__c0_0, %v_acc0__ar0, %v_v1;
	// Let(name=one__c0_0, value=1.0)
	mov.f32 %v_one__c0_0, 0f3F800000;
	// Assign(name=v4__gn__c0_0, op=ElementwiseImpl('maximum'))
	max.f32 %v_v4__gn__c0_0, %v_acc1__c0_0, %v_v4__c0_0;
	// Assign(name=v4__dg__c0_0, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg__c0_0, %v_acc1__c0_0, %v_v4__gn__c0_0;
	// Assign(name=v4__alpha__c0_0, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f1, %v_v4__dg__c0_0, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__alpha__c0_0, %f1;
	// Assign(name=v4__dg_o__c0_0, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg_o__c0_0, %v_v4__c0_0, %v_v4__gn__c0_0;
	// Assign(name=v4__beta__c0_0, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f2, %v_v4__dg_o__c0_0, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__beta__c0_0, %f2;
	// Assign(name=v4__acc3_sa__c0_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sa__c0_0, %v_acc3__c0_0, %v_v4__alpha__c0_0;
	// Assign(name=v4__acc3_sb__c0_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sb__c0_0, %v_one__c0_0, %v_v4__beta__c0_0;
	// Accum(name=acc3__c0_0, value=v4__acc3_sb__c0_0)
	add.rn.f32 %v_acc3__c0_0, %v_v4__acc3_sa__c0_0, %v_v4__acc3_sb__c0_0;
	// Assign(name=v4__acc5__sum_sa__c0_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sa__c0_0, %v_acc5__sum__c0_0, %v_v4__alpha__c0_0;
	// Load(names=in7__bc0, in7__bc1, input=v)
	mul.lo.s32 %r30, %v_a5_b, 32;
	mul.lo.s32 %r31, %v_a5_u, 2;
	add.s32 %r32, %r30, %r31;
	add.s32 %r33, %r32, 0;
	mad.lo.s32 %r34, %v_a1, 64, %r33;
	mul.wide.s32 %rd24, %r34, 4;
	add.s64 %rd25, %g_v, %rd24;
	ld.global.v2.f32 {%v_in7__bc0, %v_in7__bc1}, [%rd25];
	// Assign(name=v4__acc5__sum_sb__c0_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sb__c0_0, %v_in7__bc0, %v_v4__beta__c0_0;
	// Accum(name=acc5__sum__c0_0, value=v4__acc5__sum_sb__c0_0)
	add.rn.f32 %v_acc5__sum__c0_0, %v_v4__acc5__sum_sa__c0_0, %v_v4__acc5__sum_sb__c0_0;
	// Accum(name=acc1__c0_0, value=v4__c0_0)
	max.f32 %v_acc1__c0_0, %v_acc1__c0_0, %v_v4__c0_0;
	// Assign(name=v4__c0_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__c0_1, %v_acc0__ar0, %v_v1;
	// Let(name=one__c0_1, value=1.0)
	mov.f32 %v_one__c0_1, 0f3F800000;
	// Assign(name=v4__gn__c0_1, op=ElementwiseImpl('maximum'))
	max.f32 %v_v4__gn__c0_1, %v_acc1__c0_1, %v_v4__c0_1;
	// Assign(name=v4__dg__c0_1, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg__c0_1, %v_acc1__c0_1, %v_v4__gn__c0_1;
	// Assign(name=v4__alpha__c0_1, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f3, %v_v4__dg__c0_1, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__alpha__c0_1, %f3;
	// Assign(name=v4__dg_o__c0_1, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg_o__c0_1, %v_v4__c0_1, %v_v4__gn__c0_1;
	// Assign(name=v4__beta__c0_1, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f4, %v_v4__dg_o__c0_1, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__beta__c0_1, %f4;
	// Assign(name=v4__acc3_sa__c0_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sa__c0_1, %v_acc3__c0_1, %v_v4__alpha__c0_1;
	// Assign(name=v4__acc3_sb__c0_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sb__c0_1, %v_one__c0_1, %v_v4__beta__c0_1;
	// Accum(name=acc3__c0_1, value=v4__acc3_sb__c0_1)
	add.rn.f32 %v_acc3__c0_1, %v_v4__acc3_sa__c0_1, %v_v4__acc3_sb__c0_1;
	// Assign(name=v4__acc5__sum_sa__c0_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sa__c0_1, %v_acc5__sum__c0_1, %v_v4__alpha__c0_1;
	// Assign(name=v4__acc5__sum_sb__c0_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sb__c0_1, %v_in7__bc1, %v_v4__beta__c0_1;
	// Accum(name=acc5__sum__c0_1, value=v4__acc5__sum_sb__c0_1)
	add.rn.f32 %v_acc5__sum__c0_1, %v_v4__acc5__sum_sa__c0_1, %v_v4__acc5__sum_sb__c0_1;
	// Accum(name=acc1__c0_1, value=v4__c0_1)
	max.f32 %v_acc1__c0_1, %v_acc1__c0_1, %v_v4__c0_1;
	// Assign(name=v4__c1_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__c1_0, %v_acc0__ar1, %v_v1;
	// Let(name=one__c1_0, value=1.0)
	mov.f32 %v_one__c1_0, 0f3F800000;
	// Assign(name=v4__gn__c1_0, op=ElementwiseImpl('maximum'))
	max.f32 %v_v4__gn__c1_0, %v_acc1__c1_0, %v_v4__c1_0;
	// Assign(name=v4__dg__c1_0, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg__c1_0, %v_acc1__c1_0, %v_v4__gn__c1_0;
	// Assign(name=v4__alpha__c1_0, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f5, %v_v4__dg__c1_0, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__alpha__c1_0, %f5;
	// Assign(name=v4__dg_o__c1_0, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg_o__c1_0, %v_v4__c1_0, %v_v4__gn__c1_0;
	// Assign(name=v4__beta__c1_0, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f6, %v_v4__dg_o__c1_0, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__beta__c1_0, %f6;
	// Assign(name=v4__acc3_sa__c1_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sa__c1_0, %v_acc3__c1_0, %v_v4__alpha__c1_0;
	// Assign(name=v4__acc3_sb__c1_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sb__c1_0, %v_one__c1_0, %v_v4__beta__c1_0;
	// Accum(name=acc3__c1_0, value=v4__acc3_sb__c1_0)
	add.rn.f32 %v_acc3__c1_0, %v_v4__acc3_sa__c1_0, %v_v4__acc3_sb__c1_0;
	// Assign(name=v4__acc5__sum_sa__c1_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sa__c1_0, %v_acc5__sum__c1_0, %v_v4__alpha__c1_0;
	// Assign(name=v4__acc5__sum_sb__c1_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sb__c1_0, %v_in7__bc0, %v_v4__beta__c1_0;
	// Accum(name=acc5__sum__c1_0, value=v4__acc5__sum_sb__c1_0)
	add.rn.f32 %v_acc5__sum__c1_0, %v_v4__acc5__sum_sa__c1_0, %v_v4__acc5__sum_sb__c1_0;
	// Accum(name=acc1__c1_0, value=v4__c1_0)
	max.f32 %v_acc1__c1_0, %v_acc1__c1_0, %v_v4__c1_0;
	// Assign(name=v4__c1_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__c1_1, %v_acc0__ar1, %v_v1;
	// Let(name=one__c1_1, value=1.0)
	mov.f32 %v_one__c1_1, 0f3F800000;
	// Assign(name=v4__gn__c1_1, op=ElementwiseImpl('maximum'))
	max.f32 %v_v4__gn__c1_1, %v_acc1__c1_1, %v_v4__c1_1;
	// Assign(name=v4__dg__c1_1, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg__c1_1, %v_acc1__c1_1, %v_v4__gn__c1_1;
	// Assign(name=v4__alpha__c1_1, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f7, %v_v4__dg__c1_1, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__alpha__c1_1, %f7;
	// Assign(name=v4__dg_o__c1_1, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg_o__c1_1, %v_v4__c1_1, %v_v4__gn__c1_1;
	// Assign(name=v4__beta__c1_1, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f8, %v_v4__dg_o__c1_1, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__beta__c1_1, %f8;
	// Assign(name=v4__acc3_sa__c1_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sa__c1_1, %v_acc3__c1_1, %v_v4__alpha__c1_1;
	// Assign(name=v4__acc3_sb__c1_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sb__c1_1, %v_one__c1_1, %v_v4__beta__c1_1;
	// Accum(name=acc3__c1_1, value=v4__acc3_sb__c1_1)
	add.rn.f32 %v_acc3__c1_1, %v_v4__acc3_sa__c1_1, %v_v4__acc3_sb__c1_1;
	// Assign(name=v4__acc5__sum_sa__c1_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sa__c1_1, %v_acc5__sum__c1_1, %v_v4__alpha__c1_1;
	// Assign(name=v4__acc5__sum_sb__c1_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sb__c1_1, %v_in7__bc1, %v_v4__beta__c1_1;
	// Accum(name=acc5__sum__c1_1, value=v4__acc5__sum_sb__c1_1)
	add.rn.f32 %v_acc5__sum__c1_1, %v_v4__acc5__sum_sa__c1_1, %v_v4__acc5__sum_sb__c1_1;
	// Accum(name=acc1__c1_1, value=v4__c1_1)
	max.f32 %v_acc1__c1_1, %v_acc1__c1_1, %v_v4__c1_1;
	// Assign(name=v4__c2_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__c2_0, %v_acc0__ar2, %v_v1;
	// Let(name=one__c2_0, value=1.0)
	mov.f32 %v_one__c2_0, 0f3F800000;
	// Assign(name=v4__gn__c2_0, op=ElementwiseImpl('maximum'))
	max.f32 %v_v4__gn__c2_0, %v_acc1__c2_0, %v_v4__c2_0;
	// Assign(name=v4__dg__c2_0, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg__c2_0, %v_acc1__c2_0, %v_v4__gn__c2_0;
	// Assign(name=v4__alpha__c2_0, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f9, %v_v4__dg__c2_0, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__alpha__c2_0, %f9;
	// Assign(name=v4__dg_o__c2_0, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg_o__c2_0, %v_v4__c2_0, %v_v4__gn__c2_0;
	// Assign(name=v4__beta__c2_0, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f10, %v_v4__dg_o__c2_0, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__beta__c2_0, %f10;
	// Assign(name=v4__acc3_sa__c2_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sa__c2_0, %v_acc3__c2_0, %v_v4__alpha__c2_0;
	// Assign(name=v4__acc3_sb__c2_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sb__c2_0, %v_one__c2_0, %v_v4__beta__c2_0;
	// Accum(name=acc3__c2_0, value=v4__acc3_sb__c2_0)
	add.rn.f32 %v_acc3__c2_0, %v_v4__acc3_sa__c2_0, %v_v4__acc3_sb__c2_0;
	// Assign(name=v4__acc5__sum_sa__c2_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sa__c2_0, %v_acc5__sum__c2_0, %v_v4__alpha__c2_0;
	// Assign(name=v4__acc5__sum_sb__c2_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sb__c2_0, %v_in7__bc0, %v_v4__beta__c2_0;
	// Accum(name=acc5__sum__c2_0, value=v4__acc5__sum_sb__c2_0)
	add.rn.f32 %v_acc5__sum__c2_0, %v_v4__acc5__sum_sa__c2_0, %v_v4__acc5__sum_sb__c2_0;
	// Accum(name=acc1__c2_0, value=v4__c2_0)
	max.f32 %v_acc1__c2_0, %v_acc1__c2_0, %v_v4__c2_0;
	// Assign(name=v4__c2_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__c2_1, %v_acc0__ar2, %v_v1;
	// Let(name=one__c2_1, value=1.0)
	mov.f32 %v_one__c2_1, 0f3F800000;
	// Assign(name=v4__gn__c2_1, op=ElementwiseImpl('maximum'))
	max.f32 %v_v4__gn__c2_1, %v_acc1__c2_1, %v_v4__c2_1;
	// Assign(name=v4__dg__c2_1, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg__c2_1, %v_acc1__c2_1, %v_v4__gn__c2_1;
	// Assign(name=v4__alpha__c2_1, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f11, %v_v4__dg__c2_1, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__alpha__c2_1, %f11;
	// Assign(name=v4__dg_o__c2_1, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg_o__c2_1, %v_v4__c2_1, %v_v4__gn__c2_1;
	// Assign(name=v4__beta__c2_1, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f12, %v_v4__dg_o__c2_1, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__beta__c2_1, %f12;
	// Assign(name=v4__acc3_sa__c2_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sa__c2_1, %v_acc3__c2_1, %v_v4__alpha__c2_1;
	// Assign(name=v4__acc3_sb__c2_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sb__c2_1, %v_one__c2_1, %v_v4__beta__c2_1;
	// Accum(name=acc3__c2_1, value=v4__acc3_sb__c2_1)
	add.rn.f32 %v_acc3__c2_1, %v_v4__acc3_sa__c2_1, %v_v4__acc3_sb__c2_1;
	// Assign(name=v4__acc5__sum_sa__c2_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sa__c2_1, %v_acc5__sum__c2_1, %v_v4__alpha__c2_1;
	// Assign(name=v4__acc5__sum_sb__c2_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sb__c2_1, %v_in7__bc1, %v_v4__beta__c2_1;
	// Accum(name=acc5__sum__c2_1, value=v4__acc5__sum_sb__c2_1)
	add.rn.f32 %v_acc5__sum__c2_1, %v_v4__acc5__sum_sa__c2_1, %v_v4__acc5__sum_sb__c2_1;
	// Accum(name=acc1__c2_1, value=v4__c2_1)
	max.f32 %v_acc1__c2_1, %v_acc1__c2_1, %v_v4__c2_1;
	// Assign(name=v4__c3_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__c3_0, %v_acc0__ar3, %v_v1;
	// Let(name=one__c3_0, value=1.0)
	mov.f32 %v_one__c3_0, 0f3F800000;
	// Assign(name=v4__gn__c3_0, op=ElementwiseImpl('maximum'))
	max.f32 %v_v4__gn__c3_0, %v_acc1__c3_0, %v_v4__c3_0;
	// Assign(name=v4__dg__c3_0, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg__c3_0, %v_acc1__c3_0, %v_v4__gn__c3_0;
	// Assign(name=v4__alpha__c3_0, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f13, %v_v4__dg__c3_0, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__alpha__c3_0, %f13;
	// Assign(name=v4__dg_o__c3_0, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg_o__c3_0, %v_v4__c3_0, %v_v4__gn__c3_0;
	// Assign(name=v4__beta__c3_0, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f14, %v_v4__dg_o__c3_0, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__beta__c3_0, %f14;
	// Assign(name=v4__acc3_sa__c3_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sa__c3_0, %v_acc3__c3_0, %v_v4__alpha__c3_0;
	// Assign(name=v4__acc3_sb__c3_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sb__c3_0, %v_one__c3_0, %v_v4__beta__c3_0;
	// Accum(name=acc3__c3_0, value=v4__acc3_sb__c3_0)
	add.rn.f32 %v_acc3__c3_0, %v_v4__acc3_sa__c3_0, %v_v4__acc3_sb__c3_0;
	// Assign(name=v4__acc5__sum_sa__c3_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sa__c3_0, %v_acc5__sum__c3_0, %v_v4__alpha__c3_0;
	// Assign(name=v4__acc5__sum_sb__c3_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sb__c3_0, %v_in7__bc0, %v_v4__beta__c3_0;
	// Accum(name=acc5__sum__c3_0, value=v4__acc5__sum_sb__c3_0)
	add.rn.f32 %v_acc5__sum__c3_0, %v_v4__acc5__sum_sa__c3_0, %v_v4__acc5__sum_sb__c3_0;
	// Accum(name=acc1__c3_0, value=v4__c3_0)
	max.f32 %v_acc1__c3_0, %v_acc1__c3_0, %v_v4__c3_0;
	// Assign(name=v4__c3_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__c3_1, %v_acc0__ar3, %v_v1;
	// Let(name=one__c3_1, value=1.0)
	mov.f32 %v_one__c3_1, 0f3F800000;
	// Assign(name=v4__gn__c3_1, op=ElementwiseImpl('maximum'))
	max.f32 %v_v4__gn__c3_1, %v_acc1__c3_1, %v_v4__c3_1;
	// Assign(name=v4__dg__c3_1, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg__c3_1, %v_acc1__c3_1, %v_v4__gn__c3_1;
	// Assign(name=v4__alpha__c3_1, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f15, %v_v4__dg__c3_1, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__alpha__c3_1, %f15;
	// Assign(name=v4__dg_o__c3_1, op=ElementwiseImpl('subtract'))
	sub.rn.f32 %v_v4__dg_o__c3_1, %v_v4__c3_1, %v_v4__gn__c3_1;
	// Assign(name=v4__beta__c3_1, op=ElementwiseImpl('exp'))
	mul.rn.f32 %f16, %v_v4__dg_o__c3_1, 0f3FB8AA3B;
	ex2.approx.f32 %v_v4__beta__c3_1, %f16;
	// Assign(name=v4__acc3_sa__c3_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sa__c3_1, %v_acc3__c3_1, %v_v4__alpha__c3_1;
	// Assign(name=v4__acc3_sb__c3_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc3_sb__c3_1, %v_one__c3_1, %v_v4__beta__c3_1;
	// Accum(name=acc3__c3_1, value=v4__acc3_sb__c3_1)
	add.rn.f32 %v_acc3__c3_1, %v_v4__acc3_sa__c3_1, %v_v4__acc3_sb__c3_1;
	// Assign(name=v4__acc5__sum_sa__c3_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sa__c3_1, %v_acc5__sum__c3_1, %v_v4__alpha__c3_1;
	// Assign(name=v4__acc5__sum_sb__c3_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sb__c3_1, %v_in7__bc1, %v_v4__beta__c3_1;
	// Accum(name=acc5__sum__c3_1, value=v4__acc5__sum_sb__c3_1)
	add.rn.f32 %v_acc5__sum__c3_1, %v_v4__acc5__sum_sa__c3_1, %v_v4__acc5__sum_sb__c3_1;
	// Accum(name=acc1__c3_1, value=v4__c3_1)
	max.f32 %v_acc1__c3_1, %v_acc1__c3_1, %v_v4__c3_1;
	add.s32 %v_a1, %v_a1, 1;
	bra LOOP_2;
LOOP_END_3:
	// Assign(name=v9__c0_0, op=ElementwiseImpl('reciprocal'))
	rcp.rn.f32 %v_v9__c0_0, %v_acc3__c0_0;
	// Assign(name=acc5__c0_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc5__c0_0, %v_acc5__sum__c0_0, %v_v9__c0_0;
	// Write(output=matmul_1, index=(((a0_b * 32) + (a0_u * 4)) + 0), (((a5_b * 32) + (a5_u * 2)) + 0))
	mul.lo.s32 %r35, %v_a0_b, 32;
	mul.lo.s32 %r36, %v_a0_u, 4;
	add.s32 %r37, %r35, %r36;
	add.s32 %r38, %r37, 0;
	mul.lo.s32 %r39, %v_a5_b, 32;
	mul.lo.s32 %r40, %v_a5_u, 2;
	add.s32 %r41, %r39, %r40;
	add.s32 %r42, %r41, 0;
	mad.lo.s32 %r43, %r38, 64, %r42;
	mul.wide.s32 %rd26, %r43, 4;
	add.s64 %rd27, %g_matmul_1, %rd26;
	st.global.f32 [%rd27], %v_acc5__c0_0;
	// Assign(name=v9__c0_1, op=ElementwiseImpl('reciprocal'))
	rcp.rn.f32 %v_v9__c0_1, %v_acc3__c0_1;
	// Assign(name=acc5__c0_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc5__c0_1, %v_acc5__sum__c0_1, %v_v9__c0_1;
	// Write(output=matmul_1, index=(((a0_b * 32) + (a0_u * 4)) + 0), (((a5_b * 32) + (a5_u * 2)) + 1))
	mul.lo.s32 %r44, %v_a0_b, 32;
	mul.lo.s32 %r45, %v_a0_u, 4;
	add.s32 %r46, %r44, %r45;
	add.s32 %r47, %r46, 0;
	mul.lo.s32 %r48, %v_a5_b, 32;
	mul.lo.s32 %r49, %v_a5_u, 2;
	add.s32 %r50, %r48, %r49;
	add.s32 %r51, %r50, 1;
	mad.lo.s32 %r52, %r47, 64, %r51;
	mul.wide.s32 %rd28, %r52, 4;
	add.s64 %rd29, %g_matmul_1, %rd28;
	st.global.f32 [%rd29], %v_acc5__c0_1;
	// Assign(name=v9__c1_0, op=ElementwiseImpl('reciprocal'))
	rcp.rn.f32 %v_v9__c1_0, %v_acc3__c1_0;
	// Assign(name=acc5__c1_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc5__c1_0, %v_acc5__sum__c1_0, %v_v9__c1_0;
	// Write(output=matmul_1, index=(((a0_b * 32) + (a0_u * 4)) + 1), (((a5_b * 32) + (a5_u * 2)) + 0))
	mul.lo.s32 %r53, %v_a0_b, 32;
	mul.lo.s32 %r54, %v_a0_u, 4;
	add.s32 %r55, %r53, %r54;
	add.s32 %r56, %r55, 1;
	mul.lo.s32 %r57, %v_a5_b, 32;
	mul.lo.s32 %r58, %v_a5_u, 2;
	add.s32 %r59, %r57, %r58;
	add.s32 %r60, %r59, 0;
	mad.lo.s32 %r61, %r56, 64, %r60;
	mul.wide.s32 %rd30, %r61, 4;
	add.s64 %rd31, %g_matmul_1, %rd30;
	st.global.f32 [%rd31], %v_acc5__c1_0;
	// Assign(name=v9__c1_1, op=ElementwiseImpl('reciprocal'))
	rcp.rn.f32 %v_v9__c1_1, %v_acc3__c1_1;
	// Assign(name=acc5__c1_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc5__c1_1, %v_acc5__sum__c1_1, %v_v9__c1_1;
	// Write(output=matmul_1, index=(((a0_b * 32) + (a0_u * 4)) + 1), (((a5_b * 32) + (a5_u * 2)) + 1))
	mul.lo.s32 %r62, %v_a0_b, 32;
	mul.lo.s32 %r63, %v_a0_u, 4;
	add.s32 %r64, %r62, %r63;
	add.s32 %r65, %r64, 1;
	mul.lo.s32 %r66, %v_a5_b, 32;
	mul.lo.s32 %r67, %v_a5_u, 2;
	add.s32 %r68, %r66, %r67;
	add.s32 %r69, %r68, 1;
	mad.lo.s32 %r70, %r65, 64, %r69;
	mul.wide.s32 %rd32, %r70, 4;
	add.s64 %rd33, %g_matmul_1, %rd32;
	st.global.f32 [%rd33], %v_acc5__c1_1;
	// Assign(name=v9__c2_0, op=ElementwiseImpl('reciprocal'))
	rcp.rn.f32 %v_v9__c2_0, %v_acc3__c2_0;
	// Assign(name=acc5__c2_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc5__c2_0, %v_acc5__sum__c2_0, %v_v9__c2_0;
	// Write(output=matmul_1, index=(((a0_b * 32) + (a0_u * 4)) + 2), (((a5_b * 32) + (a5_u * 2)) + 0))
	mul.lo.s32 %r71, %v_a0_b, 32;
	mul.lo.s32 %r72, %v_a0_u, 4;
	add.s32 %r73, %r71, %r72;
	add.s32 %r74, %r73, 2;
	mul.lo.s32 %r75, %v_a5_b, 32;
	mul.lo.s32 %r76, %v_a5_u, 2;
	add.s32 %r77, %r75, %r76;
	add.s32 %r78, %r77, 0;
	mad.lo.s32 %r79, %r74, 64, %r78;
	mul.wide.s32 %rd34, %r79, 4;
	add.s64 %rd35, %g_matmul_1, %rd34;
	st.global.f32 [%rd35], %v_acc5__c2_0;
	// Assign(name=v9__c2_1, op=ElementwiseImpl('reciprocal'))
	rcp.rn.f32 %v_v9__c2_1, %v_acc3__c2_1;
	// Assign(name=acc5__c2_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc5__c2_1, %v_acc5__sum__c2_1, %v_v9__c2_1;
	// Write(output=matmul_1, index=(((a0_b * 32) + (a0_u * 4)) + 2), (((a5_b * 32) + (a5_u * 2)) + 1))
	mul.lo.s32 %r80, %v_a0_b, 32;
	mul.lo.s32 %r81, %v_a0_u, 4;
	add.s32 %r82, %r80, %r81;
	add.s32 %r83, %r82, 2;
	mul.lo.s32 %r84, %v_a5_b, 32;
	mul.lo.s32 %r85, %v_a5_u, 2;
	add.s32 %r86, %r84, %r85;
	add.s32 %r87, %r86, 1;
	mad.lo.s32 %r88, %r83, 64, %r87;
	mul.wide.s32 %rd36, %r88, 4;
	add.s64 %rd37, %g_matmul_1, %rd36;
	st.global.f32 [%rd37], %v_acc5__c2_1;
	// Assign(name=v9__c3_0, op=ElementwiseImpl('reciprocal'))
	rcp.rn.f32 %v_v9__c3_0, %v_acc3__c3_0;
	// Assign(name=acc5__c3_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc5__c3_0, %v_acc5__sum__c3_0, %v_v9__c3_0;
	// Write(output=matmul_1, index=(((a0_b * 32) + (a0_u * 4)) + 3), (((a5_b * 32) + (a5_u * 2)) + 0))
	mul.lo.s32 %r89, %v_a0_b, 32;
	mul.lo.s32 %r90, %v_a0_u, 4;
	add.s32 %r91, %r89, %r90;
	add.s32 %r92, %r91, 3;
	mul.lo.s32 %r93, %v_a5_b, 32;
	mul.lo.s32 %r94, %v_a5_u, 2;
	add.s32 %r95, %r93, %r94;
	add.s32 %r96, %r95, 0;
	mad.lo.s32 %r97, %r92, 64, %r96;
	mul.wide.s32 %rd38, %r97, 4;
	add.s64 %rd39, %g_matmul_1, %rd38;
	st.global.f32 [%rd39], %v_acc5__c3_0;
	// Assign(name=v9__c3_1, op=ElementwiseImpl('reciprocal'))
	rcp.rn.f32 %v_v9__c3_1, %v_acc3__c3_1;
	// Assign(name=acc5__c3_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc5__c3_1, %v_acc5__sum__c3_1, %v_v9__c3_1;
	// Write(output=matmul_1, index=(((a0_b * 32) + (a0_u * 4)) + 3), (((a5_b * 32) + (a5_u * 2)) + 1))
	mul.lo.s32 %r98, %v_a0_b, 32;
	mul.lo.s32 %r99, %v_a0_u, 4;
	add.s32 %r100, %r98, %r99;
	add.s32 %r101, %r100, 3;
	mul.lo.s32 %r102, %v_a5_b, 32;
	mul.lo.s32 %r103, %v_a5_u, 2;
	add.s32 %r104, %r102, %r103;
	add.s32 %r105, %r104, 1;
	mad.lo.s32 %r106, %r101, 64, %r105;
	mul.wide.s32 %rd40, %r106, 4;
	add.s64 %rd41, %g_matmul_1, %rd40;
	st.global.f32 [%rd41], %v_acc5__c3_1;
TILE_END_1:
	ret;
}
