.version 8.0
.target sm_89
.address_size 64


.visible .entry k_matmul_softmax_reduce_6f0029(
	.param .u64 param_div_c1,
	.param .u64 param_q,
	.param .u64 param_kt,
	.param .u64 param_v,
	.param .u64 param_matmul_1
)
{
	.reg .pred %p<4>;
	.reg .b32 %r<26>;
	.reg .b64 %rd<16>;
	.reg .f32 %f<3>;
	.reg .b32 %v__gid, %v_a0_b, %v_a5_b, %v_a0_u, %v_a5_u, %v_a1, %v_a2;
	.reg .b64 %g_div_c1, %g_q, %g_kt, %g_v, %g_matmul_1;
	.reg .f32 %v_in0, %v_v1, %v_acc3__c0_0, %v_acc5__sum__c0_0, %v_acc1__c0_0, %v_acc0__ar0, %v_in2__ar0, %v_in1__ar0, %v_v3__ar0, %v_v4__c0_0, %v_one__c0_0, %v_v4__gn__c0_0, %v_v4__dg__c0_0, %v_v4__alpha__c0_0, %v_v4__dg_o__c0_0, %v_v4__beta__c0_0, %v_v4__acc3_sa__c0_0, %v_v4__acc3_sb__c0_0, %v_v4__acc5__sum_sa__c0_0, %v_in7__bc0, %v_v4__acc5__sum_sb__c0_0, %v_v9__c0_0, %v_acc5__c0_0;

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
	// Tile[a0_b, a5_b, a0_u, a5_u] (N=4096)
	mov.u32 %r1, %ctaid.x;
	mov.u32 %r2, %ntid.x;
	mov.u32 %r3, %tid.x;
	mad.lo.u32 %v__gid, %r1, %r2, %r3;
	setp.ge.u32 %p1, %v__gid, 4096;
	@%p1 bra TILE_END_1;
	// START: decoding each axis index
	div.u32 %v_a0_b, %v__gid, 32;
	div.u32 %r4, %v__gid, 32;
	rem.u32 %v_a5_b, %r4, 1;
	div.u32 %r5, %v__gid, 32;
	rem.u32 %v_a0_u, %r5, 1;
	rem.u32 %v_a5_u, %v__gid, 32;
	// END: decoding each axis index
	// Load(names=in0, input=div_c1)
	mov.b64 %rd6, 0;
	add.s64 %rd7, %g_div_c1, %rd6;
	ld.global.f32 %v_in0, [%rd7];
	// Assign(name=v1, op=ElementwiseImpl('reciprocal'))
	rcp.rn.f32 %v_v1, %v_in0;
	// Loop(axis=Axis(name=a1, extent=Dim(value=128)))
	mov.f32 %v_acc3__c0_0, 0f00000000;
	mov.f32 %v_acc5__sum__c0_0, 0f00000000;
	mov.f32 %v_acc1__c0_0, 0fF149F2CA;
	mov.s32 %v_a1, 0;
LOOP_2:
	setp.ge.s32 %p2, %v_a1, 128;
	@%p2 bra LOOP_END_3;
	// Loop(axis=Axis(name=a2, extent=Dim(value=32)))
	mov.f32 %v_acc0__ar0, 0f00000000;
	mov.s32 %v_a2, 0;
LOOP_4:
	setp.ge.s32 %p3, %v_a2, 32;
	@%p3 bra LOOP_END_5;
	// Load(names=in2__ar0, input=q)
	mul.lo.s32 %r6, %v_a0_b, 1;
	mul.lo.s32 %r7, %v_a0_u, 1;
	add.s32 %r8, %r6, %r7;
	add.s32 %r9, %r8, 0;
	mad.lo.s32 %r10, %r9, 32, %v_a2;
	mul.wide.s32 %rd8, %r10, 4;
	add.s64 %rd9, %g_q, %rd8;
	ld.global.f32 %v_in2__ar0, [%rd9];
	// Load(names=in1__ar0, input=kt)
	mad.lo.s32 %r11, %v_a2, 128, %v_a1;
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
	// Load(names=in7__bc0, input=v)
	mul.lo.s32 %r12, %v_a5_b, 32;
	mul.lo.s32 %r13, %v_a5_u, 1;
	add.s32 %r14, %r12, %r13;
	add.s32 %r15, %r14, 0;
	mad.lo.s32 %r16, %v_a1, 32, %r15;
	mul.wide.s32 %rd12, %r16, 4;
	add.s64 %rd13, %g_v, %rd12;
	ld.global.f32 %v_in7__bc0, [%rd13];
	// Assign(name=v4__acc5__sum_sb__c0_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_v4__acc5__sum_sb__c0_0, %v_in7__bc0, %v_v4__beta__c0_0;
	// Accum(name=acc5__sum__c0_0, value=v4__acc5__sum_sb__c0_0)
	add.rn.f32 %v_acc5__sum__c0_0, %v_v4__acc5__sum_sa__c0_0, %v_v4__acc5__sum_sb__c0_0;
	// Accum(name=acc1__c0_0, value=v4__c0_0)
	max.f32 %v_acc1__c0_0, %v_acc1__c0_0, %v_v4__c0_0;
	add.s32 %v_a1, %v_a1, 1;
	bra LOOP_2;
LOOP_END_3:
	// Assign(name=v9__c0_0, op=ElementwiseImpl('reciprocal'))
	rcp.rn.f32 %v_v9__c0_0, %v_acc3__c0_0;
	// Assign(name=acc5__c0_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc5__c0_0, %v_acc5__sum__c0_0, %v_v9__c0_0;
	// Write(output=matmul_1, index=(((a0_b * 1) + (a0_u * 1)) + 0), (((a5_b * 32) + (a5_u * 1)) + 0))
	mul.lo.s32 %r17, %v_a0_b, 1;
	mul.lo.s32 %r18, %v_a0_u, 1;
	add.s32 %r19, %r17, %r18;
	add.s32 %r20, %r19, 0;
	mul.lo.s32 %r21, %v_a5_b, 32;
	mul.lo.s32 %r22, %v_a5_u, 1;
	add.s32 %r23, %r21, %r22;
	add.s32 %r24, %r23, 0;
	mad.lo.s32 %r25, %r20, 32, %r24;
	mul.wide.s32 %rd14, %r25, 4;
	add.s64 %rd15, %g_matmul_1, %rd14;
	st.global.f32 [%rd15], %v_acc5__c0_0;
TILE_END_1:
	ret;
}
