.version 8.0
.target sm_89
.address_size 64

.shared .align 16 .b8 s__a_smem[512];
.shared .align 16 .b8 s__b_smem[1024];

.visible .entry k_matmul(
	.param .u64 param_x1,
	.param .u64 param_x0,
	.param .u64 param_matmul
)
{
	.reg .pred %p<6>;
	.reg .b32 %r<90>;
	.reg .b64 %rd<12>;
	.reg .b32 %v__gid, %v__a2_ks, %v_a0_b, %v_a1_b, %v_a0_u, %v_a1_u, %v__ks, %v__fa, %v__fb, %v__ki;
	.reg .b64 %g_x1, %g_x0, %g_matmul;
	.reg .f32 %v_acc0__c0_0, %v_acc0__c1_0, %v_in1__c0_0, %v_in0__c0_0, %v_acc0__v__c0_0, %v_in0__c1_0, %v_acc0__v__c1_0;

	ld.param.u64 %rd1, [param_x1];
	cvta.to.global.u64 %g_x1, %rd1;
	ld.param.u64 %rd2, [param_x0];
	cvta.to.global.u64 %g_x0, %rd2;
	ld.param.u64 %rd3, [param_matmul];
	cvta.to.global.u64 %g_matmul, %rd3;
	// Tile[_a2_ks, a0_b, a1_b, a0_u, a1_u] (N=131072)
	mov.u32 %r1, %ctaid.x;
	mov.u32 %r2, %ntid.x;
	mov.u32 %r3, %tid.x;
	mad.lo.u32 %v__gid, %r1, %r2, %r3;
	setp.ge.u32 %p1, %v__gid, 131072;
	@%p1 bra TILE_END_1;
	// START: decoding each axis index
	div.u32 %v__a2_ks, %v__gid, 4096;
	div.u32 %r4, %v__gid, 512;
	rem.u32 %v_a0_b, %r4, 8;
	div.u32 %r5, %v__gid, 256;
	rem.u32 %v_a1_b, %r5, 2;
	div.u32 %r6, %v__gid, 32;
	rem.u32 %v_a0_u, %r6, 8;
	rem.u32 %v_a1_u, %v__gid, 32;
	// END: decoding each axis index
	// Init(name=acc0__c0_0, identity=0.0)
	mov.f32 %v_acc0__c0_0, 0f00000000;
	// Init(name=acc0__c1_0, identity=0.0)
	mov.f32 %v_acc0__c1_0, 0f00000000;
	// Smem(name=_a_smem, extents=16, 8)
	// Smem(name=_b_smem, extents=8, 32)
	// StridedLoop(axis=Axis(name=_ks, extent=Dim(value=8)), start=0)
	mov.s32 %v__ks, 0;
LOOP_2:
	setp.ge.s32 %p2, %v__ks, 8;
	@%p2 bra LOOP_END_3;
	// StridedLoop(axis=Axis(name=_fa, extent=Dim(value=32)), start=((a0_u * 32) + a1_u))
	mul.lo.s32 %r7, %v_a0_u, 32;
	add.s32 %r8, %r7, %v_a1_u;
	mov.s32 %v__fa, %r8;
LOOP_4:
	setp.ge.s32 %p3, %v__fa, 32;
	@%p3 bra LOOP_END_5;
	// CpAsyncCopy(smem=_a_smem, smem_index=((_fa * 4) / 8), ((_fa * 4) % 8))
	mul.lo.s32 %r9, %v__fa, 4;
	div.s32 %r10, %r9, 8;
	mul.lo.s32 %r11, %v__fa, 4;
	rem.s32 %r12, %r11, 8;
	mad.lo.s32 %r13, %r10, 8, %r12;
	mov.u32 %r14, s__a_smem;
	mad.lo.s32 %r15, %r13, 4, %r14;
	mul.lo.s32 %r16, %v_a0_b, 16;
	mul.lo.s32 %r17, %v__fa, 4;
	div.s32 %r18, %r17, 8;
	add.s32 %r19, %r16, %r18;
	mul.lo.s32 %r20, %v__a2_ks, 8;
	mul.lo.s32 %r21, %v__fa, 4;
	rem.s32 %r22, %r21, 8;
	add.s32 %r23, %v__ks, %r22;
	add.s32 %r24, %r20, %r23;
	mad.lo.s32 %r25, %r19, 256, %r24;
	mul.wide.s32 %rd4, %r25, 4;
	add.s64 %rd5, %g_x0, %rd4;
	cp.async.cg.shared.global [%r15], [%rd5], 16;
	add.s32 %v__fa, %v__fa, 256;
	bra LOOP_4;
LOOP_END_5:
	// StridedLoop(axis=Axis(name=_fb, extent=Dim(value=64)), start=((a0_u * 32) + a1_u))
	mul.lo.s32 %r26, %v_a0_u, 32;
	add.s32 %r27, %r26, %v_a1_u;
	mov.s32 %v__fb, %r27;
LOOP_6:
	setp.ge.s32 %p4, %v__fb, 64;
	@%p4 bra LOOP_END_7;
	// CpAsyncCopy(smem=_b_smem, smem_index=((_fb * 4) / 32), ((_fb * 4) % 32))
	mul.lo.s32 %r28, %v__fb, 4;
	div.s32 %r29, %r28, 32;
	mul.lo.s32 %r30, %v__fb, 4;
	rem.s32 %r31, %r30, 32;
	mad.lo.s32 %r32, %r29, 32, %r31;
	mov.u32 %r33, s__b_smem;
	mad.lo.s32 %r34, %r32, 4, %r33;
	mul.lo.s32 %r35, %v__a2_ks, 8;
	mul.lo.s32 %r36, %v__fb, 4;
	div.s32 %r37, %r36, 32;
	add.s32 %r38, %v__ks, %r37;
	add.s32 %r39, %r35, %r38;
	mul.lo.s32 %r40, %v_a1_b, 32;
	mul.lo.s32 %r41, %v__fb, 4;
	rem.s32 %r42, %r41, 32;
	add.s32 %r43, %r40, %r42;
	mad.lo.s32 %r44, %r39, 64, %r43;
	mul.wide.s32 %rd6, %r44, 4;
	add.s64 %rd7, %g_x1, %rd6;
	cp.async.cg.shared.global [%r34], [%rd7], 16;
	add.s32 %v__fb, %v__fb, 256;
	bra LOOP_6;
LOOP_END_7:
	cp.async.commit_group;
	cp.async.wait_group 0;
	// Sync(barrier_id=0, count=None)
	bar.sync 0;
	// Loop(axis=Axis(name=_ki, extent=Dim(value=8)))
	mov.s32 %v__ki, 0;
LOOP_8:
	setp.ge.s32 %p5, %v__ki, 8;
	@%p5 bra LOOP_END_9;
	// Load(names=in1__c0_0, input=_b_smem)
	mul.lo.s32 %r45, %v_a1_b, 32;
	mul.lo.s32 %r46, %v_a1_u, 1;
	add.s32 %r47, %r45, %r46;
	add.s32 %r48, %r47, 0;
	mul.lo.s32 %r49, %v_a1_b, 32;
	sub.s32 %r50, %r48, %r49;
	mad.lo.s32 %r51, %v__ki, 32, %r50;
	mov.u32 %r52, s__b_smem;
	mad.lo.s32 %r53, %r51, 4, %r52;
	ld.shared.f32 %v_in1__c0_0, [%r53];
	// Load(names=in0__c0_0, input=_a_smem)
	mul.lo.s32 %r54, %v_a0_b, 16;
	mul.lo.s32 %r55, %v_a0_u, 2;
	add.s32 %r56, %r54, %r55;
	add.s32 %r57, %r56, 0;
	mul.lo.s32 %r58, %v_a0_b, 16;
	sub.s32 %r59, %r57, %r58;
	mad.lo.s32 %r60, %r59, 8, %v__ki;
	mov.u32 %r61, s__a_smem;
	mad.lo.s32 %r62, %r60, 4, %r61;
	ld.shared.f32 %v_in0__c0_0, [%r62];
	// Assign(name=acc0__v__c0_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__v__c0_0, %v_in1__c0_0, %v_in0__c0_0;
	// Accum(name=acc0__c0_0, value=acc0__v__c0_0)
	add.rn.f32 %v_acc0__c0_0, %v_acc0__c0_0, %v_acc0__v__c0_0;
	// Load(names=in0__c1_0, input=_a_smem)
	mul.lo.s32 %r63, %v_a0_b, 16;
	mul.lo.s32 %r64, %v_a0_u, 2;
	add.s32 %r65, %r63, %r64;
	add.s32 %r66, %r65, 1;
	mul.lo.s32 %r67, %v_a0_b, 16;
	sub.s32 %r68, %r66, %r67;
	mad.lo.s32 %r69, %r68, 8, %v__ki;
	mov.u32 %r70, s__a_smem;
	mad.lo.s32 %r71, %r69, 4, %r70;
	ld.shared.f32 %v_in0__c1_0, [%r71];
	// Assign(name=acc0__v__c1_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__v__c1_0, %v_in1__c0_0, %v_in0__c1_0;
	// Accum(name=acc0__c1_0, value=acc0__v__c1_0)
	add.rn.f32 %v_acc0__c1_0, %v_acc0__c1_0, %v_acc0__v__c1_0;
	add.s32 %v__ki, %v__ki, 1;
	bra LOOP_8;
LOOP_END_9:
	// Sync(barrier_id=0, count=None)
	bar.sync 0;
	add.s32 %v__ks, %v__ks, 8;
	bra LOOP_2;
LOOP_END_3:
	// Write(output=matmul, index=(((a0_b * 16) + (a0_u * 2)) + 0), (((a1_b * 32) + (a1_u * 1)) + 0))
	mul.lo.s32 %r72, %v_a0_b, 16;
	mul.lo.s32 %r73, %v_a0_u, 2;
	add.s32 %r74, %r72, %r73;
	add.s32 %r75, %r74, 0;
	mul.lo.s32 %r76, %v_a1_b, 32;
	mul.lo.s32 %r77, %v_a1_u, 1;
	add.s32 %r78, %r76, %r77;
	add.s32 %r79, %r78, 0;
	mad.lo.s32 %r80, %r75, 64, %r79;
	mul.wide.s32 %rd8, %r80, 4;
	add.s64 %rd9, %g_matmul, %rd8;
	red.global.add.f32 [%rd9], %v_acc0__c0_0;
	// Write(output=matmul, index=(((a0_b * 16) + (a0_u * 2)) + 1), (((a1_b * 32) + (a1_u * 1)) + 0))
	mul.lo.s32 %r81, %v_a0_b, 16;
	mul.lo.s32 %r82, %v_a0_u, 2;
	add.s32 %r83, %r81, %r82;
	add.s32 %r84, %r83, 1;
	mul.lo.s32 %r85, %v_a1_b, 32;
	mul.lo.s32 %r86, %v_a1_u, 1;
	add.s32 %r87, %r85, %r86;
	add.s32 %r88, %r87, 0;
	mad.lo.s32 %r89, %r84, 64, %r88;
	mul.wide.s32 %rd10, %r89, 4;
	add.s64 %rd11, %g_matmul, %rd10;
	red.global.add.f32 [%rd11], %v_acc0__c1_0;
TILE_END_1:
	ret;
}
