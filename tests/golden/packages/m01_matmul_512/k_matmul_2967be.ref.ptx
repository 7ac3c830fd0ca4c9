.version 8.0
.target sm_89
.address_size 64

.extern .shared .align 16 .b8 s_pool[];

.visible .entry k_matmul_2967be(
	.param .u64 param_x1,
	.param .u64 param_x0,
	.param .u64 param_matmul
)
{
	.reg .pred %p<7>;
	.reg .b32 %r<345>;
	.reg .b64 %rd<26>;
	.reg .b32 %v__gid, %v_a0_b, %v_a1_b, %v_a0_u, %v_a1_u, %v__ks, %v__ki;
	.reg .b64 %g_x1, %g_x0, %g_matmul;
	.reg .f32 %v_acc0__c0_0, %v_acc0__c0_1, %v_acc0__c1_0, %v_acc0__c1_1, %v_in1__c0_0, %v_in0__c0_0, %v_acc0__v__c0_0, %v_in1__c0_1, %v_acc0__v__c0_1, %v_in0__c1_0, %v_acc0__v__c1_0, %v_acc0__v__c1_1;

	ld.param.u64 %rd1, [param_x1];
	cvta.to.global.u64 %g_x1, %rd1;
	ld.param.u64 %rd2, [param_x0];
	cvta.to.global.u64 %g_x0, %rd2;
	ld.param.u64 %rd3, [param_matmul];
	cvta.to.global.u64 %g_matmul, %rd3;
	// Tile[a0_b, a1_b, a0_u, a1_u] (N=65536)
	mov.u32 %r1, %ctaid.x;
	mov.u32 %r2, %ntid.x;
	mov.u32 %r3, %tid.x;
	mad.lo.u32 %v__gid, %r1, %r2, %r3;
	setp.ge.u32 %p1, %v__gid, 65536;
	@%p1 bra TILE_END_1;
	// START: decoding each axis index
	div.u32 %v_a0_b, %v__gid, 4096;
	div.u32 %r4, %v__gid, 512;
	rem.u32 %v_a1_b, %r4, 8;
	div.u32 %r5, %v__gid, 32;
	rem.u32 %v_a0_u, %r5, 16;
	rem.u32 %v_a1_u, %v__gid, 32;
	// END: decoding each axis index
	// Init(name=acc0__c0_0, identity=0.0)
	mov.f32 %v_acc0__c0_0, 0f00000000;
	// Init(name=acc0__c0_1, identity=0.0)
	mov.f32 %v_acc0__c0_1, 0f00000000;
	// Init(name=acc0__c1_0, identity=0.0)
	mov.f32 %v_acc0__c1_0, 0f00000000;
	// Init(name=acc0__c1_1, identity=0.0)
	mov.f32 %v_acc0__c1_1, 0f00000000;
	// Smem(name=_a_smem, extents=96, 64)  (pool + 0)
	// Smem(name=_b_smem, extents=192, 64)  (pool + 24576)
	// CpAsyncCopy(smem=_a_smem, smem_index=0, 0)
	mul.lo.s32 %r6, %v_a0_u, 32;
	add.s32 %r7, %r6, %v_a1_u;
	mul.lo.s32 %r8, %r7, 4;
	div.s32 %r9, %r8, 64;
	mul.lo.s32 %r10, %r9, 64;
	mul.lo.s32 %r11, %v_a0_u, 32;
	add.s32 %r12, %r11, %v_a1_u;
	mul.lo.s32 %r13, %r12, 4;
	rem.s32 %r14, %r13, 64;
	add.s32 %r15, %r10, %r14;
	add.s32 %r16, 0, %r15;
	mov.u32 %r17, s_pool;
	mad.lo.s32 %r18, %r16, 4, %r17;
	mul.lo.s32 %r19, %v_a0_b, 32;
	mul.lo.s32 %r20, %v_a0_u, 32;
	add.s32 %r21, %r20, %v_a1_u;
	mul.lo.s32 %r22, %r21, 4;
	div.s32 %r23, %r22, 64;
	add.s32 %r24, %r23, 0;
	add.s32 %r25, %r19, %r24;
	mul.lo.s32 %r26, %v_a0_u, 32;
	add.s32 %r27, %r26, %v_a1_u;
	mul.lo.s32 %r28, %r27, 4;
	rem.s32 %r29, %r28, 64;
	add.s32 %r30, 0, %r29;
	mad.lo.s32 %r31, %r25, 512, %r30;
	mul.wide.s32 %rd4, %r31, 4;
	add.s64 %rd5, %g_x0, %rd4;
	cp.async.cg.shared.global [%r18], [%rd5], 16;
	// CpAsyncCopy(smem=_b_smem, smem_index=0, 0)
	mul.lo.s32 %r32, %v_a0_u, 32;
	add.s32 %r33, %r32, %v_a1_u;
	mul.lo.s32 %r34, %r33, 4;
	div.s32 %r35, %r34, 64;
	mul.lo.s32 %r36, %r35, 64;
	mul.lo.s32 %r37, %v_a0_u, 32;
	add.s32 %r38, %r37, %v_a1_u;
	mul.lo.s32 %r39, %r38, 4;
	rem.s32 %r40, %r39, 64;
	add.s32 %r41, %r36, %r40;
	add.s32 %r42, 0, %r41;
	mov.u32 %r43, s_pool;
	add.s32 %r44, %r43, 24576;
	mad.lo.s32 %r45, %r42, 4, %r44;
	mul.lo.s32 %r46, %v_a0_u, 32;
	add.s32 %r47, %r46, %v_a1_u;
	mul.lo.s32 %r48, %r47, 4;
	div.s32 %r49, %r48, 64;
	add.s32 %r50, %r49, 0;
	add.s32 %r51, 0, %r50;
	mul.lo.s32 %r52, %v_a1_b, 64;
	mul.lo.s32 %r53, %v_a0_u, 32;
	add.s32 %r54, %r53, %v_a1_u;
	mul.lo.s32 %r55, %r54, 4;
	rem.s32 %r56, %r55, 64;
	add.s32 %r57, %r52, %r56;
	mad.lo.s32 %r58, %r51, 512, %r57;
	mul.wide.s32 %rd6, %r58, 4;
	add.s64 %rd7, %g_x1, %rd6;
	cp.async.cg.shared.global [%r45], [%rd7], 16;
	// CpAsyncCopy(smem=_b_smem, smem_index=32, 0)
	mul.lo.s32 %r59, %v_a0_u, 32;
	add.s32 %r60, %r59, %v_a1_u;
	mul.lo.s32 %r61, %r60, 4;
	div.s32 %r62, %r61, 64;
	mul.lo.s32 %r63, %r62, 64;
	mul.lo.s32 %r64, %v_a0_u, 32;
	add.s32 %r65, %r64, %v_a1_u;
	mul.lo.s32 %r66, %r65, 4;
	rem.s32 %r67, %r66, 64;
	add.s32 %r68, %r63, %r67;
	add.s32 %r69, 2048, %r68;
	mov.u32 %r70, s_pool;
	add.s32 %r71, %r70, 24576;
	mad.lo.s32 %r72, %r69, 4, %r71;
	mul.lo.s32 %r73, %v_a0_u, 32;
	add.s32 %r74, %r73, %v_a1_u;
	mul.lo.s32 %r75, %r74, 4;
	div.s32 %r76, %r75, 64;
	add.s32 %r77, %r76, 32;
	add.s32 %r78, 0, %r77;
	mul.lo.s32 %r79, %v_a1_b, 64;
	mul.lo.s32 %r80, %v_a0_u, 32;
	add.s32 %r81, %r80, %v_a1_u;
	mul.lo.s32 %r82, %r81, 4;
	rem.s32 %r83, %r82, 64;
	add.s32 %r84, %r79, %r83;
	mad.lo.s32 %r85, %r78, 512, %r84;
	mul.wide.s32 %rd8, %r85, 4;
	add.s64 %rd9, %g_x1, %rd8;
	cp.async.cg.shared.global [%r72], [%rd9], 16;
	cp.async.commit_group;
	// CpAsyncCopy(smem=_a_smem, smem_index=((1 * 32) + 0), 0)
	mul.lo.s32 %r86, %v_a0_u, 32;
	add.s32 %r87, %r86, %v_a1_u;
	mul.lo.s32 %r88, %r87, 4;
	div.s32 %r89, %r88, 64;
	mul.lo.s32 %r90, %r89, 64;
	mul.lo.s32 %r91, %v_a0_u, 32;
	add.s32 %r92, %r91, %v_a1_u;
	mul.lo.s32 %r93, %r92, 4;
	rem.s32 %r94, %r93, 64;
	add.s32 %r95, %r90, %r94;
	add.s32 %r96, 2048, %r95;
	mov.u32 %r97, s_pool;
	mad.lo.s32 %r98, %r96, 4, %r97;
	mul.lo.s32 %r99, %v_a0_b, 32;
	mul.lo.s32 %r100, %v_a0_u, 32;
	add.s32 %r101, %r100, %v_a1_u;
	mul.lo.s32 %r102, %r101, 4;
	div.s32 %r103, %r102, 64;
	add.s32 %r104, %r103, 0;
	add.s32 %r105, %r99, %r104;
	mul.lo.s32 %r106, %v_a0_u, 32;
	add.s32 %r107, %r106, %v_a1_u;
	mul.lo.s32 %r108, %r107, 4;
	rem.s32 %r109, %r108, 64;
	add.s32 %r110, 64, %r109;
	mad.lo.s32 %r111, %r105, 512, %r110;
	mul.wide.s32 %rd10, %r111, 4;
	add.s64 %rd11, %g_x0, %rd10;
	cp.async.cg.shared.global [%r98], [%rd11], 16;
	// CpAsyncCopy(smem=_b_smem, smem_index=((1 * 64) + 0), 0)
	mul.lo.s32 %r112, %v_a0_u, 32;
	add.s32 %r113, %r112, %v_a1_u;
	mul.lo.s32 %r114, %r113, 4;
	div.s32 %r115, %r114, 64;
	mul.lo.s32 %r116, %r115, 64;
	mul.lo.s32 %r117, %v_a0_u, 32;
	add.s32 %r118, %r117, %v_a1_u;
	mul.lo.s32 %r119, %r118, 4;
	rem.s32 %r120, %r119, 64;
	add.s32 %r121, %r116, %r120;
	add.s32 %r122, 4096, %r121;
	mov.u32 %r123, s_pool;
	add.s32 %r124, %r123, 24576;
	mad.lo.s32 %r125, %r122, 4, %r124;
	mul.lo.s32 %r126, %v_a0_u, 32;
	add.s32 %r127, %r126, %v_a1_u;
	mul.lo.s32 %r128, %r127, 4;
	div.s32 %r129, %r128, 64;
	add.s32 %r130, %r129, 0;
	add.s32 %r131, 64, %r130;
	mul.lo.s32 %r132, %v_a1_b, 64;
	mul.lo.s32 %r133, %v_a0_u, 32;
	add.s32 %r134, %r133, %v_a1_u;
	mul.lo.s32 %r135, %r134, 4;
	rem.s32 %r136, %r135, 64;
	add.s32 %r137, %r132, %r136;
	mad.lo.s32 %r138, %r131, 512, %r137;
	mul.wide.s32 %rd12, %r138, 4;
	add.s64 %rd13, %g_x1, %rd12;
	cp.async.cg.shared.global [%r125], [%rd13], 16;
	// CpAsyncCopy(smem=_b_smem, smem_index=((1 * 64) + 32), 0)
	mul.lo.s32 %r139, %v_a0_u, 32;
	add.s32 %r140, %r139, %v_a1_u;
	mul.lo.s32 %r141, %r140, 4;
	div.s32 %r142, %r141, 64;
	mul.lo.s32 %r143, %r142, 64;
	mul.lo.s32 %r144, %v_a0_u, 32;
	add.s32 %r145, %r144, %v_a1_u;
	mul.lo.s32 %r146, %r145, 4;
	rem.s32 %r147, %r146, 64;
	add.s32 %r148, %r143, %r147;
	add.s32 %r149, 6144, %r148;
	mov.u32 %r150, s_pool;
	add.s32 %r151, %r150, 24576;
	mad.lo.s32 %r152, %r149, 4, %r151;
	mul.lo.s32 %r153, %v_a0_u, 32;
	add.s32 %r154, %r153, %v_a1_u;
	mul.lo.s32 %r155, %r154, 4;
	div.s32 %r156, %r155, 64;
	add.s32 %r157, %r156, 32;
	add.s32 %r158, 64, %r157;
	mul.lo.s32 %r159, %v_a1_b, 64;
	mul.lo.s32 %r160, %v_a0_u, 32;
	add.s32 %r161, %r160, %v_a1_u;
	mul.lo.s32 %r162, %r161, 4;
	rem.s32 %r163, %r162, 64;
	add.s32 %r164, %r159, %r163;
	mad.lo.s32 %r165, %r158, 512, %r164;
	mul.wide.s32 %rd14, %r165, 4;
	add.s64 %rd15, %g_x1, %rd14;
	cp.async.cg.shared.global [%r152], [%rd15], 16;
	cp.async.commit_group;
	// StridedLoop(axis=Axis(name=_ks, extent=Dim(value=512)), start=0)
	mov.s32 %v__ks, 0;
LOOP_2:
	setp.ge.s32 %p2, %v__ks, 512;
	@%p2 bra LOOP_END_3;
	// CpAsyncCopy(smem=_a_smem, smem_index=(((((_ks / 64) + 2) % 3) * 32) + 0), 0)
	div.s32 %r166, %v__ks, 64;
	add.s32 %r167, %r166, 2;
	rem.s32 %r168, %r167, 3;
	mul.lo.s32 %r169, %r168, 32;
	add.s32 %r170, %r169, 0;
	mad.lo.s32 %r171, %r170, 64, 0;
	mul.lo.s32 %r172, %v_a0_u, 32;
	add.s32 %r173, %r172, %v_a1_u;
	mul.lo.s32 %r174, %r173, 4;
	div.s32 %r175, %r174, 64;
	mul.lo.s32 %r176, %r175, 64;
	mul.lo.s32 %r177, %v_a0_u, 32;
	add.s32 %r178, %r177, %v_a1_u;
	mul.lo.s32 %r179, %r178, 4;
	rem.s32 %r180, %r179, 64;
	add.s32 %r181, %r176, %r180;
	add.s32 %r182, %r171, %r181;
	mov.u32 %r183, s_pool;
	mad.lo.s32 %r184, %r182, 4, %r183;
	mul.lo.s32 %r185, %v_a0_b, 32;
	mul.lo.s32 %r186, %v_a0_u, 32;
	add.s32 %r187, %r186, %v_a1_u;
	mul.lo.s32 %r188, %r187, 4;
	div.s32 %r189, %r188, 64;
	add.s32 %r190, %r189, 0;
	add.s32 %r191, %r185, %r190;
	add.s32 %r192, %v__ks, 128;
	setp.lt.s32 %p3, %r192, 512;
	add.s32 %r193, %v__ks, 128;
	selp.s32 %r194, %r193, 448, %p3;
	mul.lo.s32 %r195, %v_a0_u, 32;
	add.s32 %r196, %r195, %v_a1_u;
	mul.lo.s32 %r197, %r196, 4;
	rem.s32 %r198, %r197, 64;
	add.s32 %r199, %r194, %r198;
	mad.lo.s32 %r200, %r191, 512, %r199;
	mul.wide.s32 %rd16, %r200, 4;
	add.s64 %rd17, %g_x0, %rd16;
	cp.async.cg.shared.global [%r184], [%rd17], 16;
	// CpAsyncCopy(smem=_b_smem, smem_index=(((((_ks / 64) + 2) % 3) * 64) + 0), 0)
	div.s32 %r201, %v__ks, 64;
	add.s32 %r202, %r201, 2;
	rem.s32 %r203, %r202, 3;
	mul.lo.s32 %r204, %r203, 64;
	add.s32 %r205, %r204, 0;
	mad.lo.s32 %r206, %r205, 64, 0;
	mul.lo.s32 %r207, %v_a0_u, 32;
	add.s32 %r208, %r207, %v_a1_u;
	mul.lo.s32 %r209, %r208, 4;
	div.s32 %r210, %r209, 64;
	mul.lo.s32 %r211, %r210, 64;
	mul.lo.s32 %r212, %v_a0_u, 32;
	add.s32 %r213, %r212, %v_a1_u;
	mul.lo.s32 %r214, %r213, 4;
	rem.s32 %r215, %r214, 64;
	add.s32 %r216, %r211, %r215;
	add.s32 %r217, %r206, %r216;
	mov.u32 %r218, s_pool;
	add.s32 %r219, %r218, 24576;
	mad.lo.s32 %r220, %r217, 4, %r219;
	add.s32 %r221, %v__ks, 128;
	setp.lt.s32 %p4, %r221, 512;
	add.s32 %r222, %v__ks, 128;
	selp.s32 %r223, %r222, 448, %p4;
	mul.lo.s32 %r224, %v_a0_u, 32;
	add.s32 %r225, %r224, %v_a1_u;
	mul.lo.s32 %r226, %r225, 4;
	div.s32 %r227, %r226, 64;
	add.s32 %r228, %r227, 0;
	add.s32 %r229, %r223, %r228;
	mul.lo.s32 %r230, %v_a1_b, 64;
	mul.lo.s32 %r231, %v_a0_u, 32;
	add.s32 %r232, %r231, %v_a1_u;
	mul.lo.s32 %r233, %r232, 4;
	rem.s32 %r234, %r233, 64;
	add.s32 %r235, %r230, %r234;
	mad.lo.s32 %r236, %r229, 512, %r235;
	mul.wide.s32 %rd18, %r236, 4;
	add.s64 %rd19, %g_x1, %rd18;
	cp.async.cg.shared.global [%r220], [%rd19], 16;
	// CpAsyncCopy(smem=_b_smem, smem_index=(((((_ks / 64) + 2) % 3) * 64) + 32), 0)
	div.s32 %r237, %v__ks, 64;
	add.s32 %r238, %r237, 2;
	rem.s32 %r239, %r238, 3;
	mul.lo.s32 %r240, %r239, 64;
	add.s32 %r241, %r240, 32;
	mad.lo.s32 %r242, %r241, 64, 0;
	mul.lo.s32 %r243, %v_a0_u, 32;
	add.s32 %r244, %r243, %v_a1_u;
	mul.lo.s32 %r245, %r244, 4;
	div.s32 %r246, %r245, 64;
	mul.lo.s32 %r247, %r246, 64;
	mul.lo.s32 %r248, %v_a0_u, 32;
	add.s32 %r249, %r248, %v_a1_u;
	mul.lo.s32 %r250, %r249, 4;
	rem.s32 %r251, %r250, 64;
	add.s32 %r252, %r247, %r251;
	add.s32 %r253, %r242, %r252;
	mov.u32 %r254, s_pool;
	add.s32 %r255, %r254, 24576;
	mad.lo.s32 %r256, %r253, 4, %r255;
	add.s32 %r257, %v__ks, 128;
	setp.lt.s32 %p5, %r257, 512;
	add.s32 %r258, %v__ks, 128;
	selp.s32 %r259, %r258, 448, %p5;
	mul.lo.s32 %r260, %v_a0_u, 32;
	add.s32 %r261, %r260, %v_a1_u;
	mul.lo.s32 %r262, %r261, 4;
	div.s32 %r263, %r262, 64;
	add.s32 %r264, %r263, 32;
	add.s32 %r265, %r259, %r264;
	mul.lo.s32 %r266, %v_a1_b, 64;
	mul.lo.s32 %r267, %v_a0_u, 32;
	add.s32 %r268, %r267, %v_a1_u;
	mul.lo.s32 %r269, %r268, 4;
	rem.s32 %r270, %r269, 64;
	add.s32 %r271, %r266, %r270;
	mad.lo.s32 %r272, %r265, 512, %r271;
	mul.wide.s32 %rd20, %r272, 4;
	add.s64 %rd21, %g_x1, %rd20;
	cp.async.cg.shared.global [%r256], [%rd21], 16;
	cp.async.commit_group;
	cp.async.wait_group 2;
	// Sync(barrier_id=0, count=None)
	bar.sync 0;
	// Loop(axis=Axis(name=_ki, extent=Dim(value=64)))
	mov.s32 %v__ki, 0;
LOOP_4:
	setp.ge.s32 %p6, %v__ki, 64;
	@%p6 bra LOOP_END_5;
	// Load(names=in1__c0_0, input=_b_smem)
	div.s32 %r273, %v__ks, 64;
	rem.s32 %r274, %r273, 3;
	mul.lo.s32 %r275, %r274, 64;
	add.s32 %r276, %r275, %v__ki;
	mul.lo.s32 %r277, %v_a1_b, 64;
	mul.lo.s32 %r278, %v_a1_u, 2;
	add.s32 %r279, %r277, %r278;
	add.s32 %r280, %r279, 0;
	mul.lo.s32 %r281, %v_a1_b, 64;
	sub.s32 %r282, %r280, %r281;
	mad.lo.s32 %r283, %r276, 64, %r282;
	mov.u32 %r284, s_pool;
	add.s32 %r285, %r284, 24576;
	mad.lo.s32 %r286, %r283, 4, %r285;
	ld.shared.f32 %v_in1__c0_0, [%r286];
	// Load(names=in0__c0_0, input=_a_smem)
	div.s32 %r287, %v__ks, 64;
	rem.s32 %r288, %r287, 3;
	mul.lo.s32 %r289, %r288, 32;
	mul.lo.s32 %r290, %v_a0_b, 32;
	mul.lo.s32 %r291, %v_a0_u, 2;
	add.s32 %r292, %r290, %r291;
	add.s32 %r293, %r292, 0;
	mul.lo.s32 %r294, %v_a0_b, 32;
	sub.s32 %r295, %r293, %r294;
	add.s32 %r296, %r289, %r295;
	mad.lo.s32 %r297, %r296, 64, %v__ki;
	mov.u32 %r298, s_pool;
	mad.lo.s32 %r299, %r297, 4, %r298;
	ld.shared.f32 %v_in0__c0_0, [%r299];
	// Assign(name=acc0__v__c0_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__v__c0_0, %v_in1__c0_0, %v_in0__c0_0;
	// Accum(name=acc0__c0_0, value=acc0__v__c0_0)
	add.rn.f32 %v_acc0__c0_0, %v_acc0__c0_0, %v_acc0__v__c0_0;
	// Load(names=in1__c0_1, input=_b_smem)
	div.s32 %r300, %v__ks, 64;
	rem.s32 %r301, %r300, 3;
	mul.lo.s32 %r302, %r301, 64;
	add.s32 %r303, %r302, %v__ki;
	mul.lo.s32 %r304, %v_a1_b, 64;
	mul.lo.s32 %r305, %v_a1_u, 2;
	add.s32 %r306, %r304, %r305;
	add.s32 %r307, %r306, 1;
	mul.lo.s32 %r308, %v_a1_b, 64;
	sub.s32 %r309, %r307, %r308;
	mad.lo.s32 %r310, %r303, 64, %r309;
	mov.u32 %r311, s_pool;
	add.s32 %r312, %r311, 24576;
	mad.lo.s32 %r313, %r310, 4, %r312;
	ld.shared.f32 %v_in1__c0_1, [%r313];
	// Assign(name=acc0__v__c0_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__v__c0_1, %v_in1__c0_1, %v_in0__c0_0;
	// Accum(name=acc0__c0_1, value=acc0__v__c0_1)
	add.rn.f32 %v_acc0__c0_1, %v_acc0__c0_1, %v_acc0__v__c0_1;
	// Load(names=in0__c1_0, input=_a_smem)
	div.s32 %r314, %v__ks, 64;
	rem.s32 %r315, %r314, 3;
	mul.lo.s32 %r316, %r315, 32;
	mul.lo.s32 %r317, %v_a0_b, 32;
	mul.lo.s32 %r318, %v_a0_u, 2;
	add.s32 %r319, %r317, %r318;
	add.s32 %r320, %r319, 1;
	mul.lo.s32 %r321, %v_a0_b, 32;
	sub.s32 %r322, %r320, %r321;
	add.s32 %r323, %r316, %r322;
	mad.lo.s32 %r324, %r323, 64, %v__ki;
	mov.u32 %r325, s_pool;
	mad.lo.s32 %r326, %r324, 4, %r325;
	ld.shared.f32 %v_in0__c1_0, [%r326];
	// Assign(name=acc0__v__c1_0, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__v__c1_0, %v_in1__c0_0, %v_in0__c1_0;
	// Accum(name=acc0__c1_0, value=acc0__v__c1_0)
	add.rn.f32 %v_acc0__c1_0, %v_acc0__c1_0, %v_acc0__v__c1_0;
	// Assign(name=acc0__v__c1_1, op=ElementwiseImpl('multiply'))
	mul.rn.f32 %v_acc0__v__c1_1, %v_in1__c0_1, %v_in0__c1_0;
	// Accum(name=acc0__c1_1, value=acc0__v__c1_1)
	add.rn.f32 %v_acc0__c1_1, %v_acc0__c1_1, %v_acc0__v__c1_1;
	add.s32 %v__ki, %v__ki, 1;
	bra LOOP_4;
LOOP_END_5:
	// Sync(barrier_id=0, count=None)
	bar.sync 0;
	add.s32 %v__ks, %v__ks, 64;
	bra LOOP_2;
LOOP_END_3:
	// Write(output=matmul, index=(((a0_b * 32) + (a0_u * 2)) + 0), (((a1_b * 64) + (a1_u * 2)) + 0))
	mul.lo.s32 %r327, %v_a0_b, 32;
	mul.lo.s32 %r328, %v_a0_u, 2;
	add.s32 %r329, %r327, %r328;
	add.s32 %r330, %r329, 0;
	mul.lo.s32 %r331, %v_a1_b, 64;
	mul.lo.s32 %r332, %v_a1_u, 2;
	add.s32 %r333, %r331, %r332;
	add.s32 %r334, %r333, 0;
	mad.lo.s32 %r335, %r330, 512, %r334;
	mul.wide.s32 %rd22, %r335, 4;
	add.s64 %rd23, %g_matmul, %rd22;
	st.global.v2.f32 [%rd23], {%v_acc0__c0_0, %v_acc0__c0_1};
	// Write(output=matmul, index=(((a0_b * 32) + (a0_u * 2)) + 1), (((a1_b * 64) + (a1_u * 2)) + 0))
	mul.lo.s32 %r336, %v_a0_b, 32;
	mul.lo.s32 %r337, %v_a0_u, 2;
	add.s32 %r338, %r336, %r337;
	add.s32 %r339, %r338, 1;
	mul.lo.s32 %r340, %v_a1_b, 64;
	mul.lo.s32 %r341, %v_a1_u, 2;
	add.s32 %r342, %r340, %r341;
	add.s32 %r343, %r342, 0;
	mad.lo.s32 %r344, %r339, 512, %r343;
	mul.wide.s32 %rd24, %r344, 4;
	add.s64 %rd25, %g_matmul, %rd24;
	st.global.v2.f32 [%rd25], {%v_acc0__c1_0, %v_acc0__c1_1};
TILE_END_1:
	ret;
}
