"""Stage 3: walk the statement tree, one handler per statement class.

The Walker dispatches each statement to its handler by class and carries the
context handlers share: the emitter, the kernel (its parameters), the
declared Smem arrays, the register fragments, and the values of the loops
being unrolled.  Any statement class without a handler fails loudly with
``NotImplementedError`` -- the reference's behaviour
(thompiler/walk.py:48-52 of the reference).

Two hooks let a tuned family reuse the generic handlers for the parts of a
kernel it does not rewrite: ``load_hook`` / ``write_hook`` may serve a Load
(or take a Write) themselves and return True, e.g. to read a row that the
family keeps resident in registers.
"""

from __future__ import annotations

from collections import Counter
from typing import Any, Callable

from thompiler import ir
from thompiler.emitter import Emitter
from thompiler.handlers.blocks import emit_cond, emit_loop, emit_strided_loop, emit_tile
from thompiler.handlers.blockscale import emit_block_scale_load
from thompiler.handlers.carry import StepBegin, StepEnd, emit_carry, emit_pre, emit_step_begin, emit_step_end
from thompiler.handlers.async_copy import (emit_mbarrier_arrive, emit_mbarrier_arrive_expect_tx, emit_mbarrier_init,
                                           emit_mbarrier_wait, emit_set_max_nreg, emit_tma_descriptor, emit_tma_load)
from thompiler.handlers.compute import emit_assign, emit_let, emit_load, emit_select, emit_write, emit_zero_prologue
from thompiler.handlers.cp_async import emit_cp_async_commit, emit_cp_async_copy, emit_cp_async_wait
from thompiler.handlers.fragments import (emit_fragment_apply, emit_fragment_promote, emit_fragment_repack,
                                         emit_fragment_row_reduce)
from thompiler.handlers.memory import emit_smem, emit_sync
from thompiler.handlers.mma import emit_ldmatrix_load, emit_mma_sync, emit_reg_fragment, emit_reg_store
from thompiler.handlers.wgmma import (emit_wgmma_commit, emit_wgmma_descriptor, emit_wgmma_fence,
                                      emit_wgmma_mma, emit_wgmma_wait)
from thompiler.handlers.reduce import emit_accum, emit_init, emit_tree_halve, emit_warp_shuffle
from thompiler.load import KernelInfo


class Walker:
    def __init__(self, em: Emitter, kernel: KernelInfo) -> None:
        self.em = em
        self.kernel = kernel
        self.smem: dict = {}
        self.fragments: dict = {}
        self.consts: dict[str, int] = {}
        self.wgmma = None                      # tensor-memory plan of Wgmma* accumulators
        self.load_hook: Callable[[Any, ir.Load], bool] | None = None
        self.write_hook: Callable[[Any, ir.Write], bool] | None = None
        self._writes = Counter(s.output for s in ir.walk_stmts(kernel.body) if isinstance(s, ir.Write))

    def body(self, stmts) -> None:
        for s in stmts:
            self.stmt(s)

    def stmt(self, s) -> None:
        handler = HANDLERS.get(type(s))
        if handler is None:
            kind = s.kind if isinstance(s, ir.Opaque) else type(s).__name__
            raise NotImplementedError(f"IR statement {kind} has no handler")
        handler(self, s)

    def smem_rewritten(self, bufs) -> bool:
        """Is one of these shared arrays written by more than one statement?"""
        return any(self._writes[b] > 1 for b in bufs)


HANDLERS: dict[type, Callable[[Walker, Any], None]] = {
    ir.Tile: emit_tile,
    ir.StridedLoop: emit_strided_loop,
    ir.Loop: emit_loop,
    ir.Cond: emit_cond,
    ir.Load: emit_load,
    ir.Assign: emit_assign,
    ir.Let: emit_let,
    ir.Write: emit_write,
    ir.Accum: emit_accum,
    ir.Init: emit_init,
    ir.WarpShuffle: emit_warp_shuffle,
    ir.TreeHalve: emit_tree_halve,
    ir.Smem: emit_smem,
    ir.BlockScaleLoad: emit_block_scale_load,
    ir.Sync: emit_sync,
    ir.CpAsyncCopy: emit_cp_async_copy,
    ir.CpAsyncCommit: emit_cp_async_commit,
    ir.CpAsyncWait: emit_cp_async_wait,
    ir.RegFragment: emit_reg_fragment,
    ir.LdmatrixLoad: emit_ldmatrix_load,
    ir.MmaSyncPtx: emit_mma_sync,
    ir.RegStore: emit_reg_store,
    ir.Select: emit_select,
    ir.ZeroPrologue: emit_zero_prologue,
    ir.TmaDescriptor: emit_tma_descriptor,
    ir.TmaLoad: emit_tma_load,
    ir.MbarrierInit: emit_mbarrier_init,
    ir.MbarrierArriveExpectTx: emit_mbarrier_arrive_expect_tx,
    ir.MbarrierArrive: emit_mbarrier_arrive,
    ir.MbarrierWait: emit_mbarrier_wait,
    ir.SetMaxNReg: emit_set_max_nreg,
    ir.WgmmaDescriptor: emit_wgmma_descriptor,
    ir.WgmmaFence: emit_wgmma_fence,
    ir.WgmmaMma: emit_wgmma_mma,
    ir.WgmmaCommit: emit_wgmma_commit,
    ir.WgmmaWait: emit_wgmma_wait,
    ir.FragmentPromote: emit_fragment_promote,
    ir.FragmentRowReduce: emit_fragment_row_reduce,
    ir.FragmentApply: emit_fragment_apply,
    ir.FragmentRepack: emit_fragment_repack,
    ir.Carry: emit_carry,
    ir.Pre: emit_pre,
    StepBegin: emit_step_begin,
    StepEnd: emit_step_end,
}
