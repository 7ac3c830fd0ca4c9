"""The pipeline: KernelInfo -> PTX text.

``compile_kernel`` first asks the family recognisers (thompiler.families)
whether the kernel is one of the shapes this backend has a hand-tuned
sm_100a body for (full sums, row reductions with an elementwise pass,
pointwise maps, f16 tensor-core matmuls, attention).  A recognised kernel
is emitted by its family; anything else goes through the generic
statement-by-statement lowering.  Both produce one module with one entry
named after the IR kernel and taking meta.json's ``arg_order`` pointers, and
both are correct under meta.json's launch.  A family may add a tuned launch
record (``// @thompiler-launch {...}``) that this backend's runner honours.

``compile_kernel(kernel, tuned=False)`` (``compile.py --generic``) forces the
generic lowering.  Nothing here reads the environment.
"""

from __future__ import annotations

from thompiler import prologue
from thompiler.emitter import Emitter
from thompiler.load import KernelInfo
from thompiler.walk import Walker


def compile_generic(kernel: KernelInfo) -> str:
    from thompiler.handlers import wgmma
    em = Emitter()
    prologue.emit_param_loads(em, kernel)
    w = Walker(em, kernel)
    w.wgmma = wgmma.plan(kernel)
    if w.wgmma is not None:
        wgmma.prologue(w, w.wgmma)
    w.body(kernel.body)
    if w.wgmma is not None:
        wgmma.epilogue(w, w.wgmma)
    em.ins("ret")
    return em.render(prologue.header(), kernel.name, prologue.params(kernel))


def compile_kernel(kernel: KernelInfo, tuned: bool = True) -> str:
    if tuned:
        from thompiler import families
        family = families.recognise(kernel)
        if family is not None:
            return family.emit()
    return compile_generic(kernel)
