"""Stage 2: module header, entry signature and parameter loads.

Every module targets Blackwell: ``.target sm_100a`` (the arch-specific
target that unlocks tcgen05 / TMEM) with PTX ISA 8.8, the version CUDA 12.9's
ptxas reads.  The entry takes the kernel's buffers as ``.param .u64``
pointers in meta.json's ``arg_order`` -- the same contract as the reference
(thompiler/prologue.py:20-39 of the reference) -- so a runner that knows
nothing about this backend still launches it.
"""

from __future__ import annotations

from thompiler.emitter import Emitter
from thompiler.load import KernelInfo

PTX_VERSION = "8.8"
PTX_TARGET = "sm_100a"


def param_symbol(buffer: str) -> str:
    return f"p_{buffer}"


def header() -> list[str]:
    return [f".version {PTX_VERSION}", f".target {PTX_TARGET}", ".address_size 64"]


def params(kernel: KernelInfo) -> list[str]:
    return [f".param .u64 {param_symbol(p.name)}" for p in kernel.params]


def emit_param_loads(em: Emitter, kernel: KernelInfo) -> None:
    """Each pointer param -> a global address in %g_<buffer>."""
    for p in kernel.params:
        raw = em.tmp("b64")
        em.ins(f"ld.param.u64 {raw}, [{param_symbol(p.name)}]")
        em.ins(f"cvta.to.global.u64 {em.buffer_reg(p.name)}, {raw}")
