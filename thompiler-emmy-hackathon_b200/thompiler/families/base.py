"""Shared frame of the tuned families.

A tuned kernel is still one module with one entry named after the IR
kernel and taking meta.json's ``arg_order`` pointers.  Its body has two
paths:

  * the tuned path, taken when the launch matches what the family planned
    for (``guard``: e.g. the CTA size the IR's reduction tree assumes);
  * the generic lowering of the same IR, taken otherwise, so the module is
    correct under any launch -- in particular meta.json's.

Both paths live in one Walker (Smem arrays and IR value registers are
shared by name; only one path runs).  A family may record a tuned launch
(grid / block / shared memory / tensor maps) as the module's sidecar.
"""

from __future__ import annotations

from thompiler import prologue
from thompiler.emitter import Emitter
from thompiler.load import KernelInfo
from thompiler.walk import Walker


class TunedKernel:
    family = "tuned"

    def __init__(self, kernel: KernelInfo) -> None:
        self.k = kernel
        self.em = Emitter()
        self.w = Walker(self.em, kernel)

    # subclasses implement these -------------------------------------------
    def guard(self, generic_label: str) -> None:
        """Branch to ``generic_label`` when the launch does not suit the tuned path."""

    def emit_tuned(self) -> None:
        raise NotImplementedError

    def sidecar(self) -> dict | None:
        return None

    # ----------------------------------------------------------------------
    def emit(self) -> str:
        em, w = self.em, self.w
        em.note(f"family: {self.family}")
        prologue.emit_param_loads(em, self.k)
        generic = em.label("generic")
        self.exit = em.label("exit")
        self.guard(generic)
        self.emit_tuned()
        em.place(self.exit)
        em.ins("ret")
        em.place(generic)
        em.note("generic lowering of the same IR (any launch geometry)")
        w.load_hook = w.write_hook = None
        w.consts.clear()
        w.body(self.k.body)
        em.ins("ret")
        side = self.sidecar()
        if side is not None:
            # keep what the generic path's statements recorded (IR-level tensor maps)
            side = dict(em.sidecar or {}, **side, family=self.family)
        em.sidecar = side if side is not None else em.sidecar
        return em.render(prologue.header(), self.k.name, prologue.params(self.k))

    # helpers ----------------------------------------------------------------
    def special(self, reg: str) -> str:
        r = self.em.tmp("b32")
        self.em.ins(f"mov.u32 {r}, {reg}")
        return r
