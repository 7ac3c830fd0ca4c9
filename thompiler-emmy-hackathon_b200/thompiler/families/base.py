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
from thompiler.families.tuning import TUNING
from thompiler.load import KernelInfo
from thompiler.walk import Walker


class TunedKernel:
    family = "tuned"

    def __init__(self, kernel: KernelInfo) -> None:
        self.k = kernel
        self.em = Emitter()
        self.w = Walker(self.em, kernel)
        self.pdl = False            # set by pdl_wait: the tuned body waits for the previous grid

    # programmatic dependent launch ----------------------------------------------
    def pdl_trigger(self) -> None:
        """Let the stream's next kernel launch (its CTAs start and set up while this grid runs;
        it still waits for this grid's completion before touching global data)."""
        if TUNING.pdl:
            self.em.ins("griddepcontrol.launch_dependents")

    def pdl_wait(self) -> None:
        """Wait until the stream's previous grid has completed and its writes are visible: every
        thread of a tuned body runs this before its first access to global data, so the launch
        may be a programmatic dependent one (the launch record's ``pdl``)."""
        if TUNING.pdl:
            self.em.ins("griddepcontrol.wait")
            self.pdl = True

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
        if self.pdl:                 # the generic path too waits for the previous grid first
            em.ins("griddepcontrol.wait")
        w.load_hook = w.write_hook = None
        w.consts.clear()
        w.body(self.k.body)
        em.ins("ret")
        side = self.sidecar()
        if side is not None:
            # keep what the generic path's statements recorded (IR-level tensor maps)
            side = dict(em.sidecar or {}, **side, family=self.family)
        if self.pdl:
            # both paths wait for the previous grid before touching global data, so any launch of
            # the module (the tuned one or meta.json's) may overlap the stream's previous kernel
            side = dict(side if side is not None else (em.sidecar or {}), pdl=True)
        em.sidecar = side if side is not None else em.sidecar
        return em.render(prologue.header(), self.k.name, prologue.params(self.k))

    # helpers ----------------------------------------------------------------
    def special(self, reg: str) -> str:
        r = self.em.tmp("b32")
        self.em.ins(f"mov.u32 {r}, {reg}")
        return r
