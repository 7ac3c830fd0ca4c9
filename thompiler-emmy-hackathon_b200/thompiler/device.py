"""Compiled kernels launched on device-resident buffers.

``DeviceKernel(ir_path)`` compiles one IR file with this backend, JIT-loads
the module through the runner and plans its launch (the tuned launch a
family recorded, else meta.json's).  Calling it launches the kernel on
device pointers given by buffer name, in meta.json's ``arg_order``, on the
given CUDA stream -- the path for callers that keep data in HBM (PyTorch
tensors: pass ``t.data_ptr()``).  Tensor maps a tuned launch reads live in
the module as a few sets, one per set of buffers (``runner.TensorMaps``):
a call on buffers the module already has a set for uploads nothing, and
calls on different buffers may be in flight together on any streams.
"""

from __future__ import annotations

import json
import re
from pathlib import Path

from thompiler import runner
from thompiler.compiler import compile_kernel
from thompiler.load import load


class DeviceKernel:
    def __init__(self, ir_path: str | Path, device: int = 0, honour_meta: bool = False, tuned: bool = True,
                 ptx: str | None = None):
        ir_path = self.ir_path = Path(ir_path)
        meta = json.loads((ir_path.parent / "meta.json").read_text())
        self.info = load(ir_path, meta)
        self.kmeta = next(k for k in meta["kernels"] if k["entry"] == self.info.name)
        self.ptx = ptx if ptx is not None else compile_kernel(self.info, tuned=tuned)
        self.module = runner.load_module(self.ptx, device)
        self.fn = self.module.function(self.info.name)
        self.plan = runner.plan_launch(self.module, self.kmeta, honour_meta=honour_meta)
        self.arg_order = list(self.kmeta["arg_order"])
        self.tmaps = runner.TensorMaps(self.module, self.plan, self.arg_order) if self.plan.tmaps else None

    @property
    def family(self) -> str:
        side = self.module.sidecar or {}
        if side.get("family"):
            return side["family"]
        m = re.search(r"// family: ([\w-]+)", self.ptx)
        return m.group(1) if m else "generic"

    def __call__(self, ptrs: dict[str, int], stream: int = 0) -> None:
        """Launch on device pointers.  A tuned launch whose kernel waits for the previous grid
        before touching global data (``plan.pdl``) is issued as a programmatic dependent launch:
        its CTAs may start, and set up, while the stream's previous kernel finishes."""
        args = [ptrs[n] for n in self.arg_order]
        pdl = self.plan.pdl
        if self.tmaps is None:
            self.fn.launch(self.plan.grid, self.plan.block, self.plan.smem, args, stream, overlap=pdl)
            return
        k = self.tmaps.bind(ptrs, stream)
        self.fn.launch(self.plan.grid, self.plan.block, self.plan.smem, args, stream, overlap=pdl)
        self.tmaps.launched(k, stream)

    def error_word(self) -> int:
        """The module's error word (0: no bounded wait gave up, no guarded access was skipped)."""
        return runner.read_error_word(self.module, self.plan)

    def clear_error(self) -> None:
        """Zero the error word and the family's self-resetting counters (``runner.clear_error_word``)."""
        runner.clear_error_word(self.module, self.plan)

    def close(self) -> None:
        self.module.unload()
