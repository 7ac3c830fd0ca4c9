"""Stage 1: read a Kernel IR file and its launch contract.

``load(path)`` returns a ``KernelInfo`` with everything later stages need:
the entry name (the IR KernelOp's ``name``), the parameters in the order of
``meta.json``'s ``arg_order`` (the contract; emmy may reorder arguments, so
the IR node's input list is not used), each parameter's IR shape and dtype,
the statement tree, and the launch the contract prescribes (grid, block,
dynamic shared memory, zero_outputs).

Behaviour follows the reference loader (thompiler/load.py:40-91 of the
reference): exactly one KernelOp per file, the kernel found in meta.json by
its entry name, by-value scalars and non-static shapes rejected.  It also
records which parameters the body writes, so the read-only ones can be
loaded through the non-coherent cache.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from math import prod
from pathlib import Path

from thompiler import ir
from thompiler.lowering.types import Ty, dtype_of


@dataclass
class Param:
    name: str
    shape: tuple[int, ...]       # IR shape; () for a 0-d result
    ty: Ty
    written: bool                # the body stores into it (Write / RegStore)
    meta: dict = field(default_factory=dict)   # the meta.json arg record

    @property
    def nelems(self) -> int:
        return prod(self.shape) if self.shape else 1

    @property
    def nbytes(self) -> int:
        return self.nelems * self.ty.nbytes


@dataclass
class KernelInfo:
    name: str
    params: list[Param]
    body: tuple
    dynamic_smem_bytes: int
    grid: tuple[int, int, int] = (1, 1, 1)
    block: tuple[int, int, int] = (1, 1, 1)
    zero_outputs: tuple[str, ...] = ()
    meta: dict = field(default_factory=dict)   # the whole meta.json
    ir_path: Path | None = None

    def param(self, name: str) -> Param | None:
        return next((p for p in self.params if p.name == name), None)

    @property
    def threads_per_cta(self) -> int:
        return prod(self.block)

    @property
    def ctas(self) -> int:
        return prod(self.grid)


def written_buffers(body: tuple) -> set[str] | None:
    """Names the body stores into; None when an unknown statement might."""
    out: set[str] = set()
    for s in ir.walk_stmts(body):
        if isinstance(s, ir.Write):
            out.add(s.output)
        elif isinstance(s, ir.RegStore):
            out.add(s.dst_buffer)
        elif isinstance(s, ir.Opaque):
            return None
    return out


def load(ir_path: str | Path, meta: dict | None = None) -> KernelInfo:
    ir_path = Path(ir_path)
    graph = ir.Graph.from_dict(json.loads(ir_path.read_text()))
    if meta is None:
        meta = json.loads((ir_path.parent / "meta.json").read_text())
    return load_graph(graph, meta, ir_path)


def load_graph(graph: ir.Graph, meta: dict, ir_path: Path | None = None) -> KernelInfo:
    if len(graph.kernels) != 1:
        raise NotImplementedError(f"{ir_path}: expected one KernelOp, found {len(graph.kernels)}")
    kop = graph.kernels[0]
    kmeta = next((k for k in meta["kernels"] if k["entry"] == kop.name), None)
    if kmeta is None:
        raise ValueError(f"kernel {kop.name!r} is not listed in meta.json")
    args = {a["name"]: a for a in kmeta["args"]}
    written = written_buffers(kop.body)
    params = []
    for name in kmeta["arg_order"]:
        rec = args.get(name, {})
        if rec.get("scalar", False):
            raise NotImplementedError(f"by-value kernel argument {name!r} in meta.json")
        t = graph.buffer(name)
        if t is None:
            raise ValueError(f"arg {name!r} from arg_order has no buffer in the IR")
        if not all(isinstance(d, int) for d in t.shape):
            raise NotImplementedError(f"{name}: non-static shape {t.shape}")
        params.append(Param(name, tuple(int(d) for d in t.shape), dtype_of(t.dtype, f"param {name}"),
                            True if written is None else name in written, rec))

    def dims(v) -> tuple[int, int, int]:
        v = list(v) + [1, 1, 1]
        return (int(v[0]), int(v[1]), int(v[2]))

    return KernelInfo(
        name=kop.name, params=params, body=kop.body,
        dynamic_smem_bytes=int(kmeta.get("smem_bytes", 0)),
        grid=dims(kmeta.get("grid", [1])), block=dims(kmeta.get("block", [1])),
        zero_outputs=tuple(kmeta.get("zero_outputs", ())), meta=meta, ir_path=ir_path)
