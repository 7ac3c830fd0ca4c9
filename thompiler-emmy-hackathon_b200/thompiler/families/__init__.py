"""Hand-tuned sm_100a kernel families, chosen by recognising the IR's shape.

``recognise(kernel)`` returns an object with ``emit() -> str`` for a kernel
this backend has a tuned body for, else None (generic lowering).
"""

from __future__ import annotations

from thompiler.load import KernelInfo


def recognise(kernel: KernelInfo):
    """The families are tried in order; a family module is imported only when the kernel passes
    a cheap necessary condition of its recogniser (the statement kinds it requires), so a
    ``compile.py`` process loads the tuned code it can use and no more."""
    import importlib

    from thompiler import ir
    body = kernel.body
    tile = body[0] if len(body) == 1 and isinstance(body[0], ir.Tile) else None
    kinds = {type(s) for s in ir.walk_stmts(body)}
    mma = ir.MmaSyncPtx in kinds and ir.RegStore in kinds               # matmul: warp-level MMAs
    top_loop = tile is not None and any(isinstance(s, ir.Loop) for s in tile.body)   # attention
    flat = tile is not None and all(isinstance(s, (ir.Load, ir.Assign, ir.Let, ir.Write))
                                    for s in tile.body)                  # pointwise
    simt_mm = ir.CpAsyncCopy in kinds and ir.MmaSyncPtx not in kinds    # f32 matmul on the FMA pipes
    for name, maybe in (("strided", True), ("matmul_pair", mma), ("matmul", mma), ("matmul_f32", simt_mm),
                        ("attention", top_loop), ("pointwise", flat)):
        if maybe:
            k = importlib.import_module(f"thompiler.families.{name}").recognise(kernel)
            if k is not None:
                return k
    return None
