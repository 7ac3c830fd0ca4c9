"""Synthetic problem packages at any size, in the shipped Kernel IR vocabulary.

emmy cannot run here, and the benchmark shapes (1M-element and 2^30-element
sums, [8192, 4096] row ops, 4096^3 matmuls, [8, 16, 2048, 128] attention)
have no shipped IR.  This module writes packages in the exact format of the
reference's problem set (tools/generate.py:74-205 of the reference): a
``<entry>.ir.json`` graph whose KernelOp body is the repr text of the
statement tree, and a ``meta.json`` launch contract with ``arg_order``,
``grid``, ``block``, ``smem_bytes``, ``zero_outputs``, per-arg records and
``rtol`` / ``atol``.

The schedules are emmy's own for these families, with the extents
substituted (the shipped r01 and r02 IRs differ only in ``Dim(1024)`` vs
``Dim(65536)``): one CTA of T threads striding a whole array for sums, one
row per CTA for row reductions.  An arg may carry an ``init`` record
(``{"dist": "uniform", "low", "high", "seed"}``) for non-normal inputs;
``seed`` args keep the runner's standard-normal meaning.
"""

from __future__ import annotations

import dataclasses
import json
from pathlib import Path

from thompiler import ir

F32T = ir.DataType("f32", "float32", 4)
F16T = ir.DataType("f16", "float16", 2)

# Constructor fields in the order emmy's repr writes them (the shipped IR).
EMMY_FIELDS = {
    "Tile": ("axes", "body", "block_threads", "aux_threads", "raster_axes", "raster_group", "raster_orient"),
    "Loop": ("axis", "body", "unroll", "seed"),
    "StridedLoop": ("axis", "start", "step", "body", "unroll", "end", "seed"),
    "Axis": ("name", "extent", "window"),
}


def to_repr(o) -> str:
    if isinstance(o, ir.DataType):
        return f"DataType(name={o.name!r}, np=dtype({o.np!r}), nbytes={o.nbytes})"
    if isinstance(o, ir.ElementwiseImpl):
        return f"ElementwiseImpl({o.name!r})"
    if isinstance(o, ir.Dim):
        return f"Dim({o.value!r})"
    if isinstance(o, tuple):
        inner = ", ".join(to_repr(x) for x in o)
        return f"({inner},)" if len(o) == 1 else f"({inner})"
    if ir.is_record(o) or dataclasses.is_dataclass(o):
        name = type(o).__name__
        names = EMMY_FIELDS.get(name) or list(ir.field_names(o))
        return f"{name}(" + ", ".join(f"{n}={to_repr(getattr(o, n))}" for n in names) + ")"
    return repr(o)


# ---- small builders ------------------------------------------------------------

def V(n):
    return ir.Var(n)


def L(v, dt="int"):
    return ir.Literal(v, dt)


def B(op, a, b):
    return ir.BinaryExpr(op, a, b)


def E(name):
    return ir.ElementwiseImpl(name)


def axis(name, n):
    return ir.Axis(name, ir.Dim(n), None)


def assign(name, op, *args, dt=F32T):
    return ir.Assign(name, E(op), tuple(args), dt)


def combine_block(states, partners, combine, T):
    """WarpShuffle + per-warp slots + barrier + TreeHalve, as emmy schedules it."""
    warps = T // 32
    out = [ir.WarpShuffle(tuple(states), tuple(partners), tuple(combine), 32, F32T)]
    out += [ir.Smem(f"{s}_smem", (warps,), "float", 0) for s in states]
    out.append(ir.Cond(B("==", V("lane"), L(0)),
                       tuple(ir.Write(f"{s}_smem", (V("warp"),), (s,), F32T, False, "NONE") for s in states), ()))
    out.append(ir.Sync(0, None, False))
    out.append(ir.TreeHalve(tuple(f"{s}_smem" for s in states), tuple(states), tuple(partners), tuple(combine),
                            warps, "warp", F32T, 0, None, None))
    return out


def add_combine(s):
    return (assign(s, "add", s, f"{s}__o", dt=None),)


def softmax_combine():
    """The online-softmax merge of two (max, sum) states (f02's combine_states)."""
    a, b, o, ob = "acc0", "acc1", "acc0__o", "acc1__o"

    def c(name, op, *args):
        return assign(name, op, *args, dt=None)

    return (c(f"{o}__gn", "maximum", a, o), c(f"{o}__dg", "subtract", a, f"{o}__gn"),
            c(f"{o}__alpha", "exp", f"{o}__dg"), c(f"{o}__dg_o", "subtract", o, f"{o}__gn"),
            c(f"{o}__beta", "exp", f"{o}__dg_o"), c(f"{o}__acc1_sa", "multiply", f"{o}__alpha", b),
            c(f"{o}__acc1_sb", "multiply", f"{o}__beta", ob),
            c(b, "add", f"{o}__acc1_sa", f"{o}__acc1_sb"), c(a, "copy", f"{o}__gn"))


# ---- packages ---------------------------------------------------------------------

def _graph(inputs: dict, consts: dict, out_name: str, out_shape, kernel_name: str, body, dtype="f32") -> dict:
    nodes = {}
    for n, (shape, dt) in inputs.items():
        nodes[n] = {"op": "InputOp", "op_fields": {}, "inputs": [], "outputs": [{"name": n, "shape": list(shape),
                                                                              "dtype": dt}]}
    for n, (value, dt) in consts.items():
        nodes[n] = {"op": "ConstantOp", "op_fields": {"name": n, "value": value}, "inputs": [],
                    "outputs": [{"name": n, "shape": [1], "dtype": dt}]}
    nodes[out_name] = {"op": "KernelOp",
                       "op_fields": {"body": [to_repr(body)], "name": kernel_name, "zero_delegated": [], "serial": []},
                       "inputs": list(consts) + list(inputs),
                       "outputs": [{"name": out_name, "shape": list(out_shape), "dtype": dtype}]}
    return {"inputs": list(inputs), "outputs": [out_name], "nodes": nodes}


def _write(outdir: Path, pid: str, code: str, entry: str, graph: dict, kmeta: dict, rtol: float, atol: float) -> Path:
    outdir = Path(outdir)
    outdir.mkdir(parents=True, exist_ok=True)
    (outdir / f"{entry}.ir.json").write_text(json.dumps(graph, indent=1))
    meta = {"id": pid, "code": code, "rtol": rtol, "atol": atol, "graph_inputs": graph["inputs"],
            "graph_outputs": graph["outputs"], "kernels": [dict(kmeta, entry=entry, final=True)]}
    (outdir / "meta.json").write_text(json.dumps(meta, indent=1))
    return outdir


def sum_package(outdir, n: int, kind: str = "sum", T: int = 128, init: dict | None = None) -> Path:
    """Full sum (r01 / r02) or mean (r03) of an f32 vector, one CTA of T threads."""
    co, a0 = "a0_co", "a0"
    l1 = ir.StridedLoop(axis(a0, n), V(co), L(T), (
        ir.Load(("in0",), "x", (V(a0),), F32T),
        ir.Accum("acc0", "in0", E("add"), F32T, (a0,), None)), False, None, True)
    if kind == "mean":
        tail_body = (ir.Load(("in1",), "mean_keepdim_count", (L(0),), F32T),
                     assign("v0", "divide", "acc0", "in1"), ir.Write("mean", (), ("v0",), F32T, False, "NONE"))
        out, consts = "mean", {"mean_keepdim_count": (float(n), "f32")}
    else:
        tail_body = (ir.Write("sum_1", (), ("acc0",), F32T, False, "NONE"),)
        out, consts = "sum_1", {}
    body = ir.Tile((axis(co, T),), (l1, *combine_block(["acc0"], ["acc0__o"], add_combine("acc0"), T),
                                    ir.Cond(B("==", V(co), L(0)), tail_body, ())), T, 0, None, None, "m")
    entry = "k_sum_1_reduce" if kind == "sum" else "k_mean_reduce"
    g = _graph({"x": ((n,), "f32")}, consts, out, (), entry, body)
    xrec = {"name": "x", "dtype": "f32", "shape": [n], "seed": 0}
    if init:
        xrec["init"] = init
    args = [xrec] + [{"name": c, "dtype": "f32", "shape": [1], "data": [v]} for c, (v, _) in consts.items()]
    args.append({"name": out, "dtype": "f32", "shape": [1], "output": True})
    kmeta = {"node": out, "arg_order": ["x"] + list(consts) + [out], "grid": [1, 1, 1], "block": [T, 1, 1],
             "smem_bytes": 0, "zero_outputs": [], "args": args}
    code = f"torch.rand({n}).sum()" if kind == "sum" else f"torch.rand({n}).mean()"
    return _write(outdir, f"synth_{kind}_{n}", code, entry, g, kmeta, 1e-5, 1e-6)


def pointwise_package(outdir, n: int, kind: str = "relu_mul", U: int = 4, T: int = 256) -> Path:
    """Pointwise f32 kernel over n elements in the schedule of the reference's p01 / p03
    problems: one thread per U consecutive elements (``a0 * U + u``), each element's Loads and
    Assigns in turn, one Write of the U results.  kind: "add" (x0 + x1, p01) or "relu_mul"
    (relu(x0) * x1, p03)."""
    if n % U or (n // U) % T:
        raise ValueError("pointwise_package needs n a multiple of U * T")
    a0 = "a0"
    body = []
    outs = []
    for u in range(U):
        idx = (B("+", B("*", V(a0), L(U)), L(u)),)
        body.append(ir.Load((f"in0__u{u}",), "x0", idx, F32T))
        if kind == "relu_mul":
            body.append(assign(f"v0__u{u}", "relu", f"in0__u{u}"))
            body.append(ir.Load((f"in1__u{u}",), "x1", idx, F32T))
            body.append(assign(f"v1__u{u}", "multiply", f"v0__u{u}", f"in1__u{u}"))
            outs.append(f"v1__u{u}")
        else:
            body.append(ir.Load((f"in1__u{u}",), "x1", idx, F32T))
            body.append(assign(f"v0__u{u}", "add", f"in0__u{u}", f"in1__u{u}"))
            outs.append(f"v0__u{u}")
    out = "mul" if kind == "relu_mul" else "add"
    body.append(ir.Write(out, (B("+", B("*", V(a0), L(U)), L(0)),), tuple(outs), F32T, False, "NONE"))
    tile = ir.Tile((axis(a0, n // U),), tuple(body), T, 0, None, None, "m")
    entry = f"k_{out}_pointwise"
    g = _graph({"x0": ((n,), "f32"), "x1": ((n,), "f32")}, {}, out, (n,), entry, tile)
    args = [{"name": "x0", "dtype": "f32", "shape": [n], "seed": 0},
            {"name": "x1", "dtype": "f32", "shape": [n], "seed": 1},
            {"name": out, "dtype": "f32", "shape": [n], "output": True}]
    kmeta = {"node": out, "arg_order": ["x0", "x1", out], "grid": [n // U // T, 1, 1], "block": [T, 1, 1],
             "smem_bytes": 0, "zero_outputs": [], "args": args}
    code = (f"torch.relu(torch.randn({n})) * torch.randn({n})" if kind == "relu_mul"
            else f"torch.randn({n}) + torch.randn({n})")
    return _write(outdir, f"synth_{kind}_{n}", code, entry, g, kmeta, 0, 0)


def matmul_package(outdir, M: int, N: int, K: int, b_layout: str = "col", out_dtype: str = "f32",
                   init: dict | None = None) -> Path:
    """C[M, N] = A[M, K] @ B with f16 inputs on the warp-level tensor cores (mma.sync m16n8k16),
    in the vocabulary of the reference's t01 / t02 problems.

    B is stored column-major (``b_layout="col"``: a [N, K] buffer, the ``b_trans`` ldmatrix path)
    or row-major (``"row"``: [K, N]).  Schedule: a 64 x 64 output tile per CTA of 4 warps, each
    warp a 16 x 64 strip (eight n8 accumulators); K in steps of 64 staged through two 64 x 64
    f16 slabs in shared memory with 16-byte cp.async copies and the B128 swizzle; per k16 step
    one ldmatrix.x4 of A, four paired ldmatrix.x4 of B and eight mma.sync."""
    if M % 64 or N % 64 or K % 64:
        raise ValueError("matmul_package needs M, N, K multiples of 64")
    col = b_layout == "col"
    F16 = F16T
    a0b, a1b, a0u, ln = "a0_b", "a1_b", "a0_u", "_lane"
    tid = B("+", B("*", V(a0u), L(32)), V(ln))            # thread index in the CTA (0..127)
    body = [ir.RegFragment("_a", "a", (16, 8, 16), F16, 1, None),
            ir.RegFragment("_b", "b", (16, 8, 16), F16, 8, None),
            ir.RegFragment("_c", "c", (16, 8, 16), F32T, 8, None),
            ir.Smem("_a_smem", (64, 64), "__half", 1024),
            ir.Smem("_b_smem", (64, 64), "__half", 1024)]
    copies = []
    for i in range(4):
        chunk = B("+", tid, L(128 * i))                      # 16-byte chunk 0..511 of a 64 x 64 slab
        row, c8 = B("/", chunk, L(8)), B("*", B("%", chunk, L(8)), L(8))
        copies.append(ir.CpAsyncCopy("_a_smem", (L(0), L(0)), "x0",
                                     (B("+", B("*", V(a0b), L(64)), row), B("+", V("_ks"), c8)), 16, "B128",
                                     (row, c8), None))
        if col:
            src = (B("+", B("*", V(a1b), L(64)), row), B("+", V("_ks"), c8))
        else:
            src = (B("+", V("_ks"), row), B("+", B("*", V(a1b), L(64)), c8))
        copies.append(ir.CpAsyncCopy("_b_smem", (L(0), L(0)), "x1", src, 16, "B128", (row, c8), None))
    inner = [ir.LdmatrixLoad("_a", "_a_smem", (B("*", V(a0u), L(16)), V("_kk")), "a", 64, "B128", True, None,
                             None, False, None, False, None, (), 0, "m16n8k16", None)]
    for j in range(4):
        idx = (L(16 * j), V("_kk")) if col else (V("_kk"), L(16 * j))
        inner.append(ir.LdmatrixLoad(f"_b[{2 * j}]", "_b_smem", idx, "b", 64, "B128", True, None, None, col,
                                     f"_b[{2 * j + 1}]", False, None, (), 0, "m16n8k16", None))
    inner.append(ir.Loop(axis("_r0", 8), (ir.MmaSyncPtx("_c[_r0]", "_a", "_b[_r0]", (16, 8, 16), "f16", "f32",
                                                       False, None, None),), True, False))
    ks = ir.StridedLoop(axis("_ks", K), L(0), L(64), (
        *copies, ir.CpAsyncCommit(), ir.CpAsyncWait(0), ir.Sync(0, None, False),
        ir.StridedLoop(axis("_kk", 64), L(0), L(16), tuple(inner), False, None, False),
        ir.Sync(0, None, False)), False, None, False)
    body.append(ks)
    out = "matmul"
    for j in range(8):
        body.append(ir.RegStore(out, (B("+", B("*", V(a0b), L(64)), B("*", V(a0u), L(16))),
                                      B("+", B("*", V(a1b), L(64)), L(8 * j))), f"_c[{j}]", (16, 8, 16), 0, None,
                                (), None, None, False, "m16n8k16", False, None, "NONE", None, None))
    tile = ir.Tile((axis(a0b, M // 64), axis(a1b, N // 64), axis(a0u, 4), axis(ln, 32)), tuple(body), 128, 0,
                   None, None, "m")
    entry = "k_matmul_f16"
    bshape = (N, K) if col else (K, N)
    g = _graph({"x0": ((M, K), "f16"), "x1": (bshape, "f16")}, {}, out, (M, N), entry, tile, dtype=out_dtype)
    args = [{"name": "x1", "dtype": "f16", "shape": list(bshape), "seed": 1},
            {"name": "x0", "dtype": "f16", "shape": [M, K], "seed": 0},
            {"name": out, "dtype": out_dtype, "shape": [M, N], "output": True}]
    if init:
        for a in args[:2]:
            a["init"] = dict(init, seed=a["seed"])
    kmeta = {"node": out, "arg_order": ["x1", "x0", out], "grid": [(M // 64) * (N // 64), 1, 1],
             "block": [128, 1, 1], "smem_bytes": 0, "zero_outputs": [], "args": args}
    bexpr = f"torch.randn({N}, {K}, dtype=torch.float16).T" if col else f"torch.randn({K}, {N}, dtype=torch.float16)"
    code = f"(torch.randn({M}, {K}, dtype=torch.float16) @ {bexpr})" + (".float()" if out_dtype == "f32" else "")
    return _write(outdir, f"synth_matmul_{M}x{N}x{K}_{b_layout}", code, entry, g, kmeta, 2e-2, 2e-3)


def attention_package(outdir, B: int, H: int, S: int, D: int, dtype: str = "f16", T: int = 128) -> Path:
    """softmax(Q K^T * scale) V over [B, H, S, D] tensors (non-causal), one output element per
    thread, in the vocabulary and schedule of the reference's a01 / a02 problems (online
    softmax over the key loop, the QK dot recomputed per output column, ``1/scale`` passed as
    the constant ``div_c1``).  f16 inputs are widened to f32 with ``copy`` Assigns and the f32
    result is narrowed to the output dtype -- the only f16 arithmetic the reference lowers."""
    half = dtype == "f16"
    DT = F16T if half else F32T
    b, h, a0, a5, a1, a2 = "a_b", "a_h", "a0", "a5", "a1", "a2"

    def ld(name, buf, idx):
        if not half:
            return [ir.Load((name,), buf, idx, F32T)]
        return [ir.Load((name + "h",), buf, idx, F16T), ir.Assign(name, E("copy"), (name + "h",), F32T)]

    inner = ir.Loop(axis(a2, D), (
        *ld("in2", "q", (V(b), V(h), V(a0), V(a2))), *ld("in1", "k", (V(b), V(h), V(a1), V(a2))),
        assign("v3", "multiply", "in1", "in2"),
        ir.Accum("acc0", "v3", E("add"), F32T, (a2,), None)), False, True)
    outer = ir.Loop(axis(a1, S), (
        inner, assign("v4", "multiply", "acc0", "v1"), ir.Let("one", L(1.0, "float"), F32T),
        assign("v4__gn", "maximum", "acc1", "v4"), assign("v4__dg", "subtract", "acc1", "v4__gn"),
        assign("v4__alpha", "exp", "v4__dg"), assign("v4__dg_o", "subtract", "v4", "v4__gn"),
        assign("v4__beta", "exp", "v4__dg_o"), assign("v4__acc3_sa", "multiply", "acc3", "v4__alpha"),
        assign("v4__acc3_sb", "multiply", "one", "v4__beta"),
        ir.Accum("acc3", "v4__acc3_sb", E("add"), F32T, (a1,), "v4__acc3_sa"),
        assign("v4__acc5__sum_sa", "multiply", "acc5__sum", "v4__alpha"),
        *ld("in7", "v", (V(b), V(h), V(a1), V(a5))),
        assign("v4__acc5__sum_sb", "multiply", "in7", "v4__beta"),
        ir.Accum("acc5__sum", "v4__acc5__sum_sb", E("add"), F32T, (a1,), "v4__acc5__sum_sa"),
        ir.Accum("acc1", "v4", E("maximum"), F32T, (a1,), None)), False, True)
    tail = [assign("v9", "reciprocal", "acc3"), assign("acc5", "multiply", "acc5__sum", "v9")]
    if half:
        tail.append(ir.Assign("out", E("copy"), ("acc5",), F16T))
    tail.append(ir.Write("attn", (V(b), V(h), V(a0), V(a5)), ("out" if half else "acc5",), DT, False, "NONE"))
    body = ir.Tile((axis(b, B), axis(h, H), axis(a0, S), axis(a5, D)), (
        ir.Load(("in0",), "div_c1", (L(0),), F32T), assign("v1", "reciprocal", "in0"), outer, *tail),
        T, 0, None, None, "m")
    shape = (B, H, S, D)
    entry = "k_attention"
    g = _graph({"q": (shape, dtype), "k": (shape, dtype), "v": (shape, dtype)},
               {"div_c1": (float(D) ** 0.5, "f32")}, "attn", shape, entry, body, dtype=dtype)
    args = [{"name": "div_c1", "dtype": "f32", "shape": [1], "data": [float(D) ** 0.5]},
            {"name": "q", "dtype": dtype, "shape": list(shape), "seed": 0},
            {"name": "k", "dtype": dtype, "shape": list(shape), "seed": 1},
            {"name": "v", "dtype": dtype, "shape": list(shape), "seed": 2},
            {"name": "attn", "dtype": dtype, "shape": list(shape), "output": True}]
    n = B * H * S * D
    kmeta = {"node": "attn", "arg_order": [a["name"] for a in args], "grid": [-(-n // T), 1, 1],
             "block": [T, 1, 1], "smem_bytes": 0, "zero_outputs": [], "args": args}
    code = (f"q, k, v = (torch.randn({B}, {H}, {S}, {D}, dtype=torch.float16) for _ in range(3)); "
            f"torch.softmax(q @ k.transpose(-1, -2) / {float(D) ** 0.5}, dim=-1) @ v")
    return _write(outdir, f"synth_attention_{B}x{H}x{S}x{D}", code, entry, g, kmeta, 2e-2, 2e-3)


def row_package(outdir, kind: str, rows: int, cols: int, T: int = 128, eps: float = 1e-6,
                init: dict | None = None, w_init: dict | None = None) -> Path:
    """Row softmax / RMSNorm / L2-normalise / row sum of x[rows, cols], one row per CTA (f01/f02/f03/r04)."""
    # axis and value names as emmy writes them for f01 / f02 / f03 / r04 (the softmax's second
    # pass walks its own axis a3; the L2-norm's first pass loads in0, the RMSNorm's in2)
    a0, co, a1 = "a0", "a1_co", "a1"
    a2 = "a3" if kind == "softmax" else "a2"
    x_at = lambda v: ir.Load(("in0",), "x", (V(a0), V(v)), F32T)  # noqa: E731
    consts: dict = {}
    inputs = {"x": ((rows, cols), "f32")}
    if kind == "softmax":
        l1 = ir.StridedLoop(axis(a1, cols), V(co), L(T), (
            ir.Let("one", L(1.0, "float"), F32T), x_at(a1),
            assign("in0__gn", "maximum", "acc0", "in0"), assign("in0__dg", "subtract", "acc0", "in0__gn"),
            assign("in0__alpha", "exp", "in0__dg"), assign("in0__dg_o", "subtract", "in0", "in0__gn"),
            assign("in0__beta", "exp", "in0__dg_o"), assign("in0__acc1_sa", "multiply", "acc1", "in0__alpha"),
            assign("in0__acc1_sb", "multiply", "in0__beta", "one"),
            ir.Accum("acc1", "in0__acc1_sb", E("add"), F32T, (a1,), "in0__acc1_sa"),
            ir.Accum("acc0", "in0", E("maximum"), F32T, (a1,), None)), False, None, True)
        states, partners, comb = ["acc0", "acc1"], ["acc0__o", "acc1__o"], softmax_combine()
        mid = [assign("v2", "reciprocal", "acc1")]
        tail = ir.StridedLoop(axis(a2, cols), V(co), L(T), (
            ir.Load(("in2",), "x", (V(a0), V(a2)), F32T), assign("v3", "subtract", "in2", "acc0"),
            assign("v4", "exp", "v3"), assign("v5", "multiply", "v2", "v4"),
            ir.Write("softmax", (V(a0), V(a2)), ("v5",), F32T, False, "NONE")), False, None, True)
        out, code = "softmax", f"torch.softmax(torch.randn({rows}, {cols}), dim=-1)"
    elif kind in ("rmsnorm", "l2norm", "rowsum"):
        sq = kind != "rowsum"
        sq_in = 2 if kind == "rmsnorm" else 0
        l1 = ir.StridedLoop(axis(a1, cols), V(co), L(T), (
            (ir.Load((f"in{sq_in}",), "x", (V(a0), V(a1)), F32T),
             assign(f"v{sq_in // 2}", "multiply", f"in{sq_in}", f"in{sq_in}"),
             ir.Accum("acc0", f"v{sq_in // 2}", E("add"), F32T, (a1,), None)) if sq else
            (x_at(a1), ir.Accum("acc0", "in0", E("add"), F32T, (a1,), None))), False, None, True)
        states, partners, comb = ["acc0"], ["acc0__o"], add_combine("acc0")
        if kind == "rmsnorm":
            consts = {"mean_count": (float(cols), "f32"), "add_c1": (float(eps), "f32")}
            inputs["w"] = ((cols,), "f32")
            mid = [ir.Load(("in1",), "mean_count", (L(0),), F32T), assign("v0", "reciprocal", "in1"),
                   assign("v2", "multiply", "acc0", "v0"), ir.Load(("in0",), "add_c1", (L(0),), F32T),
                   assign("v3", "add", "in0", "v2"), assign("v4", "sqrt", "v3"), assign("v5", "reciprocal", "v4")]
            tail = ir.StridedLoop(axis(a2, cols), V(co), L(T), (
                ir.Load(("in3",), "x", (V(a0), V(a2)), F32T), assign("v6", "multiply", "in3", "v5"),
                ir.Load(("in4",), "w", (V(a2),), F32T), assign("v7", "multiply", "in4", "v6"),
                ir.Write("mul_1", (V(a0), V(a2)), ("v7",), F32T, False, "NONE")), False, None, True)
            out = "mul_1"
            code = (f"x = torch.randn({rows}, {cols}); w = torch.rand({cols}) + 0.5; "
                    f"x / torch.sqrt((x * x).mean(-1, keepdim=True) + {eps}) * w")
        elif kind == "l2norm":
            mid = [assign("v1", "sqrt", "acc0"), assign("v2", "reciprocal", "v1")]
            tail = ir.StridedLoop(axis(a2, cols), V(co), L(T), (
                ir.Load(("in1",), "x", (V(a0), V(a2)), F32T), assign("v3", "multiply", "in1", "v2"),
                ir.Write("div", (V(a0), V(a2)), ("v3",), F32T, False, "NONE")), False, None, True)
            out = "div"
            code = f"x = torch.randn({rows}, {cols}); x / torch.sqrt((x * x).sum(-1, keepdim=True))"
        else:
            mid = []
            tail = ir.Cond(B("==", V(co), L(0)), (ir.Write("sum_1", (V(a0),), ("acc0",), F32T, False, "NONE"),), ())
            out = "sum_1"
            code = f"torch.randn({rows}, {cols}).sum(-1)"
    else:
        raise ValueError(f"row op {kind!r}")
    body = ir.Tile((axis(a0, rows), axis(co, T)),
                   (l1, *combine_block(states, partners, comb, T), *mid, tail), T, 0, None, None, "m")
    entry = {"softmax": "k_softmax_rows", "rmsnorm": "k_rmsnorm_rows", "l2norm": "k_l2norm_rows",
             "rowsum": "k_sum_rows"}[kind]
    out_shape = (rows,) if kind == "rowsum" else (rows, cols)
    g = _graph(inputs, consts, out, out_shape, entry, body)
    args = [{"name": c, "dtype": "f32", "shape": [1], "data": [v]} for c, (v, _) in consts.items()]
    xrec = {"name": "x", "dtype": "f32", "shape": [rows, cols], "seed": 0}
    if init:
        xrec["init"] = init
    args.append(xrec)
    if "w" in inputs:
        wrec = {"name": "w", "dtype": "f32", "shape": [cols], "seed": 1}
        if w_init:
            wrec["init"] = w_init
        args.append(wrec)
    args.append({"name": out, "dtype": "f32", "shape": list(out_shape), "output": True})
    kmeta = {"node": out, "arg_order": [a["name"] for a in args], "grid": [rows, 1, 1], "block": [T, 1, 1],
             "smem_bytes": 0, "zero_outputs": [], "args": args}
    return _write(outdir, f"synth_{kind}_{rows}x{cols}", code, entry, g, kmeta, 1e-5, 1e-6)
