"""Test packages in the IR vocabulary the reference compiler does not lower (the statements
marked * in its TASK.md: TMA copies, mbarriers, Select, ZeroPrologue, built-in and call
expressions).  No emmy-generated sample of these exists, so the packages are written here from
the IR reference's field lists, in the repr format of the shipped kernels."""

from __future__ import annotations

from pathlib import Path

from thompiler import ir
from thompiler.synth import B, E, F16T, F32T, L, V, _graph, _write, assign, axis

N, TILE, T = 256, 64, 256            # x[N, N] f32, one CTA per TILE x TILE tile, T threads


def tma_transpose_package(outdir: Path, swizzle=None) -> Path:
    """y = x^T: each CTA loads its 64 x 64 tile of x into shared memory with one TMA box copy
    (TmaDescriptor / MbarrierInit / MbarrierArriveExpectTx / TmaLoad / MbarrierWait), then
    each thread writes 16 elements of the transposed tile."""
    tiles = (N // TILE) ** 2
    per = TILE * TILE // T
    ty = B("/", V("t"), L(N // TILE))
    tx = B("%", V("t"), L(N // TILE))
    e = B("+", B("*", V("lane"), L(per)), V("j"))          # this thread's j-th element of the tile
    r, c = B("/", e, L(TILE)), B("%", e, L(TILE))
    body = (
        ir.Smem("buf", (TILE, TILE), "float", 1024),
        ir.Smem("bar", (1,), "uint64_t", 8),
        ir.TmaDescriptor("dx", "x", (N, N), (TILE, TILE), swizzle, F32T),
        ir.MbarrierInit("bar", L(1), L(0)),
        ir.Sync(0, None, False),
        ir.Cond(B("==", V("lane"), L(0)), (
            ir.MbarrierArriveExpectTx("bar", L(TILE * TILE * 4), L(0)),
            ir.TmaLoad("buf", (L(0), L(0)), "dx", (B("*", ty, L(TILE)), B("*", tx, L(TILE))), "bar", L(0)),
        ), ()),
        ir.MbarrierWait("bar", L(0), L(0)),
        ir.Loop(axis("j", per), (
            ir.Load(("v",), "buf", (r, c), F32T),
            ir.Write("y", (B("+", B("*", tx, L(TILE)), c), B("+", B("*", ty, L(TILE)), r)), ("v",), F32T,
                     False, "NONE"),
        ), False, False),
    )
    tile = ir.Tile((axis("t", tiles), axis("lane", T)), body, T, 0, None, None, "m")
    g = _graph({"x": ((N, N), "f32")}, {}, "y", (N, N), "k_tma_transpose", tile)
    args = [{"name": "x", "dtype": "f32", "shape": [N, N], "seed": 0},
            {"name": "y", "dtype": "f32", "shape": [N, N], "output": True}]
    kmeta = {"node": "y", "arg_order": ["x", "y"], "grid": [tiles, 1, 1], "block": [T, 1, 1], "smem_bytes": 0,
             "zero_outputs": [], "args": args}
    return _write(outdir, "sm90_tma_transpose", "x.t()", "k_tma_transpose", g, kmeta, 0, 0)


M = 4096                             # elements of the Select kernel


def select_package(outdir: Path) -> Path:
    """y[i] = x[min(i, 99)] if i < 100 else x[i]^2, with i read back from the built-ins, the flat
    offset of y from a FlatIndex, int casts; and ZeroPrologue clearing the first 64 words of z."""
    i = B("+", B("*", ir.Builtin("blockIdx.x"), L(T)), ir.Builtin("threadIdx.x"))
    body = (
        ir.ZeroPrologue("z", L(64)),
        ir.Let("i", ir.CastExpr("int", i), ir.DataType("i32", "int32", 4)),
        ir.Let("f", ir.FlatIndex("y", (V("a0"),)), ir.DataType("i32", "int32", 4)),
        ir.Load(("lo",), "x", (ir.FuncCallExpr("min", (V("i"), L(99))),), F32T),
        ir.Load(("v",), "x", (V("a0"),), F32T),
        assign("sq", "multiply", "v", "v"),
        ir.Select("s", (ir.Branch("lo", B("<", V("i"), L(100))), ir.Branch("sq", None))),
        ir.Write("y", (V("f"),), ("s",), F32T, False, "NONE"),
    )
    tile = ir.Tile((axis("a0", M),), body, T, 0, None, None, "m")
    g = _graph({"x": ((M,), "f32"), "z": ((M,), "f32")}, {}, "y", (M,), "k_select", tile)
    args = [{"name": "x", "dtype": "f32", "shape": [M], "seed": 0},
            {"name": "z", "dtype": "f32", "shape": [M], "seed": 1},
            {"name": "y", "dtype": "f32", "shape": [M], "output": True}]
    kmeta = {"node": "y", "arg_order": ["x", "z", "y"], "grid": [M // T, 1, 1], "block": [T, 1, 1],
             "smem_bytes": 0, "zero_outputs": [], "args": args}
    return _write(outdir, "sm90_select", "select", "k_select", g, kmeta, 0, 0)


def stuck_wait_package(outdir: Path, n: int = 64) -> Path:
    """y = x after an MbarrierWait that nothing completes (count 1, no arrival): the bounded wait
    must give up, record its bit in the error word and let the kernel finish."""
    body = (
        ir.Smem("bar", (1,), "uint64_t", 8),
        ir.MbarrierInit("bar", L(1), L(0)),
        ir.Sync(0, None, False),
        ir.MbarrierWait("bar", L(0), L(0)),
        ir.Load(("v",), "x", (V("a0"),), F32T),
        ir.Write("y", (V("a0"),), ("v",), F32T, False, "NONE"),
    )
    tile = ir.Tile((axis("a0", n),), body, n, 0, None, None, "m")
    g = _graph({"x": ((n,), "f32")}, {}, "y", (n,), "k_stuck_wait", tile)
    args = [{"name": "x", "dtype": "f32", "shape": [n], "seed": 0},
            {"name": "y", "dtype": "f32", "shape": [n], "output": True}]
    kmeta = {"node": "y", "arg_order": ["x", "y"], "grid": [1, 1, 1], "block": [n, 1, 1], "smem_bytes": 0,
             "zero_outputs": [], "args": args}
    return _write(outdir, "sm90_stuck_wait", "x", "k_stuck_wait", g, kmeta, 0, 0)


ROWS, COLS = 256, 24


def scan_package(outdir: Path) -> Path:
    """Carried state (Carry, Pre), one thread per row of x[ROWS, COLS]:
    y[r, j] = x[r, 0] + ... + x[r, j] and t[r] = the row total (read after the loop), and f[r] =
    the (COLS + 1)-th Fibonacci number from a two-cell carrier whose step reads cell 0 after
    setting it (a read within a step sees the previous state)."""
    f32 = F32T
    step = (
        ir.Pre("prev", "acc", ()),
        ir.Load(("v",), "x", (V("r"), V("j")), f32),
        assign("s", "add", "prev", "v"),
        ir.Carry("acc", "s", (), L(0.0, "float"), f32),
        ir.Write("y", (V("r"), V("j")), ("s",), f32, False, "NONE"),
        ir.Pre("fb", "fib", (L(1),)),
        ir.Carry("fib", "fb", (L(0),), L(0.0, "float"), f32),
        ir.Pre("fa", "fib", (L(0),)),                    # the previous step's cell 0, not fb
        assign("fs", "add", "fa", "fb"),
        ir.Carry("fib", "fs", (L(1),), L(1.0, "float"), f32),
    )
    body = (
        ir.Loop(axis("j", COLS), step, False, False),
        ir.Pre("tot", "acc", ()),
        ir.Write("t", (V("r"),), ("tot",), f32, False, "NONE"),
        ir.Pre("fn", "fib", (L(1),)),
        ir.Write("f", (V("r"),), ("fn",), f32, False, "NONE"),
    )
    tile = ir.Tile((axis("r", ROWS),), body, 128, 0, None, None, "m")
    g = _graph({"x": ((ROWS, COLS), "f32")}, {}, "y", (ROWS, COLS), "k_scan", tile)
    g["nodes"]["y"]["outputs"] += [{"name": "t", "shape": [ROWS], "dtype": "f32"},
                                   {"name": "f", "shape": [ROWS], "dtype": "f32"}]
    g["outputs"] = ["y", "t", "f"]
    args = [{"name": "x", "dtype": "f32", "shape": [ROWS, COLS], "seed": 0},
            {"name": "y", "dtype": "f32", "shape": [ROWS, COLS], "output": True},
            {"name": "t", "dtype": "f32", "shape": [ROWS], "output": True},
            {"name": "f", "dtype": "f32", "shape": [ROWS], "output": True}]
    kmeta = {"node": "y", "arg_order": ["x", "y", "t", "f"], "grid": [ROWS // 128, 1, 1], "block": [128, 1, 1],
             "smem_bytes": 0, "zero_outputs": [], "args": args}
    return _write(outdir, "sm90_scan", "x.cumsum(-1)", "k_scan", g, kmeta, 1e-5, 1e-5)


def wgmma_gemm_package(outdir: Path, M: int, N: int, K: int, BN: int = 128, n_wg: int = 1,
                       trans_b: bool = False, tail_overwrite: bool = False, out_scale: float | None = None) -> Path:
    """y[M, N] = x0[M, K] @ B (f16 in, f32 out) in the warpgroup vocabulary of sm_90 kernels:
    WgmmaDescriptor / WgmmaFence / WgmmaMma / WgmmaCommit / WgmmaWait with an m64 accumulator
    RegFragment and a RegStore of it, the operands staged by TMA with the 128-byte swizzle.

    B is x1[N, K] (K-major) or, with ``trans_b``, x1[K, N] (MN-major, loaded as 64 x 64 boxes).
    A CTA of ``n_wg`` warpgroups computes a (64 n_wg) x BN tile, warpgroup g its rows
    64g..64g+63; K runs in blocks of 64, four k16 MMAs per block, the first of them
    overwriting the accumulator (``scale_d`` false at kb = kk = 0).  With ``tail_overwrite``
    one more MMA after the loop, with ``scale_d`` 0, replaces the result by the product of
    the last 16 columns of K alone: y = x0[:, K-16:] @ B[K-16:, :].  With ``out_scale`` y is f16,
    out_scale * (x0 @ B) through a RegStore epilogue Lambda."""
    if M % (64 * n_wg) or N % BN or K % 64 or BN % 64:
        raise ValueError("wgmma_gemm_package: M, N, K and BN must be whole tiles")
    F16 = F16T
    rows = 64 * n_wg
    t, wg = V("t"), B("/", V("t"), L(128))
    if trans_b:
        bshape, b_s = (K, N), ir.Smem("b_s", (BN // 64, 64, 64), "__half", 1024)
        db = ir.TmaDescriptor("db", "x1", bshape, (64, 64), "B128", F16)
        b_loads = tuple(ir.TmaLoad("b_s", (L(j), L(0), L(0)), "db", (V("kb"), B("+", B("*", V("tn"), L(BN)), L(64 * j))),
                                   "bar", L(0)) for j in range(BN // 64))
    else:
        bshape, b_s = (N, K), ir.Smem("b_s", (BN, 64), "__half", 1024)
        db = ir.TmaDescriptor("db", "x1", bshape, (BN, 64), "B128", F16)
        b_loads = (ir.TmaLoad("b_s", (L(0), L(0)), "db", (B("*", V("tn"), L(BN)), V("kb")), "bar", L(0)),)

    def descs(k0):
        """Descriptors of the k16 slice starting at column k0 of the staged 64-wide K block."""
        a = ir.WgmmaDescriptor("ad", "a_s", (B("*", wg, L(64)), k0), "B128", L(16), L(1024))
        if trans_b:      # MN-major: the slice is rows k0..k0+15 of each 64 x 64 box, boxes 8 KiB apart
            b = ir.WgmmaDescriptor("bd", "b_s", (L(0), k0, L(0)), "B128", L(8192), L(1024))
        else:
            b = ir.WgmmaDescriptor("bd", "b_s", (L(0), k0), "B128", L(16), L(1024))
        return a, b

    def mma(scale):
        return ir.WgmmaMma(("acc",), "bd", (64, BN, 16), "f16", "ad", None, scale, False, trans_b)

    kstep = (*descs(B("*", V("kk"), L(16))), ir.WgmmaFence(),
             mma(B("||", B("!=", V("kb"), L(0)), B("!=", V("kk"), L(0)))))
    body = [
        ir.Smem("a_s", (rows, 64), "__half", 1024), b_s,
        ir.Smem("bar", (1,), "uint64_t", 8),
        ir.TmaDescriptor("da", "x0", (M, K), (rows, 64), "B128", F16), db,
        ir.MbarrierInit("bar", L(1), L(0)),
        ir.Sync(0, None, False),
        ir.RegFragment("acc", "c", (64, BN, 16), F32T, 1, None),
        ir.StridedLoop(axis("kb", K), L(0), L(64), (
            ir.Cond(B("==", t, L(0)), (
                ir.MbarrierArriveExpectTx("bar", L((rows + BN) * 64 * 2), L(0)),
                ir.TmaLoad("a_s", (L(0), L(0)), "da", (B("*", V("tm"), L(rows)), V("kb")), "bar", L(0)),
                *b_loads), ()),
            ir.MbarrierWait("bar", B("/", V("kb"), L(64)), L(0)),
            ir.Loop(axis("kk", 4), kstep, True, False),
            ir.WgmmaCommit(),
            ir.WgmmaWait(L(0)),
            ir.Sync(0, None, False)), False, None, False),
    ]
    if tail_overwrite:
        body += [*descs(L(3 * 16)), ir.WgmmaFence(), mma(L(0)), ir.WgmmaCommit(), ir.WgmmaWait(L(0))]
    epilogue = None
    if out_scale is not None:
        epilogue = ir.Lambda(("v",), (ir.Let("sc", L(float(out_scale), "float"), F32T),
                                      assign("o", "multiply", "v", "sc")), ("o",))
    body.append(ir.RegStore("y", (B("+", B("*", V("tm"), L(rows)), B("*", wg, L(64))), B("*", V("tn"), L(BN))),
                            "acc", (64, BN, 16), 0, epilogue, (), None, None, False, "m64nNk16", False, None, "NONE",
                            None, None))
    out_dtype = "f32" if out_scale is None else "f16"
    tile = ir.Tile((axis("tm", M // rows), axis("tn", N // BN), axis("t", 128 * n_wg)), tuple(body), 128 * n_wg, 0,
                   None, None, "m")
    entry = "k_wgmma_gemm"
    g = _graph({"x0": ((M, K), "f16"), "x1": (bshape, "f16")}, {}, "y", (M, N), entry, tile, out_dtype)
    args = [{"name": "x0", "dtype": "f16", "shape": [M, K], "seed": 0},
            {"name": "x1", "dtype": "f16", "shape": list(bshape), "seed": 1},
            {"name": "y", "dtype": out_dtype, "shape": [M, N], "output": True}]
    kmeta = {"node": "y", "arg_order": ["x0", "x1", "y"], "grid": [(M // rows) * (N // BN), 1, 1],
             "block": [128 * n_wg, 1, 1], "smem_bytes": 0, "zero_outputs": [], "args": args}
    return _write(outdir, "sm90_wgmma_gemm", "x0 @ x1", entry, g, kmeta, 1e-3, 1e-3)


def _copy_tile(smem: str, src: str, row0, tid):
    """Four 16-byte cp.async copies per thread of 128: a 64 x 64 f16 tile of ``src`` (rows row0..)
    into ``smem`` with the 128-byte swizzle."""
    out = []
    for i in range(4):
        chunk = B("+", tid, L(128 * i))
        row, c8 = B("/", chunk, L(8)), B("*", B("%", chunk, L(8)), L(8))
        out.append(ir.CpAsyncCopy(smem, (L(0), L(0)), src, (B("+", row0, row), c8), 16, "B128", (row, c8), None))
    return out


def _ldm(frag, smem, idx, role, b_trans=False, pair=None):
    return ir.LdmatrixLoad(frag, smem, idx, role, 64, "B128", True, None, None, b_trans, pair, False, None, (), 0,
                           "m16n8k16", None)


def _unrolled(var, n, body):
    return ir.Loop(axis(var, n), tuple(body), True, False)


FRAGMENT_ATTENTION_EXTRAS = ("causal", "causal_pred", "bias", "bias_cols", "bias_index")


def fragment_attention_package(outdir: Path, S: int = 256, D: int = 64, extra: str | None = None) -> Path:
    """o = softmax(q k^T / sqrt(D)) v for one head (q, k, v f16 [S, D], o f32), written with the
    register-fragment statements on mma.sync m16n8k16: per warp a 16-query strip, keys in blocks
    of 64 staged by cp.async; FragmentApply scales the scores (a scalar argument, in place),
    subtracts the running row maximum (a row argument) with an exp ``post``, rescales the
    output strip and divides it by the row sums at the end; FragmentRowReduce gives the block's
    row maxima and sums; FragmentRepack turns the probabilities into the A fragments of P V.

    ``extra`` adds one FragmentApply whose argument is a function of each score's (query, key)
    coordinates (row_base = the warp's first query, col_base = the fragment's first key):
      causal       -- a ``mask`` Lambda: add 0 where key <= query, -1e30 elsewhere (scores);
      causal_pred  -- a ``mask`` predicate key <= query (1 / 0) multiplying the probabilities;
      bias         -- a ``bias`` from the f32 [S, S] buffer ``bias`` at (query, key), added;
      bias_cols    -- a ``bias`` from the f32 [S] buffer ``kbias`` at (key), added;
      bias_index   -- the same [S, S] bias through an explicit (buffer, (row, col)) index."""
    if S % 64 or D != 64:
        raise ValueError("fragment_attention_package: S a multiple of 64, D = 64")
    if extra not in (None, *FRAGMENT_ATTENTION_EXTRAS):
        raise ValueError(f"fragment_attention_package: extra {extra!r}")
    F16 = F16T
    tid = B("+", B("*", V("_w"), L(32)), V("_lane"))
    sfr = tuple(f"s[{n}]" for n in range(8))
    frags = [ir.RegFragment("qa", "a", (16, 8, 16), F16, 4, None), ir.RegFragment("kb", "b", (16, 8, 16), F16, 8, None),
             ir.RegFragment("s", "c", (16, 8, 16), F32T, 8, None), ir.RegFragment("pa", "a", (16, 8, 16), F16, 4, None),
             ir.RegFragment("vb", "b", (16, 8, 16), F16, 8, None), ir.RegFragment("o", "c", (16, 8, 16), F32T, 8, None)]
    smem = [ir.Smem(n, (64, 64), "__half", 1024) for n in ("q_s", "k_s", "v_s")]
    load_q = [*_copy_tile("q_s", "q", B("*", V("qb"), L(64)), tid), ir.CpAsyncCommit(), ir.CpAsyncWait(0),
              ir.Sync(0, None, False),
              _unrolled("_kq", 4, [_ldm("qa[_kq]", "q_s", (B("*", V("_w"), L(16)), B("*", V("_kq"), L(16))), "a")])]
    init = [ir.Let(n, L(v, "float"), F32T) for n, v in (("m_t", -1e30), ("m_b", -1e30), ("l_t", 0.0), ("l_b", 0.0))]
    row = ("frag", "row")
    block = [
        *_copy_tile("k_s", "k", V("_kv"), tid), *_copy_tile("v_s", "v", V("_kv"), tid),
        ir.CpAsyncCommit(), ir.CpAsyncWait(0), ir.Sync(0, None, False),
        _unrolled("_z", 8, [ir.FragmentApply("s[_z]", E("copy"), (L(0.0, "float"),), ("scalar",), False, None, None,
                                             None, None)]),
        _unrolled("_kk", 4, [
            _unrolled("_j", 4, [_ldm("kb[_j * 2]", "k_s", (B("*", V("_j"), L(16)), B("*", V("_kk"), L(16))), "b",
                                     True, "kb[_j * 2 + 1]")]),
            _unrolled("_n", 8, [ir.MmaSyncPtx("s[_n]", "qa[_kk]", "kb[_n]", (16, 8, 16), "f16", "f32", False, None,
                                              None)])]),
        _unrolled("_c", 8, [ir.FragmentApply("s[_c]", E("multiply"), (L(1.0 / D ** 0.5, "float"),), ("scalar",), True,
                                             None, None, None, None)]),
        *_coordinate_apply(extra, "scores"),
        ir.FragmentRowReduce("mx_t", "mx_b", sfr, E("maximum"), None, F32T),
        assign("mn_t", "maximum", "m_t", "mx_t"), assign("mn_b", "maximum", "m_b", "mx_b"),
        assign("d_t", "subtract", "m_t", "mn_t"), assign("d_b", "subtract", "m_b", "mn_b"),
        assign("al_t", "exp", "d_t"), assign("al_b", "exp", "d_b"),
        _unrolled("_e", 8, [ir.FragmentApply("s[_e]", E("subtract"), ("s[_e]", ("mn_t", "mn_b")), row, False,
                                             ir.FragLayout(4, (0, 0, 1, 1), (1, 2), None, (), None, None), E("exp"),
                                             None, None)]),
        *_coordinate_apply(extra, "probabilities"),
        ir.FragmentRowReduce("ls_t", "ls_b", sfr, E("add"), ir.FragLayout(4, (0, 0, 1, 1), (1, 2), None, (), None,
                                                                           None), F32T),
        assign("lt1", "multiply", "l_t", "al_t"), assign("lb1", "multiply", "l_b", "al_b"),
        assign("l_t", "add", "lt1", "ls_t"), assign("l_b", "add", "lb1", "ls_b"),
        assign("m_t", "copy", "mn_t"), assign("m_b", "copy", "mn_b"),
        _unrolled("_r", 8, [ir.FragmentApply("o[_r]", E("multiply"), ("o[_r]", ("al_t", "al_b")), row, False, None,
                                             None, None, None)]),
        _unrolled("_p", 4, [ir.FragmentRepack("pa[_p]", sfr, "f16", "m16n8k16", V("_p"))]),
        _unrolled("_kk", 4, [
            _unrolled("_j", 4, [_ldm("vb[_j * 2]", "v_s", (B("*", V("_kk"), L(16)), B("*", V("_j"), L(16))), "b",
                                     False, "vb[_j * 2 + 1]")]),
            _unrolled("_n", 8, [ir.MmaSyncPtx("o[_n]", "pa[_kk]", "vb[_n]", (16, 8, 16), "f16", "f32", False, None,
                                              None)])]),
        ir.Sync(0, None, False),
    ]
    finish = [_unrolled("_f", 8, [
        ir.FragmentApply("o[_f]", E("divide"), ("o[_f]", ("l_t", "l_b")), row, False, None, None, None, None),
        ir.RegStore("o", (B("+", B("*", V("qb"), L(64)), B("*", V("_w"), L(16))), B("*", V("_f"), L(8))), "o[_f]",
                    (16, 8, 16), 0, None, (), None, None, False, "m16n8k16", False, None, "NONE", None, None)])]
    body = (*frags, *smem, *load_q, *init, ir.StridedLoop(axis("_kv", S), L(0), L(64), tuple(block), False, None, False),
            *finish)
    tile = ir.Tile((axis("qb", S // 64), axis("_w", 4), axis("_lane", 32)), body, 128, 0, None, None, "m")
    entry = "k_fragment_attention"
    inputs = {"q": ((S, D), "f16"), "k": ((S, D), "f16"), "v": ((S, D), "f16")}
    args = [{"name": n, "dtype": "f16", "shape": [S, D], "seed": i} for i, n in enumerate(("q", "k", "v"))]
    if extra in ("bias", "bias_index"):
        inputs["bias"] = ((S, S), "f32")
        args.append({"name": "bias", "dtype": "f32", "shape": [S, S], "seed": 3})
    elif extra == "bias_cols":
        inputs["kbias"] = ((S,), "f32")
        args.append({"name": "kbias", "dtype": "f32", "shape": [S], "seed": 3})
    g = _graph(inputs, {}, "o", (S, D), entry, tile)
    args.append({"name": "o", "dtype": "f32", "shape": [S, D], "output": True})
    kmeta = {"node": "o", "arg_order": [a["name"] for a in args], "grid": [S // 64, 1, 1], "block": [128, 1, 1],
             "smem_bytes": 0, "zero_outputs": [], "args": args}
    return _write(outdir, "sm90_fragment_attention", "softmax(q @ k.T / 8) @ v", entry, g, kmeta, 2e-2, 2e-3)


def _coordinate_apply(extra: str | None, stage: str) -> list:
    """The FragmentApply of ``extra`` at its stage (on the scaled scores, or on the
    probabilities), over the 8 score fragments of the warp's 16 x 64 block."""
    row_base = B("+", B("*", V("qb"), L(64)), B("*", V("_w"), L(16)))
    col_base = B("+", V("_kv"), B("*", V("_x"), L(8)))
    if extra is None or (stage == "probabilities") != (extra == "causal_pred"):
        return []
    if extra == "causal":
        arg, kind, op = ir.Lambda(("qr", "kc"), (ir.Select("mv", (ir.Branch(L(0.0, "float"), B("<=", V("kc"), V("qr"))),
                                                                ir.Branch(L(-1e30, "float"), None))),), ("mv",)), \
            "mask", "add"
    elif extra == "causal_pred":
        arg, kind, op = B("<=", V("col"), V("row")), "mask", "multiply"
    elif extra == "bias":
        arg, kind, op = "bias", "bias", "add"
    elif extra == "bias_cols":
        arg, kind, op = "kbias", "bias", "add"
    else:
        arg, kind, op = ("bias", (V("row"), V("col"))), "bias", "add"
    return [_unrolled("_x", 8, [ir.FragmentApply("s[_x]", E(op), (arg,), (kind,), True, None, None, row_base,
                                                 col_base)])]


def promote_matmul_package(outdir: Path, M: int = 128, N: int = 128, K: int = 512) -> Path:
    """y = x0 @ x1^T (x1 [N, K]) accumulated in f16 fragments (mma.sync with f16 C) for each K block
    of 64 and promoted into f32 shadows after the block (FragmentPromote, which also zeroes the
    f16 ones).  Inputs are integers in -2..2, so every f16 partial (at most 256 in magnitude) and
    every f32 sum is exact: the result equals the integer product bit for bit."""
    if M % 64 or N % 64 or K % 64:
        raise ValueError("promote_matmul_package: M, N, K multiples of 64")
    F16 = F16T
    tid = B("+", B("*", V("_w"), L(32)), V("_lane"))
    body = [ir.RegFragment("a", "a", (16, 8, 16), F16, 1, None), ir.RegFragment("b", "b", (16, 8, 16), F16, 8, None),
            ir.RegFragment("c16", "c", (16, 8, 16), F16, 8, None), ir.RegFragment("c", "c", (16, 8, 16), F32T, 8, None),
            ir.Smem("a_s", (64, 64), "__half", 1024), ir.Smem("b_s", (64, 64), "__half", 1024)]
    ks = [*_copy_tile("a_s", "x0", B("*", V("bm"), L(64)), tid)]
    for i in range(4):                     # B rows bn*64.., columns kb..kb+63
        chunk = B("+", tid, L(128 * i))
        r, c8 = B("/", chunk, L(8)), B("*", B("%", chunk, L(8)), L(8))
        ks.append(ir.CpAsyncCopy("b_s", (L(0), L(0)), "x1", (B("+", B("*", V("bn"), L(64)), r), B("+", V("kb"), c8)),
                                 16, "B128", (r, c8), None))
    # the A copies read columns kb.. too
    ks[:4] = [ir.CpAsyncCopy(c.smem, c.smem_index, c.src, (c.src_index[0], B("+", V("kb"), c.src_index[1])), 16,
                             "B128", c.lane_index, None) for c in ks[:4]]
    ks += [ir.CpAsyncCommit(), ir.CpAsyncWait(0), ir.Sync(0, None, False),
           _unrolled("_kk", 4, [
               _ldm("a", "a_s", (B("*", V("_w"), L(16)), B("*", V("_kk"), L(16))), "a"),
               _unrolled("_j", 4, [_ldm("b[_j * 2]", "b_s", (B("*", V("_j"), L(16)), B("*", V("_kk"), L(16))), "b",
                                        True, "b[_j * 2 + 1]")]),
               _unrolled("_n", 8, [ir.MmaSyncPtx("c16[_n]", "a", "b[_n]", (16, 8, 16), "f16", "f16", False, None,
                                                 None)])]),
           _unrolled("_q", 8, [ir.FragmentPromote("c[_q]", "c16[_q]")]),
           ir.Sync(0, None, False)]
    body.append(ir.StridedLoop(axis("kb", K), L(0), L(64), tuple(ks), False, None, False))
    body.append(_unrolled("_s", 8, [ir.RegStore("y", (B("+", B("*", V("bm"), L(64)), B("*", V("_w"), L(16))),
                                                      B("+", B("*", V("bn"), L(64)), B("*", V("_s"), L(8)))), "c[_s]",
                                                (16, 8, 16), 0, None, (), None, None, False, "m16n8k16", False, None,
                                                "NONE", None, None)]))
    tile = ir.Tile((axis("bm", M // 64), axis("bn", N // 64), axis("_w", 4), axis("_lane", 32)), tuple(body), 128, 0,
                   None, None, "m")
    entry = "k_promote_matmul"
    g = _graph({"x0": ((M, K), "f16"), "x1": ((N, K), "f16")}, {}, "y", (M, N), entry, tile)
    ints = {"dist": "integers", "low": -2, "high": 2}
    args = [{"name": "x0", "dtype": "f16", "shape": [M, K], "seed": 0, "init": dict(ints, seed=0)},
            {"name": "x1", "dtype": "f16", "shape": [N, K], "seed": 1, "init": dict(ints, seed=1)},
            {"name": "y", "dtype": "f32", "shape": [M, N], "output": True}]
    kmeta = {"node": "y", "arg_order": ["x0", "x1", "y"], "grid": [(M // 64) * (N // 64), 1, 1], "block": [128, 1, 1],
             "smem_bytes": 0, "zero_outputs": [], "args": args}
    return _write(outdir, "sm90_promote_matmul", "x0 @ x1.T", entry, g, kmeta, 0, 0)


EPILOGUE_FORMS = ("bias_relu_mask", "guarded", "atomic", "extra")


def epilogue_matmul_package(outdir: Path, form: str, M: int = 128, N: int = 128, K: int = 256) -> Path:
    """An mma.sync GEMM (f32 accumulators, cp.async-staged 64 x 64 tiles, a 16 x 64 strip per warp)
    whose result leaves through the fused RegStore forms: ``x0 @ x1^T`` with x0 [M, K], x1 [N, K]
    integers in -2..2, so every accumulator is an exact integer.

    * ``bias_relu_mask``: y f16 [M, N] = (col <= row) ? relu(0.5 acc + bias[col]) : 0, an epilogue
      Lambda with the element's row and column bound (Let, Assign, a Load of the bias, Select);
    * ``guarded``: y f32 [M - 28, N - 38], the tiles past its edges dropped by ``m_guard`` /
      ``n_guard``;
    * ``atomic``: K split over four CTAs per tile, each adding its partial product into y f32 [M, N]
      (zeroed before the launch) with ``red.global.add``;
    * ``extra``: a second accumulator d = x0 @ x2^T passed through ``extra_frags``; y = acc * d."""
    if form not in EPILOGUE_FORMS or M % 64 or N % 64 or K % 64:
        raise ValueError("epilogue_matmul_package: a known form and M, N, K multiples of 64")
    F16 = F16T
    ks_n = 4 if form == "atomic" else 1
    if K % (64 * ks_n):
        raise ValueError("epilogue_matmul_package: K must split into whole blocks")
    tid = B("+", B("*", V("_w"), L(32)), V("_lane"))
    srcs = ["x1"] + (["x2"] if form == "extra" else [])
    accs = ["c"] + (["d"] if form == "extra" else [])
    body = [ir.RegFragment("a", "a", (16, 8, 16), F16, 1, None)]
    body += [ir.RegFragment(f"b{i}", "b", (16, 8, 16), F16, 8, None) for i in range(len(srcs))]
    body += [ir.RegFragment(n, "c", (16, 8, 16), F32T, 8, None) for n in accs]
    body += [ir.Smem("a_s", (64, 64), "__half", 1024)]
    body += [ir.Smem(f"b{i}_s", (64, 64), "__half", 1024) for i in range(len(srcs))]
    ks = []
    for i in range(4):
        chunk = B("+", tid, L(128 * i))
        r, c8 = B("/", chunk, L(8)), B("*", B("%", chunk, L(8)), L(8))
        ks.append(ir.CpAsyncCopy("a_s", (L(0), L(0)), "x0", (B("+", B("*", V("bm"), L(64)), r), B("+", V("kb"), c8)),
                                 16, "B128", (r, c8), None))
        for j, src in enumerate(srcs):
            ks.append(ir.CpAsyncCopy(f"b{j}_s", (L(0), L(0)), src,
                                     (B("+", B("*", V("bn"), L(64)), r), B("+", V("kb"), c8)), 16, "B128", (r, c8),
                                     None))
    mmas = [_ldm("a", "a_s", (B("*", V("_w"), L(16)), B("*", V("_kk"), L(16))), "a")]
    for j, acc in enumerate(accs):
        mmas += [_unrolled("_j", 4, [_ldm(f"b{j}[_j * 2]", f"b{j}_s", (B("*", V("_j"), L(16)), B("*", V("_kk"), L(16))),
                                          "b", True, f"b{j}[_j * 2 + 1]")]),
                 _unrolled("_n", 8, [ir.MmaSyncPtx(f"{acc}[_n]", "a", f"b{j}[_n]", (16, 8, 16), "f16", "f32", False,
                                                   None, None)])]
    ks += [ir.CpAsyncCommit(), ir.CpAsyncWait(0), ir.Sync(0, None, False), _unrolled("_kk", 4, mmas),
           ir.Sync(0, None, False)]
    if ks_n == 1:
        body.append(ir.StridedLoop(axis("kb", K), L(0), L(64), tuple(ks), False, None, False))
    else:               # CTA ks of the tile covers K columns ks * K / 4 .. (ks + 1) * K / 4
        k0 = B("*", V("ks"), L(K // ks_n))
        body.append(ir.StridedLoop(axis("kb", K), k0, L(64), tuple(ks), False, B("+", k0, L(K // ks_n)), False))
    epilogue, extra, m_guard, n_guard, atomic = None, (), None, None, False
    out_shape, out_dtype = (M, N), "f32"
    if form == "bias_relu_mask":
        out_dtype = "f16"
        epilogue = ir.Lambda(("v", "row", "col"), (
            ir.Let("half", L(0.5, "float"), F32T),
            assign("sv", "multiply", "v", "half"),
            ir.Load(("bv",), "bias", (V("col"),), F32T),
            assign("tv", "add", "sv", "bv"),
            assign("uv", "relu", "tv"),
            ir.Select("ov", (ir.Branch("uv", B("<=", V("col"), V("row"))), ir.Branch(L(0.0, "float"), None)))),
            ("ov",))
    elif form == "guarded":
        out_shape = (M - 28, N - 38)
        m_guard, n_guard = L(M - 28), L(N - 38)
    elif form == "atomic":
        atomic = True
    else:
        epilogue = ir.Lambda(("v", "w"), (assign("pv", "multiply", "v", "w"),), ("pv",))
        extra = ("d[_s]",)
    body.append(_unrolled("_s", 8, [ir.RegStore("y", (B("+", B("*", V("bm"), L(64)), B("*", V("_w"), L(16))),
                                                      B("+", B("*", V("bn"), L(64)), B("*", V("_s"), L(8)))), "c[_s]",
                                                (16, 8, 16), 0, epilogue, extra, m_guard, n_guard, atomic, "m16n8k16",
                                                False, None, "NONE", None, None)]))
    axes = (axis("bm", M // 64), axis("bn", N // 64)) + ((axis("ks", ks_n),) if ks_n > 1 else ())
    tile = ir.Tile(axes + (axis("_w", 4), axis("_lane", 32)), tuple(body), 128, 0, None, None, "m")
    entry = f"k_epilogue_{form}"
    inputs = {"x0": ((M, K), "f16"), **{s: ((N, K), "f16") for s in srcs}}
    ints = {"dist": "integers", "low": -2, "high": 2}
    args = [{"name": n, "dtype": "f16", "shape": list(shape), "seed": i, "init": dict(ints, seed=i)}
            for i, (n, (shape, _)) in enumerate(inputs.items())]
    order = list(inputs)
    if form == "bias_relu_mask":
        inputs["bias"] = ((N,), "f32")
        args.append({"name": "bias", "dtype": "f32", "shape": [N], "seed": 7})
        order.append("bias")
    args.append({"name": "y", "dtype": out_dtype, "shape": list(out_shape), "output": True})
    g = _graph(inputs, {}, "y", out_shape, entry, tile, out_dtype)
    kmeta = {"node": "y", "arg_order": order + ["y"], "grid": [(M // 64) * (N // 64) * ks_n, 1, 1],
             "block": [128, 1, 1], "smem_bytes": 0, "zero_outputs": ["y"] if atomic else [], "args": args}
    return _write(outdir, f"sm90_epilogue_{form}", "x0 @ x1.T", entry, g, kmeta, 1e-3, 1e-3)



def blockscaled_matmul_package(outdir: Path, M: int = 128, N: int = 128, K: int = 128) -> Path:
    """y = dequant(xa) @ dequant(xb)^T with block-scaled fp4 operands: xa [M, K/2] and xb [N, K/2]
    hold two e2m1 codes per byte (the lower k in the low nibble), sa [M, K/32] and sb [N, K/32]
    one ue8m0 scale (2^(e - 127)) per 32 consecutive k.  Per warp a 16-row strip of a 64 x 64
    tile: both operand tiles staged into byte Smem arrays by cp.async, then per 64-deep K step an
    fp4 LdmatrixLoad of A, BlockScaleLoad of its scales, and for each of 8 column atoms an fp4
    LdmatrixLoad of B, its BlockScaleLoad and one block-scaled m16n8k64 MmaSyncPtx into f32."""
    if M % 64 or N % 64 or K % 64:
        raise ValueError("blockscaled_matmul_package: M, N, K multiples of 64")
    KB = K // 2
    tid = B("+", B("*", V("_w"), L(32)), V("_lane"))
    body = [ir.RegFragment("fa", "a", (16, 8, 64), "e2m1", 1, None),
            ir.RegFragment("fb", "b", (16, 8, 64), "e2m1", 8, None),
            ir.RegFragment("sfa", "a", (16, 8, 64), "ue8m0", 1, None),
            ir.RegFragment("sfb", "b", (16, 8, 64), "ue8m0", 8, None),
            ir.RegFragment("c", "c", (16, 8, 64), F32T, 8, None),
            ir.Smem("a_s", (64, KB), "uint8_t", 16), ir.Smem("b_s", (64, KB), "uint8_t", 16)]
    per_row = KB // 16                                # 16-byte chunks per tile row
    for smem, src, blk in (("a_s", "xa", "bm"), ("b_s", "xb", "bn")):
        for i in range(64 * per_row // 128):
            chunk = B("+", tid, L(128 * i))
            r, c = B("/", chunk, L(per_row)), B("*", B("%", chunk, L(per_row)), L(16))
            body.append(ir.CpAsyncCopy(smem, (r, c), src, (B("+", B("*", V(blk), L(64)), r), c), 16, "NONE", None, 0))
    body += [ir.CpAsyncCommit(), ir.CpAsyncWait(0), ir.Sync(0, None, False)]

    def ldm(frag, smem, idx, role):
        return ir.LdmatrixLoad(frag, smem, idx, role, KB, "NONE", True, None, None, False, None, False, None, (), 0,
                               "m16n8k64", None)
    row0 = B("*", V("_w"), L(16))
    body.append(_unrolled("_ks", K // 64, [
        ldm("fa", "a_s", (row0, B("*", V("_ks"), L(32))), "a"),
        ir.BlockScaleLoad("sfa", "sa", (B("+", B("*", V("bm"), L(64)), row0), B("*", V("_ks"), L(2))), "a", 0),
        _unrolled("_j", 8, [
            ldm("fb[_j]", "b_s", (B("*", V("_j"), L(8)), B("*", V("_ks"), L(32))), "b"),
            ir.BlockScaleLoad("sfb[_j]", "sb", (B("+", B("*", V("bn"), L(64)), B("*", V("_j"), L(8))),
                                                B("*", V("_ks"), L(2))), "b", 0),
            ir.MmaSyncPtx("c[_j]", "fa", "fb[_j]", (16, 8, 64), "e2m1", "f32", False, "sfa", "sfb[_j]")])]))
    body.append(_unrolled("_s", 8, [ir.RegStore("y", (B("+", B("*", V("bm"), L(64)), row0),
                                                      B("+", B("*", V("bn"), L(64)), B("*", V("_s"), L(8)))), "c[_s]",
                                                (16, 8, 16), 0, None, (), None, None, False, "m16n8k16", False, None,
                                                "NONE", None, None)]))
    tile = ir.Tile((axis("bm", M // 64), axis("bn", N // 64), axis("_w", 4), axis("_lane", 32)), tuple(body), 128, 0,
                   None, None, "m")
    entry = "k_blockscaled_matmul"
    g = _graph({"xa": ((M, KB), "u8"), "xb": ((N, KB), "u8"), "sa": ((M, K // 32), "u8"),
                "sb": ((N, K // 32), "u8")}, {}, "y", (M, N), entry, tile)
    codes = {"dist": "integers", "low": 0, "high": 255}
    scales = {"dist": "integers", "low": 124, "high": 130}
    args = [{"name": "xa", "dtype": "u8", "shape": [M, KB], "seed": 0, "init": dict(codes, seed=0)},
            {"name": "xb", "dtype": "u8", "shape": [N, KB], "seed": 1, "init": dict(codes, seed=1)},
            {"name": "sa", "dtype": "u8", "shape": [M, K // 32], "seed": 2, "init": dict(scales, seed=2)},
            {"name": "sb", "dtype": "u8", "shape": [N, K // 32], "seed": 3, "init": dict(scales, seed=3)},
            {"name": "y", "dtype": "f32", "shape": [M, N], "output": True}]
    kmeta = {"node": "y", "arg_order": [a["name"] for a in args], "grid": [(M // 64) * (N // 64), 1, 1],
             "block": [128, 1, 1], "smem_bytes": 0, "zero_outputs": [], "args": args}
    return _write(outdir, "sm90_blockscaled_matmul", "dequant(xa) @ dequant(xb).T", entry, g, kmeta, 1e-5, 1e-5)


def dequant_fp4(codes: "np.ndarray", scales: "np.ndarray") -> "np.ndarray":
    """The float64 values of packed fp4 rows (two e2m1 codes per byte, low nibble first) scaled by
    ue8m0 bytes, one per 32 values -- the numpy statement of the block-scaled operands."""
    import numpy as np
    from thompiler.handlers.blockscale import e2m1_value
    table = np.array([e2m1_value(n) for n in range(16)])
    nib = np.stack([codes & 15, codes >> 4], axis=-1).reshape(codes.shape[0], -1)
    vals = table[nib]
    sc = np.exp2(scales.astype(np.float64) - 127.0)
    return vals * np.repeat(sc, 32, axis=1)


def window_package(outdir: Path, W: int = 4) -> Path:
    """Carried state indexed at run time, one thread per row of x[ROWS, COLS]: a ring of W cells
    holds the row's last W values, cell j % W written at step j, so the step reads the value of
    step j - W from the same cell before setting it: y[r, j] = x[r, j] - x[r, j - W] (0 for
    j < W), and t[r] = the cell of the last step (x[r, COLS - 1]), read after the loop."""
    f32 = F32T
    cell = (B("%", V("j"), L(W)),)
    step = (
        ir.Pre("old", "win", cell),
        ir.Load(("v",), "x", (V("r"), V("j")), f32),
        assign("d", "subtract", "v", "old"),
        ir.Carry("win", "v", cell, L(0.0, "float"), f32),
        ir.Write("y", (V("r"), V("j")), ("d",), f32, False, "NONE"),
    )
    body = (
        ir.Loop(axis("j", COLS), step, False, False),
        ir.Pre("last", "win", (L((COLS - 1) % W),)),
        ir.Write("t", (V("r"),), ("last",), f32, False, "NONE"),
    )
    tile = ir.Tile((axis("r", ROWS),), body, 128, 0, None, None, "m")
    g = _graph({"x": ((ROWS, COLS), "f32")}, {}, "y", (ROWS, COLS), "k_window", tile)
    g["nodes"]["y"]["outputs"] += [{"name": "t", "shape": [ROWS], "dtype": "f32"}]
    g["outputs"] = ["y", "t"]
    args = [{"name": "x", "dtype": "f32", "shape": [ROWS, COLS], "seed": 0},
            {"name": "y", "dtype": "f32", "shape": [ROWS, COLS], "output": True},
            {"name": "t", "dtype": "f32", "shape": [ROWS], "output": True}]
    kmeta = {"node": "y", "arg_order": ["x", "y", "t"], "grid": [ROWS // 128, 1, 1], "block": [128, 1, 1],
             "smem_bytes": 0, "zero_outputs": [], "args": args}
    return _write(outdir, "sm90_window", f"x - shifted(x, {W})", "k_window", g, kmeta, 0, 0)


def chained_matmul_package(outdir: Path) -> Path:
    """y = f16(x0 @ x1^T) @ x2^T on one 64 x 64 tile (x0, x1, x2 f16 [64, 64], K-major B operands):
    the first product's C fragments go to a shared array with the 128-byte swizzle (RegStore
    into shared memory, rounded to f16), which the second product reads back as A fragments
    with ldmatrix under the same swizzle -- the staging a chained contraction needs."""
    F16 = F16T
    tid = B("+", B("*", V("_w"), L(32)), V("_lane"))
    row0 = B("*", V("_w"), L(16))
    frags = [ir.RegFragment("a", "a", (16, 8, 16), F16, 4, None), ir.RegFragment("b", "b", (16, 8, 16), F16, 8, None),
             ir.RegFragment("c", "c", (16, 8, 16), F32T, 8, None), ir.RegFragment("pa", "a", (16, 8, 16), F16, 4, None),
             ir.RegFragment("b2", "b", (16, 8, 16), F16, 8, None), ir.RegFragment("c2", "c", (16, 8, 16), F32T, 8, None)]
    smem = [ir.Smem(n, (64, 64), "__half", 1024) for n in ("a_s", "b_s", "p_s", "b2_s")]
    copies = [*_copy_tile("a_s", "x0", L(0), tid), *_copy_tile("b_s", "x1", L(0), tid),
              *_copy_tile("b2_s", "x2", L(0), tid), ir.CpAsyncCommit(), ir.CpAsyncWait(0), ir.Sync(0, None, False)]

    def gemm(afr, asmem, bfr, bsmem, cfr):
        return _unrolled("_kk", 4, [
            _ldm(f"{afr}[_kk]", asmem, (row0, B("*", V("_kk"), L(16))), "a"),
            _unrolled("_j", 4, [_ldm(f"{bfr}[_j * 2]", bsmem, (B("*", V("_j"), L(16)), B("*", V("_kk"), L(16))), "b",
                                     True, f"{bfr}[_j * 2 + 1]")]),
            _unrolled("_n", 8, [ir.MmaSyncPtx(f"{cfr}[_n]", f"{afr}[_kk]", f"{bfr}[_n]", (16, 8, 16), "f16", "f32",
                                              False, None, None)])])

    def store(dst, cfr, swizzle):
        return _unrolled("_s", 8, [ir.RegStore(dst, (row0, B("*", V("_s"), L(8))), f"{cfr}[_s]", (16, 8, 16), 0, None,
                                               (), None, None, False, "m16n8k16", False, None, swizzle, None, None)])
    body = (*frags, *smem, *copies, gemm("a", "a_s", "b", "b_s", "c"), store("p_s", "c", "B128"),
            ir.Sync(0, None, False), gemm("pa", "p_s", "b2", "b2_s", "c2"), store("y", "c2", "NONE"))
    tile = ir.Tile((axis("_w", 4), axis("_lane", 32)), body, 128, 0, None, None, "m")
    entry = "k_chained_matmul"
    g = _graph({"x0": ((64, 64), "f16"), "x1": ((64, 64), "f16"), "x2": ((64, 64), "f16")}, {}, "y", (64, 64), entry,
               tile)
    args = [{"name": n, "dtype": "f16", "shape": [64, 64], "seed": i} for i, n in enumerate(("x0", "x1", "x2"))]
    args.append({"name": "y", "dtype": "f32", "shape": [64, 64], "output": True})
    kmeta = {"node": "y", "arg_order": ["x0", "x1", "x2", "y"], "grid": [1, 1, 1], "block": [128, 1, 1],
             "smem_bytes": 0, "zero_outputs": [], "args": args}
    return _write(outdir, "sm90_chained_matmul", "(x0 @ x1.T).half() @ x2.T", entry, g, kmeta, 2e-2, 2e-3)
