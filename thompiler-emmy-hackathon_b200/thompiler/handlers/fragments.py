"""Register-fragment operations on tensor-core accumulators: FragmentPromote, FragmentRowReduce,
FragmentApply, FragmentRepack.

The IR reference (TASK.md:149-157 of the reference) defines these for C fragments held in
registers; the reference compiler lowers none of them.  Every accumulator this backend keeps
in registers has the same per-thread geometry, whatever its width: registers come in groups
of four per 8 columns, with g = lane / 4 and t = lane % 4

    register 4i + 0, 4i + 1  ->  top row    (g, or 16q + g in warp q of a warpgroup), columns 8i + 2t, 8i + 2t + 1
    register 4i + 2, 4i + 3  ->  bottom row (the top row + 8),                            the same columns

(an m16n8 ``mma.sync`` C fragment is one group; an m64nN warpgroup accumulator N/8 of them),
and a row's 8i + 2t columns are spread over the four lanes of a quad (xor 1, xor 2).  A
packed f16 accumulator holds each register pair (4i + 2j, 4i + 2j + 1) as one f16x2 word.
Hence:

* ``FragmentPromote(dst, src)``: dst[2j] += lo(src[j]), dst[2j + 1] += hi(src[j]) (f16 -> f32
  exactly, one ``add.rn.f32`` each), then src[j] = 0;
* ``FragmentRowReduce(top, bot, frags, op)``: ``top`` = op over the top-row registers of every
  fragment, ``bot`` the same for the bottom rows, each then combined across the quad by
  ``shfl.sync.bfly`` over the layout's ``reduce_xors`` (default 1, 2), so that every lane of
  the quad holds its rows' reduction over all the fragments' columns.  op: maximum, minimum, add;
* ``FragmentApply(out, op, args, kinds, in_place, post, row_base, col_base)``: for every
  element e of ``out``, out[e] = post(op(out[e] if in_place, arg_1[e], ...)), where an argument
  of kind ``frag`` is the same element of another fragment, ``row`` a (top, bottom) pair of
  per-row values (FragmentRowReduce's results) taken by the element's row, and ``scalar`` one
  value (a name or a literal).  ``mask`` and ``bias`` arguments are functions of the element's
  coordinates in the output: row = row_base + the element's row (g or g + 8, plus 16 (warp % 4)
  in a warpgroup accumulator), col = col_base + its column (8i + 2t + j):

  - ``mask``: a predicate (an index expression in which ``Var('row')`` and ``Var('col')`` are
    those coordinates), giving 1.0 where it holds and 0.0 where it does not; or an ``ir.Lambda``
    with parameters (row, col) and one result, whose body (Load / Assign / Let / Select) gives
    the operand -- e.g. a Select of 0 or -1e30 for an additive causal mask;
  - ``bias``: a global load at the coordinates -- a buffer name (a 2-D buffer read at (row,
    col); a 1-D one at (col), one value per column broadcast over the rows, as a linear layer's
    bias), a (buffer, index) pair whose index is written in ``Var('row')`` / ``Var('col')``, or
    an ``ir.Lambda`` as for a mask.  The loaded value is widened to f32.
* ``FragmentRepack(frag, srcs, ab_dtype, part)``: the 16 x 16 A fragment of an m16n8k16 MMA
  from two f32 C fragments (columns 0-7 and 8-15 of its K): a0 = (c0[0], c0[1]), a1 =
  (c0[2], c0[3]), a2 = (c1[0], c1[1]), a3 = (c1[2], c1[3]), each pair rounded to f16x2 (or
  bf16x2) with ``cvt.rn``; ``part`` p picks srcs[2p], srcs[2p + 1] from a longer list.

A FragLayout, when given, must agree with this geometry (element rows 0, 0, 1, 1 per group);
a fragment written here that is a warpgroup accumulator is marked for its next WgmmaFence.
"""

from __future__ import annotations

from typing import TYPE_CHECKING

from thompiler import ir
from thompiler.handlers.compute import apply_op
from thompiler.handlers.mma import fragment_regs
from thompiler.lowering import expr
from thompiler.lowering.types import F16, F32

if TYPE_CHECKING:
    from thompiler.walk import Walker

REDUCE_OPS = ("maximum", "minimum", "add")


def _op_name(op, what: str) -> str:
    name = op.name if isinstance(op, ir.ElementwiseImpl) else op
    if not isinstance(name, str):
        raise ValueError(f"{what}: operation {op!r}")
    return name


def _accumulator(w: "Walker", ref: str, what: str) -> list[str]:
    frag, regs = fragment_regs(w, ref)
    if frag.role != "c" or frag.ty is not F32 or len(regs) % 4:
        raise NotImplementedError(f"{what}: {ref} is not an f32 accumulator fragment")
    return regs


def _check_layout(layout, n: int, what: str) -> tuple[int, ...]:
    """The lane xors of a FragLayout (1, 2 by default), after checking its element rows."""
    if layout is None:
        return (1, 2)
    if not isinstance(layout, ir.FragLayout):
        raise NotImplementedError(f"{what}: layout {layout!r}")
    rows = tuple(int(r) for r in layout.elem_row)
    if rows and (len(rows) % 4 or rows != (0, 0, 1, 1) * (len(rows) // 4)):
        raise NotImplementedError(f"{what}: element rows {rows} differ from the accumulator layout")
    if layout.n_elems and int(layout.n_elems) not in (4, n):
        raise NotImplementedError(f"{what}: {layout.n_elems} elements per atom, the fragment has {n}")
    xors = tuple(int(x) for x in layout.reduce_xors) or (1, 2)
    if sorted(xors) != [1, 2]:
        raise NotImplementedError(f"{what}: lane xors {xors} (a row spans the quad: 1 and 2)")
    return xors


def _written(w: "Walker", ref: str) -> None:
    from thompiler.handlers.wgmma import fragment_written
    fragment_written(w, ref.split("[", 1)[0])


def emit_fragment_promote(w: "Walker", s: ir.FragmentPromote) -> None:
    em = w.em
    em.note(f"FragmentPromote {s.dst} += {s.src}")
    dst = _accumulator(w, s.dst, "FragmentPromote")
    frag, src = fragment_regs(w, s.src)
    if frag.role != "c" or frag.ty is not F16 or 2 * len(src) != len(dst):
        raise ValueError(f"FragmentPromote: {s.src} is not the packed f16 shadow of {s.dst}")
    for j, word in enumerate(src):
        lo, hi = em.tmp("b16"), em.tmp("b16")
        em.ins(f"mov.b32 {{{lo}, {hi}}}, {word}")
        for half, r in ((lo, dst[2 * j]), (hi, dst[2 * j + 1])):
            f = em.tmp("f32")
            em.ins(f"cvt.f32.f16 {f}, {half}")
            em.ins(f"add.rn.f32 {r}, {r}, {f}")
        em.ins(f"mov.b32 {word}, 0")
    _written(w, s.dst)
    _written(w, s.src)


def emit_fragment_row_reduce(w: "Walker", s: ir.FragmentRowReduce) -> None:
    em = w.em
    op = _op_name(s.op, "FragmentRowReduce")
    em.note(f"FragmentRowReduce {s.top}, {s.bot} = {op} over {', '.join(s.frags)}")
    if op not in REDUCE_OPS:
        raise NotImplementedError(f"FragmentRowReduce with {op}")
    if s.dtype is not None and getattr(s.dtype, "name", s.dtype) != "f32":
        raise NotImplementedError(f"FragmentRowReduce in {s.dtype}")
    if not s.frags:
        raise ValueError("FragmentRowReduce over no fragments")
    regs = [_accumulator(w, f, "FragmentRowReduce") for f in s.frags]
    xors = _check_layout(s.layout, len(regs[0]), "FragmentRowReduce")
    out = []
    for name, half in ((s.top, 0), (s.bot, 2)):
        vals = [r[4 * i + half + k] for r in regs for i in range(len(r) // 4) for k in (0, 1)]
        acc = em.tmp("f32")
        apply_op(w, op, acc, [vals[0], vals[1]], F32)
        for v in vals[2:]:
            apply_op(w, op, acc, [acc, v], F32)
        out.append((name, acc))
    for x in xors:
        for _, acc in out:
            other = em.tmp("f32")
            em.ins(f"shfl.sync.bfly.b32 {other}, {acc}, {x}, 31, -1")
            apply_op(w, op, acc, [acc, other], F32)
    for name, acc in out:
        em.ins(f"mov.f32 {em.value(name, 'f32')}, {acc}")


def _scalar(w: "Walker", arg, what: str) -> str:
    em = w.em
    if isinstance(arg, str):
        return em.get(arg)
    value = arg.value if isinstance(arg, ir.Literal) else arg
    if isinstance(value, (int, float)) and not isinstance(value, bool):
        r = em.tmp("f32")
        em.ins(f"mov.f32 {r}, {F32.imm(value)}")
        return r
    raise NotImplementedError(f"{what}: scalar argument {ir.pretty(arg)}")


def emit_fragment_apply(w: "Walker", s: ir.FragmentApply) -> None:
    em = w.em
    op = _op_name(s.op, "FragmentApply")
    post = None if s.post is None else _op_name(s.post, "FragmentApply post")
    em.note(f"FragmentApply {s.out} = {post + '(' if post else ''}{op}({'out, ' if s.in_place else ''}"
            f"{', '.join(ir.pretty(a) if not isinstance(a, str) else a for a in s.args)}){')' if post else ''}")
    out = _accumulator(w, s.out, "FragmentApply")
    _check_layout(s.layout, len(out), "FragmentApply")
    kinds = tuple(s.kinds) or ("frag",) * len(s.args)
    if len(kinds) != len(s.args):
        raise ValueError(f"FragmentApply: {len(s.args)} arguments with {len(kinds)} kinds")
    operands = []                       # per argument: element index -> register
    for arg, kind in zip(s.args, kinds):
        if kind == "frag":
            regs = _accumulator(w, arg, "FragmentApply")
            if len(regs) != len(out):
                raise ValueError(f"FragmentApply: {arg} has {len(regs)} registers, {s.out} {len(out)}")
            operands.append(lambda e, regs=regs: regs[e])
        elif kind == "row":
            if not (isinstance(arg, tuple) and len(arg) == 2):
                raise ValueError(f"FragmentApply: a row argument is a (top, bottom) pair, got {arg!r}")
            top, bot = (_scalar(w, x, "FragmentApply") for x in arg)
            operands.append(lambda e, top=top, bot=bot: top if e % 4 < 2 else bot)
        elif kind == "scalar":
            r = _scalar(w, arg, "FragmentApply")
            operands.append(lambda e, r=r: r)
        elif kind in ("mask", "bias"):
            if s.row_base is None or s.col_base is None:
                raise ValueError(f"FragmentApply: a {kind} argument needs row_base and col_base")
            operands.append(lambda e, arg=arg, kind=kind: _coordinate_operand(w, s, len(out), e, arg, kind))
        else:
            raise NotImplementedError(f"FragmentApply argument of kind {kind!r}")
    arity = ir.ElementwiseImpl(op).arity
    if arity != len(operands) + bool(s.in_place):
        raise ValueError(f"FragmentApply: {op} takes {arity} operands, given {len(operands) + bool(s.in_place)}")
    for e, dst in enumerate(out):
        vals = ([dst] if s.in_place else []) + [f(e) for f in operands]
        r = em.tmp("f32")
        apply_op(w, op, r, vals, F32)
        if post is not None:
            r2 = em.tmp("f32")
            apply_op(w, post, r2, [r], F32)
            r = r2
        em.ins(f"mov.f32 {dst}, {r}")
    _written(w, s.out)


def _element_coords(w: "Walker", s: ir.FragmentApply, nregs: int, e: int) -> tuple:
    """Index expressions of element e's row and column in the output (see the module docstring)."""
    from thompiler.handlers.mma import _lane_expr
    lane = ir.Var("lane")
    g = _lane_expr("/", lane, 4)
    if nregs > 4:                            # a warpgroup accumulator: warp q holds rows 16q ..
        g = ir.BinaryExpr("+", g, _lane_expr("*", _lane_expr("%", ir.Var("warp"), 4), 16))
    t2 = _lane_expr("*", _lane_expr("%", lane, 4), 2)
    i, r = divmod(e, 4)
    row = ir.BinaryExpr("+", s.row_base, g if r < 2 else _lane_expr("+", g, 8))
    col = ir.BinaryExpr("+", s.col_base, _lane_expr("+", t2, 8 * i + (r % 2)))
    return row, col


def _bind_coords(w: "Walker", names: tuple, row, col) -> None:
    from thompiler.lowering import expr as ex
    em = w.em
    for name, e in zip(names, (row, col)):
        em.ins(f"mov.s32 {em.value(name, 'b32')}, {ex.int_operand(w, e)}")


def _coordinate_operand(w: "Walker", s: ir.FragmentApply, nregs: int, e: int, arg, kind: str) -> str:
    """The f32 register holding a mask or bias argument's value at element e."""
    from thompiler.handlers.mma import _param_name
    from thompiler.lowering import address
    from thompiler.lowering import expr as ex
    em = w.em
    row, col = _element_coords(w, s, nregs, e)
    out = em.tmp("f32")
    if isinstance(arg, ir.Lambda):
        params = tuple(_param_name(p) for p in arg.params)
        if len(params) != 2:
            raise ValueError(f"FragmentApply {kind}: a Lambda takes (row, col), got {len(params)} parameters")
        _bind_coords(w, params, row, col)
        for st in arg.body:
            if not isinstance(st, (ir.Load, ir.Assign, ir.Let, ir.Select)):
                raise NotImplementedError(f"FragmentApply {kind}: statement {type(st).__name__} in a Lambda")
            w.stmt(st)
        results = [_param_name(r) for r in arg.results]
        if len(results) != 1:
            raise NotImplementedError(f"FragmentApply {kind}: a Lambda with {len(results)} results")
        reg = em.get(results[0])
        cls = em.named[reg]
        if cls == "f32":
            em.ins(f"mov.f32 {out}, {reg}")
        elif cls == "b16":
            em.ins(f"cvt.f32.f16 {out}, {reg}")
        elif cls == "b32":
            em.ins(f"cvt.rn.f32.s32 {out}, {reg}")
        elif cls == "pred":
            em.ins(f"selp.f32 {out}, 0f3F800000, 0f00000000, {reg}")
        else:
            raise TypeError(f"FragmentApply {kind}: a .{cls} result")
        return out
    if kind == "mask":
        _bind_coords(w, ("row", "col"), row, col)
        p = ex.pred_operand(w, arg)
        em.ins(f"selp.f32 {out}, 0f3F800000, 0f00000000, {p}")
        return out
    # bias: a global load at the element's coordinates
    if isinstance(arg, str):
        prm = w.kernel.param(arg)
        if prm is None:
            raise ValueError(f"FragmentApply bias: {arg!r} is not a kernel parameter")
        if len(prm.shape) == 2:
            idx = (row, col)
        elif len(prm.shape) == 1:
            idx = (col,)
        else:
            raise NotImplementedError(f"FragmentApply bias from a {len(prm.shape)}-d buffer")
        buf = arg
    elif isinstance(arg, tuple) and len(arg) == 2 and isinstance(arg[0], str):
        buf, idx = arg[0], tuple(arg[1])
        _bind_coords(w, ("row", "col"), row, col)
    else:
        raise NotImplementedError(f"FragmentApply bias argument {arg!r}")
    prm = w.kernel.param(buf)
    if prm is None:
        raise ValueError(f"FragmentApply bias: {buf!r} is not a kernel parameter")
    addr = address.global_address(w, prm, idx)
    ld = "ld.global" if prm.written else "ld.global.nc"      # a buffer the kernel writes: coherent loads
    if prm.ty is F32:
        em.ins(f"{ld}.f32 {out}, [{addr}]")
    elif prm.ty is F16:
        h = em.tmp("b16")
        em.ins(f"{ld}.b16 {h}, [{addr}]")
        em.ins(f"cvt.f32.f16 {out}, {h}")
    else:
        raise NotImplementedError(f"FragmentApply bias from a {prm.ty.name} buffer")
    return out


def emit_fragment_repack(w: "Walker", s: ir.FragmentRepack) -> None:
    em = w.em
    em.note(f"FragmentRepack {s.frag} <- {', '.join(s.srcs)}")
    if s.fragment_layout not in ("m16n8k16", None):
        raise NotImplementedError(f"FragmentRepack to layout {s.fragment_layout}")
    if s.ab_dtype not in ("f16", "bf16"):
        raise NotImplementedError(f"FragmentRepack to {s.ab_dtype}")
    srcs = tuple(s.srcs)
    if s.part is not None:
        part = expr.int_operand(w, s.part) if isinstance(s.part, ir.Expr) else str(int(s.part))
        if not expr.is_imm(part):
            raise NotImplementedError(f"FragmentRepack: part {ir.pretty(s.part)} must fold to a constant")
        srcs = srcs[2 * int(part):2 * int(part) + 2]
    if len(srcs) != 2:
        raise ValueError(f"FragmentRepack: an A fragment takes two C fragments, got {len(srcs)}")
    frag, dst = fragment_regs(w, s.frag)
    if frag.role != "a" or frag.ty.nbytes != 2 or len(dst) != 4:
        raise ValueError(f"FragmentRepack: {s.frag} is not a 16-bit m16n8k16 A fragment")
    c0, c1 = (_accumulator(w, c, "FragmentRepack") for c in srcs)
    if len(c0) != 4 or len(c1) != 4:
        raise NotImplementedError("FragmentRepack from accumulators wider than m16n8")
    for d, (lo, hi) in zip(dst, ((c0[0], c0[1]), (c0[2], c0[3]), (c1[0], c1[1]), (c1[2], c1[3]))):
        em.ins(f"cvt.rn.{s.ab_dtype}x2.f32 {d}, {hi}, {lo}")
