"""Reductions: Accum / Init and the cross-thread combines.

WarpShuffle folds the per-lane states of ``length`` lanes with an XOR
butterfly of ``shfl.sync.bfly`` (the IR's ``combine_states`` Assigns are
replayed after each exchange), as the IR reference specifies; f64 states
move as two 32-bit halves and f16 states in the low half of a 32-bit word.

TreeHalve folds ``length`` partial states that the warps left in shared
memory and gives every thread the result.  The reference walks a shared
tree with one CTA barrier per level and a final broadcast read
(thompiler/handlers/reduce.py:87-133 of the reference).  For ``length <= 32``
this backend instead has every warp read the ``length`` slots into its
lanes and fold them with the same XOR butterfly: lane 0 combines exactly
the operands the tree combines at slot 0, in the same order, so lane 0's
value is bit-identical to the tree root, and a final ``shfl.idx`` from
lane 0 hands that value to the whole warp.  No barrier and no shared
store is needed.  Wider trees keep the barrier form.
"""

from __future__ import annotations

from typing import TYPE_CHECKING

from thompiler import ir
from thompiler.handlers.compute import arg_type, emit_assign
from thompiler.handlers.memory import emit_sync
from thompiler.lowering import address, expr, ops
from thompiler.lowering.types import F16, F64, dtype_of

if TYPE_CHECKING:
    from thompiler.walk import Walker

WARP = 32


def emit_accum(w: "Walker", acc: ir.Accum) -> None:
    em = w.em
    em.note(acc.pretty())
    op = acc.op.name
    if op not in ops.ACCUM_OPS:
        raise NotImplementedError(f"Accum with op {op!r}")
    ty = dtype_of(acc.dtype, f"Accum {acc.name}")
    if arg_type(w, acc.value) != ty:
        raise TypeError(f"Accum {acc.name}: {ty.name} accumulator, {arg_type(w, acc.value).name} value")
    reg = em.get(acc.name)
    base = em.get(acc.base) if acc.base is not None else reg
    em.ins(f"{ops.instruction(ops.BINARY, op, ty)} {reg}, {base}, {em.get(acc.value)}")


def emit_init(w: "Walker", init: ir.Init) -> None:
    em = w.em
    em.note(init.pretty())
    ty = dtype_of(init.dtype, f"Init {init.name}")
    em.ins(f"mov.{ty.mov} {em.value(init.name, ty.reg)}, {ty.imm(init.identity)}")


def shuffle(w: "Walker", mode: str, dst: str, src: str, lane_arg: str, clamp: str, mask: str, ty) -> None:
    """dst = shfl.sync.<mode>(src) for a value of any supported width."""
    em = w.em
    if ty.nbytes == 4:
        em.ins(f"shfl.sync.{mode}.b32 {dst}, {src}, {lane_arg}, {clamp}, {mask}")
    elif ty is F64:
        lo, hi = em.tmp("b32"), em.tmp("b32")
        em.ins(f"mov.b64 {{{lo}, {hi}}}, {src}")
        em.ins(f"shfl.sync.{mode}.b32 {lo}, {lo}, {lane_arg}, {clamp}, {mask}")
        em.ins(f"shfl.sync.{mode}.b32 {hi}, {hi}, {lane_arg}, {clamp}, {mask}")
        em.ins(f"mov.b64 {dst}, {{{lo}, {hi}}}")
    elif ty is F16:
        t = em.tmp("b32")
        em.ins(f"cvt.u32.u16 {t}, {src}")
        em.ins(f"shfl.sync.{mode}.b32 {t}, {t}, {lane_arg}, {clamp}, {mask}")
        em.ins(f"cvt.u16.u32 {dst}, {t}")
    else:
        raise NotImplementedError(f"shuffle of {ty.name}")


def butterfly(w: "Walker", states: tuple, partners: tuple, combine: tuple, length: int, ty) -> None:
    em = w.em
    mask = em.tmp("b32")
    em.ins(f"activemask.b32 {mask}")
    step = length // 2
    while step:
        em.note(f"butterfly: exchange with lane ^ {step}")
        for s, o in zip(states, partners, strict=True):
            shuffle(w, "bfly", em.value(o, ty.reg), em.get(s), str(step), "0x1f", mask, ty)
        for a in combine:
            emit_assign(w, a)
        step //= 2


def _check_pow2(length: int, what: str, upper: int | None = None) -> None:
    if length < 1 or length & (length - 1) or (upper is not None and length > upper):
        raise ValueError(f"{what} length {length} is not a power of two"
                         + (f" <= {upper}" if upper else ""))


def emit_warp_shuffle(w: "Walker", sh: ir.WarpShuffle) -> None:
    w.em.note(sh.pretty())
    length = int(sh.length)
    _check_pow2(length, "WarpShuffle", WARP)
    ty = dtype_of(sh.dtype, "WarpShuffle")
    butterfly(w, tuple(sh.state), tuple(sh.state_b), tuple(sh.combine_states), length, ty)


def emit_tree_halve(w: "Walker", tree: ir.TreeHalve) -> None:
    em = w.em
    em.note(tree.pretty())
    length = int(tree.length)
    _check_pow2(length, "TreeHalve")
    ty = dtype_of(tree.dtype, "TreeHalve")

    def slot(index) -> tuple:
        if tree.inner is None:
            return (index,)
        var, scale = tree.inner
        return (ir.BinaryExpr("+", ir.BinaryExpr("*", index, ir.Literal(int(scale), "int")), ir.Var(var)),)

    if length <= WARP and tree.inner is None:
        # every lane reads slot (lane % length); the butterfly's lane 0 is the tree root.
        # (With ``inner``, lanes of one warp may belong to different trees: barrier form.)
        lane = em.get("lane")
        idx_name = f"__slot_{tree.tid_var}"
        idx = em.value(idx_name, "b32")
        em.ins(f"and.b32 {idx}, {lane}, {length - 1}")
        for buf, s in zip(tree.bufs, tree.state, strict=True):
            space, addr, _, _ = address.access(w, buf, slot(ir.Var(idx_name)))
            em.ins(f"ld.{space}.{ty.mov} {em.value(s, ty.reg)}, [{addr}]")
        butterfly(w, tuple(tree.state), tuple(tree.state_b), tuple(tree.combine_states), length, ty)
        full = em.tmp("b32")
        em.ins(f"activemask.b32 {full}")
        for s in tree.state:
            r = em.get(s)
            shuffle(w, "idx", r, r, "0", "0x1f", full, ty)
        if w.smem_rewritten(tree.bufs):
            emit_sync(w, ir.Sync(barrier_id=tree.barrier_id, count=tree.barrier_count))
        return

    barrier = ir.Sync(barrier_id=tree.barrier_id, count=tree.barrier_count)
    tid = ir.Var(tree.tid_var)
    step = length // 2
    while step:
        active = expr.pred_operand(w, ir.BinaryExpr("<", tid, ir.Literal(step, "int")))
        skip = em.label("tree_skip")
        em.ins(f"@!{active} bra {skip}")
        partner = ir.BinaryExpr("+", tid, ir.Literal(step, "int"))
        for buf, s, o in zip(tree.bufs, tree.state, tree.state_b, strict=True):
            space, a1, _, _ = address.access(w, buf, slot(tid))
            em.ins(f"ld.{space}.{ty.mov} {em.value(s, ty.reg)}, [{a1}]")
            space, a2, _, _ = address.access(w, buf, slot(partner))
            em.ins(f"ld.{space}.{ty.mov} {em.value(o, ty.reg)}, [{a2}]")
        for a in tree.combine_states:
            emit_assign(w, a)
        for buf, s in zip(tree.bufs, tree.state, strict=True):
            space, a1, _, _ = address.access(w, buf, slot(tid))
            em.ins(f"st.{space}.{ty.mov} [{a1}], {em.get(s)}")
        em.place(skip)
        emit_sync(w, barrier)
        step //= 2
    root = ir.Var(tree.inner[0]) if tree.inner is not None else ir.Literal(0, "int")
    for buf, s in zip(tree.bufs, tree.state, strict=True):
        space, a, _, _ = address.access(w, buf, (root,))
        em.ins(f"ld.{space}.{ty.mov} {em.get(s)}, [{a}]")
