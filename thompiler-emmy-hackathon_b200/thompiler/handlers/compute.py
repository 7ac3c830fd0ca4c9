"""Leaf statements that read, compute and write: Load, Assign, Let, Write.

Load / Write move one value or a group of consecutive values (a vector
access of at most 16 bytes).  Global reads of buffers the kernel never
writes go through the read-only non-coherent path (``ld.global.nc``).
Assign lowers one elementwise op with ``.rn`` arithmetic (bit-exact against
CPU float math), ``exp`` as ``ex2.approx(x * log2 e)`` (the reference's
lowering, thompiler/handlers/compute.py:77-83 of the reference), ``relu`` as
``max(x, 0)``, and a change of dtype (spelled ``copy``) as ``cvt``.
f16 values compute natively where sm_100a has the instruction and through
f32 otherwise.
"""

from __future__ import annotations

import math
from typing import TYPE_CHECKING

from thompiler import ir
from thompiler.lowering import address, expr, ops
from thompiler.lowering.types import F16, F32, I32, REG_VALUE_TYPE, Ty, dtype_of

if TYPE_CHECKING:
    from thompiler.walk import Walker

MAX_VECTOR_BYTES = 16
LOG2_E = math.log2(math.e)


def check_vector(width: int, ty: Ty, what: str) -> None:
    if width not in (1, 2, 4) and not (ty.nbytes == 2 and width == 8):
        raise NotImplementedError(f"{what}: vector of width {width}")
    if width > 1 and width * ty.nbytes > MAX_VECTOR_BYTES:
        raise NotImplementedError(f"{what}: {width} x {ty.name} is over {MAX_VECTOR_BYTES} bytes")


def emit_load(w: "Walker", load: ir.Load) -> None:
    em = w.em
    em.note(load.pretty())
    if w.load_hook is not None and w.load_hook(w, load):
        return
    space, addr, ty, readonly = address.access(w, load.input, load.index)
    width = len(load.names)
    check_vector(width, ty, f"Load from {load.input}")
    regs = [em.value(n, ty.reg) for n in load.names]
    op = "ld.global.nc" if (space == "global" and readonly) else f"ld.{space}"
    if width == 1:
        em.ins(f"{op}.{ty.mov} {regs[0]}, [{addr}]")
    else:
        em.ins(f"{op}.v{width}.{ty.mov} {{{', '.join(regs)}}}, [{addr}]")


def arg_type(w: "Walker", name: str) -> Ty:
    return REG_VALUE_TYPE[w.em.cls_of(name)]


def apply_op(w: "Walker", op: str, dst: str, args: list[str], ty: Ty) -> None:
    """dst = op(args) on values of type ``ty`` (dst already declared)."""
    em = w.em
    if ty is F16 and not ops.f16_native(op) and op not in ("relu",):
        # no f16 instruction: widen, compute in f32, round back once
        wide = [em.tmp("f32") for _ in args]
        for r, a in zip(wide, args):
            em.ins(f"cvt.f32.f16 {r}, {a}")
        out = em.tmp("f32")
        apply_op(w, op, out, wide, F32)
        em.ins(f"cvt.rn.f16.f32 {dst}, {out}")
        return
    if op == "relu":
        if ty is F16:
            zero = em.tmp("b16")
            em.ins(f"mov.b16 {zero}, 0x0000")
            em.ins(f"max.f16 {dst}, {args[0]}, {zero}")
        else:
            em.ins(f"{ops.instruction(ops.BINARY, 'maximum', ty)} {dst}, {args[0]}, {ty.imm(0)}")
        return
    if op == "exp":
        if ty is not F32:
            raise NotImplementedError(f"exp on {ty.name} values")
        t = em.tmp("f32")
        em.ins(f"mul.rn.f32 {t}, {args[0]}, {F32.imm(LOG2_E)}")
        em.ins(f"ex2.approx.f32 {dst}, {t}")
        return
    if op in ops.UNARY:
        em.ins(f"{ops.instruction(ops.UNARY, op, ty)} {dst}, {args[0]}")
        return
    if op in ops.BINARY:
        em.ins(f"{ops.instruction(ops.BINARY, op, ty)} {dst}, {args[0]}, {args[1]}")
        return
    raise NotImplementedError(f"operation {op!r}")


def emit_assign(w: "Walker", a: ir.Assign) -> None:
    em = w.em
    em.note(a.pretty())
    op = a.op.name
    if len(a.args) != a.op.arity:
        raise ValueError(f"{op} takes {a.op.arity} args, got {a.args}")
    tys = {arg_type(w, x) for x in a.args}
    if len(tys) != 1:
        raise TypeError(f"Assign {a.name}: args of mixed types {sorted(t.name for t in tys)}")
    (ty,) = tys
    out_ty = ty if a.dtype is None else dtype_of(a.dtype, f"Assign {a.name}")
    args = [em.get(x) for x in a.args]
    if out_ty != ty:
        if op != "copy":
            raise TypeError(f"Assign {a.name}: {op} on {ty.name} args with a {out_ty.name} result")
        em.ins(f"{ops.convert(ty, out_ty)} {em.value(a.name, out_ty.reg)}, {args[0]}")
        return
    dst = em.value(a.name, ty.reg)
    apply_op(w, op, dst, args, ty)


def emit_write(w: "Walker", wr: ir.Write) -> None:
    em = w.em
    em.note(wr.pretty())
    if w.write_hook is not None and w.write_hook(w, wr):
        return
    width = len(wr.values)
    if wr.atomic and width != 1:
        raise NotImplementedError(f"atomic Write of width {width}")
    values = [em.get(v) for v in wr.values]
    space, addr, ty, _ = address.access(w, wr.output, wr.index, wr.swizzle)
    check_vector(width, ty, f"Write to {wr.output}")
    vtys = {arg_type(w, v) for v in wr.values}
    if vtys != {ty}:
        raise TypeError(f"Write to {ty.name} buffer {wr.output} of {sorted(t.name for t in vtys)} values")
    if wr.atomic:
        if space != "global":
            raise NotImplementedError(f"atomic Write to shared array {wr.output}")
        suffix = "noftz.f16" if ty is F16 else ty.ptx
        em.ins(f"red.global.add.{suffix} [{addr}], {values[0]}")
    elif width == 1:
        em.ins(f"st.{space}.{ty.mov} [{addr}], {values[0]}")
    else:
        em.ins(f"st.{space}.v{width}.{ty.mov} [{addr}], {{{', '.join(values)}}}")


def emit_let(w: "Walker", let: ir.Let) -> None:
    em = w.em
    em.note(let.pretty())
    v = let.value
    if isinstance(v, ir.FlatIndex):
        # the row-major element offset of a coordinate, against the buffer's (or Smem array's) shape
        p = w.kernel.param(v.buffer)
        shape = tuple(p.shape) if p is not None else (w.smem[v.buffer].extents if v.buffer in w.smem else None)
        if shape is None:
            raise ValueError(f"Let {let.name}: FlatIndex of unknown buffer {v.buffer}")
        if not shape:
            shape = (1,)
        off = address.flat_index(w, tuple(int(x) for x in shape), tuple(v.index), v.buffer)
        em.ins(f"mov.s32 {em.value(let.name, 'b32')}, {off}")
        return
    if isinstance(v, ir.Literal) and v.dtype == "float":
        ty = dtype_of(let.dtype, f"Let {let.name}")
        em.ins(f"mov.{ty.mov} {em.value(let.name, ty.reg)}, {ty.imm(float(v.value))}")
        return
    if expr.value_type(w, v) is I32:
        if let.dtype is not None and getattr(let.dtype, "name", let.dtype) not in ("i32", "int32"):
            raise NotImplementedError(f"Let {let.name} of integer dtype {let.dtype}")
        val = expr.int_operand(w, v)
        em.ins(f"mov.s32 {em.value(let.name, 'b32')}, {val}")
        return
    raise NotImplementedError(f"Let {let.name} = {ir.pretty(v)}")


def _branch_fields(b) -> tuple:
    """(value, select) of a Select arm: a Branch, any constructor with those fields, or a pair."""
    if isinstance(b, ir.Branch):
        return b.value, b.select
    if isinstance(b, ir.Opaque):
        f = {k: v for k, v in b.fields if isinstance(k, str)}
        if "value" in f:
            return f["value"], f.get("select")
    if isinstance(b, tuple) and len(b) == 2:
        return b
    raise NotImplementedError(f"Select branch {b!r}")


def emit_select(w: "Walker", s: ir.Select) -> None:
    """``name`` = the value of the first branch whose predicate holds (the last branch when
    none does): a chain of ``selp`` from the last branch back to the first."""
    em = w.em
    em.note(s.pretty())
    arms = [_branch_fields(b) for b in s.branches]
    if not arms:
        raise ValueError(f"Select {s.name} has no branches")

    def operand(v):
        if isinstance(v, str):
            return em.get(v), arg_type(w, v)
        if isinstance(v, ir.Var) and v.name not in w.consts:
            return em.get(v.name), arg_type(w, v.name)
        if isinstance(v, ir.Literal) and v.dtype == "float":
            return F32.imm(float(v.value)), F32
        return expr.int_operand(w, v), I32

    vals = [operand(v) for v, _ in arms]
    tys = {t for _, t in vals}
    if len(tys) != 1:
        raise TypeError(f"Select {s.name}: branches of mixed types {sorted(t.name for t in tys)}")
    (ty,) = tys
    cur = vals[-1][0]
    for (v, sel), (op, _) in zip(reversed(arms[:-1]), reversed(vals[:-1])):
        if sel is None:
            cur = op
            continue
        pr = expr.pred_operand(w, sel)
        nxt = em.tmp(ty.reg)
        em.ins(f"selp.{ty.reg} {nxt}, {op}, {cur}, {pr}")
        cur = nxt
    dst = em.value(s.name, ty.reg)
    em.ins(f"mov.{ty.mov} {dst}, {cur}")


def emit_zero_prologue(w: "Walker", z: ir.ZeroPrologue) -> None:
    """Zero ``words`` 32-bit words of buffer ``dst`` (another kernel's atomic accumulator) with a
    grid-stride loop over every thread of the launch."""
    em = w.em
    em.note(z.pretty())
    p = w.kernel.param(z.dst)
    if p is None:
        raise ValueError(f"ZeroPrologue: {z.dst} is not a kernel buffer")
    words = expr.int_operand(w, z.words)
    if expr.is_imm(words) and int(words) * 4 > p.nelems * p.ty.nbytes:
        raise ValueError(f"ZeroPrologue: {words} words overrun {z.dst} ({p.nelems * p.ty.nbytes} bytes)")
    gid, stride, a = em.tmp("b32"), em.tmp("b32"), em.tmp("b32")
    em.ins(f"mov.u32 {gid}, %ctaid.x")
    em.ins(f"mov.u32 {a}, %ntid.x")
    t = em.tmp("b32")
    em.ins(f"mov.u32 {t}, %tid.x")
    em.ins(f"mad.lo.u32 {gid}, {gid}, {a}, {t}")
    em.ins(f"mov.u32 {stride}, %nctaid.x")
    em.ins(f"mul.lo.u32 {stride}, {stride}, {a}")
    top, done = em.label("zp"), em.label("zp_done")
    q = em.tmp("pred")
    em.place(top)
    em.ins(f"setp.ge.u32 {q}, {gid}, {words}")
    em.ins(f"@{q} bra {done}")
    ad = em.tmp("b64")
    em.ins(f"mad.wide.u32 {ad}, {gid}, 4, {em.buffer_reg(z.dst)}")
    em.ins(f"st.global.u32 [{ad}], 0")
    em.ins(f"add.u32 {gid}, {gid}, {stride}")
    em.ins(f"bra {top}")
    em.place(done)
