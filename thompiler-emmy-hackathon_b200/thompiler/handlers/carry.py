"""Carried state: Carry, Pre (and Loop.carries).

The IR reference (TASK.md:104-105 of the reference) defines carried state for loops that pass
values from one step to the next (a scan): ``Carry(name, value, index, seed, dtype)`` sets
the next value of cell ``index`` of carrier ``name``; ``Pre(name, carrier, index)`` reads a
cell -- inside the carrying loop the previous step's value (the seed on the first step), after
the loop the final value.  Reads within a step see the previous state, and cells a step does
not set keep their values.  The reference compiler has no lowering for these.

A Carry belongs to its innermost enclosing loop (``Loop.carries``, when the IR lists it, must
name only carriers the body sets).  Every cell (carrier, constant index) of that loop is two
registers: ``cur`` is seeded before the loop, copied to ``next`` when a step starts and
replaced by ``next`` when it ends; ``Carry`` writes ``next``, ``Pre`` reads ``cur``.

A carrier whose cells some Carry or Pre indexes at run time (an index that does not fold to a
constant) keeps its cells in two per-thread ``.local`` arrays instead, ``cur`` and ``next``,
over the index range the expressions can reach: each index coordinate is bounded by interval
arithmetic over the axes it reads (a Tile, Loop or StridedLoop variable of extent E spans 0 ..
E - 1; + - * of bounded terms, / and % by positive constants), and the cells are that box,
flattened row-major.  The same steps apply, element-wise: seed every cell, copy ``cur`` to
``next`` at a step's start and back at its end.  An index the arithmetic cannot bound is
refused at compile time.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING, Any

from thompiler import ir
from thompiler.lowering import expr
from thompiler.lowering.types import F32, I32, REG_VALUE_TYPE, dtype_of

if TYPE_CHECKING:
    from thompiler.walk import Walker


@dataclass(frozen=True)
class StepBegin(ir.Stmt):
    """Internal: the start of one step of a carrying loop (next := cur for its cells)."""
    cells: tuple = ()


@dataclass(frozen=True)
class StepEnd(ir.Stmt):
    """Internal: the end of one step of a carrying loop (cur := next for its cells)."""
    cells: tuple = ()


def _const(w: "Walker", e: Any) -> int:
    if isinstance(e, bool):
        raise NotImplementedError("a boolean carried-state cell index")
    if isinstance(e, int):
        return e
    if isinstance(e, ir.Literal) and isinstance(e.value, int):
        return int(e.value)
    if isinstance(e, ir.Var) and e.name in w.consts:
        return w.consts[e.name]
    if isinstance(e, ir.BinaryExpr) and e.op in ("+", "-", "*", "/", "%"):
        return expr.fold(e.op, _const(w, e.left), _const(w, e.right))
    raise NotImplementedError(f"carried-state cell {ir.pretty(e)}: only indices that fold to a constant are lowered")


def cell_key(w: "Walker", carrier: str, index) -> tuple:
    idx = index if isinstance(index, tuple) else (index,)
    return (carrier, tuple(_const(w, i) for i in idx))


def carries_in(stmts) -> list:
    """The Carry statements a loop with body ``stmts`` owns: those not inside a nested loop (a
    Carry belongs to its innermost enclosing loop)."""
    out = []
    for s in stmts:
        if isinstance(s, ir.Carry):
            out.append(s)
        elif isinstance(s, ir.Cond):
            out += carries_in(s.body) + carries_in(s.else_body)
    return out


def _operand(w: "Walker", v, ty) -> str:
    em = w.em
    if isinstance(v, str):
        return em.get(v)
    if isinstance(v, ir.Var) and v.name not in w.consts:
        return em.get(v.name)
    if isinstance(v, ir.Literal):
        return ty.imm(float(v.value) if ty.is_float else int(v.value))
    if ty is I32:
        return expr.int_operand(w, v)
    raise NotImplementedError(f"carried value {ir.pretty(v)}")


def _folds(w: "Walker", index) -> bool:
    try:
        cell_key(w, "", index)
        return True
    except NotImplementedError:
        return False


def axis_extents(body) -> dict:
    """Extent of every axis variable the kernel declares (Tile, Loop and StridedLoop axes)."""
    out = {}
    for s in ir.walk_stmts(body):
        axes = s.axes if isinstance(s, ir.Tile) else (s.axis,) if isinstance(s, (ir.Loop, ir.StridedLoop)) else ()
        for a in axes:
            try:
                out[a.name] = int(a.size)
            except Exception:               # a dynamic extent bounds nothing
                pass
    return out


def _bounds(w: "Walker", e, extents: dict):
    """(lo, hi) an integer index expression can take, or None when it cannot be bounded."""
    if isinstance(e, bool):
        return None
    if isinstance(e, int):
        return e, e
    if isinstance(e, ir.Literal) and isinstance(e.value, int) and not isinstance(e.value, bool):
        return int(e.value), int(e.value)
    if isinstance(e, ir.Var):
        if e.name in w.consts:
            return w.consts[e.name], w.consts[e.name]
        n = extents.get(e.name)
        return (0, n - 1) if n else None
    if isinstance(e, ir.BinaryExpr) and e.op in ("+", "-", "*", "/", "%"):
        a, b = _bounds(w, e.left, extents), _bounds(w, e.right, extents)
        if a is None or b is None:
            return None
        if e.op == "+":
            return a[0] + b[0], a[1] + b[1]
        if e.op == "-":
            return a[0] - b[1], a[1] - b[0]
        if e.op == "*":
            v = [a[i] * b[j] for i in (0, 1) for j in (0, 1)]
            return min(v), max(v)
        if b[0] != b[1] or b[0] <= 0 or a[0] < 0:     # / and % by a positive constant of a non-negative
            return None
        if e.op == "/":
            return a[0] // b[0], a[1] // b[0]
        return (a[0], a[1]) if a[1] < b[0] else (0, b[0] - 1)
    return None


class LocalCells:
    """A run-time indexed carrier: ``cur`` and ``next`` per-thread .local arrays over a box of cells."""

    def __init__(self, w: "Walker", name: str, ty, lo: tuple, hi: tuple):
        self.name, self.ty, self.lo = name, ty, lo
        self.shape = tuple(h - l + 1 for l, h in zip(lo, hi))
        self.n = 1
        for d in self.shape:
            self.n *= d
        em, size = w.em, max(ty.nbytes, 4)
        self.stride = size
        self.arrays = []
        for part in ("cur", "next"):
            arr = f"thl_{name}_{part}"
            em.local(f".local .align 8 .b8 {arr}[{self.n * size}]")
            base = em.tmp("b64")
            em.ins(f"mov.u64 {base}, {arr}")
            self.arrays.append(base)

    def address(self, w: "Walker", index, part: int) -> str:
        em = w.em
        idx = index if isinstance(index, tuple) else (index,)
        if len(idx) != len(self.shape):
            raise ValueError(f"carrier {self.name}: a {len(idx)}-d index for {len(self.shape)}-d cells")
        flat = None
        for e, lo, extent in zip(idx, self.lo, self.shape):
            term = expr.int_operand(w, ir.BinaryExpr("-", e, ir.Literal(lo, "int")))
            if flat is None:
                flat = term
            else:
                f2 = em.tmp("b32")
                em.ins(f"mad.lo.s32 {f2}, {flat}, {extent}, {term}")
                flat = f2
        off, addr = em.tmp("b64"), em.tmp("b64")
        em.ins(f"mul.wide.s32 {off}, {flat}, {self.stride}")
        em.ins(f"add.u64 {addr}, {self.arrays[part]}, {off}")
        return addr

    def copy(self, w: "Walker", src: int, dst: int) -> None:
        em, t = w.em, self.ty
        v = em.tmp(t.reg)
        for i in range(self.n):
            em.ins(f"ld.local.{t.mov} {v}, [{self.arrays[src]}+{i * self.stride}]")
            em.ins(f"st.local.{t.mov} [{self.arrays[dst]}+{i * self.stride}], {v}")


def open_cells(w: "Walker", loop) -> tuple:
    """Declare and seed the cells of a carrying loop; the (begin, end) markers for its body."""
    carriers = set(getattr(loop, "carries", ()) or ())
    em = w.em
    w.carry_cells = getattr(w, "carry_cells", {})
    w.carry_local = getattr(w, "carry_local", {})
    owned = carries_in(loop.body)
    # carriers with a run-time index anywhere in the kernel: cells in .local arrays
    dynamic = {c.name for c in owned if not _folds(w, c.index)}
    dynamic |= {p.carrier for p in ir.walk_stmts(w.kernel.body) if isinstance(p, ir.Pre)
                and p.carrier in {c.name for c in owned} and not _folds(w, p.index)}
    local_keys = []
    if dynamic:
        extents = axis_extents(w.kernel.body)
        for name in sorted(dynamic):
            refs = [c.index for c in owned if c.name == name]
            refs += [p.index for p in ir.walk_stmts(w.kernel.body) if isinstance(p, ir.Pre) and p.carrier == name]
            boxes = []
            for index in refs:
                idx = index if isinstance(index, tuple) else (index,)
                bs = [_bounds(w, e, extents) for e in idx]
                if any(b is None for b in bs):
                    raise NotImplementedError(
                        f"carried-state cell {name}[{', '.join(ir.pretty(e) for e in idx)}]: a run-time index "
                        "must be bounded by axis extents (+ - * and / % by constants)")
                boxes.append(bs)
            if len({len(b) for b in boxes}) != 1:
                raise ValueError(f"carrier {name} indexed with different ranks")
            lo = tuple(min(b[d][0] for b in boxes) for d in range(len(boxes[0])))
            hi = tuple(max(b[d][1] for b in boxes) for d in range(len(boxes[0])))
            c0 = next(c for c in owned if c.name == name)
            ty = dtype_of(c0.dtype, f"Carry {name}") if c0.dtype is not None else F32
            cells = LocalCells(w, name, ty, lo, hi)
            seed = c0.seed if c0.seed is not None else ir.Literal(0.0 if ty.is_float else 0,
                                                                  "float" if ty.is_float else "int")
            sv = em.tmp(ty.reg)
            em.ins(f"mov.{ty.mov} {sv}, {_operand(w, seed, ty)}")
            for i in range(cells.n):
                em.ins(f"st.local.{ty.mov} [{cells.arrays[0]}+{i * cells.stride}], {sv}")
            w.carry_local[name] = cells
            local_keys.append(("local", name))
    cells = {}
    for c in owned:
        if c.name in dynamic:
            continue
        key = cell_key(w, c.name, c.index)
        if key in cells:
            continue
        ty = dtype_of(c.dtype, f"Carry {c.name}") if c.dtype is not None else F32
        cells[key] = (c, ty)
    missing = carriers - {k[0] for k in cells} - dynamic
    if missing:
        raise ValueError(f"loop over {loop.axis.name} carries {sorted(missing)} but never sets them")
    keys = list(local_keys)
    for key, (c, ty) in cells.items():
        tag = "_".join(str(i) for i in key[1]) or "s"
        cur = em.value(f"{key[0]}__cell_{tag}", ty.reg)
        nxt = em.tmp(ty.reg)
        seed = c.seed if c.seed is not None else ir.Literal(0.0 if ty.is_float else 0, "float" if ty.is_float else "int")
        em.ins(f"mov.{ty.mov} {cur}, {_operand(w, seed, ty)}")
        w.carry_cells[key] = (cur, nxt, ty)
        keys.append(key)
    return StepBegin(tuple(keys)), StepEnd(tuple(keys))


def emit_step_begin(w: "Walker", s: StepBegin) -> None:
    for key in s.cells:
        if key[0] == "local":
            w.carry_local[key[1]].copy(w, 0, 1)
            continue
        cur, nxt, ty = w.carry_cells[key]
        w.em.ins(f"mov.{ty.mov} {nxt}, {cur}")


def emit_step_end(w: "Walker", s: StepEnd) -> None:
    for key in s.cells:
        if key[0] == "local":
            w.carry_local[key[1]].copy(w, 1, 0)
            continue
        cur, nxt, ty = w.carry_cells[key]
        w.em.ins(f"mov.{ty.mov} {cur}, {nxt}")


def emit_carry(w: "Walker", c: ir.Carry) -> None:
    em = w.em
    em.note(c.pretty())
    local = getattr(w, "carry_local", {}).get(c.name)
    if local is not None:
        v = _operand(w, c.value, local.ty)
        em.ins(f"st.local.{local.ty.mov} [{local.address(w, c.index, 1)}], {v}")
        return
    key = cell_key(w, c.name, c.index)
    cell = getattr(w, "carry_cells", {}).get(key)
    if cell is None:
        raise ValueError(f"Carry {c.name}{list(key[1])} outside a loop that carries {c.name}")
    cur, nxt, ty = cell
    v = _operand(w, c.value, ty)
    if isinstance(c.value, str) and REG_VALUE_TYPE[em.cls_of(c.value)] is not ty:
        raise TypeError(f"Carry {c.name}: a {REG_VALUE_TYPE[em.cls_of(c.value)].name} value into a {ty.name} cell")
    em.ins(f"mov.{ty.mov} {nxt}, {v}")


def emit_pre(w: "Walker", p: ir.Pre) -> None:
    em = w.em
    em.note(p.pretty())
    local = getattr(w, "carry_local", {}).get(p.carrier)
    if local is not None:
        em.ins(f"ld.local.{local.ty.mov} {em.value(p.name, local.ty.reg)}, [{local.address(w, p.index, 0)}]")
        return
    key = cell_key(w, p.carrier, p.index)
    cell = getattr(w, "carry_cells", {}).get(key)
    if cell is None:
        raise ValueError(f"Pre {p.name}: carrier {p.carrier}{list(key[1])} is not carried by an enclosing or "
                         "earlier loop")
    cur, _, ty = cell
    em.ins(f"mov.{ty.mov} {em.value(p.name, ty.reg)}, {cur}")
