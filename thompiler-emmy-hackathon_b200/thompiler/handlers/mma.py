"""Warp-level tensor-core statements: RegFragment, LdmatrixLoad, MmaSyncPtx,
RegStore (the generic lowering; the tuned matmul family replaces whole
kernels of these by tcgen05).  RegFragment and RegStore also take the m64
warpgroup accumulators of the Wgmma* statements (handlers/wgmma.py): N/2
f32 registers per thread, warp q of the group holding rows 16q + g and
16q + g + 8, registers 4i..4i+3 at columns 8i + 2t, 8i + 2t + 1.

A fragment family is ``count`` members of ``nregs`` registers each, named
``%fr_<frag>_<member>_<slot>``.  The IR indexes families by expressions of
unrolled loop variables (``_a0_s[_r0]``), which are constants by the time a
reference is lowered.

Lane geometry.  The m16n8k16 operand layouts are fixed by the PTX ISA
(``mma.sync`` fragment layouts and ``ldmatrix``): with g = lane / 4 and
t = lane % 4, A's register i holds rows g (+8 for i odd) and columns
2t, 2t+1 (+8 for i >= 2); B's register i holds k = 2t, 2t+1 (+8 for i = 1)
at column n = g; C's registers 0,1 are row g, columns 2t, 2t+1 and 2,3 the
same at row g+8.  ``ldmatrix`` hands thread T element (T/4, 2(T%4)+{0,1}) of
matrix i in register i (transposed with ``.trans``), matrix i's eight row
addresses coming from lanes 8i..8i+7.  Solving for the row each lane must
address gives, per form (and the same table as the reference's
thompiler/handlers/mma.py:129-199, since both follow from the ISA):

  A 16x16                    x4        row lane%16,               col 8*(lane/16)
  B pair, smem [K][N]        x4.trans  row lane%16,               col 8*(lane/16)
  B pair, smem [N][K]        x4        row lane%8 + 8*(lane/16),  col 8*((lane/8)%2)
  B single, smem [N][K]      x2        row lane%8,                col 8*((lane/8)%2)
  B single, smem [K][N]      x2.trans  row lane%16,               col 0
"""

from __future__ import annotations

import ast
import dataclasses
import re
from dataclasses import dataclass
from typing import TYPE_CHECKING

from thompiler import ir
from thompiler.lowering import address, expr
from thompiler.lowering.types import F16, F32, Ty, dtype_of

if TYPE_CHECKING:
    from thompiler.walk import Walker

REF = re.compile(r"^(?P<name>\w+)(?:\[(?P<index>[^\]]+)\])?$")


@dataclass
class Fragment:
    name: str
    role: str
    ty: Ty
    count: int
    nregs: int
    cls: str       # register class: f32 for an f32 accumulator, else b32 (packed halves)

    def regs(self, member: int) -> list[str]:
        return [f"%fr_{self.name}_{member}_{s}" for s in range(self.nregs)]


def operand_regs(role: str, shape: tuple, ty: Ty) -> int:
    m, n, k = shape
    if role in ("a", "b"):
        if ty.nbytes != 2:
            raise NotImplementedError(f"mma operand {role} of {ty.name}")
        return (m * k if role == "a" else k * n) // 64
    if role == "c":
        threads = 128 if m == 64 else 32          # an m64 accumulator spans a warpgroup (wgmma)
        return (m * n) // (threads * (2 if ty.nbytes == 2 else 1))
    raise ValueError(f"mma role {role!r}")


def emit_reg_fragment(w: "Walker", f: ir.RegFragment) -> None:
    em = w.em
    em.note(f"RegFragment {f.role}:{getattr(f.dtype, 'name', f.dtype)} {f.name}[{f.count}]")
    if f.name in w.fragments:
        raise ValueError(f"fragment {f.name} declared twice")
    ty = dtype_of(f.dtype, f"RegFragment {f.name}")
    shape = tuple(int(x) for x in f.shape)
    nregs = int(f.nregs) if f.nregs else operand_regs(f.role, shape, ty)
    cls = "f32" if (f.role == "c" and ty is F32) else "b32"
    frag = Fragment(f.name, f.role, ty, int(f.count), nregs, cls)
    w.fragments[f.name] = frag
    for m in range(frag.count):
        for r in frag.regs(m):
            em.declare(r, cls)
            if f.role == "c":
                em.ins(f"mov.{'f32' if cls == 'f32' else 'b32'} {r}, {'0f00000000' if cls == 'f32' else '0'}")
    if f.role == "c":
        from thompiler.handlers.wgmma import fragment_written
        fragment_written(w, f.name)


def _const_index(w: "Walker", text: str, ref: str) -> int:
    def ev(node: ast.AST) -> int:
        if isinstance(node, ast.Constant) and isinstance(node.value, int):
            return node.value
        if isinstance(node, ast.Name) and node.id in w.consts:
            return w.consts[node.id]
        if isinstance(node, ast.BinOp) and isinstance(node.op, (ast.Add, ast.Sub, ast.Mult)):
            a, b = ev(node.left), ev(node.right)
            return a + b if isinstance(node.op, ast.Add) else a - b if isinstance(node.op, ast.Sub) else a * b
        raise NotImplementedError(f"{ref}: fragment index {text!r} is not a compile-time constant")
    return ev(ast.parse(text, mode="eval").body)


def fragment_regs(w: "Walker", ref: str) -> tuple[Fragment, list[str]]:
    m = REF.match(ref)
    if m is None:
        raise ValueError(f"not a fragment reference: {ref!r}")
    frag = w.fragments.get(m["name"])
    if frag is None:
        raise KeyError(f"fragment {m['name']!r} used before its RegFragment")
    member = 0 if m["index"] is None else _const_index(w, m["index"], ref)
    if not 0 <= member < frag.count:
        raise IndexError(f"{ref}: member {member} of a family of {frag.count}")
    return frag, frag.regs(member)


def indexes_fragment(var: str, node: object) -> bool:
    """Does ``var`` occur in the index of a fragment reference under ``node``?"""
    if isinstance(node, str):
        m = REF.match(node)
        return bool(m and m["index"] and re.search(rf"\b{re.escape(var)}\b", m["index"]))
    if isinstance(node, tuple):
        return any(indexes_fragment(var, x) for x in node)
    if dataclasses.is_dataclass(node) and not isinstance(node, type):
        return any(indexes_fragment(var, getattr(node, f.name)) for f in dataclasses.fields(node))
    return False


def _lane_expr(op: str, a, n: int):
    return ir.BinaryExpr(op, a, ir.Literal(n, "int"))


def emit_ldmatrix_load(w: "Walker", ld: ir.LdmatrixLoad) -> None:
    em = w.em
    em.note(f"LdmatrixLoad {ld.frag}{' + ' + ld.pair_frag if ld.pair_frag else ''} <- {ld.src_buffer}")
    if (not ld.staged or ld.fragment_layout != "m16n8k16" or ld.byte_slab or ld.gmem_guard is not None
            or ld.k_zero is not None or ld.scale_buffer is not None):
        raise NotImplementedError("LdmatrixLoad form: unstaged, guarded, scaled or not m16n8k16")
    arr = w.smem.get(ld.src_buffer)
    if arr is None:
        raise ValueError(f"LdmatrixLoad from {ld.src_buffer!r}, which is not an Smem array")
    if arr.ty.nbytes != 2:
        raise NotImplementedError(f"ldmatrix of {arr.ty.name} elements")
    frag, regs = fragment_regs(w, ld.frag)
    if frag.role != ld.role:
        raise ValueError(f"LdmatrixLoad role {ld.role} into a {frag.role} fragment")
    if ld.pair_frag is not None:
        if ld.role != "b":
            raise ValueError("a paired ldmatrix loads two B fragments")
        regs = regs + fragment_regs(w, ld.pair_frag)[1]
    ldm = int(ld.ldm) or arr.extents[-1]
    lane = ir.Var("lane")
    pair = ld.pair_frag is not None
    if ld.role == "a" or (ld.role == "b" and not ld.b_trans):
        row = _lane_expr("%", lane, 16)
    elif pair:
        row = ir.BinaryExpr("+", _lane_expr("%", lane, 8), _lane_expr("*", _lane_expr("/", lane, 16), 8))
    else:
        row = _lane_expr("%", lane, 8)
    if ld.role == "a" or (pair and not ld.b_trans):
        col = _lane_expr("*", _lane_expr("/", lane, 16), 8)
    elif ld.b_trans:
        col = _lane_expr("*", _lane_expr("%", _lane_expr("/", lane, 8), 2), 8)
    else:
        col = None
    nmat = 4 if (ld.role == "a" or pair) else 2
    trans = ld.role == "b" and not ld.b_trans
    if len(regs) != nmat:
        raise ValueError(f"ldmatrix .x{nmat} into {len(regs)} registers ({ld.frag})")
    offset = _lane_expr("*", row, ldm)
    if col is not None:
        offset = ir.BinaryExpr("+", offset, col)
    base = address.flat_index(w, arr.extents, tuple(ld.src_index), arr.name)
    elem = expr.add_ints(w, base, expr.int_operand(w, offset))
    addr = address.shared_element_address(w, arr, elem, ld.swizzle)
    em.ins(f"ldmatrix.sync.aligned.m8n8.x{nmat}{'.trans' if trans else ''}.shared.b16 "
           f"{{{', '.join(regs)}}}, [{addr}]")


def emit_mma_sync(w: "Walker", mma: ir.MmaSyncPtx) -> None:
    em = w.em
    shape = tuple(int(x) for x in mma.shape)
    em.note(f"MmaSyncPtx {mma.c_frag} += {mma.a_frag} @ {mma.b_frag}")
    if shape != (16, 8, 16) or mma.ab_dtype not in ("f16", "bf16") or mma.c_dtype not in ("f32", "f16"):
        raise NotImplementedError(f"MmaSyncPtx m{shape[0]}n{shape[1]}k{shape[2]} {mma.ab_dtype}->{mma.c_dtype}")
    if mma.b_row_major or mma.block_scaled:
        raise NotImplementedError("MmaSyncPtx with a row-major B (Volta) or block scales")
    ops_ = []
    for role, ref in (("c", mma.c_frag), ("a", mma.a_frag), ("b", mma.b_frag)):
        frag, regs = fragment_regs(w, ref)
        want = mma.c_dtype if role == "c" else mma.ab_dtype
        if frag.role != role or frag.ty.name != want or len(regs) != operand_regs(role, shape, frag.ty):
            raise ValueError(f"MmaSyncPtx operand {role}: {ref} is {len(regs)} x {frag.ty.name} {frag.role}")
        ops_.append("{" + ", ".join(regs) + "}")
    c, a, b = ops_
    ab = mma.ab_dtype
    em.ins(f"mma.sync.aligned.m16n8k16.row.col.{mma.c_dtype}.{ab}.{ab}.{mma.c_dtype} {c}, {a}, {b}, {c}")


def emit_reg_store(w: "Walker", st: ir.RegStore) -> None:
    em = w.em
    em.note(f"RegStore {st.dst_buffer} <- {st.frag}")
    if (st.fragment_layout not in ("m16n8k16", "m64nNk16") or st.volta_interleaved or st.epilogue is not None
            or st.extra_frags or st.m_guard is not None or st.n_guard is not None or st.atomic
            or st.swizzle not in ("NONE", None)):
        raise NotImplementedError("RegStore form: epilogue, guards, atomics, swizzle or Volta layout")
    shape = tuple(int(x) for x in st.shape)
    wide = len(shape) == 3 and shape[0] == 64 and shape[2] == 16 and shape[1] % 8 == 0
    if shape != (16, 8, 16) and not wide:
        raise NotImplementedError(f"RegStore of shape {st.shape}")
    p = w.kernel.param(st.dst_buffer)
    if p is None:
        raise NotImplementedError(f"RegStore to {st.dst_buffer!r}, which is not a kernel parameter")
    if p.ty not in (F32, F16):
        raise NotImplementedError(f"RegStore to a {p.ty.name} buffer")
    frag, regs = fragment_regs(w, st.frag)
    want = shape[1] // 2 if wide else 4
    if frag.role != "c" or frag.ty is not F32 or len(regs) != want:
        raise ValueError(f"RegStore of {st.frag}: not an f32 accumulator of {want} registers")
    index = list(st.dst_index)
    if len(index) < 2:
        raise ValueError(f"RegStore to {st.dst_buffer}: {len(index)}-d index")
    rdim = len(index) - 2 if st.row_dim is None else int(st.row_dim)
    cdim = len(index) - 1 if st.col_dim is None else int(st.col_dim)
    if cdim != len(index) - 1:
        raise NotImplementedError("RegStore with N not on the last dimension")
    row_stride = 1
    for e in p.shape[rdim + 1:]:
        row_stride *= e
    if st.ldm and int(st.ldm) != row_stride:
        raise NotImplementedError(f"RegStore ldm={st.ldm}, but the row stride is {row_stride}")
    lane = ir.Var("lane")
    g = _lane_expr("/", lane, 4)
    if wide:                     # a warpgroup accumulator: warp q of the group holds rows 16q..16q+15
        g = ir.BinaryExpr("+", g, _lane_expr("*", _lane_expr("%", ir.Var("warp"), 4), 16))
    col = _lane_expr("*", _lane_expr("%", lane, 4), 2)
    for dr, dc, (lo, hi) in ((dr, 8 * i, regs[4 * i + (2 if dr else 0):4 * i + (4 if dr else 2)])
                             for i in range(len(regs) // 4) for dr in (0, 8)):
        idx = list(index)
        idx[rdim] = ir.BinaryExpr("+", st.dst_index[rdim], g if dr == 0 else _lane_expr("+", g, dr))
        idx[cdim] = ir.BinaryExpr("+", st.dst_index[cdim], col if dc == 0 else _lane_expr("+", col, dc))
        addr = address.global_address(w, p, tuple(idx))
        if p.ty is F32:
            em.ins(f"st.global.v2.f32 [{addr}], {{{lo}, {hi}}}")
        else:
            packed = em.tmp("b32")
            em.ins(f"cvt.rn.f16x2.f32 {packed}, {hi}, {lo}")
            em.ins(f"st.global.b32 [{addr}], {packed}")
