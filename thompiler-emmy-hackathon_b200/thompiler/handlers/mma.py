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
import re
from dataclasses import dataclass
from typing import TYPE_CHECKING

from thompiler import ir
from thompiler.lowering import address, expr
from thompiler.lowering.types import E2M1, F16, F32, FRAGMENT_TYPES, UE8M0, Ty, dtype_of

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
    if ty is UE8M0:                               # block scales: four bytes in one register
        return 1
    if ty is E2M1 and role in ("a", "b"):         # fp4: eight values per register
        return (m * k if role == "a" else k * n) // 256
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
    ty = FRAGMENT_TYPES.get(str(getattr(f.dtype, "name", f.dtype))) or dtype_of(f.dtype, f"RegFragment {f.name}")
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
        raise NotImplementedError(f"{ref}: member {text!r} must fold to a constant when the kernel is compiled")
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
    if ir.is_record(node):
        return any(indexes_fragment(var, getattr(node, f)) for f in node._fields)
    return False


def _lane_expr(op: str, a, n: int):
    return ir.BinaryExpr(op, a, ir.Literal(n, "int"))


def emit_ldmatrix_load(w: "Walker", ld: ir.LdmatrixLoad) -> None:
    em = w.em
    em.note(f"LdmatrixLoad {ld.frag}{' + ' + ld.pair_frag if ld.pair_frag else ''} <- {ld.src_buffer}")
    if fragment_regs(w, ld.frag)[0].ty is E2M1:
        from thompiler.handlers.blockscale import emit_ldmatrix_fp4
        emit_ldmatrix_fp4(w, ld)
        return
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
            raise ValueError("an x4 ldmatrix of B fills exactly two fragments, not one")
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
    if mma.block_scaled:
        from thompiler.handlers.blockscale import emit_block_scaled_mma
        emit_block_scaled_mma(w, mma)
        return
    if shape != (16, 8, 16) or mma.ab_dtype not in ("f16", "bf16") or mma.c_dtype not in ("f32", "f16"):
        raise NotImplementedError(f"MmaSyncPtx m{shape[0]}n{shape[1]}k{shape[2]} {mma.ab_dtype}->{mma.c_dtype}")
    if mma.b_row_major:
        raise NotImplementedError("MmaSyncPtx with a row-major B (Volta)")
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


EPILOGUE_STMTS = (ir.Load, ir.Assign, ir.Let, ir.Select)


def _param_name(p) -> str:
    name = p.name if isinstance(p, ir.Var) else p
    if not isinstance(name, str):
        raise ValueError(f"Lambda parameter {p!r}")
    return name


def _epilogue_value(w: "Walker", lam: ir.Lambda, elems: list[str], row: str, col: str) -> tuple[str, Ty]:
    """One fragment element through a RegStore epilogue: the Lambda's leading parameters are bound
    to ``elems`` (the element of the stored fragment, then the same element of each extra
    fragment); two further parameters, when declared, to the element's destination row and
    column (s32).  The body (Load / Assign / Let / Select) is lowered for this element, and the
    register of its one result is returned with the result's type."""
    em = w.em
    params = [_param_name(p) for p in lam.params]
    if len(params) not in (len(elems), len(elems) + 2):
        raise ValueError(f"RegStore epilogue takes {len(params)} parameters for {len(elems)} fragments "
                         f"(one per fragment, optionally then row and column)")
    for name, reg in zip(params, elems):
        em.ins(f"mov.f32 {em.value(name, 'f32')}, {reg}")
    if len(params) == len(elems) + 2:
        em.ins(f"mov.s32 {em.value(params[-2], 'b32')}, {row}")
        em.ins(f"mov.s32 {em.value(params[-1], 'b32')}, {col}")
    for s in lam.body:
        if not isinstance(s, EPILOGUE_STMTS):
            kind = s.kind if isinstance(s, ir.Opaque) else type(s).__name__
            raise NotImplementedError(f"RegStore epilogue statement {kind} (only Load, Assign, Let, Select)")
        w.stmt(s)
    results = [_param_name(r) for r in lam.results]
    if len(results) != 1:
        raise NotImplementedError(f"RegStore epilogue with {len(results)} results")
    reg = em.get(results[0])
    cls = em.named[reg]
    if cls not in ("f32", "b16"):
        raise TypeError(f"RegStore epilogue result {results[0]} is a .{cls} value, not a float")
    out = em.tmp(cls)            # the result's name is rebound by the next element's evaluation
    em.ins(f"mov.{'f32' if cls == 'f32' else 'b16'} {out}, {reg}")
    return out, (F32 if cls == "f32" else F16)


def _to(w: "Walker", reg: str, have: Ty, want: Ty) -> str:
    if have is want:
        return reg
    out = w.em.tmp(want.reg)
    w.em.ins(f"{'cvt.rn.f16.f32' if want is F16 else 'cvt.f32.f16'} {out}, {reg}")
    return out


def _plus(addr: str, nbytes: int) -> str:
    base, _, off = addr.partition("+")
    return f"{base}+{int(off or 0) + nbytes}"


def _reg_store_shared(w: "Walker", st: ir.RegStore) -> None:
    """A C fragment into a shared array (row-major by its extents, after ``swizzle``: the layout
    ldmatrix and cp.async read with the same mode), as f32 or rounded to f16 -- e.g. a product
    staged for the next MMA's A operand.  Each register pair is one 8- (f32) or 4-byte (f16
    pair) store: its two columns share a swizzle chunk."""
    em = w.em
    arr = w.smem[st.dst_buffer]
    if st.epilogue is not None or st.extra_frags or st.m_guard is not None or st.n_guard is not None or st.atomic:
        raise NotImplementedError("RegStore into shared memory: epilogues, guards and atomics are for global outputs")
    shape = tuple(int(x) for x in st.shape)
    if shape != (16, 8, 16):
        raise NotImplementedError(f"RegStore of shape {st.shape} into shared memory")
    if arr.ty not in (F32, F16):
        raise NotImplementedError(f"RegStore into a {arr.ty.name} shared array")
    frag, regs = fragment_regs(w, st.frag)
    if frag.role != "c" or frag.ty is not F32 or len(regs) != 4:
        raise ValueError(f"RegStore of {st.frag}: not an f32 m16n8 accumulator")
    index = list(st.dst_index)
    if len(index) != len(arr.extents):
        raise ValueError(f"RegStore to {arr.name}: {len(index)}-d index for a {len(arr.extents)}-d array")
    lane = ir.Var("lane")
    g = _lane_expr("/", lane, 4)
    col = _lane_expr("*", _lane_expr("%", lane, 4), 2)
    for dr in (0, 8):
        idx = list(index)
        idx[-2] = ir.BinaryExpr("+", index[-2], g if dr == 0 else _lane_expr("+", g, dr))
        idx[-1] = ir.BinaryExpr("+", index[-1], col)
        flat = address.flat_index(w, arr.extents, tuple(idx), arr.name)
        addr = address.shared_element_address(w, arr, flat, st.swizzle or "NONE")
        lo, hi = regs[2 if dr else 0], regs[3 if dr else 1]
        if arr.ty is F32:
            em.ins(f"st.shared.v2.f32 [{addr}], {{{lo}, {hi}}}")
        else:
            packed = em.tmp("b32")
            em.ins(f"cvt.rn.f16x2.f32 {packed}, {hi}, {lo}")
            em.ins(f"st.shared.b32 [{addr}], {packed}")


def emit_reg_store(w: "Walker", st: ir.RegStore) -> None:
    """A C fragment (an m16n8 ``mma.sync`` accumulator or an m64nN warpgroup one) to global
    memory, each lane storing its registers at the rows and columns of the accumulator layout.

    Plain form: a two-element store per register pair (``st.global.v2.f32``, or one f16x2 word
    for an f16 buffer).  Fused form, when any of these is given:

    * ``epilogue``: an ``ir.Lambda`` evaluated per element (``_epilogue_value``), its result
      rounded to the buffer's type: the fused pointwise tail of TASK.md:159 of the IR
      reference;
    * ``extra_frags``: further accumulators of the same geometry whose same element is passed
      to the epilogue;
    * ``m_guard`` / ``n_guard``: the element is stored only where its destination row is below
      ``m_guard`` and its column below ``n_guard`` (exclusive bounds on the destination
      coordinates; ragged edges of M and N);
    * ``atomic``: ``red.global.add`` of each element instead of a store (split-K partial sums).

    Guarded and atomic stores, and rows of an odd length, go element by element; an epilogue
    alone keeps the pair stores."""
    em = w.em
    em.note(f"RegStore {st.dst_buffer} <- {st.frag}")
    if st.fragment_layout not in ("m16n8k16", "m64nNk16") or st.volta_interleaved:
        raise NotImplementedError("RegStore form: Volta (interleaved) layout, which no MMA of this backend produces")
    if st.dst_buffer in w.smem:
        _reg_store_shared(w, st)
        return
    if st.swizzle not in ("NONE", None):
        raise NotImplementedError(f"RegStore with swizzle {st.swizzle} into global memory (shared arrays only)")
    if st.epilogue is not None and not isinstance(st.epilogue, ir.Lambda):
        raise NotImplementedError(f"RegStore epilogue {type(st.epilogue).__name__} (a Lambda expected)")
    if st.extra_frags and st.epilogue is None:
        raise ValueError("RegStore extra_frags without an epilogue to read them")
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
    extra = []
    for ref in st.extra_frags:
        f2, r2 = fragment_regs(w, ref)
        if f2.role != "c" or f2.ty is not F32 or len(r2) != want:
            raise ValueError(f"RegStore extra fragment {ref}: not an f32 accumulator of {want} registers")
        extra.append(r2)
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
    guarded = st.m_guard is not None or st.n_guard is not None
    wants_coords = st.epilogue is not None and len(st.epilogue.params) == 1 + len(extra) + 2
    # a pair store needs the pair's first element at an even offset: an odd row stride goes element by element
    by_element = guarded or st.atomic or row_stride % 2 == 1
    lane = ir.Var("lane")
    g = _lane_expr("/", lane, 4)
    if wide:                     # a warpgroup accumulator: warp q of the group holds rows 16q..16q+15
        g = ir.BinaryExpr("+", g, _lane_expr("*", _lane_expr("%", ir.Var("warp"), 4), 16))
    col = _lane_expr("*", _lane_expr("%", lane, 4), 2)
    for i in range(len(regs) // 4):
        for dr in (0, 8):
            k = 4 * i + (2 if dr else 0)
            row_e = ir.BinaryExpr("+", st.dst_index[rdim], g if dr == 0 else _lane_expr("+", g, dr))
            col_e = ir.BinaryExpr("+", st.dst_index[cdim], col if i == 0 else _lane_expr("+", col, 8 * i))
            idx = list(index)
            idx[rdim], idx[cdim] = row_e, col_e
            addr = address.global_address(w, p, tuple(idx))
            row_r = col_r = None
            if wants_coords:
                row_r, col_r = expr.int_operand(w, row_e), expr.int_operand(w, col_e)
            vals = []
            for j in (0, 1):
                v, ty = regs[k + j], F32
                if st.epilogue is not None:
                    c_j = col_r
                    if j and wants_coords:
                        c_j = em.tmp("b32")
                        em.ins(f"add.s32 {c_j}, {col_r}, 1")
                    v, ty = _epilogue_value(w, st.epilogue, [v] + [r[k + j] for r in extra], row_r, c_j)
                vals.append((v, ty))
            if not by_element:
                if p.ty is F32:
                    lo, hi = (_to(w, v, ty, F32) for v, ty in vals)
                    em.ins(f"st.global.v2.f32 [{addr}], {{{lo}, {hi}}}")
                    continue
                packed = em.tmp("b32")
                if vals[0][1] is F32 and vals[1][1] is F32:
                    em.ins(f"cvt.rn.f16x2.f32 {packed}, {vals[1][0]}, {vals[0][0]}")
                else:
                    lo, hi = (_to(w, v, ty, F16) for v, ty in vals)
                    em.ins(f"mov.b32 {packed}, {{{lo}, {hi}}}")
                em.ins(f"st.global.b32 [{addr}], {packed}")
                continue
            vals = [_to(w, v, ty, p.ty) for v, ty in vals]
            row_ok = None
            if st.m_guard is not None:
                row_ok = expr.pred_operand(w, ir.BinaryExpr("<", row_e, st.m_guard))
            for j in (0, 1):
                pred = row_ok
                if st.n_guard is not None:
                    col_j = col_e if j == 0 else ir.BinaryExpr("+", col_e, ir.Literal(1, "int"))
                    col_ok = expr.pred_operand(w, ir.BinaryExpr("<", col_j, st.n_guard))
                    if pred is None:
                        pred = col_ok
                    else:
                        both = em.tmp("pred")
                        em.ins(f"and.pred {both}, {row_ok}, {col_ok}")
                        pred = both
                at = addr if j == 0 else _plus(addr, p.ty.nbytes)
                guard = f"@{pred} " if pred is not None else ""
                if st.atomic:
                    op = "red.global.add.f32" if p.ty is F32 else "red.global.add.noftz.f16"
                else:
                    op = "st.global.f32" if p.ty is F32 else "st.global.b16"
                em.ins(f"{guard}{op} [{at}], {vals[j]}")
