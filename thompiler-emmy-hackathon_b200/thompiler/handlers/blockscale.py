"""Block-scaled fp4 tensor-core statements: fp4 LdmatrixLoad, BlockScaleLoad and the block-scaled
MmaSyncPtx (m16n8k64, e2m1 x e2m1 with ue8m0 scales per 32 K elements, f32 accumulator).

The IR reference (TASK.md:151-152 of the reference) names these for the block-scaled fp4
``mma.sync`` of sm_120; sm_100a has no block-scaled ``mma.sync`` (its block-scaled MMAs are
``tcgen05.mma`` kinds, CTA-wide with operands in shared and tensor memory), and no shipped
problem or emmy sample fixes the statements' lane conventions.  This backend states them as
follows and lowers the MMA on the FMA pipes of the warp that issues it -- the same result, in
f32, as the hardware's (every dequantised operand, e2m1 x 2^k, is exact in f32).

Fragments (g = lane / 4, t = lane % 4; a 32-bit register holds eight fp4 values, the one for the
lowest k in its lowest nibble -- the order of packed fp4 bytes in memory):
  * A, 16 x 64, four registers: register i holds row g + 8 (i % 2), k = 32 (i / 2) + 8 t .. + 7;
  * B, 64 x 8, two registers: register i holds column g, k = 32 i + 8 t .. + 7;
  * C, 16 x 8 f32, the m16n8 accumulator of the other MMAs (rows g, g + 8; columns 2t, 2t + 1);
  * scales, one register of ue8m0 bytes (value 2^(e - 127); e = 0 is 2^-127, e = 255 NaN):
    for A, bytes (row g, K block 0), (row g, block 1), (row g + 8, block 0), (row g + 8, block
    1); for B, bytes (column g, block 0), (column g, block 1).
``LdmatrixLoad`` of an fp4 fragment reads packed bytes from a byte Smem array with ``ldmatrix``
(.b16 units, four fp4 values each): A as x4 with the lane address row lane % 16, byte column 16
(lane / 16); B stored [N][K/2] as x2 with row lane % 8, byte column 16 ((lane / 8) % 2) -- which
gives exactly the register contents above.  ``BlockScaleLoad(frag, src_buffer, src_index, role,
ldm)`` reads the lane's scale bytes from a byte buffer (a kernel parameter or an Smem array)
laid out [rows][K / 32]: src_index is (first row, first K block) of the 16-row A atom or the
8-column B atom.

The MMA: each lane writes its dequantised operands to a per-warp scratch in shared memory (A 16
x 64 and B 64 x 8 f32, 6 KB per warp), the warp synchronises, and each lane accumulates its
four C elements over k = 0 .. 63 with ``fma.rn.f32``.
"""

from __future__ import annotations

import struct
from typing import TYPE_CHECKING

from thompiler import ir
from thompiler.handlers.mma import _lane_expr, fragment_regs
from thompiler.lowering import address, expr
from thompiler.lowering.types import E2M1, F32, U8, UE8M0

if TYPE_CHECKING:
    from thompiler.walk import Walker

E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
SCRATCH_PER_WARP = (16 * 64 + 64 * 8) * 4
SCRATCH = "thc_bs_scratch"
TABLE = "thc_e2m1"


def _f32_bits(v: float) -> str:
    return "0x%08X" % struct.unpack("<I", struct.pack("<f", v))[0]


def e2m1_value(nibble: int) -> float:
    """The value of one fp4 (e2m1) code: sign bit 3, exponent bits 2-1, mantissa bit 0."""
    v = E2M1_VALUES[nibble & 7]
    return -v if nibble & 8 else v


def emit_ldmatrix_fp4(w: "Walker", ld: ir.LdmatrixLoad) -> None:
    em = w.em
    arr = w.smem.get(ld.src_buffer)
    if arr is None or arr.ty is not U8:
        raise NotImplementedError(f"fp4 LdmatrixLoad from {ld.src_buffer!r}: a byte Smem array expected")
    if ld.pair_frag is not None or ld.b_trans or ld.swizzle not in ("NONE", None):
        raise NotImplementedError("fp4 LdmatrixLoad: paired, transposed or swizzled form")
    frag, regs = fragment_regs(w, ld.frag)
    want = 4 if ld.role == "a" else 2
    if frag.role != ld.role or len(regs) != want:
        raise ValueError(f"fp4 LdmatrixLoad into {ld.frag}: {len(regs)} registers, role {frag.role}")
    ldm = int(ld.ldm) or arr.extents[-1]
    if ldm % 16:
        raise ValueError(f"fp4 LdmatrixLoad: rows of {ldm} bytes are not 16-byte aligned")
    lane = ir.Var("lane")
    if ld.role == "a":
        row, col = _lane_expr("%", lane, 16), _lane_expr("*", _lane_expr("/", lane, 16), 16)
    else:
        row, col = _lane_expr("%", lane, 8), _lane_expr("*", _lane_expr("%", _lane_expr("/", lane, 8), 2), 16)
    offset = ir.BinaryExpr("+", _lane_expr("*", row, ldm), col)
    base = address.flat_index(w, arr.extents, tuple(ld.src_index), arr.name)
    elem = expr.add_ints(w, base, expr.int_operand(w, offset))
    addr = address.shared_element_address(w, arr, elem, "NONE")
    em.ins(f"ldmatrix.sync.aligned.m8n8.x{want}.shared.b16 {{{', '.join(regs)}}}, [{addr}]")


def emit_block_scale_load(w: "Walker", s: ir.BlockScaleLoad) -> None:
    em = w.em
    em.note(f"BlockScaleLoad {s.frag} <- {s.src_buffer}")
    frag, regs = fragment_regs(w, s.frag)
    if frag.ty is not UE8M0 or len(regs) != 1:
        raise ValueError(f"BlockScaleLoad into {s.frag}: not a one-register ue8m0 fragment")
    if s.role not in ("a", "b"):
        raise ValueError(f"BlockScaleLoad role {s.role!r}")
    if len(s.src_index) != 2:
        raise ValueError(f"BlockScaleLoad index {s.src_index}: (first row, first K block) expected")
    lane = ir.Var("lane")
    g = _lane_expr("/", lane, 4)
    r0, k0 = s.src_index
    cells = [(ir.BinaryExpr("+", r0, g), k0), (ir.BinaryExpr("+", r0, g), _lane_expr("+", k0, 1))]
    if s.role == "a":
        g8 = _lane_expr("+", g, 8)
        cells += [(ir.BinaryExpr("+", r0, g8), k0), (ir.BinaryExpr("+", r0, g8), _lane_expr("+", k0, 1))]
    prm, arr = w.kernel.param(s.src_buffer), w.smem.get(s.src_buffer)
    if prm is None and arr is None:
        raise ValueError(f"BlockScaleLoad from {s.src_buffer!r}: no parameter or Smem array of that name")
    ty = prm.ty if prm is not None else arr.ty
    if ty is not U8:
        raise NotImplementedError(f"BlockScaleLoad from a {ty.name} buffer (bytes expected)")
    rows = prm.shape[-1] if prm is not None else arr.extents[-1]
    if s.ldm and int(s.ldm) != rows:
        raise NotImplementedError(f"BlockScaleLoad ldm={s.ldm}, but the buffer's rows hold {rows} scales")
    out = regs[0]
    em.ins(f"mov.b32 {out}, 0")
    for i, idx in enumerate(cells):
        b = em.tmp("b32")
        if prm is not None:
            a = address.global_address(w, prm, idx)
            em.ins(f"ld.global{'.nc' if not prm.written else ''}.u8 {b}, [{a}]")
        else:
            elem = address.flat_index(w, arr.extents, idx, arr.name)
            a = address.shared_element_address(w, arr, elem, "NONE")
            em.ins(f"ld.shared.u8 {b}, [{a}]")
        if i:
            em.ins(f"shl.b32 {b}, {b}, {8 * i}")
        em.ins(f"or.b32 {out}, {out}, {b}")


def _declare_scratch(w: "Walker") -> None:
    em = w.em
    if getattr(w, "_bs_scratch", False):
        return
    threads = max(w.kernel.threads_per_cta,
                  max((int(t.block_threads or 0) for t in ir.walk_stmts(w.kernel.body) if isinstance(t, ir.Tile)),
                      default=0))
    warps = -(-threads // 32)
    em.module(f".shared .align 16 .b8 {SCRATCH}[{warps * SCRATCH_PER_WARP}]")
    table = ", ".join(_f32_bits(e2m1_value(n)) for n in range(16))
    em.module(f".const .align 4 .b32 {TABLE}[16] = {{{table}}}")
    w._bs_scratch = True


def _scale(w: "Walker", word: str, byte: int) -> str:
    """f32 2^(e - 127) of byte ``byte`` of a ue8m0 register (e = 0: 2^-127; e = 255: NaN)."""
    em = w.em
    e, f, p = em.tmp("b32"), em.tmp("b32"), em.tmp("pred")
    em.ins(f"bfe.u32 {e}, {word}, {8 * byte}, 8")
    em.ins(f"shl.b32 {f}, {e}, 23")
    em.ins(f"setp.eq.u32 {p}, {e}, 0")
    em.ins(f"@{p} mov.b32 {f}, 0x00400000")
    em.ins(f"setp.eq.u32 {p}, {e}, 255")
    em.ins(f"@{p} mov.b32 {f}, 0x7FC00000")
    out = em.tmp("f32")
    em.ins(f"mov.b32 {out}, {f}")
    return out


def emit_block_scaled_mma(w: "Walker", mma: ir.MmaSyncPtx) -> None:
    em = w.em
    shape = tuple(int(x) for x in mma.shape)
    if shape != (16, 8, 64) or mma.ab_dtype not in ("e2m1", "fp4") or mma.c_dtype != "f32" or mma.b_row_major:
        raise NotImplementedError(f"block-scaled MmaSyncPtx m{shape[0]}n{shape[1]}k{shape[2]} {mma.ab_dtype}"
                                  f"->{mma.c_dtype} (m16n8k64 e2m1 -> f32 is lowered)")
    c_f, c = fragment_regs(w, mma.c_frag)
    a_f, a = fragment_regs(w, mma.a_frag)
    b_f, b = fragment_regs(w, mma.b_frag)
    if c_f.role != "c" or c_f.ty is not F32 or len(c) != 4:
        raise ValueError(f"block-scaled MmaSyncPtx: {mma.c_frag} is not an m16n8 f32 accumulator")
    if a_f.ty is not E2M1 or len(a) != 4 or b_f.ty is not E2M1 or len(b) != 2:
        raise ValueError(f"block-scaled MmaSyncPtx: {mma.a_frag} / {mma.b_frag} are not fp4 A / B fragments")
    sa_f, sa = fragment_regs(w, mma.sfa_frag)
    sb_f, sb = fragment_regs(w, mma.sfb_frag)
    if sa_f.ty is not UE8M0 or sb_f.ty is not UE8M0:
        raise ValueError("block-scaled MmaSyncPtx: the scale fragments are not ue8m0")
    _declare_scratch(w)
    tid, lane, g, t, base = em.tmp("b32"), em.tmp("b32"), em.tmp("b32"), em.tmp("b32"), em.tmp("b32")
    em.ins(f"mov.u32 {tid}, %tid.x")
    em.ins(f"and.b32 {lane}, {tid}, 31")
    em.ins(f"shr.u32 {g}, {lane}, 2")
    em.ins(f"and.b32 {t}, {lane}, 3")
    em.ins(f"shr.u32 {base}, {tid}, 5")
    em.ins(f"mul.lo.u32 {base}, {base}, {SCRATCH_PER_WARP}")
    sbase = em.tmp("b32")
    em.ins(f"mov.u32 {sbase}, {SCRATCH}")
    em.ins(f"add.u32 {base}, {base}, {sbase}")
    a_s, b_s = base, em.tmp("b32")
    em.ins(f"add.u32 {b_s}, {base}, {16 * 64 * 4}")
    tab = em.tmp("b64")
    em.ins(f"mov.u64 {tab}, {TABLE}")
    scale_a = {(r, kb): _scale(w, sa[0], 2 * r + kb) for r in (0, 1) for kb in (0, 1)}
    scale_b = {kb: _scale(w, sb[0], kb) for kb in (0, 1)}

    def decode(word: str, j: int, scale: str) -> str:
        nib, off, ad = em.tmp("b32"), em.tmp("b64"), em.tmp("b64")
        em.ins(f"bfe.u32 {nib}, {word}, {4 * j}, 4")
        em.ins(f"mul.wide.u32 {off}, {nib}, 4")
        em.ins(f"add.u64 {ad}, {tab}, {off}")
        v = em.tmp("f32")
        em.ins(f"ld.const.f32 {v}, [{ad}]")
        em.ins(f"mul.rn.f32 {v}, {v}, {scale}")
        return v

    # A[row][k] at (row * 64 + k) * 4; this lane's row g + 8 (i % 2), k = 32 (i / 2) + 8 t + j
    t32, g4 = em.tmp("b32"), em.tmp("b32")
    em.ins(f"shl.b32 {t32}, {t}, 5")                   # 8 t floats = 32 t bytes
    em.ins(f"mad.lo.u32 {g4}, {g}, 256, {a_s}")         # row g: 64 floats
    ga = em.tmp("b32")
    em.ins(f"add.u32 {ga}, {g4}, {t32}")
    for i in range(4):
        r, kb = i % 2, i // 2
        off = (8 * r * 64 + 32 * kb) * 4
        for j in range(8):
            em.ins(f"st.shared.f32 [{ga}+{off + 4 * j}], {decode(a[i], j, scale_a[(r, kb)])}")
    # B[k][n] at (k * 8 + n) * 4; this lane's column g, k = 32 i + 8 t + j
    gb = em.tmp("b32")
    em.ins(f"shl.b32 {gb}, {g}, 2")
    em.ins(f"add.u32 {gb}, {gb}, {b_s}")
    tk = em.tmp("b32")
    em.ins(f"shl.b32 {tk}, {t}, 8")                     # 8 t rows of 8 floats = 256 t bytes
    em.ins(f"add.u32 {gb}, {gb}, {tk}")
    for i in range(2):
        for j in range(8):
            off = ((32 * i + j) * 8) * 4
            em.ins(f"st.shared.f32 [{gb}+{off}], {decode(b[i], j, scale_b[i])}")
    em.ins("bar.warp.sync -1")
    # C: rows g, g + 8; columns 2t, 2t + 1
    ra, rb = em.tmp("b32"), em.tmp("b32")
    em.ins(f"mad.lo.u32 {ra}, {g}, 256, {a_s}")
    em.ins(f"shl.b32 {rb}, {t}, 3")
    em.ins(f"add.u32 {rb}, {rb}, {b_s}")
    for k in range(64):
        a0, a1, b0, b1 = (em.tmp("f32") for _ in range(4))
        em.ins(f"ld.shared.f32 {a0}, [{ra}+{4 * k}]")
        em.ins(f"ld.shared.f32 {a1}, [{ra}+{4 * (8 * 64 + k)}]")
        em.ins(f"ld.shared.v2.f32 {{{b0}, {b1}}}, [{rb}+{4 * 8 * k}]")
        em.ins(f"fma.rn.f32 {c[0]}, {a0}, {b0}, {c[0]}")
        em.ins(f"fma.rn.f32 {c[1]}, {a0}, {b1}, {c[1]}")
        em.ins(f"fma.rn.f32 {c[2]}, {a1}, {b0}, {c[2]}")
        em.ins(f"fma.rn.f32 {c[3]}, {a1}, {b1}, {c[3]}")
    em.ins("bar.warp.sync -1")                          # the scratch is rewritten by the next MMA
