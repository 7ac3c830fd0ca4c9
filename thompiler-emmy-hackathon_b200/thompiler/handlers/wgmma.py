"""Warpgroup tensor-core statements lowered onto tcgen05: WgmmaDescriptor, WgmmaFence,
WgmmaMma, WgmmaCommit, WgmmaWait.

The IR reference (TASK.md:163-171 of the reference) defines these after sm_90's ``wgmma``: the
four warps of a warpgroup issue one ``wgmma.mma_async`` m64nNk16 cell together and its 64 x N
f32 accumulator lives in their registers (thread t of warp q holds rows 16q + t/4 and
16q + t/4 + 8, columns 8i + 2(t%4) + {0, 1} in registers 4i..4i+3).  ``wgmma`` does not exist
on sm_100a, and the reference compiler lowers none of these statements.  Here:

* the accumulator fragments get a home in tensor memory.  Every C fragment family that a
  WgmmaMma names is given N columns per member (f32), each warpgroup its own column range; the
  kernel prologue allocates them (``tcgen05.alloc``, a power of two of at least 32 columns)
  and the end of the kernel frees them.  An M = 64 tcgen05 accumulator keeps rows 16q..16q+15
  in TMEM lanes 32q..32q+15, so warp q of the warpgroup reaches its own rows through its lane
  quarter, and ``tcgen05.ld`` / ``tcgen05.st`` of shape 16x256b move exactly the register
  layout above (four registers per 8 columns);
* ``WgmmaDescriptor`` builds a tcgen05 shared-memory descriptor (start address >> 4, leading
  and stride byte offsets >> 4, version 1, layout 0 / 6 / 4 / 2 for no / 32 / 64 / 128-byte
  swizzle) for the Smem element at ``smem_index``;
* ``WgmmaFence`` stores every accumulator whose registers were written since they last matched
  tensor memory (a per-member predicate, set by RegFragment's zero fill), fences the
  thread's shared-memory writes for the tensor core (``fence.proxy.async``), and arrives on
  the warpgroup's fence mbarrier (128 arrivals); the warpgroup's first thread waits for it;
* ``WgmmaMma`` is one ``tcgen05.mma.cta_group::1.kind::f16`` issued by the warpgroup's first
  thread, M = 64, N from the shape, A / B K- or MN-major from ``trans_a`` / ``trans_b``, the
  accumulate predicate from ``scale_d``.  A descriptor whose operand would reach past its
  Smem array, or that is not 16-byte aligned, skips the MMA and sets bit 2 of the error word;
* ``WgmmaCommit`` has nothing left to do (completion is tracked at the wait);
* ``WgmmaWait`` commits the warpgroup's MMAs to its completion mbarrier, waits for them and
  loads the accumulators back into registers.  It waits for all of them, which satisfies any
  ``group`` count.

Every wait is bounded (bit 1 of the error word on expiry), so a fence or wait that part of a
warpgroup skips ends in an error report, not a hang.  Accumulators in f16, A from registers
(``a_frag``), and an MN-major operand without swizzle are refused at compile time.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import TYPE_CHECKING

from thompiler import ir
from thompiler.handlers.async_copy import ERR_WAIT_TIMEOUT, WAIT_LIMIT, _flag
from thompiler.lowering import expr, ops
from thompiler.lowering.address import flat_index, shared_element_address
from thompiler.lowering.types import F32, dtype_of

if TYPE_CHECKING:
    from thompiler.load import KernelInfo
    from thompiler.walk import Walker

ERR_MMA_SKIPPED = 4
WG_THREADS = 128
LAYOUT = {None: 0, "": 0, "NONE": 0, 0: 0, "B32": 6, 32: 6, "B64": 4, 64: 4, "B128": 2, 128: 2}
SPAN = {0: None, 6: 32, 4: 64, 2: 128}
BASE_SLOT = "thc_wg_tmem"
FENCE_BAR = "thc_wg_fence"
DONE_BAR = "thc_wg_done"


def _base_name(ref: str) -> str:
    return ref.split("[", 1)[0].strip()


def _pow2_at_least(n: int) -> int:
    p = 32
    while p < n:
        p *= 2
    return p


@dataclass
class Desc:
    reg: str              # the 64-bit descriptor
    arr: object           # the Smem array it points into
    offset: str           # byte offset of its start in the array (register or immediate)
    layout: int
    lbo: int
    sbo: int


@dataclass
class WgPlan:
    """Tensor-memory columns of the warpgroup accumulators of one kernel."""
    frags: dict[str, tuple[int, int, int]]     # name -> (first column, N, count)
    cols_per_wg: int
    n_wg: int
    ncols: int
    descs: dict[str, Desc] = field(default_factory=dict)

    def columns(self, name: str, member: int) -> tuple[int, int]:
        first, n, _ = self.frags[name]
        return first + member * n, n

    def members(self):
        for name, (_, n, count) in self.frags.items():
            for m in range(count):
                yield name, m


def plan(kernel: "KernelInfo") -> WgPlan | None:
    """The accumulator columns of ``kernel``, or None when it has no WgmmaMma."""
    stmts = list(ir.walk_stmts(kernel.body))
    mmas = [s for s in stmts if isinstance(s, ir.WgmmaMma)]
    if not mmas:
        return None
    names = {_base_name(r) for s in mmas for r in s.c_frags}
    frags: dict[str, tuple[int, int, int]] = {}
    col = 0
    for s in stmts:
        if isinstance(s, ir.RegFragment) and s.name in names:
            shape = tuple(int(x) for x in s.shape)
            if s.role != "c" or shape[0] != 64:
                raise ValueError(f"WgmmaMma accumulator {s.name} is a {s.role} fragment of shape {shape}, "
                                 "not an m64 C fragment")
            if dtype_of(s.dtype, f"RegFragment {s.name}") is not F32:
                raise NotImplementedError(f"WgmmaMma accumulator {s.name}: only f32 accumulators")
            n = shape[1]
            if n % 8 or not 8 <= n <= 256:
                raise ValueError(f"WgmmaMma accumulator {s.name}: N={n} (a multiple of 8 in 8..256)")
            if s.name in frags:
                raise ValueError(f"fragment {s.name} declared twice")
            frags[s.name] = (col, n, int(s.count))
            col += n * int(s.count)
    missing = names - set(frags)
    if missing:
        raise ValueError(f"WgmmaMma accumulators {sorted(missing)} have no RegFragment")
    threads = kernel.threads_per_cta
    if kernel.block[1:] != (1, 1) or threads % WG_THREADS:
        raise NotImplementedError(f"Wgmma statements in a CTA of {kernel.block} threads "
                                  "(a 1-d block of whole warpgroups)")
    tiles = [s for s in kernel.body if isinstance(s, ir.Tile)]
    if len(tiles) != 1 or tiles[0].n_elements != kernel.ctas * threads:
        raise NotImplementedError("Wgmma statements need one Tile whose cells fill the launch exactly "
                                  "(every thread of a warpgroup reaches its fences and waits)")
    n_wg = threads // WG_THREADS
    if col * n_wg > 512:
        raise ValueError(f"{n_wg} warpgroups x {col} accumulator columns exceed tensor memory (512)")
    return WgPlan(frags, col, n_wg, _pow2_at_least(col * n_wg))


def _regs(w: "Walker", name: str, member: int) -> list[str]:
    frag = w.fragments.get(name)
    if frag is None:
        raise KeyError(f"fragment {name!r} used before its RegFragment")
    return frag.regs(member)


def dirty(name: str, member: int) -> str:
    return f"%wgd_{name}_{member}"


def prologue(w: "Walker", p: WgPlan) -> None:
    """Tensor-memory allocation and the warpgroup barriers, before the Tile."""
    em = w.em
    em.note(f"warpgroup accumulators: {p.n_wg} x {p.cols_per_wg} tensor-memory columns (alloc {p.ncols})")
    em.module(f".shared .align 4 .b32 {BASE_SLOT}")
    em.module(f".shared .align 8 .b64 {FENCE_BAR}[{p.n_wg}]")
    em.module(f".shared .align 8 .b64 {DONE_BAR}[{p.n_wg}]")
    tid, warp, wg, q = em.tmps("b32", 4)
    pw, p0 = em.tmp("pred"), em.tmp("pred")
    em.ins(f"mov.u32 {tid}, %tid.x")
    em.ins(f"shr.u32 {warp}, {tid}, 5")
    em.ins(f"setp.eq.u32 {pw}, {warp}, 0")
    skip = em.label("wg_noalloc")
    em.ins(f"@!{pw} bra {skip}")
    em.ins(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{BASE_SLOT}], {p.ncols}")
    em.ins("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned")
    em.place(skip)
    em.ins(f"setp.eq.u32 {p0}, {tid}, 0")
    for i in range(p.n_wg):
        em.ins(f"@{p0} mbarrier.init.shared::cta.b64 [{FENCE_BAR}+{8 * i}], {WG_THREADS}")
        em.ins(f"@{p0} mbarrier.init.shared::cta.b64 [{DONE_BAR}+{8 * i}], 1")
    em.ins(f"@{p0} fence.mbarrier_init.release.cluster")
    em.ins("tcgen05.fence::before_thread_sync")
    em.ins("bar.sync 0")
    em.ins("tcgen05.fence::after_thread_sync")
    base = em.tmp("b32")
    em.ins(f"ld.shared.u32 {base}, [{BASE_SLOT}]")
    em.ins(f"div.u32 {wg}, {tid}, {WG_THREADS}")
    tmd = em.declare("%wg_tmd", "b32")               # the warpgroup's columns, lane 0 (the MMA's D)
    em.ins(f"mad.lo.u32 {tmd}, {wg}, {p.cols_per_wg}, {base}")
    tm = em.declare("%wg_tm", "b32")                 # the same columns at this warp's lane quarter
    em.ins(f"and.b32 {q}, {warp}, 3")
    em.ins(f"shl.b32 {q}, {q}, 21")                  # (32 * q) << 16
    em.ins(f"add.u32 {tm}, {tmd}, {q}")
    fb, db = em.declare("%wg_fb", "b32"), em.declare("%wg_db", "b32")
    off = em.tmp("b32")
    em.ins(f"shl.b32 {off}, {wg}, 3")
    em.ins(f"mov.u32 {fb}, {FENCE_BAR}")
    em.ins(f"add.u32 {fb}, {fb}, {off}")
    em.ins(f"mov.u32 {db}, {DONE_BAR}")
    em.ins(f"add.u32 {db}, {db}, {off}")
    em.ins(f"mov.u32 {em.declare('%wg_fph', 'b32')}, 0")
    em.ins(f"mov.u32 {em.declare('%wg_dph', 'b32')}, 0")
    lead = em.declare("%wg_el", "pred")              # the warpgroup's first thread issues its MMAs
    r = em.tmp("b32")
    em.ins(f"rem.u32 {r}, {tid}, {WG_THREADS}")
    em.ins(f"setp.eq.u32 {lead}, {r}, 0")
    for name, m in p.members():
        em.ins(f"setp.ne.u32 {em.declare(dirty(name, m), 'pred')}, 0, 0")
    em.ins(f"mov.u32 {em.declare('%wg_base', 'b32')}, {base}")


def _bounded_wait(w: "Walker", bar: str, parity: str) -> None:
    em = w.em
    top, done = em.label("wgw"), em.label("wgw_done")
    n, ok, more = em.tmp("b32"), em.tmp("pred"), em.tmp("pred")
    em.ins(f"mov.u32 {n}, 0")
    em.place(top)
    em.ins(f"mbarrier.try_wait.parity.shared::cta.b64 {ok}, [{bar}], {parity}")
    em.ins(f"@{ok} bra {done}")
    em.ins(f"add.u32 {n}, {n}, 1")
    em.ins(f"setp.lt.u32 {more}, {n}, {WAIT_LIMIT}")
    em.ins(f"@{more} bra {top}")
    _flag(w, ERR_WAIT_TIMEOUT)
    em.place(done)


def _wait_done(w: "Walker") -> None:
    """Commit the warpgroup's MMAs to its completion barrier and wait for them (all threads)."""
    em = w.em
    em.ins("@%wg_el tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%wg_db]")
    par = em.tmp("b32")
    em.ins(f"and.b32 {par}, %wg_dph, 1")
    _bounded_wait(w, "%wg_db", par)
    em.ins("add.u32 %wg_dph, %wg_dph, 1")
    em.ins("tcgen05.fence::after_thread_sync")


def _chunks(n8: int):
    """Split n8 column groups of 8 into power-of-two runs (the .x counts tcgen05.ld/st take)."""
    start = 0
    for bit in (32, 16, 8, 4, 2, 1):
        while n8 - start >= bit:
            yield start, bit
            start += bit


def _move(w: "Walker", name: str, member: int, store: bool) -> None:
    """tcgen05.st (store) or tcgen05.ld of one accumulator member, skipped unless it is dirty
    (a store) or clean (a load)."""
    em = w.em
    p: WgPlan = w.wgmma
    col, n = p.columns(name, member)
    regs = _regs(w, name, member)
    if len(regs) != n // 2:
        raise ValueError(f"accumulator {name}[{member}] has {len(regs)} registers, not {n // 2}")
    skip = em.label("wg_skip")
    d = dirty(name, member)
    em.ins(f"@{'!' if store else ''}{d} bra {skip}")
    for c8, x in _chunks(n // 8):
        part = regs[4 * c8:4 * (c8 + x)]
        addr = "%wg_tm" if col + 8 * c8 == 0 else f"%wg_tm+{col + 8 * c8}"
        if store:
            em.ins(f"tcgen05.st.sync.aligned.16x256b.x{x}.b32 [{addr}], {{{', '.join(part)}}}")
        else:
            em.ins(f"tcgen05.ld.sync.aligned.16x256b.x{x}.b32 {{{', '.join(part)}}}, [{addr}]")
    if store:
        em.ins(f"setp.ne.u32 {d}, 0, 0")
    em.place(skip)


def epilogue(w: "Walker", p: WgPlan) -> None:
    """After the Tile: no MMA in flight, every thread done with tensor memory, then free it."""
    em = w.em
    em.note("warpgroup accumulators: release tensor memory")
    _wait_done(w)
    em.ins("tcgen05.fence::before_thread_sync")
    em.ins("bar.sync 0")
    em.ins("tcgen05.fence::after_thread_sync")
    t, pw = em.tmp("b32"), em.tmp("pred")
    em.ins(f"mov.u32 {t}, %tid.x")
    em.ins(f"shr.u32 {t}, {t}, 5")
    em.ins(f"setp.eq.u32 {pw}, {t}, 0")
    skip = em.label("wg_nofree")
    em.ins(f"@!{pw} bra {skip}")
    em.ins(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 %wg_base, {p.ncols}")
    em.place(skip)


def _need(w: "Walker", what: str) -> WgPlan:
    p = getattr(w, "wgmma", None)
    if p is None:
        raise ValueError(f"{what} in a kernel without a WgmmaMma")
    return p


def emit_wgmma_descriptor(w: "Walker", d: ir.WgmmaDescriptor) -> None:
    em = w.em
    em.note(d.pretty())
    p = _need(w, "WgmmaDescriptor")
    arr = w.smem.get(d.smem)
    if arr is None:
        raise ValueError(f"WgmmaDescriptor {d.name}: {d.smem} is not a declared Smem array")
    sw = d.swizzle.upper() if isinstance(d.swizzle, str) else d.swizzle
    if sw not in LAYOUT:
        raise NotImplementedError(f"WgmmaDescriptor {d.name}: swizzle {d.swizzle!r}")
    layout = LAYOUT[sw]
    lbo, sbo = int(expr_value(d.lbo_bytes)), int(expr_value(d.sbo_bytes))
    for what, v in (("leading", lbo), ("stride", sbo)):
        if v < 0 or v % 16 or v >= (1 << 18):
            raise ValueError(f"WgmmaDescriptor {d.name}: {what} byte offset {v} (a multiple of 16 below 2^18)")
    flat = flat_index(w, arr.extents, tuple(d.smem_index), d.smem)
    if expr.is_imm(flat):
        offset = str(int(flat) * arr.ty.nbytes)
    else:
        offset = em.tmp("b32")
        em.ins(f"mul.lo.s32 {offset}, {flat}, {arr.ty.nbytes}")
    addr = shared_element_address(w, arr, flat)
    sa = em.tmp("b32")
    base, _, off = addr.partition("+")
    if base.startswith("%"):
        em.ins(f"add.u32 {sa}, {base}, {off or 0}")
    else:
        em.ins(f"mov.u32 {sa}, {base}")
        if off:
            em.ins(f"add.u32 {sa}, {sa}, {off}")
    lo, hi = em.tmp("b32"), em.tmp("b32")
    em.ins(f"shr.u32 {lo}, {sa}, 4")
    em.ins(f"and.b32 {lo}, {lo}, 16383")
    em.ins(f"or.b32 {lo}, {lo}, {((lbo >> 4) & 0x3FFF) << 16}")
    em.ins(f"mov.u32 {hi}, {((sbo >> 4) & 0x3FFF) | (1 << 14) | (layout << 29)}")
    reg = em.declare(f"%wgdesc_{d.name}", "b64")
    em.ins(f"mov.b64 {reg}, {{{lo}, {hi}}}")
    p.descs[d.name] = Desc(reg, arr, offset, layout, lbo, sbo)


def expr_value(v):
    """An int from an IR literal or a plain number (byte offsets are compile-time values)."""
    if isinstance(v, ir.Literal):
        return v.value
    if isinstance(v, (int, float)):
        return v
    raise NotImplementedError(f"a run-time descriptor byte offset: {ir.pretty(v)}")


def _extent(desc: Desc, rows: int, mn_major: bool, what: str) -> int:
    """Bytes from the descriptor's start that one k16 step of a ``rows``-row f16 operand reads."""
    span = SPAN[desc.layout]
    if not mn_major:
        if rows % 8:
            raise ValueError(f"{what}: {rows} rows (a multiple of 8)")
        if span is None:                  # 8 x 16-byte core matrices: two along K, rows/8 down
            return (rows // 8 - 1) * desc.sbo + desc.lbo + 128
        return (rows // 8 - 1) * desc.sbo + 7 * span + 32
    if span is None:
        raise NotImplementedError(f"{what}: an MN-major operand without swizzle")
    per_atom = span // 2                  # f16 elements of MN in one swizzle row
    atoms = -(-rows // per_atom)
    return (atoms - 1) * desc.lbo + desc.sbo + 8 * span


def emit_wgmma_fence(w: "Walker", s: ir.WgmmaFence) -> None:
    em = w.em
    em.note("WgmmaFence: accumulators written since the last sync go to tensor memory")
    p = _need(w, "WgmmaFence")
    for name, m in p.members():
        _move(w, name, m, store=True)
    em.ins("tcgen05.wait::st.sync.aligned")
    em.ins("fence.proxy.async.shared::cta")
    em.ins("tcgen05.fence::before_thread_sync")
    em.ins("mbarrier.arrive.shared::cta.b64 _, [%wg_fb]")
    skip = em.label("wgf")
    em.ins(f"@!%wg_el bra {skip}")
    par = em.tmp("b32")
    em.ins(f"and.b32 {par}, %wg_fph, 1")
    _bounded_wait(w, "%wg_fb", par)
    em.ins("tcgen05.fence::after_thread_sync")
    em.place(skip)
    em.ins("add.u32 %wg_fph, %wg_fph, 1")


def _member(w: "Walker", ref: str) -> tuple[str, int]:
    from thompiler.handlers.mma import REF, _const_index
    m = REF.match(ref)
    if m is None:
        raise ValueError(f"not a fragment reference: {ref!r}")
    return m["name"], 0 if m["index"] is None else _const_index(w, m["index"], ref)


def _idesc(n: int, ab: str, a_mn: bool, b_mn: bool) -> int:
    """kind::f16 instruction descriptor, M = 64, f32 accumulator."""
    fmt = {"f16": 0, "bf16": 1}[ab]
    return ((1 << 4) | (fmt << 7) | (fmt << 10) | (int(a_mn) << 15) | (int(b_mn) << 16)
            | ((n >> 3) << 17) | ((64 >> 4) << 24))


def emit_wgmma_mma(w: "Walker", s: ir.WgmmaMma) -> None:
    em = w.em
    em.note(s.pretty())
    p = _need(w, "WgmmaMma")
    shape = tuple(int(x) for x in s.shape)
    if len(shape) != 3 or shape[0] != 64 or shape[2] != 16:
        raise NotImplementedError(f"WgmmaMma of shape {shape} (m64nNk16)")
    n = shape[1]
    if s.ab_dtype not in ("f16", "bf16"):
        raise NotImplementedError(f"WgmmaMma with {s.ab_dtype} operands")
    if s.a_frag is not None or s.a_desc is None:
        raise NotImplementedError("WgmmaMma with A in registers (tcgen05 reads A from shared or tensor memory)")
    cols = []
    for ref in s.c_frags:
        name, member = _member(w, ref)
        if name not in p.frags:
            raise ValueError(f"WgmmaMma accumulator {ref} is not planned")
        cols.append(p.columns(name, member))
    first = cols[0][0]
    at = first
    for c, width in cols:
        if c != at:
            raise NotImplementedError(f"WgmmaMma accumulators {s.c_frags} are not adjacent in tensor memory")
        at += width
    if at - first != n:
        raise ValueError(f"WgmmaMma N={n} over accumulators of {at - first} columns")
    bad = em.tmp("pred")
    em.ins(f"setp.ne.u32 {bad}, 0, 0")
    regs = {}
    for role, name, rows, mn in (("A", s.a_desc, 64, bool(s.trans_a)), ("B", s.b_desc, n, bool(s.trans_b))):
        d = p.descs.get(name)
        if d is None:
            raise ValueError(f"WgmmaMma operand {role}: descriptor {name!r} is not built before use")
        ext = _extent(d, rows, mn, f"WgmmaMma operand {role} ({name})")
        last = d.arr.nbytes - ext              # the last start offset the operand fits from
        if expr.is_imm(d.offset):
            if int(d.offset) % 16 or int(d.offset) > last:
                raise ValueError(f"WgmmaMma operand {role}: {ext} bytes from byte {d.offset} of "
                                 f"{d.arr.name} ({d.arr.nbytes} bytes), or not 16-byte aligned")
        else:
            t, q = em.tmp("b32"), em.tmp("pred")
            em.ins(f"and.b32 {t}, {d.offset}, 15")
            em.ins(f"setp.ne.u32 {q}, {t}, 0")
            em.ins(f"or.pred {bad}, {bad}, {q}")
            if last < 0:
                raise ValueError(f"WgmmaMma operand {role}: {ext} bytes do not fit {d.arr.name}")
            em.ins(f"setp.gt.s32 {q}, {d.offset}, {last}")
            em.ins(f"or.pred {bad}, {bad}, {q}")
        regs[role] = d.reg
    acc = em.tmp("pred")
    sd = s.scale_d
    if isinstance(sd, (bool, int)) or (isinstance(sd, ir.Literal) and isinstance(sd.value, (bool, int))):
        v = int(sd.value if isinstance(sd, ir.Literal) else sd)
        em.ins(f"setp.ne.u32 {acc}, {v}, 0")
    elif isinstance(sd, ir.BinaryExpr) and sd.op in (*ops.COMPARE, *ops.LOGIC):
        em.ins(f"mov.pred {acc}, {expr.pred_operand(w, sd)}")
    else:
        op = expr.int_operand(w, sd)
        em.ins(f"setp.ne.s32 {acc}, {op}, 0")
    _flag(w, ERR_MMA_SKIPPED, bad)
    go = em.tmp("pred")
    em.ins(f"not.pred {go}, {bad}")
    em.ins(f"and.pred {go}, {go}, %wg_el")
    dt = "%wg_tmd" if first == 0 else f"%wg_tmd+{first}"
    em.ins(f"@{go} tcgen05.mma.cta_group::1.kind::f16 [{dt}], {regs['A']}, {regs['B']}, "
           f"{_idesc(n, s.ab_dtype, bool(s.trans_a), bool(s.trans_b))}, {acc}")


def emit_wgmma_commit(w: "Walker", s: ir.WgmmaCommit) -> None:
    _need(w, "WgmmaCommit")
    w.em.note("WgmmaCommit: the MMAs issued so far complete at the next WgmmaWait")


def emit_wgmma_wait(w: "Walker", s: ir.WgmmaWait) -> None:
    em = w.em
    em.note(f"WgmmaWait({ir.pretty(s.group)}): all of the warpgroup's MMAs, then accumulators to registers")
    p = _need(w, "WgmmaWait")
    _wait_done(w)
    for name, m in p.members():
        _move(w, name, m, store=False)
    em.ins("tcgen05.wait::ld.sync.aligned")


def fragment_written(w: "Walker", name: str) -> None:
    """Registers of ``name`` were written outside the tensor core: mark its members dirty."""
    p = getattr(w, "wgmma", None)
    if p is None or name not in p.frags:
        return
    for m in range(p.frags[name][2]):
        w.em.ins(f"setp.eq.u32 {dirty(name, m)}, 0, 0")
