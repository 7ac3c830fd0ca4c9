"""Blackwell building blocks shared by the tcgen05 families.

* shared-memory matrix descriptors (64-bit): bits 0-13 start address >> 4,
  16-29 leading byte offset >> 4, 32-45 stride byte offset >> 4, 46-47
  version (1 on sm_100), 61-63 layout (2 = 128-byte swizzle) -- the layout
  CUTLASS documents for sm100 UMMA descriptors;
* the kind::f16 instruction descriptor (32-bit): D format (f32 = 1) at bit 4,
  A / B formats at 7 / 10 (f16 = 0), A / B major-ness at 15 / 16 (1 =
  MN-major), N >> 3 at bit 17, M >> 4 at bit 24;
* bounded mbarrier waits: every wait gives up after ``WAIT_LIMIT`` rounds of
  ``mbarrier.try_wait``, records a code in the module's error word and jumps
  to the kernel's common exit -- no kernel here can hang its GPU; a wait run
  by a whole warp makes that decision for all its lanes at once.
"""

from __future__ import annotations

WAIT_LIMIT = 1 << 18          # try_wait rounds (~4 us each while the phase is open): ~1 s
SWIZZLE_128B = 2
TMAP_SETS = 8                 # tensor-map sets a tuned module keeps (launches in flight on other buffers)
TMAP_RING, TMAP_TABLE = "thc_tmap_ring", "thc_tmap_ptr"


def declare_tmap_ring(em, nmaps: int) -> None:
    """Module globals of TMAP_SETS sets of ``nmaps`` tensor maps and the buffer addresses each set
    is encoded for (the runner fills them: thr_tmap_bind)."""
    em.module(f".global .align 64 .b8 {TMAP_RING}[{TMAP_SETS * nmaps * 128}]")
    em.module(f".global .align 8 .u64 {TMAP_TABLE}[{TMAP_SETS * nmaps}]")


def select_tmap_set(em, params: list[str], generic: str) -> str:
    """Guard code: a register with the index of the set whose recorded addresses equal the kernel
    parameters ``params`` (in map order); no such set (or a null first parameter) branches to the
    generic lowering.  The whole table is loaded first (independent loads, one memory latency),
    then compared."""
    p = em.tmp("pred")
    raws = []
    for name in params:
        r = em.tmp("b64")
        em.ins(f"ld.param.u64 {r}, [p_{name}]")
        raws.append(r)
    em.ins(f"setp.eq.u64 {p}, {raws[0]}, 0")
    em.ins(f"@{p} bra {generic}")
    n = len(params)
    table = [em.tmp("b64") for _ in range(TMAP_SETS * n)]
    for j in range(0, len(table) - 1, 2):
        em.ins(f"ld.global.nc.v2.u64 {{{table[j]}, {table[j + 1]}}}, [{TMAP_TABLE}+{8 * j}]")
    if len(table) % 2:
        em.ins(f"ld.global.nc.u64 {table[-1]}, [{TMAP_TABLE}+{8 * (len(table) - 1)}]")
    sel, hit, eq = em.tmp("b32"), em.tmp("pred"), em.tmp("pred")
    em.ins(f"mov.u32 {sel}, {TMAP_SETS}")
    for k in reversed(range(TMAP_SETS)):            # the lowest matching set wins
        for i, raw in enumerate(raws):
            if i == 0:
                em.ins(f"setp.eq.u64 {hit}, {raw}, {table[k * n]}")
            else:
                em.ins(f"setp.eq.and.u64 {hit}, {raw}, {table[k * n + i]}, {hit}")
        em.ins(f"selp.u32 {sel}, {k}, {sel}, {hit}")
    em.ins(f"setp.eq.u32 {eq}, {sel}, {TMAP_SETS}")
    em.ins(f"@{eq} bra {generic}")
    return sel


def tmap_address(em, sel: str, nmaps: int, i: int) -> str:
    """Generic address of map ``i`` of the selected set."""
    r, off = em.tmp("b64"), em.tmp("b64")
    em.ins(f"mov.u64 {r}, {TMAP_RING}")
    em.ins(f"cvta.global.u64 {r}, {r}")
    em.ins(f"mul.wide.u32 {off}, {sel}, {nmaps * 128}")
    em.ins(f"add.u64 {r}, {r}, {off}")
    if i:
        em.ins(f"add.u64 {r}, {r}, {128 * i}")
    return r


def elect_one(em, pred: str) -> None:
    """Set ``pred`` in one lane of the warp (the lowest; run where all 32 lanes are converged).

    The single-thread instructions of the tuned bodies (``tcgen05.mma`` / ``commit``, TMA loads
    and stores) are guarded by ``elect.sync`` rather than by a lane-id comparison: with it a
    warp issues a ``tcgen05.mma`` 128x128x16 in 23-25 cycles, against 46-48 under
    ``setp.eq lane, 0`` (clock stamps after each of 48 back-to-back MMAs), and a 128x128x16 MMA
    executes in 64 -- under the comparison the issuing warp, not the tensor pipe, set the pace
    of the attention's key loop."""
    em.ins(f"elect.sync {em.tmp('b32')}|{pred}, 0xffffffff")


def desc_hi(sbo: int, layout: int = SWIZZLE_128B) -> int:
    """High word: stride byte offset, version 1, layout type."""
    return ((sbo >> 4) & 0x3FFF) | (1 << 14) | (layout << 29)


def idesc_f16(m: int, n: int, a_mn_major: bool = False, b_mn_major: bool = False) -> int:
    """kind::f16 instruction descriptor: f16 A and B, f32 accumulator."""
    return ((1 << 4) | ((1 if a_mn_major else 0) << 15) | ((1 if b_mn_major else 0) << 16)
            | ((n >> 3) << 17) | ((m >> 4) << 24))


class Kit:
    """PTX helpers bound to one emitter, error word and exit label."""

    def __init__(self, em, errp: str, end: str):
        self.em, self.errp, self.end = em, errp, end
        self.q = em.tmp("pred")

    def wait(self, bar: str, parity: str, code: int, cluster: bool = False, warp: bool = True) -> None:
        """Bounded wait for the phase of parity ``parity`` of the barrier at ``bar``; ``cluster``
        acquires at cluster scope (the barrier's arrivals come from the other CTA of a pair).

        ``warp`` (the default): all 32 lanes of the warp run this wait, and they decide together
        -- the warp leaves the loop once every lane has seen the phase complete (``vote.sync.all``
        each round), and gives up with all lanes at once, so the warp-wide ``.sync.aligned``
        instructions after a wait never meet a warp split between the exit and the work.  A wait
        that a single lane runs passes ``warp=False``."""
        em = self.em
        sem = ".acquire.cluster" if cluster else ""
        top, ok = em.label("wait"), em.label("waited")
        n = em.tmp("b32")
        em.ins(f"mov.u32 {n}, 0")
        em.place(top)
        em.ins(f"mbarrier.try_wait.parity{sem}.shared::cta.b64 {self.q}, [{bar}], {parity}")
        if warp:
            em.ins(f"vote.sync.all.pred {self.q}, {self.q}, -1")
        em.ins(f"@{self.q} bra {ok}")
        em.ins(f"add.u32 {n}, {n}, 1")
        em.ins(f"setp.lt.u32 {self.q}, {n}, {WAIT_LIMIT}")
        em.ins(f"@{self.q} bra {top}")
        em.ins(f"atom.global.or.b32 {em.tmp('b32')}, [{self.errp}], {1 << code}")
        em.ins(f"bra {self.end}")
        em.place(ok)

    def desc(self, saddr: str, lbo: int, hi_reg: str) -> str:
        """A 64-bit descriptor register for the tile at shared address ``saddr``."""
        em = self.em
        lo, d = em.tmp("b32"), em.tmp("b64")
        em.ins(f"shr.u32 {lo}, {saddr}, 4")
        em.ins(f"and.b32 {lo}, {lo}, 16383")
        em.ins(f"or.b32 {lo}, {lo}, {(lbo >> 4) << 16}")
        em.ins(f"mov.b64 {d}, {{{lo}, {hi_reg}}}")
        return d

    def desc_add(self, d: str, byte_offset: int) -> str:
        """The descriptor ``d`` advanced by ``byte_offset`` bytes of start address.

        Only the low word changes: the start-address field (bits 0-13, address >> 4) plus the
        offset is the advanced tile's own address >> 4, below 2^14 inside 227 KB of shared
        memory, so nothing carries into the offset fields above it.  One 32-bit add per MMA
        operand instead of a 64-bit one (measured +0.6 % on the attention kernel, whose issuing
        warp is on its critical path)."""
        if byte_offset == 0:
            return d
        em = self.em
        lo, hi, r = em.tmp("b32"), em.tmp("b32"), em.tmp("b64")
        em.ins(f"mov.b64 {{{lo}, {hi}}}, {d}")
        em.ins(f"add.u32 {lo}, {lo}, {byte_offset >> 4}")
        em.ins(f"mov.b64 {r}, {{{lo}, {hi}}}")
        return r

    def parity(self, counter: str, period: int, flip: bool = False) -> str:
        """((counter / period) & 1) [^ 1]: the phase parity of a ring slot's use."""
        em = self.em
        r = em.tmp("b32")
        if period == 1:
            em.ins(f"and.b32 {r}, {counter}, 1")
        else:
            em.ins(f"div.u32 {r}, {counter}, {period}")
            em.ins(f"and.b32 {r}, {r}, 1")
        if flip:
            em.ins(f"xor.b32 {r}, {r}, 1")
        return r
