"""Tuned family: f16 tensor-core matmul on tcgen05 (t01 / t02 / the matmul
benchmark shapes).

Recognised IR: a Tile whose body stages two f16 operands through shared
memory with CpAsyncCopy, loads them with LdmatrixLoad (role a from one
parameter, role b from the other) and accumulates with MmaSyncPtx
m16n8k16 f16 -> f32, storing the accumulators with RegStore -- the warp-level
tensor-core schedule of the reference's tests/problems/t01_matmul_f16 and
t02_matmul_f16_to_f32 (k_to__partial).  What it computes is
C[M, N] = A[M, K] @ B with B stored [N, K] (b_trans: "column-major") or
[K, N]; a 3-D output [S, M, N] is the split-K form: slice s holds
A[:, sK/S:(s+1)K/S] @ B[sK/S:(s+1)K/S, :].

Tuned body (one persistent CTA per SM, 192 threads, warp-specialised):

  warp 0   TMA producer: per K block of 64, waits for the stage to be empty and
           loads the A tile (128 x 64) and the B tile (BN x 64, or 64 x BN) with
           cp.async.bulk.tensor into a 128B-swizzled stage, completing on the
           stage's mbarrier (expect_tx);
  warp 1   MMA issuer: allocates TMEM (2 accumulators of BN f32 columns), and for
           each K block issues 4 x tcgen05.mma.cta_group::1.kind::f16 (M=128,
           N=BN, K=16) from shared-memory descriptors, then tcgen05.commit to the
           stage's "empty" mbarrier; after the last block, commit to the
           accumulator's "full" mbarrier;
  warps 2-5 epilogue: tcgen05.ld 32x32b of their TMEM lane quarter, convert,
           stage 32-row x 64-byte boxes in per-warp 64B-swizzled shared buffers
           and store them with cp.async.bulk.tensor (bulk groups); arrive on the
           accumulator's "empty" mbarrier, so the MMA of the next tile (other
           accumulator) overlaps this epilogue.

Tiles are handed out round-robin (tile = ctaid + i * nctaid), M fastest, so
the CTAs in flight share B column tiles in L2.  Every mbarrier wait is
bounded: on expiry the thread records a code in the module's ``thc_error``
word and leaves through the common exit, which releases TMEM.

Tensor maps live in module ``.global`` variables that the runner fills (the
tuned launch lists them in the module's sidecar) together with the pointers
they were encoded for; the kernel takes the tuned path only when its
``%ntid.x`` is 192 and its A / B pointers are the ones the maps describe,
otherwise it runs the generic lowering of the IR, which needs nothing but
meta.json's launch.
"""

from __future__ import annotations

from thompiler import ir
from thompiler.families.base import TunedKernel
from thompiler.families.kit import (TMAP_RING, TMAP_SETS, TMAP_TABLE, declare_tmap_ring, elect_one,
                                    select_tmap_set, tmap_address)
from thompiler.families.tuning import TUNING
from thompiler.lowering.types import F16, F32
from thompiler.load import KernelInfo

SM_COUNT = 148
THREADS = 192
BM, BK = 128, 64
SMEM_LIMIT = 227 * 1024
WAIT_LIMIT = 1 << 18          # try_wait rounds before a wait gives up (~4 us each while open: ~1 s)
EPI_WARPS = 4
STAGE_TILE = 2048             # one epilogue store box: 32 rows x 64 bytes


def _desc_hi(sbo: int, layout: int = 2) -> int:
    """High 32 bits of a tcgen05 shared-memory descriptor: SBO, version 1, layout."""
    return ((sbo >> 4) & 0x3FFF) | (1 << 14) | (layout << 29)


def idesc_f16(n: int, b_mn_major: bool) -> int:
    """Instruction descriptor, kind::f16: f16 A/B, f32 D, M = 128, N = n."""
    return (1 << 4) | ((1 if b_mn_major else 0) << 16) | ((n >> 3) << 17) | ((BM >> 4) << 24)


class TcMatmul(TunedKernel):
    family = "tcgen05-matmul"
    tail_ranks = 1               # CTAs sharing one output tile (2 for the CTA-pair kernel)

    def __init__(self, kernel: KernelInfo, a, b, c, M, N, K, S, b_kmajor, static_smem):
        super().__init__(kernel)
        self.a, self.b, self.c = a, b, c
        self.M, self.N, self.K, self.S = M, N, K, S
        self.Ks = K // S
        self.b_kmajor = b_kmajor
        self.static_smem = static_smem
        self.BN = self.pick_bn()
        self.a_bytes = BM * BK * 2
        self.b_bytes = self.BN * BK * 2
        stage = self.a_bytes + self.b_bytes
        self.staging = EPI_WARPS * 2 * STAGE_TILE        # per-warp double-buffered store staging
        room = SMEM_LIMIT - static_smem - 2048 - self.staging
        self.stages = max(2, min(6, room // stage))
        forced = TUNING.matmul_stages
        if 2 <= forced <= room // stage:
            self.stages = forced
        self.smem = self.stages * stage + self.staging + 1024 + 256
        self.tiles = (M // BM) * (N // self.BN) * S
        self.ctas = min(self.tiles, SM_COUNT)
        # the last, partial wave: its `rem` tiles are cut along K into `parts` units each, so one
        # round of 1/parts of a tile replaces a round of whole tiles on `rem` of the SMs
        kblocks = self.Ks // BK
        rem = self.tiles % SM_COUNT if self.tiles > SM_COUNT else 0
        # a part must be long enough to pay for its partial's round trip through L2: the last part
        # to arrive reads all `parts` partials (128 KB each at N = 256), so at least 16 K blocks
        parts = min(kblocks // 16, SM_COUNT // rem) if rem else 1
        if S != 1 or c.ty is not F32 or parts < 2 or not TUNING.matmul_split_tail:
            rem, parts = 0, 1
        self.rem, self.parts = rem, parts
        self.full_tiles = self.tiles - rem
        self.units = self.full_tiles + rem * parts

    def pick_bn(self) -> int:
        forced = TUNING.matmul_bn                                   # force the tile width
        if forced and self.N % forced == 0 and forced % 16 == 0 and 16 <= forced <= 256:
            return forced
        best, best_score = None, -1.0
        # measured on B200 (cta_group::1, TMA-store epilogue): N = 128 tiles are shared-memory
        # bound (0.65 of N = 256 at 4096^3); N = 192 trails N = 256 by 7 % even where it
        # balances the waves better (8192 x 3072 x 1024)
        for bn, pref in ((256, 1.0), (192, 0.85), (128, 0.65), (64, 0.4)):
            if self.N % bn:
                continue
            tiles = (self.M // BM) * (self.N // bn) * self.S
            waves = -(-tiles // SM_COUNT)
            score = pref * tiles / (waves * SM_COUNT) if tiles >= SM_COUNT else pref * tiles / SM_COUNT
            if score > best_score + 1e-9:
                best, best_score = bn, score
        return best

    # ---- recognition ------------------------------------------------------------

    @classmethod
    def match(cls, kernel: KernelInfo):
        body = kernel.body
        if len(body) != 1 or not isinstance(body[0], ir.Tile):
            return None
        stmts = list(ir.walk_stmts(body[0].body))
        kinds = {type(s) for s in stmts}
        if ir.MmaSyncPtx not in kinds or ir.RegStore not in kinds:
            return None
        if kinds & {ir.Write, ir.Accum, ir.WarpShuffle, ir.TreeHalve, ir.Opaque, ir.Assign, ir.Load}:
            return None
        for s in stmts:
            if isinstance(s, ir.MmaSyncPtx) and (tuple(s.shape) != (16, 8, 16) or s.ab_dtype != "f16"
                                                 or s.c_dtype != "f32" or s.b_row_major or s.block_scaled):
                return None
        fed = {}
        for s in stmts:
            if isinstance(s, ir.CpAsyncCopy):
                if fed.setdefault(s.smem, s.src) != s.src:
                    return None
        roles, trans = {}, set()
        for s in stmts:
            if isinstance(s, ir.LdmatrixLoad):
                src = fed.get(s.src_buffer)
                if src is None or roles.setdefault(s.role, src) != src:
                    return None
                if s.role == "b":
                    trans.add(bool(s.b_trans))
        if set(roles) != {"a", "b"} or len(trans) != 1:
            return None
        stores = [s for s in stmts if isinstance(s, ir.RegStore)]
        # a fused store (epilogue, extra fragments, edge guards, atomic accumulation) is not the plain
        # product this schedule writes: those kernels take the generic lowering
        if any(s.epilogue is not None or s.extra_frags or s.m_guard is not None or s.n_guard is not None
               or s.atomic or s.volta_interleaved or s.swizzle not in ("NONE", None) for s in stores):
            return None
        outs = {s.dst_buffer for s in stores}
        if len(outs) != 1:
            return None
        a, b, c = kernel.param(roles["a"]), kernel.param(roles["b"]), kernel.param(outs.pop())
        if a is None or b is None or c is None or len(kernel.params) != 3:
            return None
        if a.ty is not F16 or b.ty is not F16 or a.written or b.written or c.ty not in (F32, F16):
            return None
        if len(a.shape) != 2 or len(b.shape) != 2:
            return None
        M, K = a.shape
        b_kmajor = trans.pop()
        N = b.shape[0] if b_kmajor else b.shape[1]
        if (b.shape[1] if b_kmajor else b.shape[0]) != K:
            return None
        if c.shape == (M, N):
            S = 1
        elif len(c.shape) == 3 and c.shape[1:] == (M, N) and K % c.shape[0] == 0 and c.ty is F32:
            S = c.shape[0]
        else:
            return None
        if M % BM or N % 64 or (K // S) % BK:
            return None
        # the K loop of the schedule must cover the whole (split) K range
        loops = [s for s in stmts if isinstance(s, (ir.Loop, ir.StridedLoop))
                 and any(isinstance(x, ir.MmaSyncPtx) for x in ir.walk_stmts(s.body))]
        def whole(lp):
            start = getattr(lp, "start", ir.Literal(0, "int"))
            return (lp.axis.extent.is_static and lp.axis.size == K // S and getattr(lp, "end", None) is None
                    and isinstance(start, ir.Literal) and start.value == 0)
        if not any(whole(lp) for lp in loops):
            return None
        static = sum(int(__import__("math").prod(s.extents)) * (2 if s.dtype in ("__half", "half") else 4)
                     for s in stmts if isinstance(s, ir.Smem)) if kernel.dynamic_smem_bytes == 0 else 0
        return cls(kernel, a, b, c, M, N, K, S, b_kmajor, static)

    # ---- launch ------------------------------------------------------------------

    def sidecar(self) -> dict:
        a, b = self.a, self.b
        tm_a = {"global": TMAP_RING, "param": a.name, "dtype": "f16", "dims": [self.K, self.M],
                "strides": [self.K * 2], "box": [BK, BM], "swizzle": 3}
        if self.b_kmajor:
            tm_b = {"global": TMAP_RING, "param": b.name, "dtype": "f16", "dims": [self.K, self.N],
                    "strides": [self.K * 2], "box": [BK, self.BN], "swizzle": 3}
        else:
            tm_b = {"global": TMAP_RING, "param": b.name, "dtype": "f16", "dims": [self.N, self.K],
                    "strides": [self.N * 2], "box": [64, BK], "swizzle": 3}
        esz = self.c.ty.nbytes
        tm_c = {"global": TMAP_RING, "param": self.c.name, "dtype": "f32" if esz == 4 else "f16",
                "dims": [self.N, self.S * self.M], "strides": [self.N * esz], "box": [64 // esz, 32],
                "swizzle": 2}
        side = {"grid": [self.ctas, 1, 1], "block": [THREADS, 1, 1], "smem_bytes": self.smem,
                "tmaps": [tm_a, tm_b, tm_c],
                "tmap_ptrs": {"global": TMAP_TABLE, "params": [a.name, b.name, self.c.name]},
                "tmap_sets": TMAP_SETS, "error_word": "thc_error", "tile": [BM, self.BN, BK],
                "stages": self.stages}
        if self.rem:
            side["counters"] = ["thc_tile_arrivals"]           # the split tail's (tile, rank) counters
        return side

    @property
    def tail_counters(self) -> int:
        """Split-tail arrival counters per tensor-map set: one per (tail tile, CTA of the tile's pair)."""
        return self.rem * self.tail_ranks

    @property
    def tail_ws_bytes(self) -> int:
        """Split-tail partials per tensor-map set."""
        return self.rem * self.tail_ranks * self.parts * BM * self.BN * 4

    def guard(self, generic: str) -> None:
        em = self.em
        declare_tmap_ring(em, 3)
        em.module(".global .align 4 .u32 thc_error")
        if self.rem:                 # per tensor-map set, so launches on other buffers run concurrently
            em.module(f".global .align 4 .u32 thc_tile_arrivals[{TMAP_SETS * self.tail_counters}]")
            em.module(f".global .align 16 .b8 thc_tail_ws[{TMAP_SETS * self.tail_ws_bytes}]")
        em.module(".extern .shared .align 1024 .b8 smem_pool[]")
        p = em.tmp("pred")
        r = self.special("%ntid.x")
        em.ins(f"setp.ne.u32 {p}, {r}, {THREADS}")
        em.ins(f"@{p} bra {generic}")
        # the tensor-map set encoded for these buffers (else the generic lowering)
        self.tmap_set = select_tmap_set(em, [x.name for x in (self.a, self.b, self.c)], generic)

    def tail_bases(self, cnt: str, ws: str) -> None:
        """Point ``cnt`` / ``ws`` at the selected tensor-map set's split-tail counters / partials."""
        em, t = self.em, self.em.tmp
        off = t("b64")
        em.ins(f"mov.u64 {cnt}, thc_tile_arrivals")
        em.ins(f"mul.wide.u32 {off}, {self.tmap_set}, {4 * self.tail_counters}")
        em.ins(f"add.u64 {cnt}, {cnt}, {off}")
        em.ins(f"mov.u64 {ws}, thc_tail_ws")
        em.ins(f"mul.wide.u32 {off}, {self.tmap_set}, {self.tail_ws_bytes}")
        em.ins(f"add.u64 {ws}, {ws}, {off}")

    # ---- the tuned body -------------------------------------------------------------

    def emit_tuned(self) -> None:  # noqa: C901 - one kernel, written out in order
        em = self.em
        t = em.tmp
        S_, BN, ST = self.S, self.BN, self.stages
        a_bytes, b_bytes = self.a_bytes, self.b_bytes
        tiles_m, tiles_n = self.M // BM, self.N // BN
        kblocks = self.Ks // BK
        tmem_cols = 512 if 2 * BN > 256 else 256
        ins, place, lab = em.ins, em.place, em.label
        self.pdl_trigger()

        tid, warp, lane = t("b32"), t("b32"), t("b32")
        ins(f"mov.u32 {tid}, %tid.x")
        ins(f"shr.u32 {warp}, {tid}, 5")
        ins(f"and.b32 {lane}, {tid}, 31")
        base = t("b32")
        ins(f"mov.u32 {base}, smem_pool")
        ins(f"add.u32 {base}, {base}, 1023")
        ins(f"and.b32 {base}, {base}, -1024")
        a_st = base
        b_st = t("b32")
        ins(f"add.u32 {b_st}, {base}, {ST * a_bytes}")
        # shared: A stages | B stages | epilogue staging (2 x 2 KB per epilogue warp) | barriers
        bars = t("b32")
        ins(f"add.u32 {bars}, {base}, {ST * (a_bytes + b_bytes) + self.staging}")
        full = lambda s: f"{bars}+{8 * s}"                  # noqa: E731
        empty_off, accf_off, acce_off, slot_off = 8 * ST, 16 * ST, 16 * ST + 16, 16 * ST + 32
        p, q = t("pred"), t("pred")
        # barriers
        skip = lab("mm_noinit")
        ins(f"setp.ne.u32 {p}, {tid}, 0")
        ins(f"@{p} bra {skip}")
        for s in range(ST):
            ins(f"mbarrier.init.shared::cta.b64 [{bars}+{8 * s}], 1")
            ins(f"mbarrier.init.shared::cta.b64 [{bars}+{empty_off + 8 * s}], 1")
        for b in range(2):
            ins(f"mbarrier.init.shared::cta.b64 [{bars}+{accf_off + 8 * b}], 1")
            ins(f"mbarrier.init.shared::cta.b64 [{bars}+{acce_off + 8 * b}], 128")
        tail_done_off, tail_last_off, tail_flag_off = 16 * ST + 40, 16 * ST + 48, 16 * ST + 56
        if self.rem:
            ins(f"mbarrier.init.shared::cta.b64 [{bars}+{tail_done_off}], 128")
            ins(f"mbarrier.init.shared::cta.b64 [{bars}+{tail_last_off}], 1")
        ins("fence.mbarrier_init.release.cluster")
        ins("fence.proxy.async.shared::cta")
        place(skip)
        # TMEM: warp 1 allocates
        noalloc = lab("mm_noalloc")
        ins(f"setp.ne.u32 {p}, {warp}, 1")
        ins(f"@{p} bra {noalloc}")
        slot = t("b32")
        ins(f"add.u32 {slot}, {bars}, {slot_off}")
        ins(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{slot}], {tmem_cols}")
        ins("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned")
        place(noalloc)
        ins("tcgen05.fence::before_thread_sync")
        ins("bar.sync 0")
        ins("tcgen05.fence::after_thread_sync")
        # barriers and TMEM are set up while the stream's previous kernel may still run; from
        # here on the CTA reads and writes global data
        self.pdl_wait()
        tmem = t("b32")
        ins(f"ld.shared.u32 {tmem}, [{bars}+{slot_off}]")
        cta, ncta = self.special("%ctaid.x"), self.special("%nctaid.x")
        tiles = self.tiles

        # generic addresses of the selected set's tensor maps
        tma, tmb, tmc = (tmap_address(em, self.tmap_set, 3, i) for i in range(3))
        errp = t("b64")
        ins(f"mov.u64 {errp}, thc_error")

        end = lab("mm_end")

        def wait(bar_addr: str, parity: str, code: int, warp: bool = True) -> None:
            """Bounded mbarrier wait; on expiry record ``code`` and leave.  ``warp``: the whole warp
            runs it and its lanes leave, or give up, together (as ``Kit.wait``)."""
            top, ok = lab("wait"), lab("waited")
            n = t("b32")
            ins(f"mov.u32 {n}, 0")
            place(top)
            ins(f"mbarrier.try_wait.parity.shared::cta.b64 {q}, [{bar_addr}], {parity}")
            if warp:
                ins(f"vote.sync.all.pred {q}, {q}, -1")
            ins(f"@{q} bra {ok}")
            ins(f"add.u32 {n}, {n}, 1")
            ins(f"setp.lt.u32 {q}, {n}, {WAIT_LIMIT}")
            ins(f"@{q} bra {top}")
            ins(f"atom.global.or.b32 {t('b32')}, [{errp}], {1 << code}")
            ins(f"bra {end}")
            place(ok)

        def decode(tile: str):
            tm_, tn_, ts_ = t("b32"), t("b32"), t("b32")
            r = t("b32")
            ins(f"rem.u32 {tm_}, {tile}, {tiles_m}")
            ins(f"div.u32 {r}, {tile}, {tiles_m}")
            ins(f"rem.u32 {tn_}, {r}, {tiles_n}")
            ins(f"div.u32 {ts_}, {r}, {tiles_n}")
            return tm_, tn_, ts_

        units, full_tiles, parts = self.units, self.full_tiles, self.parts

        def unit(u: str):
            """Work unit u -> (tile, first and end K block, is-whole-tile predicate, part):
            units below full_tiles are whole tiles, the rest cut the last tiles along K."""
            tile_, lo, hi_, part, v, whole = t("b32"), t("b32"), t("b32"), t("b32"), t("b32"), t("pred")
            ins(f"setp.lt.u32 {whole}, {u}, {full_tiles}")
            ins(f"mov.u32 {tile_}, {u}")
            ins(f"mov.u32 {lo}, 0")
            ins(f"mov.u32 {hi_}, {kblocks}")
            ins(f"mov.u32 {part}, 0")
            if self.rem:
                ins(f"sub.u32 {v}, {u}, {full_tiles}")
                ins(f"@!{whole} div.u32 {tile_}, {v}, {parts}")
                ins(f"@!{whole} add.u32 {tile_}, {tile_}, {full_tiles}")
                ins(f"@!{whole} rem.u32 {part}, {v}, {parts}")
                ins(f"@!{whole} mul.lo.u32 {lo}, {part}, {kblocks}")
                ins(f"@!{whole} div.u32 {lo}, {lo}, {parts}")
                ins(f"@!{whole} mad.lo.u32 {hi_}, {part}, {kblocks}, {kblocks}")
                ins(f"@!{whole} div.u32 {hi_}, {hi_}, {parts}")
            return tile_, lo, hi_, whole, part

        role_mma, role_epi = lab("mm_mma"), lab("mm_epi")
        ins(f"setp.eq.u32 {p}, {warp}, 1")
        ins(f"@{p} bra {role_mma}")
        ins(f"setp.gt.u32 {p}, {warp}, 1")
        ins(f"@{p} bra {role_epi}")

        # ---------------- producer (warp 0) ----------------
        is0 = t("pred")
        elect_one(em, is0)
        it, pu = t("b32"), t("b32")
        ins(f"mov.u32 {it}, 0")
        ins(f"mov.u32 {pu}, {cta}")
        ptop, pdone = lab("prod_tile"), lab("prod_done")
        ins(f"setp.ge.u32 {p}, {pu}, {units}")
        ins(f"@{p} bra {pdone}")
        place(ptop)
        tile, kb, kend, _, _ = unit(pu)
        tm_, tn_, ts_ = decode(tile)
        m0, n0, k0 = t("b32"), t("b32"), t("b32")
        ins(f"mul.lo.u32 {m0}, {tm_}, {BM}")
        ins(f"mul.lo.u32 {n0}, {tn_}, {BN}")
        ins(f"mul.lo.u32 {k0}, {ts_}, {self.Ks}")
        ktop = lab("prod_k")
        place(ktop)
        stage, ph, par = t("b32"), t("b32"), t("b32")
        ins(f"rem.u32 {stage}, {it}, {ST}")
        ins(f"div.u32 {ph}, {it}, {ST}")
        ins(f"and.b32 {ph}, {ph}, 1")
        ins(f"xor.b32 {par}, {ph}, 1")
        eb = t("b32")
        ins(f"mad.lo.u32 {eb}, {stage}, 8, {bars}")
        wait(f"{eb}+{empty_off}", par, 0)
        sa, sb, kc = t("b32"), t("b32"), t("b32")
        ins(f"mad.lo.u32 {sa}, {stage}, {a_bytes}, {a_st}")
        ins(f"mad.lo.u32 {sb}, {stage}, {b_bytes}, {b_st}")
        ins(f"mad.lo.u32 {kc}, {kb}, {BK}, {k0}")
        ins(f"@{is0} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{eb}], {a_bytes + b_bytes}")
        ins(f"@{is0} cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
            f"[{sa}], [{tma}, {{{kc}, {m0}}}], [{eb}]")
        if self.b_kmajor:
            ins(f"@{is0} cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
                f"[{sb}], [{tmb}, {{{kc}, {n0}}}], [{eb}]")
        else:
            for nb in range(BN // 64):
                nn = t("b32")
                ins(f"add.u32 {nn}, {n0}, {nb * 64}")
                ins(f"@{is0} cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
                    f"[{sb}+{nb * 64 * BK * 2}], [{tmb}, {{{nn}, {kc}}}], [{eb}]")
        ins(f"add.u32 {it}, {it}, 1")
        ins(f"add.u32 {kb}, {kb}, 1")
        ins(f"setp.lt.u32 {p}, {kb}, {kend}")
        ins(f"@{p} bra {ktop}")
        ins(f"add.u32 {pu}, {pu}, {ncta}")
        ins(f"setp.lt.u32 {p}, {pu}, {units}")
        ins(f"@{p} bra {ptop}")
        place(pdone)
        # drain: every stage's last load has landed before the CTA may leave
        for s in range(ST):
            used, last, lp = t("pred"), t("b32"), t("b32")
            skip_s = lab("drain_skip")
            ins(f"setp.le.u32 {used}, {it}, {s}")
            ins(f"@{used} bra {skip_s}")
            ins(f"sub.u32 {last}, {it}, 1")
            ins(f"sub.u32 {last}, {last}, {s}")
            ins(f"div.u32 {last}, {last}, {ST}")        # uses of stage s minus one
            ins(f"and.b32 {lp}, {last}, 1")
            wait(f"{bars}+{8 * s}", lp, 0)
            place(skip_s)
        ins(f"bra {end}")

        # ---------------- MMA issuer (warp 1) ----------------
        place(role_mma)
        ism = t("pred")
        elect_one(em, ism)
        it2, mu, lt = t("b32"), t("b32"), t("b32")
        ins(f"mov.u32 {it2}, 0")
        ins(f"mov.u32 {lt}, 0")
        ins(f"mov.u32 {mu}, {cta}")
        mtop, mdone = lab("mma_tile"), lab("mma_done")
        ins(f"setp.ge.u32 {p}, {mu}, {units}")
        ins(f"@{p} bra {mdone}")
        place(mtop)
        _, kb2, kend2, _, _ = unit(mu)
        kfirst = t("b32")
        ins(f"mov.u32 {kfirst}, {kb2}")
        buf, use, upar, apar = t("b32"), t("b32"), t("b32"), t("b32")
        ins(f"and.b32 {buf}, {lt}, 1")
        ins(f"shr.u32 {use}, {lt}, 1")
        ins(f"and.b32 {upar}, {use}, 1")
        ins(f"xor.b32 {apar}, {upar}, 1")
        ab = t("b32")
        ins(f"mad.lo.u32 {ab}, {buf}, 8, {bars}")
        wait(f"{ab}+{acce_off}", apar, 1)
        ins("tcgen05.fence::after_thread_sync")
        dt = t("b32")
        ins(f"mad.lo.u32 {dt}, {buf}, {BN}, {tmem}")
        mk = lab("mma_k")
        place(mk)
        st2, ph2 = t("b32"), t("b32")
        ins(f"rem.u32 {st2}, {it2}, {ST}")
        ins(f"div.u32 {ph2}, {it2}, {ST}")
        ins(f"and.b32 {ph2}, {ph2}, 1")
        fb = t("b32")
        ins(f"mad.lo.u32 {fb}, {st2}, 8, {bars}")
        wait(fb, ph2, 1)
        ins("tcgen05.fence::after_thread_sync")
        sa2, sb2 = t("b32"), t("b32")
        ins(f"mad.lo.u32 {sa2}, {st2}, {a_bytes}, {a_st}")
        ins(f"mad.lo.u32 {sb2}, {st2}, {b_bytes}, {b_st}")
        # descriptors: low word = start address >> 4 (+ LBO in bits 16..29), high word = SBO | version | layout
        adesc_lo, bdesc_lo = t("b32"), t("b32")
        ins(f"shr.u32 {adesc_lo}, {sa2}, 4")
        ins(f"and.b32 {adesc_lo}, {adesc_lo}, 16383")
        ins(f"or.b32 {adesc_lo}, {adesc_lo}, {1 << 16}")
        ins(f"shr.u32 {bdesc_lo}, {sb2}, 4")
        ins(f"and.b32 {bdesc_lo}, {bdesc_lo}, 16383")
        b_lbo = 1 if self.b_kmajor else (64 * BK * 2) >> 4
        ins(f"or.b32 {bdesc_lo}, {bdesc_lo}, {b_lbo << 16}")
        a_hi = _desc_hi(1024)
        b_hi = _desc_hi(1024)
        idesc = idesc_f16(BN, not self.b_kmajor)
        acc0, always = t("pred"), t("pred")
        ins(f"setp.ne.u32 {acc0}, {kb2}, {kfirst}")   # the unit's first MMA overwrites the accumulator
        ins(f"setp.eq.u32 {always}, {kb2}, {kb2}")
        hi_a, hi_b = t("b32"), t("b32")
        ins(f"mov.u32 {hi_a}, {a_hi}")
        ins(f"mov.u32 {hi_b}, {b_hi}")
        for k in range(BK // 16):
            ad, bd = t("b64"), t("b64")
            alo, blo = t("b32"), t("b32")
            ins(f"add.u32 {alo}, {adesc_lo}, {(k * 32) >> 4}")
            b_step = (k * 32) >> 4 if self.b_kmajor else (k * 16 * 128) >> 4
            ins(f"add.u32 {blo}, {bdesc_lo}, {b_step}")
            ins(f"mov.b64 {ad}, {{{alo}, {hi_a}}}")
            ins(f"mov.b64 {bd}, {{{blo}, {hi_b}}}")
            ins(f"@{ism} tcgen05.mma.cta_group::1.kind::f16 [{dt}], {ad}, {bd}, {idesc}, "
                f"{acc0 if k == 0 else always}")
        ins(f"@{ism} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{fb}+{empty_off}]")
        ins(f"add.u32 {it2}, {it2}, 1")
        ins(f"add.u32 {kb2}, {kb2}, 1")
        ins(f"setp.lt.u32 {p}, {kb2}, {kend2}")
        ins(f"@{p} bra {mk}")
        ins(f"@{ism} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{ab}+{accf_off}]")
        ins(f"add.u32 {lt}, {lt}, 1")
        ins(f"add.u32 {mu}, {mu}, {ncta}")
        ins(f"setp.lt.u32 {p}, {mu}, {units}")
        ins(f"@{p} bra {mtop}")
        place(mdone)
        ins(f"bra {end}")

        # ---------------- epilogue (warps 2..5) ----------------
        place(role_epi)
        quarter, row = t("b32"), t("b32")
        ins(f"and.b32 {quarter}, {warp}, 3")
        ins(f"mad.lo.u32 {row}, {quarter}, 32, {lane}")
        lane_off = t("b32")
        ins(f"shl.b32 {lane_off}, {quarter}, 21")        # (32 * quarter) << 16
        lane0 = t("pred")
        elect_one(em, lane0)
        ebase = t("b32")
        ins(f"sub.u32 {ebase}, {warp}, 2")
        ins(f"mad.lo.u32 {ebase}, {ebase}, {2 * STAGE_TILE}, {b_st}")
        ins(f"add.u32 {ebase}, {ebase}, {ST * b_bytes}")
        stage_buf = [ebase, t("b32")]
        ins(f"add.u32 {stage_buf[1]}, {ebase}, {STAGE_TILE}")
        sw = t("b32")
        ins(f"shr.u32 {sw}, {lane}, 1")
        ins(f"and.b32 {sw}, {sw}, 3")
        soff = []
        for i in range(4):
            o = t("b32")
            ins(f"xor.b32 {o}, {sw}, {i}")
            ins(f"shl.b32 {o}, {o}, 4")
            ins(f"mad.lo.u32 {o}, {lane}, 64, {o}")
            soff.append(o)
        eu, lt3, ls = t("b32"), t("b32"), t("b32")
        ins(f"mov.u32 {lt3}, 0")
        ins(f"mov.u32 {ls}, 0")
        ins(f"mov.u32 {eu}, {cta}")
        etop, edone, enext = lab("epi_tile"), lab("epi_done"), lab("epi_next")
        ins(f"setp.ge.u32 {p}, {eu}, {units}")
        ins(f"@{p} bra {edone}")
        place(etop)
        tile3, _, _, whole3, part3 = unit(eu)
        tm3, tn3, ts3 = decode(tile3)
        buf3, use3, par3 = t("b32"), t("b32"), t("b32")
        ins(f"and.b32 {buf3}, {lt3}, 1")
        ins(f"shr.u32 {use3}, {lt3}, 1")
        ins(f"and.b32 {par3}, {use3}, 1")
        ab3 = t("b32")
        ins(f"mad.lo.u32 {ab3}, {buf3}, 8, {bars}")
        wait(f"{ab3}+{accf_off}", par3, 2)
        ins("tcgen05.fence::after_thread_sync")
        taddr = t("b32")
        ins(f"mad.lo.u32 {taddr}, {buf3}, {BN}, {tmem}")
        ins(f"add.u32 {taddr}, {taddr}, {lane_off}")
        # Each warp stages its 32 rows x 64 bytes at a time in its own pair of 2 KB shared
        # buffers, laid out with the 64-byte swizzle (16-byte chunk i of row r at chunk
        # i ^ ((r >> 1) & 3)), and writes them with one TMA bulk-tensor store per box:
        # full, coalesced lines instead of 16-byte pieces of 32 different rows.
        esz = self.c.ty.nbytes
        cw = 64 // esz                                   # columns per store box
        row0, col0 = t("b32"), t("b32")
        ins(f"mad.lo.u32 {row0}, {ts3}, {self.M}, 0")
        ins(f"mad.lo.u32 {row0}, {tm3}, {BM}, {row0}")
        ins(f"mad.lo.u32 {row0}, {quarter}, 32, {row0}")
        ins(f"mul.lo.u32 {col0}, {tn3}, {BN}")

        def store_boxes(values) -> None:
            """Columns c0 .. c0 + cw of this warp's 32 rows, for each c0: ``values(c0)`` gives the
            row's cw values as b32 registers (f32, or f16 pairs), staged and stored with TMA."""
            for j, c0 in enumerate(range(0, BN, cw)):
                sbuf = stage_buf[j % 2]
                ins(f"@{lane0} cp.async.bulk.wait_group.read 1")
                ins("bar.warp.sync -1")
                v = values(c0)
                for i in range(4):
                    a_ = t("b32")
                    ins(f"add.u32 {a_}, {sbuf}, {soff[i]}")
                    ins(f"st.shared.v4.b32 [{a_}], {{{', '.join(v[4 * i:4 * i + 4])}}}")
                ins("fence.proxy.async.shared::cta")
                ins("bar.warp.sync -1")
                cc = t("b32")
                ins(f"add.u32 {cc}, {col0}, {c0}")
                ins(f"@{lane0} cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [{tmc}, {{{cc}, {row0}}}], "
                    f"[{sbuf}]")
                ins(f"@{lane0} cp.async.bulk.commit_group")

        def from_tmem(c0):
            nv = 16 if esz == 4 else 32
            v = [t("b32") for _ in range(nv)]
            tc = t("b32")
            ins(f"add.u32 {tc}, {taddr}, {c0}")
            ins(f"tcgen05.ld.sync.aligned.32x32b.x{nv}.b32 {{{', '.join(v)}}}, [{tc}]")
            ins("tcgen05.wait::ld.sync.aligned")
            if esz == 2:
                h = [t("b32") for _ in range(16)]
                for i in range(16):
                    ins(f"cvt.rn.f16x2.f32 {h[i]}, {v[2 * i + 1]}, {v[2 * i]}")
                v = h
            return v

        tail = lab("epi_tail")
        if self.rem:
            ins(f"@!{whole3} bra {tail}")
        store_boxes(from_tmem)
        ins("tcgen05.fence::before_thread_sync")
        ins(f"mbarrier.arrive.shared::cta.b64 _, [{ab3}+{acce_off}]")
        if self.rem:
            ins(f"bra {enext}")
            self._tail_epilogue(tail, enext, tile3, part3, taddr, ab3, row, lane, bars, ls, store_boxes,
                                acce_off, tail_done_off, tail_last_off, tail_flag_off, wait, p)
        place(enext)
        ins(f"add.u32 {lt3}, {lt3}, 1")
        ins(f"add.u32 {eu}, {eu}, {ncta}")
        ins(f"setp.lt.u32 {p}, {eu}, {units}")
        ins(f"@{p} bra {etop}")
        place(edone)
        ins(f"@{lane0} cp.async.bulk.wait_group 0")       # stores done before the CTA leaves

        # ---------------- common exit ----------------
        place(end)
        ins("barrier.sync 0")
        nodealloc = lab("mm_nodealloc")
        ins(f"setp.ne.u32 {p}, {warp}, 1")
        ins(f"@{p} bra {nodealloc}")
        ins("tcgen05.fence::after_thread_sync")
        ins(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {tmem}, {tmem_cols}")
        place(nodealloc)


    def _tail_epilogue(self, tail, enext, tile3, part3, taddr, ab3, row, lane, bars, ls, store_boxes,
                       acce_off, done_off, last_off, flag_off, wait, p) -> None:
        """A K part of one of the last tiles: its partial goes to the module workspace, and the
        part that arrives last adds all parts in part order (deterministic) and stores C.

        Workspace layout, per (tile, part) slot: [BN / 4 chunks][128 rows] of 16-byte chunks, so a
        warp's store or load of one chunk index touches 512 contiguous bytes.  Arrival: every
        epilogue thread fences its stores and arrives on a CTA mbarrier; thread 0 then bumps the
        tile's counter (``atom.acq_rel.gpu.inc`` wrapping at parts - 1: self-resetting) and
        publishes whether it was the last through shared memory.  No CTA waits for another."""
        em, ins, t, place = self.em, self.em.ins, self.em.tmp, self.em.place
        BN, parts = self.BN, self.parts
        place(tail)
        slot, ws, cnt = t("b32"), t("b64"), t("b64")
        ins(f"sub.u32 {slot}, {tile3}, {self.full_tiles}")
        self.tail_bases(cnt, ws)
        ins(f"mad.wide.u32 {cnt}, {slot}, 4, {cnt}")
        ins(f"mad.lo.u32 {slot}, {slot}, {parts}, {part3}")
        rowb = t("b64")                                   # this row's first chunk, 16 bytes apart per row
        ins(f"mul.wide.u32 {rowb}, {row}, 16")
        ins(f"add.u64 {rowb}, {rowb}, {ws}")
        mine = t("b64")
        ins(f"mul.wide.u32 {mine}, {slot}, {BN // 4 * 128 * 16}")
        ins(f"add.u64 {mine}, {mine}, {rowb}")
        for c0 in range(0, BN, 16):
            v = [t("b32") for _ in range(16)]
            tc = t("b32")
            ins(f"add.u32 {tc}, {taddr}, {c0}")
            ins(f"tcgen05.ld.sync.aligned.32x32b.x16.b32 {{{', '.join(v)}}}, [{tc}]")
            ins("tcgen05.wait::ld.sync.aligned")
            for i in range(4):
                ins(f"st.global.v4.b32 [{mine}+{(c0 // 4 + i) * 128 * 16}], {{{', '.join(v[4 * i:4 * i + 4])}}}")
        ins("tcgen05.fence::before_thread_sync")
        ins(f"mbarrier.arrive.shared::cta.b64 _, [{ab3}+{acce_off}]")      # the accumulator is free
        ins("fence.acq_rel.gpu")
        ins(f"mbarrier.arrive.shared::cta.b64 _, [{bars}+{done_off}]")
        par, lead, flag = t("b32"), t("pred"), t("b32")
        ins(f"and.b32 {par}, {ls}, 1")
        ins(f"add.u32 {ls}, {ls}, 1")
        ins(f"setp.eq.u32 {lead}, {row}, 0")
        notlead = em.label("tail_notlead")
        ins(f"@!{lead} bra {notlead}")
        wait(f"{bars}+{done_off}", par, 3, warp=False)     # all 128 rows of the partial are stored
        old = t("b32")
        ins(f"atom.acq_rel.gpu.global.inc.u32 {old}, [{cnt}], {parts - 1}")
        ins(f"setp.eq.u32 {p}, {old}, {parts - 1}")
        ins(f"selp.u32 {flag}, 1, 0, {p}")
        ins(f"st.shared.u32 [{bars}+{flag_off}], {flag}")
        ins(f"mbarrier.arrive.shared::cta.b64 _, [{bars}+{last_off}]")
        place(notlead)
        wait(f"{bars}+{last_off}", par, 3)
        ins(f"ld.shared.u32 {flag}, [{bars}+{flag_off}]")
        ins(f"setp.eq.u32 {p}, {flag}, 0")
        ins(f"@{p} bra {enext}")
        ins("fence.acq_rel.gpu")
        first = t("b64")                                   # part 0 of this tile
        ins(f"sub.u32 {slot}, {slot}, {part3}")
        ins(f"mul.wide.u32 {first}, {slot}, {BN // 4 * 128 * 16}")
        ins(f"add.u64 {first}, {first}, {rowb}")

        def summed(c0):
            acc = [t("f32") for _ in range(16)]
            for pp in range(parts):
                for i in range(4):
                    off = pp * (BN // 4 * 128 * 16) + (c0 // 4 + i) * 128 * 16
                    v = acc[4 * i:4 * i + 4] if pp == 0 else [t("f32") for _ in range(4)]
                    ins(f"ld.global.cg.v4.f32 {{{', '.join(v)}}}, [{first}+{off}]")
                    if pp:
                        for a_, b_ in zip(acc[4 * i:4 * i + 4], v):
                            ins(f"add.rn.f32 {a_}, {a_}, {b_}")
            out = [t("b32") for _ in range(16)]
            for o_, a_ in zip(out, acc):
                ins(f"mov.b32 {o_}, {a_}")
            return out

        store_boxes(summed)


def recognise(kernel: KernelInfo):
    return TcMatmul.match(kernel)
