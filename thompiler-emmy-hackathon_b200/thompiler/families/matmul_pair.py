"""Tuned family: the f16 tensor-core matmul of ``thompiler.families.matmul`` on CTA pairs
(tcgen05 ``cta_group::2``).

Same recognised IR and result (C[M, N] = A[M, K] @ B, B stored [N, K] or [K, N], f16 in, f32
accumulate, f32 / f16 out, the split-K [S, M, N] form).  A pair of CTAs (a ``.reqnctapercluster
2`` launch, one CTA per SM) computes a 256 x BN tile with one 2-SM MMA per K step of 16:

  CTA r of the pair   holds A rows 128 r .. 128 r + 127 of the tile and B columns
                      (BN / 2) r .. (BN / 2) r + BN / 2 - 1 (K-major: rows of B's [N, K]
                      storage) in its own shared memory, 64-deep K stages;
  leader (r = 0)      its MMA warp issues tcgen05.mma.cta_group::2 (M = 256, N = BN, K = 16)
                      for the pair; the accumulator's rows 128 r .. live in CTA r's tensor memory.

Per SM and K step this reads A 128 x 64 and half of B from shared memory -- a 256 x 256 pair tile
moves a third less operand data per FLOP through L2 and shared memory than the single-CTA
128 x 256 tile.

Warp roles per CTA (192 threads): warp 0 TMA (this CTA's halves; each load completes on the
leader's ``full`` barrier, which the leader posts both CTAs' bytes on), warp 1 the MMA issuer
(leader only; allocates the pair's TMEM in both CTAs), warps 2-5 the epilogue of this CTA's 128
rows (tcgen05.ld -> 64B-swizzled staging -> TMA store, as the single-CTA kernel).  Barriers at
the same offsets in both CTAs: ``empty`` (per stage) and ``acc_full`` (per accumulator) arrive in
both CTAs from one multicast tcgen05.commit; the leader's ``acc_empty`` takes one arrival per
epilogue warp of either CTA.  Every wait is bounded (error word + common exit); the CTAs meet
at a cluster barrier before freeing TMEM, so neither leaves while the other can still signal it.
No TMA load uses cluster multicast: each CTA loads its own halves.
"""

from __future__ import annotations

from thompiler.families.kit import Kit, desc_hi, elect_one, idesc_f16, tmap_address
from thompiler.families.matmul import BK, BM, EPI_WARPS, SM_COUNT, STAGE_TILE, TcMatmul
from thompiler.families.base import TunedKernel
from thompiler.families.tuning import TUNING
from thompiler.load import KernelInfo
from thompiler.lowering.types import F32

PM = 2 * BM                  # rows of a pair tile
PAIR_SLOTS = SM_COUNT // 2   # pairs resident at once
# pair tile widths and their efficiency relative to 256 at full waves, measured on B200: 128 is 0.71
# of 256 at 4096^3 and 192 about 0.8 at 8192 x 3072 x 1024 (0.0530 against 0.0494 ms although it
# fills 6.92 waves of pairs instead of 5.19): per flop each CTA feeds more operand bytes from
# shared memory at narrower tiles
PAIR_WIDTHS = ((256, 1.0), (192, 0.80), (128, 0.71))
SMEM_LIMIT = 227 * 1024


class TcMatmulPair(TcMatmul):
    family = "tcgen05-matmul-pair"
    tail_ranks = 2

    @classmethod
    def match(cls, kernel: KernelInfo):
        if not TUNING.matmul_pair:                                  # the single-CTA kernel instead
            return None
        one = TcMatmul.match.__func__(TcMatmul, kernel)
        if one is None or one.M % PM or kernel.grid[0] % 2:
            return None                    # the cluster launch needs an even generic grid too
        bn = cls.pair_bn(one.M, one.N, one.S, one.b_kmajor)
        if bn is None:
            return None
        return cls(kernel, one.a, one.b, one.c, one.M, one.N, one.K, one.S, one.b_kmajor, bn, one.static_smem)

    @staticmethod
    def pair_bn(M: int, N: int, S: int, b_kmajor: bool = True) -> int | None:
        """The pair tile's width: the best of wave efficiency (pair tiles over the 74 pairs
        resident at once) times the width's own efficiency.  192 needs K-major B (an MN-major B
        is loaded in 64-column boxes, and a CTA holds 96 columns)."""
        forced = TUNING.matmul_bn
        if forced in (128, 192, 256) and N % forced == 0 and (forced != 192 or b_kmajor):
            return forced
        best, best_score = None, -1.0
        for bn, pref in PAIR_WIDTHS:
            if N % bn or (bn == 192 and not b_kmajor):
                continue
            tiles = (M // PM) * (N // bn) * S
            waves = -(-tiles // PAIR_SLOTS)
            score = pref * (tiles / (waves * PAIR_SLOTS) if tiles >= PAIR_SLOTS else tiles / PAIR_SLOTS)
            if score > best_score + 1e-9:
                best, best_score = bn, score
        return best

    def __init__(self, kernel, a, b, c, M, N, K, S, b_kmajor, bn, static_smem):  # noqa: D107
        TunedKernel.__init__(self, kernel)
        self.a, self.b, self.c = a, b, c
        self.M, self.N, self.K, self.S = M, N, K, S
        self.Ks = K // S
        self.b_kmajor = b_kmajor
        self.static_smem = static_smem
        self.BN = bn
        self.HN = bn // 2                                    # B columns held by each CTA
        self.a_bytes = BM * BK * 2
        self.b_bytes = self.HN * BK * 2
        stage = self.a_bytes + self.b_bytes
        self.staging = EPI_WARPS * 2 * STAGE_TILE
        room = SMEM_LIMIT - static_smem - 2048 - self.staging
        self.stages = max(2, min(8, room // stage))
        forced = TUNING.matmul_stages
        if 2 <= forced <= room // stage:
            self.stages = forced
        self.smem = self.stages * stage + self.staging + 1024 + 256
        self.tiles = (M // PM) * (N // bn) * S
        # the last, partial wave of pair tiles: its `rem` tiles are cut along K into `parts` units,
        # as in the single-CTA kernel (each CTA of a pair keeps its own partial and counter)
        kblocks = self.Ks // BK
        rem0 = self.tiles % PAIR_SLOTS if self.tiles > PAIR_SLOTS else 0
        # the partial last wave: where its tiles halved fit one wave of pairs, each 256-wide tile
        # becomes two 256 x 128 units over the full K (no partials; measured faster than the K
        # split on 4096^3, and the only cut for a K too short to split).  B must be K-major: a half
        # unit loads the same 128-row box of B at its own column offset and its N = 128 MMA reads
        # the first 64 rows of each CTA's box.  Otherwise the tiles are cut along K into parts.
        self.hrem = 0
        if rem0 and 2 * rem0 <= PAIR_SLOTS and bn == 256 and S == 1 and b_kmajor and TUNING.matmul_half_tail:
            self.hrem = rem0
        rem = 0 if self.hrem else rem0
        parts = min(kblocks // TUNING.matmul_tail_kblocks, PAIR_SLOTS // rem) if rem else 1
        if S != 1 or c.ty is not F32 or parts < 2 or not TUNING.matmul_split_tail:
            rem, parts = 0, 1
        self.rem, self.parts = rem, parts
        self.full_tiles = self.tiles - rem - self.hrem
        self.units = self.full_tiles + rem * parts + 2 * self.hrem
        self.pairs = min(self.units, PAIR_SLOTS)
        self.ctas = 2 * self.pairs

    def sidecar(self) -> dict:
        side = super().sidecar()
        a, b = self.a, self.b
        side["tmaps"][0]["box"] = [BK, BM]
        if self.b_kmajor:
            side["tmaps"][1]["box"] = [BK, self.HN]
        side["grid"] = [self.ctas, 1, 1]
        side["cluster"] = [2, 1, 1]
        side["tile"] = [PM, self.BN, BK]
        assert side["tmap_ptrs"]["params"] == [a.name, b.name, self.c.name]
        return side

    def guard(self, generic: str) -> None:
        super().guard(generic)
        self.em.entry_attrs.append(".reqnctapercluster 2, 1, 1")

    # ---- the tuned body -------------------------------------------------------------

    def emit_tuned(self) -> None:  # noqa: C901 - one kernel, written out in order
        em = self.em
        t, ins, place, lab = em.tmp, em.ins, em.place, em.label
        BN, HN, ST = self.BN, self.HN, self.stages
        a_bytes, b_bytes = self.a_bytes, self.b_bytes
        tiles_m, tiles_n = self.M // PM, self.N // BN
        kblocks = self.Ks // BK
        mcommit = "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        tma_ld = "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        self.pdl_trigger()

        tid, warp, lane = t("b32"), t("b32"), t("b32")
        ins(f"mov.u32 {tid}, %tid.x")
        ins(f"shr.u32 {warp}, {tid}, 5")
        ins(f"and.b32 {lane}, {tid}, 31")
        rank = self.special("%cluster_ctarank")
        base = t("b32")
        ins(f"mov.u32 {base}, smem_pool")
        ins(f"add.u32 {base}, {base}, 1023")
        ins(f"and.b32 {base}, {base}, -1024")
        # shared (same offsets in both CTAs): A stages | B stages | epilogue staging | barriers
        a_st, b_st, bars = base, t("b32"), t("b32")
        ins(f"add.u32 {b_st}, {base}, {ST * a_bytes}")
        ins(f"add.u32 {bars}, {base}, {ST * (a_bytes + b_bytes) + self.staging}")
        empty_off, accf_off, acce_off, slot_off = 8 * ST, 16 * ST, 16 * ST + 16, 16 * ST + 32
        tail_done_off, tail_last_off, tail_flag_off = 16 * ST + 40, 16 * ST + 48, 16 * ST + 56
        p = t("pred")
        skip = lab("mp_noinit")
        ins(f"setp.ne.u32 {p}, {tid}, 0")
        ins(f"@{p} bra {skip}")
        for s in range(ST):
            ins(f"mbarrier.init.shared::cta.b64 [{bars}+{8 * s}], 1")
            ins(f"mbarrier.init.shared::cta.b64 [{bars}+{empty_off + 8 * s}], 1")
        for b in range(2):
            ins(f"mbarrier.init.shared::cta.b64 [{bars}+{accf_off + 8 * b}], 1")
            ins(f"mbarrier.init.shared::cta.b64 [{bars}+{acce_off + 8 * b}], {2 * EPI_WARPS}")
        if self.rem:
            ins(f"mbarrier.init.shared::cta.b64 [{bars}+{tail_done_off}], {32 * EPI_WARPS}")
            ins(f"mbarrier.init.shared::cta.b64 [{bars}+{tail_last_off}], 1")
        ins("fence.mbarrier_init.release.cluster")
        ins("fence.proxy.async.shared::cta")
        place(skip)
        # TMEM: warp 1 of both CTAs allocates the pair's 2 x BN accumulator columns
        tmem_cols = 512 if 2 * BN > 256 else 256
        noalloc = lab("mp_noalloc")
        ins(f"setp.ne.u32 {p}, {warp}, 1")
        ins(f"@{p} bra {noalloc}")
        slot = t("b32")
        ins(f"add.u32 {slot}, {bars}, {slot_off}")
        ins(f"tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [{slot}], {tmem_cols}")
        ins("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned")
        place(noalloc)
        ins("tcgen05.fence::before_thread_sync")
        ins("bar.sync 0")
        # both CTAs' barriers are initialised before either signals the other's
        ins("barrier.cluster.arrive.release")
        ins("barrier.cluster.wait.acquire")
        ins("tcgen05.fence::after_thread_sync")
        # barriers and TMEM are set up while the stream's previous kernel may still run; from
        # here on the pair reads and writes global data
        self.pdl_wait()
        tmem = t("b32")
        ins(f"ld.shared.u32 {tmem}, [{bars}+{slot_off}]")
        lbars = t("b32")                                   # the leader's barriers, cluster address
        ins(f"mapa.shared::cluster.u32 {lbars}, {bars}, 0")
        mask = t("b16")
        ins(f"mov.b16 {mask}, 3")
        lead_cta = t("pred")
        ins(f"setp.eq.u32 {lead_cta}, {rank}, 0")
        pid, npair = self.special("%clusterid.x"), self.special("%nclusterid.x")

        tma, tmb, tmc = (tmap_address(em, self.tmap_set, 3, i) for i in range(3))
        errp = t("b64")
        ins(f"mov.u64 {errp}, thc_error")
        end = lab("mp_end")
        kit = Kit(em, errp, end)

        def decode(tile: str):
            tm_, tn_, ts_, r = t("b32"), t("b32"), t("b32"), t("b32")
            ins(f"rem.u32 {tm_}, {tile}, {tiles_m}")
            ins(f"div.u32 {r}, {tile}, {tiles_m}")
            ins(f"rem.u32 {tn_}, {r}, {tiles_n}")
            ins(f"div.u32 {ts_}, {r}, {tiles_n}")
            return tm_, tn_, ts_

        units, full_tiles, parts = self.units, self.full_tiles, self.parts

        def unit(u: str):
            """Work unit u -> (pair tile, first and end K block, is-whole-tile predicate, part):
            units below full_tiles are whole tiles, the rest cut the last tiles along K into
            parts, or along N into halves (part = the half, 0 or 1)."""
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
            if self.hrem:
                ins(f"sub.u32 {v}, {u}, {full_tiles}")
                ins(f"@!{whole} shr.u32 {tile_}, {v}, 1")
                ins(f"@!{whole} add.u32 {tile_}, {tile_}, {full_tiles}")
                ins(f"@!{whole} and.b32 {part}, {v}, 1")
            return tile_, lo, hi_, whole, part

        role_mma, role_epi = lab("mp_mma"), lab("mp_epi")
        ins(f"setp.eq.u32 {p}, {warp}, 1")
        ins(f"@{p} bra {role_mma}")
        ins(f"setp.gt.u32 {p}, {warp}, 1")
        ins(f"@{p} bra {role_epi}")

        # ---------------- producer (warp 0 of each CTA: this CTA's A rows and B half) ----------------
        is0, post = t("pred"), t("pred")
        elect_one(em, is0)
        ins(f"and.pred {post}, {is0}, {lead_cta}")       # the leader posts both CTAs' bytes
        it, pu = t("b32"), t("b32")
        ins(f"mov.u32 {it}, 0")
        ins(f"mov.u32 {pu}, {pid}")
        ptop = lab("mp_prod_tile")
        ins(f"setp.ge.u32 {p}, {pu}, {units}")
        ins(f"@{p} bra {end}")
        place(ptop)
        ptile, kb, kend, pwhole, ppart = unit(pu)
        tm_, tn_, ts_ = decode(ptile)
        m0, n0, k0 = t("b32"), t("b32"), t("b32")
        ins(f"mul.lo.u32 {m0}, {tm_}, {PM}")
        ins(f"mad.lo.u32 {m0}, {rank}, {BM}, {m0}")
        ins(f"mul.lo.u32 {n0}, {tn_}, {BN}")
        if self.hrem:
            # half unit h: columns 128 h .. of the tile, 64 per CTA; the box still spans 128 rows
            # (the second 64 are not read; past N they are the tensor map's zero fill)
            nh = t("b32")
            ins(f"mad.lo.u32 {nh}, {ppart}, {BN // 2}, {n0}")
            ins(f"mad.lo.u32 {nh}, {rank}, {HN // 2}, {nh}")
        ins(f"mad.lo.u32 {n0}, {rank}, {HN}, {n0}")
        if self.hrem:
            ins(f"@!{pwhole} mov.u32 {n0}, {nh}")
        ins(f"mul.lo.u32 {k0}, {ts_}, {self.Ks}")
        ktop = lab("mp_prod_k")
        place(ktop)
        stage, eb, fb = t("b32"), t("b32"), t("b32")
        ins(f"rem.u32 {stage}, {it}, {ST}")
        ins(f"mad.lo.u32 {eb}, {stage}, 8, {bars}")
        kit.wait(f"{eb}+{empty_off}", kit.parity(it, ST, flip=True), 0)
        ins(f"mad.lo.u32 {fb}, {stage}, 8, {lbars}")
        sa, sb, kc = t("b32"), t("b32"), t("b32")
        ins(f"mad.lo.u32 {sa}, {stage}, {a_bytes}, {a_st}")
        ins(f"mad.lo.u32 {sb}, {stage}, {b_bytes}, {b_st}")
        ins(f"mad.lo.u32 {kc}, {kb}, {BK}, {k0}")
        ins(f"@{post} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{eb}], {2 * (a_bytes + b_bytes)}")
        ins(f"@{is0} {tma_ld} [{sa}], [{tma}, {{{kc}, {m0}}}], [{fb}]")
        if self.b_kmajor:
            ins(f"@{is0} {tma_ld} [{sb}], [{tmb}, {{{kc}, {n0}}}], [{fb}]")
        else:
            for nb in range(HN // 64):
                nn = t("b32")
                ins(f"add.u32 {nn}, {n0}, {nb * 64}")
                ins(f"@{is0} {tma_ld} [{sb}+{nb * 64 * BK * 2}], [{tmb}, {{{nn}, {kc}}}], [{fb}]")
        ins(f"add.u32 {it}, {it}, 1")
        ins(f"add.u32 {kb}, {kb}, 1")
        ins(f"setp.lt.u32 {p}, {kb}, {kend}")
        ins(f"@{p} bra {ktop}")
        ins(f"add.u32 {pu}, {pu}, {npair}")
        ins(f"setp.lt.u32 {p}, {pu}, {units}")
        ins(f"@{p} bra {ptop}")
        # every load of this CTA is consumed by an MMA whose completion the epilogues wait for
        # before the common exit's cluster barrier, so none is in flight when the CTAs leave
        ins(f"bra {end}")

        # ---------------- MMA issuer (the leader's warp 1, for the pair) ----------------
        place(role_mma)
        ins(f"@!{lead_cta} bra {end}")
        ism = t("pred")
        elect_one(em, ism)
        hi = t("b32")
        ins(f"mov.u32 {hi}, {desc_hi(1024)}")
        idesc = idesc_f16(PM, BN, b_mn_major=not self.b_kmajor)
        zero = t("b32")
        ins(f"mov.u32 {zero}, 0")
        always, never = t("pred"), t("pred")
        ins(f"setp.eq.u32 {always}, {zero}, 0")
        ins(f"setp.ne.u32 {never}, {zero}, 0")
        it2, mu, lt = t("b32"), t("b32"), t("b32")
        ins(f"mov.u32 {it2}, 0")
        ins(f"mov.u32 {lt}, 0")
        ins(f"mov.u32 {mu}, {pid}")
        mtop = lab("mp_mma_tile")
        ins(f"setp.ge.u32 {p}, {mu}, {units}")
        ins(f"@{p} bra {end}")
        place(mtop)
        _, kb2, kend2, mwhole, _ = unit(mu)
        idr = t("b32")
        ins(f"mov.u32 {idr}, {idesc}")
        if self.hrem:
            ins(f"@!{mwhole} mov.u32 {idr}, {idesc_f16(PM, BN // 2, b_mn_major=not self.b_kmajor)}")
        kfirst = t("b32")
        ins(f"mov.u32 {kfirst}, {kb2}")
        buf, ab = t("b32"), t("b32")
        ins(f"and.b32 {buf}, {lt}, 1")
        ins(f"mad.lo.u32 {ab}, {buf}, 8, {bars}")
        use = t("b32")
        ins(f"shr.u32 {use}, {lt}, 1")
        kit.wait(f"{ab}+{acce_off}", kit.parity(use, 1, flip=True), 1, cluster=True)
        ins("tcgen05.fence::after_thread_sync")
        dt = t("b32")
        ins(f"mad.lo.u32 {dt}, {buf}, {BN}, {tmem}")
        mk = lab("mp_mma_k")
        place(mk)
        st2, fb2 = t("b32"), t("b32")
        ins(f"rem.u32 {st2}, {it2}, {ST}")
        ins(f"mad.lo.u32 {fb2}, {st2}, 8, {bars}")
        kit.wait(fb2, kit.parity(it2, ST), 1)
        ins("tcgen05.fence::after_thread_sync")
        sa2, sb2 = t("b32"), t("b32")
        ins(f"mad.lo.u32 {sa2}, {st2}, {a_bytes}, {a_st}")
        ins(f"mad.lo.u32 {sb2}, {st2}, {b_bytes}, {b_st}")
        ad0 = kit.desc(sa2, 16, hi)
        bd0 = kit.desc(sb2, 16 if self.b_kmajor else 64 * BK * 2, hi)
        first = t("pred")
        ins(f"setp.ne.u32 {first}, {kb2}, {kfirst}")  # the unit's first MMA overwrites the accumulator
        for k in range(BK // 16):
            ad = kit.desc_add(ad0, k * 32)
            bd = kit.desc_add(bd0, k * 32 if self.b_kmajor else k * 16 * 128)
            ins(f"@{ism} tcgen05.mma.cta_group::2.kind::f16 [{dt}], {ad}, {bd}, {idr}, "
                f"{first if k == 0 else always}")
        ins(f"@{ism} {mcommit} [{fb2}+{empty_off}], {mask}")
        ins(f"add.u32 {it2}, {it2}, 1")
        ins(f"add.u32 {kb2}, {kb2}, 1")
        ins(f"setp.lt.u32 {p}, {kb2}, {kend2}")
        ins(f"@{p} bra {mk}")
        ins(f"@{ism} {mcommit} [{ab}+{accf_off}], {mask}")
        ins(f"add.u32 {lt}, {lt}, 1")
        ins(f"add.u32 {mu}, {mu}, {npair}")
        ins(f"setp.lt.u32 {p}, {mu}, {units}")
        ins(f"@{p} bra {mtop}")
        ins(f"bra {end}")

        # ---------------- epilogue (warps 2..5 of each CTA: its 128 rows) ----------------
        place(role_epi)
        quarter, row = t("b32"), t("b32")
        ins(f"and.b32 {quarter}, {warp}, 3")
        ins(f"mad.lo.u32 {row}, {quarter}, 32, {lane}")   # this thread's row of the CTA's 128
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
        ins(f"mov.u32 {eu}, {pid}")
        etop, edone, enext = lab("mp_epi_tile"), lab("mp_epi_done"), lab("mp_epi_next")
        ins(f"setp.ge.u32 {p}, {eu}, {units}")
        ins(f"@{p} bra {edone}")
        place(etop)
        tile3, _, _, whole3, part3 = unit(eu)
        tm3, tn3, ts3 = decode(tile3)
        buf3, ab3, lab3 = t("b32"), t("b32"), t("b32")
        ins(f"and.b32 {buf3}, {lt3}, 1")
        ins(f"mad.lo.u32 {ab3}, {buf3}, 8, {bars}")
        ins(f"mad.lo.u32 {lab3}, {buf3}, 8, {lbars}")
        use3 = t("b32")
        ins(f"shr.u32 {use3}, {lt3}, 1")
        kit.wait(f"{ab3}+{accf_off}", kit.parity(use3, 1), 2)
        ins("tcgen05.fence::after_thread_sync")
        taddr = t("b32")
        ins(f"mad.lo.u32 {taddr}, {buf3}, {BN}, {tmem}")
        ins(f"add.u32 {taddr}, {taddr}, {lane_off}")
        esz = self.c.ty.nbytes
        cw = 64 // esz
        row0, col0 = t("b32"), t("b32")
        ins(f"mul.lo.u32 {row0}, {ts3}, {self.M}")
        ins(f"mad.lo.u32 {row0}, {tm3}, {PM}, {row0}")
        ins(f"mad.lo.u32 {row0}, {rank}, {BM}, {row0}")
        ins(f"mad.lo.u32 {row0}, {quarter}, 32, {row0}")
        ins(f"mul.lo.u32 {col0}, {tn3}, {BN}")

        def free_accumulator() -> None:
            """This warp has read the accumulator out: one arrival on the leader's barrier."""
            ins("tcgen05.fence::before_thread_sync")
            ins("bar.warp.sync -1")
            ins(f"@{lane0} mbarrier.arrive.release.cluster.shared::cluster.b64 _, [{lab3}+{acce_off}]")

        def store_boxes(values, free_after_last: bool, width: int = BN) -> None:
            """Columns c0 .. c0 + cw of this warp's 32 rows, for each c0 < width: ``values(c0)``
            gives the row's cw values as b32 registers (f32, or f16 pairs), staged (64-byte
            swizzle) and stored with TMA."""
            for j, c0 in enumerate(range(0, width, cw)):
                sbuf = stage_buf[j % 2]
                ins(f"@{lane0} cp.async.bulk.wait_group.read 1")
                ins("bar.warp.sync -1")
                v = values(c0)
                if free_after_last and c0 + cw == width:
                    free_accumulator()
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

        tail = lab("mp_epi_tail")
        if self.rem or self.hrem:
            ins(f"@!{whole3} bra {tail}")
        store_boxes(from_tmem, True)
        if self.hrem:
            # a half unit: 128 columns of the tile, starting at 128 h
            ins(f"bra {enext}")
            place(tail)
            ins(f"mad.lo.u32 {col0}, {part3}, {BN // 2}, {col0}")
            store_boxes(from_tmem, True, BN // 2)
        if self.rem:
            ins(f"bra {enext}")
            self._pair_tail(tail, enext, tile3, part3, rank, taddr, row, bars, ls, store_boxes, free_accumulator,
                            tail_done_off, tail_last_off, tail_flag_off, kit, p)
        place(enext)
        ins(f"add.u32 {lt3}, {lt3}, 1")
        ins(f"add.u32 {eu}, {eu}, {npair}")
        ins(f"setp.lt.u32 {p}, {eu}, {units}")
        ins(f"@{p} bra {etop}")
        place(edone)
        ins(f"@{lane0} cp.async.bulk.wait_group 0")       # stores done before the CTA leaves

        # ---------------- common exit: both CTAs, then free the pair's TMEM ----------------
        place(end)
        ins("tcgen05.fence::before_thread_sync")
        ins("barrier.sync 0")
        ins("barrier.cluster.arrive.release")
        ins("barrier.cluster.wait.acquire")
        nod = lab("mp_nodealloc")
        ins(f"setp.ne.u32 {p}, {warp}, 1")
        ins(f"@{p} bra {nod}")
        ins("tcgen05.fence::after_thread_sync")
        ins(f"tcgen05.dealloc.cta_group::2.sync.aligned.b32 {tmem}, {tmem_cols}")
        place(nod)


    def _pair_tail(self, tail, enext, tile3, part3, rank, taddr, row, bars, ls, store_boxes, free_accumulator,
                   done_off, last_off, flag_off, kit, p) -> None:
        """A K part of one of the last pair tiles, for this CTA's 128 rows: its partial goes to the
        module workspace, and the part that arrives last (per tile and CTA rank) adds all parts in
        part order -- deterministic -- and stores C.

        Workspace slot (tail tile, rank, part): [BN / 4 chunks][128 rows] of 16-byte chunks, so a
        warp's store or load of one chunk index touches 512 contiguous bytes.  Arrival: every
        epilogue thread fences its stores and arrives on a CTA mbarrier; thread 0 then bumps the
        (tile, rank) counter (``atom.acq_rel.gpu.inc`` wrapping at parts - 1: self-resetting) and
        publishes through shared memory whether it was the last.  No CTA waits for another."""
        em, ins, t, place = self.em, self.em.ins, self.em.tmp, self.em.place
        BN, parts = self.BN, self.parts
        slot_bytes = BN // 4 * 128 * 16
        place(tail)
        slot, ws, cnt = t("b32"), t("b64"), t("b64")
        ins(f"sub.u32 {slot}, {tile3}, {self.full_tiles}")
        ins(f"mad.lo.u32 {slot}, {slot}, 2, {rank}")           # (tail tile, rank)
        self.tail_bases(cnt, ws)
        ins(f"mad.wide.u32 {cnt}, {slot}, 4, {cnt}")
        ins(f"mul.lo.u32 {slot}, {slot}, {parts}")             # its part 0
        rowb = t("b64")                                        # this row's first chunk, 16 bytes apart per row
        ins(f"mul.wide.u32 {rowb}, {row}, 16")
        ins(f"add.u64 {rowb}, {rowb}, {ws}")
        first, mine = t("b64"), t("b64")
        ins(f"mul.wide.u32 {first}, {slot}, {slot_bytes}")
        ins(f"add.u64 {first}, {first}, {rowb}")
        ins(f"mul.wide.u32 {mine}, {part3}, {slot_bytes}")
        ins(f"add.u64 {mine}, {mine}, {first}")
        for c0 in range(0, BN, 16):
            v = [t("b32") for _ in range(16)]
            tc = t("b32")
            ins(f"add.u32 {tc}, {taddr}, {c0}")
            ins(f"tcgen05.ld.sync.aligned.32x32b.x16.b32 {{{', '.join(v)}}}, [{tc}]")
            ins("tcgen05.wait::ld.sync.aligned")
            for i in range(4):
                ins(f"st.global.v4.b32 [{mine}+{(c0 // 4 + i) * 128 * 16}], {{{', '.join(v[4 * i:4 * i + 4])}}}")
        free_accumulator()
        ins("fence.acq_rel.gpu")
        ins(f"mbarrier.arrive.shared::cta.b64 _, [{bars}+{done_off}]")
        par, lead, flag = t("b32"), t("pred"), t("b32")
        ins(f"and.b32 {par}, {ls}, 1")
        ins(f"add.u32 {ls}, {ls}, 1")
        ins(f"setp.eq.u32 {lead}, {row}, 0")
        notlead = em.label("mp_tail_notlead")
        ins(f"@!{lead} bra {notlead}")
        kit.wait(f"{bars}+{done_off}", par, 3, warp=False)     # all 128 rows of the partial are stored
        old = t("b32")
        ins(f"atom.acq_rel.gpu.global.inc.u32 {old}, [{cnt}], {parts - 1}")
        ins(f"setp.eq.u32 {p}, {old}, {parts - 1}")
        ins(f"selp.u32 {flag}, 1, 0, {p}")
        ins(f"st.shared.u32 [{bars}+{flag_off}], {flag}")
        ins(f"mbarrier.arrive.shared::cta.b64 _, [{bars}+{last_off}]")
        place(notlead)
        kit.wait(f"{bars}+{last_off}", par, 3)
        ins(f"ld.shared.u32 {flag}, [{bars}+{flag_off}]")
        ins(f"setp.eq.u32 {p}, {flag}, 0")
        ins(f"@{p} bra {enext}")
        ins("fence.acq_rel.gpu")

        def summed(c0):
            acc = [t("f32") for _ in range(16)]
            for pp in range(parts):
                for i in range(4):
                    off = pp * slot_bytes + (c0 // 4 + i) * 128 * 16
                    v = acc[4 * i:4 * i + 4] if pp == 0 else [t("f32") for _ in range(4)]
                    ins(f"ld.global.cg.v4.f32 {{{', '.join(v)}}}, [{first}+{off}]")
                    if pp:
                        for a_, b_ in zip(acc[4 * i:4 * i + 4], v):
                            ins(f"add.rn.f32 {a_}, {a_}, {b_}")
            out = [t("b32") for _ in range(16)]
            for o_, a_ in zip(out, acc):
                ins(f"mov.b32 {o_}, {a_}")
            return out

        store_boxes(summed, False)

def recognise(kernel: KernelInfo):
    return TcMatmulPair.match(kernel)
