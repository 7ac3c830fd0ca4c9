"""Tuned family: attention, softmax(Q K^T / c) V, on a CTA pair (tcgen05 cta_group::2).

The same recognised IR and semantics as ``thompiler.families.attention``
(the a01 / a02 schedule; f16 Q, K, V, out; c from a one-element buffer),
for D = 128 and S_q a multiple of 256 (opt-in: THOMPILER_ATTN_PAIR=1; threads
per query row: THOMPILER_ATTN_PAIR_SPLIT = 1, 2 or 4).  Measured on B200, one 2-SM MMA
with A from tensor memory (M = 256 over the pair, N = 128, K = 16) takes
74 cycles -- 7,060 FLOP/cycle per SM, against 5,430 for the single-CTA
128 x 128 x 16 form with both operands in shared memory.  This kernel keeps
both of attention's products in that form:

  S = Q K^T   A = Q from TMEM (copied in from shared memory with tcgen05.cp),
              B = K: each CTA of the pair holds 64 of the block's 128 keys;
  O += P V    A = P from TMEM (written by the softmax threads over S),
              B = V: each CTA holds 64 of the 128 d columns (MN-major).

Pair p (CTAs 2p, 2p + 1 of a ``.reqnctapercluster 2`` launch) takes
pair-tiles p, p + n_pairs, ...: 256 query rows of one head, 128 per CTA.
Per CTA, 4 h softmax warps (h threads per query row, exchanging partial row
maxima and sums through shared memory), a TMA warp and an MMA warp;
only the leader CTA's MMA warp issues (for both).  TMEM per CTA: O at 0
(128 columns), S_0 / S_1 at 128 / 256 (key blocks alternate, so the
softmax of block j overlaps PV(j - 1) and S(j + 1)), Q_0 / Q_1 at 384 / 448
(tiles alternate).  MMA order: S(0), S(1), then per block j: PV(j), S(j + 2).

Barriers (same offsets in both CTAs): the leader's q_full / k_full / v_full
count both CTAs' TMA bytes (each CTA's loads signal the leader's barrier, the
leader posts the expected bytes); k_empty / v_empty / q_free / s_full / o_done
arrive in both CTAs from one multicast tcgen05.commit; p_full and o_free
live in the leader and take one arrival per softmax warp of either CTA.
p_full, s_full and o_done come in pairs indexed by the key block's parity,
so every parity wait is at most one phase away from its barrier.  All waits
are bounded (thompiler.families.kit); the CTAs meet at a cluster barrier
before exit, so neither leaves while the other can still signal it.

Measured at [8, 16, 2048, 128] it runs at 687 TFLOP/s (h = 1, 2 or 4 alike)
against the single-CTA kernel's 1064, hence opt-in.  S and PV MMAs issued
alternately average ~128 cycles per 2-SM instruction (74 for either form
alone), and with only two key blocks in flight the cross-SM round trip
(commit -> softmax -> remote arrive -> issue) stays exposed.
"""

from __future__ import annotations

import os

from thompiler.families.attention import BM, BN, LOG2E, TcAttention, _Exp2, _f32bits, _tree, POLY_PAIRS
from thompiler.families.base import TunedKernel
from thompiler.families.kit import Kit, desc_hi, idesc_f16
from thompiler.load import KernelInfo

PAIR_SLOTS = 74                     # CTA pairs resident at once: 148 SMs, one CTA per SM
KH = BN // 2                        # keys of a block held by each CTA of the pair
BAR_BYTES = 512                     # mbarriers and the TMEM address slot


class TcAttentionPair(TcAttention):
    family = "tcgen05-attention-pair"

    @classmethod
    def match(cls, kernel: KernelInfo):
        # opt-in (THOMPILER_ATTN_PAIR=1): measured on B200 at [8, 16, 2048, 128] it runs at 687
        # TFLOP/s against the single-CTA kernel's 1064 -- with only two key blocks in flight the
        # cross-SM round trip (commit -> softmax -> remote arrive -> issue) is not hidden, and S and
        # PV MMAs issued alternately average ~128 cycles per 2-SM instruction, not 74
        if os.environ.get("THOMPILER_ATTN_PAIR", "0") != "1":
            return None
        one = TcAttention.match.__func__(TcAttention, kernel)
        if one is None or one.D != 128 or one.Sq % (2 * BM):
            return None
        return cls(kernel, one.pq, one.pk, one.pv, one.pout, one.pscale, one.heads, one.Sq, one.Sk, one.D)

    def __init__(self, kernel, q, k, v, out, scale, heads, Sq, Sk, D):
        TunedKernel.__init__(self, kernel)
        self.pq, self.pk, self.pv, self.pout, self.pscale = q, k, v, out, scale
        self.heads, self.Sq, self.Sk, self.D = heads, Sq, Sk, D
        self.qt = 1
        # h softmax threads per query row (1, 2 or 4): each takes 128 / h of a key block's scores
        # and D / h of O's columns, so each SM sub-partition runs h softmax warps
        self.h = int(os.environ.get("THOMPILER_ATTN_PAIR_SPLIT", "4"))
        assert self.h in (1, 2, 4), "THOMPILER_ATTN_PAIR_SPLIT is 1, 2 or 4"
        self.q_bytes = BM * D * 2              # this CTA's 128 query rows
        self.k_bytes = KH * D * 2              # its 64 keys of a block, all d
        self.v_bytes = BN * (D // 2) * 2       # all 128 keys, its 64 d columns
        self.sm_warps = 4 * self.h
        self.w_tma, self.w_mma = self.sm_warps, self.sm_warps + 1
        self.threads = 32 * (self.sm_warps + 2)
        warps = -(-max(self.threads, kernel.threads_per_cta) // 32)
        self.maxnreg = min(255, 16384 // (32 * -(-warps // 4)) // 8 * 8)
        self.reg_split = None
        # per softmax warp a 32-row output box: 64 columns (128 B, 128-byte swizzle), or 32 (64 B,
        # unswizzled) when a thread holds 32 of O's columns
        self.box_cols = min(64, D // self.h)
        self.box_bytes = 2 * self.box_cols
        self.stage_bytes = self.sm_warps * 32 * self.box_bytes
        # h > 1: partial row maxima (two sets, alternate key blocks) and partial row sums
        self.xchg_bytes = 3 * self.h * BM * 4 if self.h > 1 else 0
        fixed = self.q_bytes + self.stage_bytes + self.xchg_bytes + 1024 + BAR_BYTES
        self.ks = self.vs = min(5, (227 * 1024 - fixed) // (self.k_bytes + self.v_bytes))
        self.smem = fixed + self.ks * self.k_bytes + self.vs * self.v_bytes
        self.pair_tiles = heads * (Sq // (2 * BM))
        self.tiles = 2 * self.pair_tiles
        self.pairs = min(self.pair_tiles, PAIR_SLOTS)

    def sidecar(self) -> dict:
        D = self.D

        def tm(name, prm, rows, box):
            return {"global": name, "param": prm.name, "dtype": "f16", "dims": [D, rows],
                    "strides": [D * 2], "box": list(box), "swizzle": 3}
        maps = [tm("thc_tmap_q", self.pq, self.heads * self.Sq, (64, BM)),
                tm("thc_tmap_k", self.pk, self.heads * self.Sk, (64, KH)),
                tm("thc_tmap_v", self.pv, self.heads * self.Sk, (64, BN)),
                tm("thc_tmap_o", self.pout, self.heads * self.Sq, (self.box_cols, 32))]
        maps[-1]["swizzle"] = 3 if self.box_bytes == 128 else 0
        return {"grid": [2 * self.pairs, 1, 1], "block": [self.threads, 1, 1], "cluster": [2, 1, 1],
                "smem_bytes": self.smem, "tmaps": maps,
                "tmap_ptrs": {"global": "thc_tmap_ptr", "params": [m["param"] for m in maps]},
                "error_word": "thc_error", "tile": [2 * BM, BN, D], "stages": [self.ks, self.vs]}

    def guard(self, generic: str) -> None:
        super().guard(generic)
        # the launch runs CTA pairs (meta.json's generic launch too: its grid, heads * S * D / threads
        # with S a multiple of 256, is even)
        self.em.entry_attrs.append(".reqnctapercluster 2, 1, 1")

    # ---- the tuned body ----------------------------------------------------------------

    def emit_tuned(self) -> None:  # noqa: C901 - one kernel, in order
        em = self.em
        t, ins, place, lab = em.tmp, em.ins, em.place, em.label
        D, n_blk = self.D, self.Sk // BN
        qb, kb, vb = self.q_bytes, self.k_bytes, self.v_bytes
        KS, VS = self.ks, self.vs
        mcommit = "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        tma = "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        remote_arrive = "mbarrier.arrive.release.cluster.shared::cluster.b64 _,"

        tid, warp, lane = t("b32"), t("b32"), t("b32")
        ins(f"mov.u32 {tid}, %tid.x")
        ins(f"shr.u32 {warp}, {tid}, 5")
        ins(f"and.b32 {lane}, {tid}, 31")
        rank = self.special("%cluster_ctarank")
        base = t("b32")
        ins(f"mov.u32 {base}, smem_pool")
        ins(f"add.u32 {base}, {base}, 1023")
        ins(f"and.b32 {base}, {base}, -1024")
        # shared (same offsets in both CTAs): Q | K ring | V ring | output staging | exchange | barriers
        q_s = base
        H = self.h
        k0, v0, stage0, xchg, bars = t("b32"), t("b32"), t("b32"), t("b32"), t("b32")
        ins(f"add.u32 {k0}, {base}, {qb}")
        ins(f"add.u32 {v0}, {base}, {qb + KS * kb}")
        ins(f"add.u32 {stage0}, {base}, {qb + KS * kb + VS * vb}")
        ins(f"add.u32 {xchg}, {stage0}, {self.stage_bytes}")
        ins(f"add.u32 {bars}, {xchg}, {self.xchg_bytes}")
        nb = 0

        def bar() -> int:
            nonlocal nb
            nb += 1
            return (nb - 1) * 8
        q_full, q_free = bar(), bar()
        k_full, k_empty = [bar() for _ in range(KS)], [bar() for _ in range(KS)]
        v_full, v_empty = [bar() for _ in range(VS)], [bar() for _ in range(VS)]
        s_full = [bar(), bar()]             # by key-block parity
        p_full = [bar(), bar()]             # leader: one arrival per softmax warp of either CTA
        o_done = [bar(), bar()]             # by the parity of the PV's key block
        o_free = bar()                      # leader: the tile's O was read out
        # h > 1, per TMEM lane quarter (the h warps sharing its rows): partial maxima written, by
        # key-block parity, and partial sums written
        mx_full = [[bar(), bar()] for _ in range(4)] if H > 1 else []
        l_full = [bar() for _ in range(4)] if H > 1 else []
        counts = {o: 1 for o in range(0, nb * 8, 8)}
        for o in p_full + [o_free]:
            counts[o] = 2 * self.sm_warps
        for o in [x for pr in mx_full for x in pr] + l_full:
            counts[o] = 32 * H
        slot_off = nb * 8
        assert slot_off + 8 <= BAR_BYTES, "barriers outgrow their shared-memory slot"
        p = t("pred")
        skip = lab("ap_noinit")
        ins(f"setp.ne.u32 {p}, {tid}, 0")
        ins(f"@{p} bra {skip}")
        for o, c in counts.items():
            ins(f"mbarrier.init.shared::cta.b64 [{bars}+{o}], {c}")
        ins("fence.mbarrier_init.release.cluster")
        ins("fence.proxy.async.shared::cta")
        place(skip)
        noalloc = lab("ap_noalloc")
        ins(f"setp.ne.u32 {p}, {warp}, {self.w_mma}")
        ins(f"@{p} bra {noalloc}")
        slot = t("b32")
        ins(f"add.u32 {slot}, {bars}, {slot_off}")
        ins(f"tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [{slot}], 512")
        ins("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned")
        place(noalloc)
        ins("tcgen05.fence::before_thread_sync")
        ins("bar.sync 0")
        # both CTAs' barriers are initialised before either signals the other's
        ins("barrier.cluster.arrive.release")
        ins("barrier.cluster.wait.acquire")
        ins("tcgen05.fence::after_thread_sync")
        tmem = t("b32")
        ins(f"ld.shared.u32 {tmem}, [{bars}+{slot_off}]")
        O_COL, S_COL, Q_COL = 0, 128, 384
        lbars = t("b32")                                    # the leader's barriers, cluster address
        ins(f"mapa.shared::cluster.u32 {lbars}, {bars}, 0")
        mask = t("b16")
        ins(f"mov.b16 {mask}, 3")
        lead_cta = t("pred")
        ins(f"setp.eq.u32 {lead_cta}, {rank}, 0")
        errp = t("b64")
        ins(f"mov.u64 {errp}, thc_error")
        end = lab("ap_end")
        kit = Kit(em, errp, end)
        tmaps = {}
        for n in ("q", "k", "v"):
            r = t("b64")
            ins(f"mov.u64 {r}, thc_tmap_{n}")
            ins(f"cvta.global.u64 {r}, {r}")
            tmaps[n] = r
        # persistent over pair-tiles: pair c takes c, c + n_pairs, ...; nt of them, nt * n_blk key blocks
        pid, npair = self.special("%clusterid.x"), self.special("%nclusterid.x")
        nt, total = t("b32"), t("b32")
        ins(f"setp.ge.u32 {p}, {pid}, {self.pair_tiles}")
        ins(f"@{p} bra {end}")
        ins(f"sub.u32 {nt}, {self.pair_tiles - 1}, {pid}")
        ins(f"div.u32 {nt}, {nt}, {npair}")
        ins(f"add.u32 {nt}, {nt}, 1")
        ins(f"mul.lo.u32 {total}, {nt}, {n_blk}")
        groups = self.Sq // (2 * BM)

        def tile_rows(tile: str) -> tuple[str, str]:
            """This CTA's first query row and the head's first key row of pair-tile ``tile``."""
            bh, qg, qrow, kvrow = t("b32"), t("b32"), t("b32"), t("b32")
            ins(f"div.u32 {bh}, {tile}, {groups}")
            ins(f"rem.u32 {qg}, {tile}, {groups}")
            ins(f"mul.lo.u32 {qrow}, {bh}, {self.Sq}")
            ins(f"mad.lo.u32 {qrow}, {qg}, {2 * BM}, {qrow}")
            ins(f"mad.lo.u32 {qrow}, {rank}, {BM}, {qrow}")
            ins(f"mul.lo.u32 {kvrow}, {bh}, {self.Sk}")
            return qrow, kvrow

        role_mma, role_sm = lab("ap_mma"), lab("ap_softmax")
        ins(f"setp.lt.u32 {p}, {warp}, {self.w_tma}")
        ins(f"@{p} bra {role_sm}")
        ins(f"setp.eq.u32 {p}, {warp}, {self.w_mma}")
        ins(f"@{p} bra {role_mma}")
        ins(f"setp.ne.u32 {p}, {warp}, {self.w_tma}")
        ins(f"@{p} bra {end}")

        # ---------------- producer (one warp per CTA: this CTA's halves) ----------------
        is0, post = t("pred"), t("pred")
        ins(f"setp.eq.u32 {is0}, {lane}, 0")
        ins(f"and.pred {post}, {is0}, {lead_cta}")       # the leader posts both CTAs' bytes

        def load_q(tile: str) -> None:
            qrow, _ = tile_rows(tile)
            ins(f"@{post} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{bars}+{q_full}], {2 * qb}")
            for db in range(D // 64):
                ins(f"@{is0} {tma} [{q_s}+{db * BM * 128}], [{tmaps['q']}, {{{db * 64}, {qrow}}}], "
                    f"[{lbars}+{q_full}]")

        def load_kv(jj: str, krow: str, vrow: str) -> None:
            for is_k, n_st, s0, nbytes, full0, empty0 in ((True, KS, k0, kb, k_full[0], k_empty[0]),
                                                          (False, VS, v0, vb, v_full[0], v_empty[0])):
                st, buf, off = t("b32"), t("b32"), t("b32")
                ins(f"rem.u32 {st}, {jj}, {n_st}")
                ins(f"mad.lo.u32 {buf}, {st}, {nbytes}, {s0}")
                ins(f"shl.b32 {off}, {st}, 3")
                eb, fb, lfb = t("b32"), t("b32"), t("b32")
                ins(f"add.u32 {eb}, {bars}, {off}")
                ins(f"add.u32 {eb}, {eb}, {empty0}")
                kit.wait(eb, kit.parity(jj, n_st, flip=True), 0)
                ins(f"add.u32 {fb}, {bars}, {off}")
                ins(f"add.u32 {fb}, {fb}, {full0}")
                ins(f"add.u32 {lfb}, {lbars}, {off}")
                ins(f"add.u32 {lfb}, {lfb}, {full0}")
                ins(f"@{post} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fb}], {2 * nbytes}")
                if is_k:              # keys krow .. krow + 63, both 64-d boxes
                    for db in range(D // 64):
                        ins(f"@{is0} {tma} [{buf}+{db * KH * 128}], [{tmaps['k']}, {{{db * 64}, {krow}}}], "
                            f"[{lfb}]")
                else:                 # all 128 keys, this CTA's 64 d columns
                    dcol = t("b32")
                    ins(f"mul.lo.u32 {dcol}, {rank}, 64")
                    ins(f"@{is0} {tma} [{buf}], [{tmaps['v']}, {{{dcol}, {vrow}}}], [{lfb}]")

        ti, tile, j, blk = t("b32"), t("b32"), t("b32"), t("b32")
        ins(f"mov.u32 {ti}, 0")
        ins(f"mov.u32 {tile}, {pid}")
        ins(f"mov.u32 {j}, 0")
        load_q(tile)
        ptile, pblk = lab("ap_prod_tile"), lab("ap_prod_blk")
        place(ptile)
        _, kvrow = tile_rows(tile)
        ins(f"mov.u32 {blk}, 0")
        place(pblk)
        krow, vrow = t("b32"), t("b32")
        ins(f"mad.lo.u32 {vrow}, {blk}, {BN}, {kvrow}")
        ins(f"mad.lo.u32 {krow}, {rank}, {KH}, {vrow}")
        load_kv(j, krow, vrow)
        # after the tile's first key block: the next tile's Q, once the MMA warp has copied this
        # tile's Q into tensor memory (q_free)
        noq = lab("ap_prod_noq")
        ins(f"setp.ne.u32 {p}, {blk}, 0")
        ins(f"@{p} bra {noq}")
        nti = t("b32")
        ins(f"add.u32 {nti}, {ti}, 1")
        ins(f"setp.ge.u32 {p}, {nti}, {nt}")
        ins(f"@{p} bra {noq}")
        kit.wait(f"{bars}+{q_free}", kit.parity(ti, 1), 9)
        ntile = t("b32")
        ins(f"add.u32 {ntile}, {tile}, {npair}")
        load_q(ntile)
        place(noq)
        ins(f"add.u32 {j}, {j}, 1")
        ins(f"add.u32 {blk}, {blk}, 1")
        ins(f"setp.lt.u32 {p}, {blk}, {n_blk}")
        ins(f"@{p} bra {pblk}")
        ins(f"add.u32 {ti}, {ti}, 1")
        ins(f"add.u32 {tile}, {tile}, {npair}")
        ins(f"setp.lt.u32 {p}, {ti}, {nt}")
        ins(f"@{p} bra {ptile}")
        ins(f"bra {end}")

        # ---------------- MMA issuer (the leader CTA's warp issues for the pair) ----------------
        place(role_mma)
        ins(f"@!{lead_cta} bra {end}")
        ism = t("pred")
        ins(f"setp.eq.u32 {ism}, {lane}, 0")
        hi = t("b32")
        ins(f"mov.u32 {hi}, {desc_hi(1024)}")
        qdesc = kit.desc(q_s, 16, hi)
        id_s = idesc_f16(2 * BM, BN)
        id_o = idesc_f16(2 * BM, D, b_mn_major=True)
        zero = t("b32")
        ins(f"mov.u32 {zero}, 0")
        always, never = t("pred"), t("pred")
        ins(f"setp.eq.u32 {always}, {zero}, 0")
        ins(f"setp.ne.u32 {never}, {zero}, 0")

        def copy_q(tt: str) -> None:
            """Tile tt's Q (both CTAs) from shared memory into TMEM buffer tt % 2."""
            kit.wait(f"{bars}+{q_full}", kit.parity(tt, 1), 4)
            ins("tcgen05.fence::after_thread_sync")
            qb_, qcol = t("b32"), t("b32")
            ins(f"and.b32 {qb_}, {tt}, 1")
            ins(f"mad.lo.u32 {qcol}, {qb_}, 64, {tmem}")
            ins(f"add.u32 {qcol}, {qcol}, {Q_COL}")
            for kk in range(D // 16):
                src = kit.desc_add(qdesc, (kk // 4) * BM * 128 + (kk % 4) * 32)
                dst = t("b32")
                ins(f"add.u32 {dst}, {qcol}, {8 * kk}")
                ins(f"@{ism} tcgen05.cp.cta_group::2.128x256b [{dst}], {src}")
            ins(f"@{ism} {mcommit} [{bars}+{q_free}], {mask}")

        def issue_s(gg: str) -> None:
            """S(gg) = Q K(gg)^T into S buffer gg % 2, Q from the TMEM buffer of gg's tile."""
            st, off, kf = t("b32"), t("b32"), t("b32")
            ins(f"rem.u32 {st}, {gg}, {KS}")
            ins(f"shl.b32 {off}, {st}, 3")
            ins(f"add.u32 {kf}, {bars}, {off}")
            ins(f"add.u32 {kf}, {kf}, {k_full[0]}")
            kit.wait(kf, kit.parity(gg, KS), 5)
            ins("tcgen05.fence::after_thread_sync")
            kbuf = t("b32")
            ins(f"mad.lo.u32 {kbuf}, {st}, {kb}, {k0}")
            kd = kit.desc(kbuf, 16, hi)
            sb, dcol, tq, qcol = t("b32"), t("b32"), t("b32"), t("b32")
            ins(f"and.b32 {sb}, {gg}, 1")
            ins(f"mad.lo.u32 {dcol}, {sb}, 128, {tmem}")
            ins(f"add.u32 {dcol}, {dcol}, {S_COL}")
            ins(f"div.u32 {tq}, {gg}, {n_blk}")
            ins(f"and.b32 {tq}, {tq}, 1")
            ins(f"mad.lo.u32 {qcol}, {tq}, 64, {tmem}")
            ins(f"add.u32 {qcol}, {qcol}, {Q_COL}")
            for kk in range(D // 16):
                a = t("b32")
                ins(f"add.u32 {a}, {qcol}, {8 * kk}")
                bb = kit.desc_add(kd, (kk // 4) * KH * 128 + (kk % 4) * 32)
                ins(f"@{ism} tcgen05.mma.cta_group::2.kind::f16 [{dcol}], [{a}], {bb}, {id_s}, "
                    f"{always if kk else never}")
            sfb = t("b32")
            ins(f"mad.lo.u32 {sfb}, {sb}, 8, {bars}")
            ins(f"@{ism} {mcommit} [{sfb}+{s_full[0]}], {mask}")
            ins(f"add.u32 {kf}, {bars}, {off}")
            ins(f"@{ism} {mcommit} [{kf}+{k_empty[0]}], {mask}")

        def issue_pv(gg: str, acc: str) -> None:  # acc: predicate, false opens a tile
            """O (+)= P(gg) V(gg): P from S buffer gg % 2 (TMEM), V this CTA's 64 d columns."""
            st, off, vf = t("b32"), t("b32"), t("b32")
            ins(f"rem.u32 {st}, {gg}, {VS}")
            ins(f"shl.b32 {off}, {st}, 3")
            ins(f"add.u32 {vf}, {bars}, {off}")
            ins(f"add.u32 {vf}, {vf}, {v_full[0]}")
            kit.wait(vf, kit.parity(gg, VS), 6)
            ins("tcgen05.fence::after_thread_sync")
            vbuf = t("b32")
            ins(f"mad.lo.u32 {vbuf}, {st}, {vb}, {v0}")
            vd = kit.desc(vbuf, BN * 128, hi)
            sb, pcol = t("b32"), t("b32")
            ins(f"and.b32 {sb}, {gg}, 1")
            ins(f"mad.lo.u32 {pcol}, {sb}, 128, {tmem}")
            ins(f"add.u32 {pcol}, {pcol}, {S_COL}")
            ocol = t("b32")
            ins(f"add.u32 {ocol}, {tmem}, {O_COL}")
            for kk in range(BN // 16):
                a = t("b32")
                ins(f"add.u32 {a}, {pcol}, {8 * kk}")
                bb = kit.desc_add(vd, kk * 16 * 128)
                ins(f"@{ism} tcgen05.mma.cta_group::2.kind::f16 [{ocol}], [{a}], {bb}, {id_o}, "
                    f"{acc if kk == 0 else always}")
            odb = t("b32")
            ins(f"mad.lo.u32 {odb}, {sb}, 8, {bars}")
            ins(f"@{ism} {mcommit} [{odb}+{o_done[0]}], {mask}")
            ins(f"add.u32 {vf}, {bars}, {off}")
            ins(f"@{ism} {mcommit} [{vf}+{v_empty[0]}], {mask}")

        def s_with_q(gg: str) -> None:
            """S(gg), after copying its tile's Q when gg opens a tile."""
            keep = lab("ap_sameq")
            r_ = t("b32")
            ins(f"rem.u32 {r_}, {gg}, {n_blk}")
            ins(f"setp.ne.u32 {p}, {r_}, 0")
            ins(f"@{p} bra {keep}")
            tt = t("b32")
            ins(f"div.u32 {tt}, {gg}, {n_blk}")
            copy_q(tt)
            place(keep)
            issue_s(gg)

        g = t("b32")
        ins(f"mov.u32 {g}, 0")
        s_with_q(g)
        one = lab("ap_one")
        ins(f"setp.lt.u32 {p}, {total}, 2")
        ins(f"@{p} bra {one}")
        g1 = t("b32")
        ins(f"mov.u32 {g1}, 1")
        s_with_q(g1)
        place(one)
        mtop = lab("ap_mma_k")
        place(mtop)
        pf = t("b32")
        ins(f"and.b32 {pf}, {g}, 1")
        ins(f"mad.lo.u32 {pf}, {pf}, 8, {bars}")
        kit.wait(f"{pf}+{p_full[0]}", kit.parity(g, 2), 7)
        ins("tcgen05.fence::after_thread_sync")
        mblk, mti, acc = t("b32"), t("b32"), t("pred")
        ins(f"rem.u32 {mblk}, {g}, {n_blk}")
        ins(f"div.u32 {mti}, {g}, {n_blk}")
        ins(f"setp.ne.u32 {acc}, {mblk}, 0")
        ready = lab("ap_o_ready")
        ins(f"@{acc} bra {ready}")
        ins(f"setp.eq.u32 {p}, {mti}, 0")
        ins(f"@{p} bra {ready}")
        pt = t("b32")
        ins(f"sub.u32 {pt}, {mti}, 1")
        kit.wait(f"{bars}+{o_free}", kit.parity(pt, 1), 8)     # the last tile's O was read
        ins("tcgen05.fence::after_thread_sync")
        place(ready)
        issue_pv(g, acc)
        g2 = t("b32")
        ins(f"add.u32 {g2}, {g}, 2")
        nos = lab("ap_nos")
        ins(f"setp.ge.u32 {p}, {g2}, {total}")
        ins(f"@{p} bra {nos}")
        s_with_q(g2)
        place(nos)
        ins(f"add.u32 {g}, {g}, 1")
        ins(f"setp.lt.u32 {p}, {g}, {total}")
        ins(f"@{p} bra {mtop}")
        ins(f"bra {end}")

        # ---------------- softmax + epilogue (warps 0 .. 4 h - 1) ----------------
        # warp w: TMEM lanes 32 (w % 4) .. (its rows of this CTA's tile), part w / 4 of each key
        # block's scores and of O's columns
        KP, DP = BN // H, D // H
        place(role_sm)
        quarter, part, r = t("b32"), t("b32"), t("b32")
        ins(f"and.b32 {quarter}, {warp}, 3")
        ins(f"shr.u32 {part}, {warp}, 2")
        ins(f"mad.lo.u32 {r}, {quarter}, 32, {lane}")
        trow = t("b32")
        ins(f"shl.b32 {trow}, {quarter}, 21")
        ins(f"add.u32 {trow}, {trow}, {tmem}")
        ocol, sbase, pbase = t("b32"), t("b32"), t("b32")
        ins(f"mad.lo.u32 {ocol}, {part}, {DP}, {trow}")
        ins(f"add.u32 {ocol}, {ocol}, {O_COL}")
        ins(f"mad.lo.u32 {sbase}, {part}, {KP}, {trow}")          # this part's scores (buffer 0)
        ins(f"add.u32 {sbase}, {sbase}, {S_COL}")
        ins(f"mad.lo.u32 {pbase}, {part}, {KP // 2}, {trow}")     # their P: key k in column k / 2
        ins(f"add.u32 {pbase}, {pbase}, {S_COL}")
        bb = self.box_bytes
        wstage, srowa, r7 = t("b32"), t("b32"), t("b32")
        ins(f"mad.lo.u32 {wstage}, {warp}, {32 * bb}, {stage0}")
        ins(f"mad.lo.u32 {srowa}, {lane}, {bb}, {wstage}")
        ins(f"and.b32 {r7}, {lane}, 7")
        if H > 1:
            # exchange slots, f32: [max set 0 | max set 1 | sums] x [part] x [row]
            xrow, xmine, qmx, ql = t("b32"), t("b32"), t("b32"), t("b32")
            ins(f"mad.lo.u32 {xrow}, {r}, 4, {xchg}")
            ins(f"mad.lo.u32 {xmine}, {part}, {BM * 4}, {xrow}")
            assert mx_full[1][0] - mx_full[0][0] == 16 and l_full[1] - l_full[0] == 8
            ins(f"mad.lo.u32 {qmx}, {quarter}, 16, {bars}")         # this quarter's mx_full[2]
            ins(f"mad.lo.u32 {ql}, {quarter}, 8, {bars}")           # and its l_full
        lead = t("pred")
        ins(f"setp.eq.u32 {lead}, {lane}, 0")
        tmap_o = t("b64")
        ins(f"mov.u64 {tmap_o}, thc_tmap_o")
        ins(f"cvta.global.u64 {tmap_o}, {tmap_o}")
        sc = t("f32")
        ins(f"ld.global.nc.f32 {sc}, [{em.buffer_reg(self.pscale.name)}]")
        ins(f"rcp.rn.f32 {sc}, {sc}")
        ins(f"mul.rn.f32 {sc}, {sc}, 0f{_f32bits(LOG2E)}")
        mref, mref8, l = t("f32"), t("f32"), t("f32")
        sti, stile, sj, blk2 = t("b32"), t("b32"), t("b32"), t("b32")
        ins(f"mov.u32 {sti}, 0")
        ins(f"mov.u32 {stile}, {pid}")
        ins(f"mov.u32 {sj}, 0")
        stile_top = lab("ap_sm_tile")
        place(stile_top)
        ins(f"mov.f32 {mref}, 0fFF800000")
        ins(f"mov.f32 {mref8}, 0fFF800000")
        ins(f"mov.f32 {l}, 0f00000000")
        ins(f"mov.u32 {blk2}, 0")
        stop = lab("ap_sm_blk")
        place(stop)
        sb, sfb, scol, pcol = t("b32"), t("b32"), t("b32"), t("b32")
        ins(f"and.b32 {sb}, {sj}, 1")
        ins(f"mad.lo.u32 {sfb}, {sb}, 8, {bars}")
        ins(f"mad.lo.u32 {scol}, {sb}, 128, {sbase}")
        ins(f"mad.lo.u32 {pcol}, {sb}, 128, {pbase}")
        kit.wait(f"{sfb}+{s_full[0]}", kit.parity(sj, 2), 2)
        ins("tcgen05.fence::after_thread_sync")
        srow = [t("f32") for _ in range(KP)]
        for c in range(KP // 32):
            a = t("b32")
            ins(f"add.u32 {a}, {scol}, {32 * c}")
            ins(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(srow[32 * c:32 * c + 32])}}}, [{a}]")
        ins("tcgen05.wait::ld.sync.aligned")
        mx = _tree(em, "max.f32", srow, arity=3)
        if H > 1:
            # the row's H partial maxima (set sj % 2); the barrier also orders every part's score
            # loads before any part's P stores (P columns of part h cover scores of part h / 2)
            xs, mb = t("b32"), t("b32")
            ins(f"mad.lo.u32 {xs}, {sb}, {H * BM * 4}, {xmine}")
            ins(f"st.shared.f32 [{xs}], {mx}")
            ins(f"mad.lo.u32 {mb}, {sb}, 8, {qmx}")
            ins("tcgen05.fence::before_thread_sync")
            ins(f"mbarrier.arrive.shared::cta.b64 _, [{mb}+{mx_full[0][0]}]")
            kit.wait(f"{mb}+{mx_full[0][0]}", kit.parity(sj, 2), 10)
            ins("tcgen05.fence::after_thread_sync")
            xr = t("b32")
            ins(f"mad.lo.u32 {xr}, {sb}, {H * BM * 4}, {xrow}")
            mx = t("f32")
            ins(f"ld.shared.f32 {mx}, [{xr}]")
            for hp in range(1, H):
                o_ = t("f32")
                ins(f"ld.shared.f32 {o_}, [{xr}+{hp * BM * 4}]")
                ins(f"max.f32 {mx}, {mx}, {o_}")
        mnew = t("f32")
        ins(f"mul.rn.f32 {mnew}, {mx}, {sc}")
        norescale, noowait = lab("ap_norescale"), lab("ap_first")
        ins(f"setp.gt.f32 {p}, {mnew}, {mref8}")
        ins(f"@!{p} bra {norescale}")
        alpha, dm = t("f32"), t("f32")
        ins(f"sub.rn.f32 {dm}, {mref}, {mnew}")
        ins(f"ex2.approx.ftz.f32 {alpha}, {dm}")
        ins(f"mul.rn.f32 {l}, {l}, {alpha}")
        ins(f"setp.eq.u32 {p}, {blk2}, 0")
        ins(f"@{p} bra {noowait}")
        # O holds PV(sj - 1) once its o_done fires (PV(sj - 2) finished before S(sj) did)
        prevb, odb = t("b32"), t("b32")
        ins(f"sub.u32 {prevb}, {sj}, 1")
        ins(f"and.b32 {odb}, {prevb}, 1")
        ins(f"mad.lo.u32 {odb}, {odb}, 8, {bars}")
        kit.wait(f"{odb}+{o_done[0]}", kit.parity(prevb, 2), 3)
        ins("tcgen05.fence::after_thread_sync")
        for c in range(DP // 16):
            ov = [t("f32") for _ in range(16)]
            a = t("b32")
            ins(f"add.u32 {a}, {ocol}, {16 * c}")
            ins(f"tcgen05.ld.sync.aligned.32x32b.x16.b32 {{{', '.join(ov)}}}, [{a}]")
            ins("tcgen05.wait::ld.sync.aligned")
            for x in ov:
                ins(f"mul.rn.f32 {x}, {x}, {alpha}")
            ins(f"tcgen05.st.sync.aligned.32x32b.x16.b32 [{a}], {{{', '.join(ov)}}}")
        ins("tcgen05.wait::st.sync.aligned")
        place(noowait)
        ins(f"mov.f32 {mref}, {mnew}")
        ins(f"add.rn.f32 {mref8}, {mnew}, 0f41000000")
        place(norescale)
        negm = t("f32")
        ins(f"neg.f32 {negm}, {mref}")
        pair = t("b64"), t("b64")
        ins(f"mov.b64 {pair[0]}, {{{sc}, {sc}}}")
        ins(f"mov.b64 {pair[1]}, {{{negm}, {negm}}}")
        ex2 = _Exp2(em) if POLY_PAIRS else None
        for c in range(KP // 16):
            sv = srow[16 * c:16 * c + 16]
            packs = []
            for k in range(8):
                x0, x1 = sv[2 * k], sv[2 * k + 1]
                d = t("b64")
                ins(f"mov.b64 {d}, {{{x0}, {x1}}}")
                ins(f"fma.rn.ftz.f32x2 {d}, {d}, {pair[0]}, {pair[1]}")
                if k < POLY_PAIRS:
                    d = ex2.pair(d, x0, x1)
                else:
                    ins(f"mov.b64 {{{x0}, {x1}}}, {d}")
                    ins(f"ex2.approx.ftz.f32 {x0}, {x0}")
                    ins(f"ex2.approx.ftz.f32 {x1}, {x1}")
                    d = t("b64")
                    ins(f"mov.b64 {d}, {{{x0}, {x1}}}")
                packs.append(d)
            sp = _tree(em, "add.rn.f32x2", packs, kind="b64")
            lo, hi2 = t("f32"), t("f32")
            ins(f"mov.b64 {{{lo}, {hi2}}}, {sp}")
            ins(f"add.rn.f32 {lo}, {lo}, {hi2}")
            ins(f"add.rn.f32 {l}, {l}, {lo}")
            hp = [t("b32") for _ in range(8)]
            for k in range(8):
                ins(f"cvt.rn.f16x2.f32 {hp[k]}, {sv[2 * k + 1]}, {sv[2 * k]}")
            a2 = t("b32")
            ins(f"add.u32 {a2}, {pcol}, {8 * c}")
            ins(f"tcgen05.st.sync.aligned.32x32b.x8.b32 [{a2}], {{{', '.join(hp)}}}")
        # P(sj) (and any O rescale) complete: one arrival per warp on the leader's p_full
        ins("tcgen05.wait::st.sync.aligned")
        ins("tcgen05.fence::before_thread_sync")
        ins("bar.warp.sync -1")
        pfr = t("b32")
        ins(f"mad.lo.u32 {pfr}, {sb}, 8, {lbars}")
        ins(f"@{lead} {remote_arrive} [{pfr}+{p_full[0]}]")
        ins(f"add.u32 {sj}, {sj}, 1")
        ins(f"add.u32 {blk2}, {blk2}, 1")
        ins(f"setp.lt.u32 {p}, {blk2}, {n_blk}")
        ins(f"@{p} bra {stop}")
        # epilogue: the row sum (H > 1: the parts' sums, added in part order by every part), the
        # tile's last PV done -> this part's O columns into registers -> o_free to the leader ->
        # O / l as f16 through the warp's 32-row box, one TMA store per box
        if H > 1:
            ins(f"st.shared.f32 [{xmine}+{2 * H * BM * 4}], {l}")
            ins(f"mbarrier.arrive.shared::cta.b64 _, [{ql}+{l_full[0]}]")
            kit.wait(f"{ql}+{l_full[0]}", kit.parity(sti, 1), 11)
            ins(f"ld.shared.f32 {l}, [{xrow}+{2 * H * BM * 4}]")
            for hp in range(1, H):
                o_ = t("f32")
                ins(f"ld.shared.f32 {o_}, [{xrow}+{(2 * H + hp) * BM * 4}]")
                ins(f"add.rn.f32 {l}, {l}, {o_}")
        inv = t("f32")
        ins(f"rcp.rn.f32 {inv}, {l}")
        lastb, odl = t("b32"), t("b32")
        ins(f"sub.u32 {lastb}, {sj}, 1")
        ins(f"and.b32 {odl}, {lastb}, 1")
        ins(f"mad.lo.u32 {odl}, {odl}, 8, {bars}")
        kit.wait(f"{odl}+{o_done[0]}", kit.parity(lastb, 2), 3)
        ins("tcgen05.fence::after_thread_sync")
        ov = [t("f32") for _ in range(DP)]
        for c in range(DP // 32):
            a = t("b32")
            ins(f"add.u32 {a}, {ocol}, {32 * c}")
            ins(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ov[32 * c:32 * c + 32])}}}, [{a}]")
        ins("tcgen05.wait::ld.sync.aligned")
        ins("tcgen05.fence::before_thread_sync")
        ins("bar.warp.sync -1")
        ins(f"@{lead} {remote_arrive} [{lbars}+{o_free}]")
        qrow_s, _ = tile_rows(stile)
        orow, oc0 = t("b32"), t("b32")
        ins(f"mad.lo.u32 {orow}, {quarter}, 32, {qrow_s}")       # the warp's first row
        ins(f"mul.lo.u32 {oc0}, {part}, {DP}")                   # and its first column
        bcols = self.box_cols
        for hb in range(DP // bcols):
            ins(f"@{lead} cp.async.bulk.wait_group.read 0")
            ins("bar.warp.sync -1")
            for c in range(bcols // 8):
                oh = [t("b32") for _ in range(4)]
                for k in range(4):
                    x0, x1 = ov[bcols * hb + 8 * c + 2 * k], ov[bcols * hb + 8 * c + 2 * k + 1]
                    ins(f"mul.rn.f32 {x0}, {x0}, {inv}")
                    ins(f"mul.rn.f32 {x1}, {x1}, {inv}")
                    ins(f"cvt.rn.f16x2.f32 {oh[k]}, {x1}, {x0}")
                if bb == 128:
                    # 16-byte chunk c of row r at chunk c ^ (r % 8): the 128-byte swizzle
                    ch = t("b32")
                    ins(f"xor.b32 {ch}, {r7}, {c}")
                    ins(f"mad.lo.u32 {ch}, {ch}, 16, {srowa}")
                    ins(f"st.shared.v4.b32 [{ch}], {{{', '.join(oh)}}}")
                else:
                    ins(f"st.shared.v4.b32 [{srowa}+{16 * c}], {{{', '.join(oh)}}}")
            ins("fence.proxy.async.shared::cta")
            ins("bar.warp.sync -1")
            oc = t("b32")
            ins(f"add.u32 {oc}, {oc0}, {bcols * hb}")
            ins(f"@{lead} cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [{tmap_o}, "
                f"{{{oc}, {orow}}}], [{wstage}]")
            ins(f"@{lead} cp.async.bulk.commit_group")
        ins(f"add.u32 {sti}, {sti}, 1")
        ins(f"add.u32 {stile}, {stile}, {npair}")
        ins(f"setp.lt.u32 {p}, {sti}, {nt}")
        ins(f"@{p} bra {stile_top}")
        ins(f"@{lead} cp.async.bulk.wait_group 0")

        # ---------------- common exit: both CTAs, then free the pair's TMEM ----------------
        place(end)
        ins("tcgen05.fence::before_thread_sync")
        ins("barrier.sync 0")
        ins("barrier.cluster.arrive.release")
        ins("barrier.cluster.wait.acquire")
        nod = lab("ap_nodealloc")
        ins(f"setp.ne.u32 {p}, {warp}, {self.w_mma}")
        ins(f"@{p} bra {nod}")
        ins("tcgen05.fence::after_thread_sync")
        ins(f"tcgen05.dealloc.cta_group::2.sync.aligned.b32 {tmem}, 512")
        place(nod)


def recognise(kernel: KernelInfo):
    return TcAttentionPair.match(kernel)
