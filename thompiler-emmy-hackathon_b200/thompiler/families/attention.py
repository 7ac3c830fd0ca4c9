"""Tuned family: attention, softmax(Q K^T / c) V, on tcgen05 (the a01 / a02
family at the benchmark shape [8, 16, 2048, 128], f16 in and out).

Recognised IR: the a02 schedule of the reference's problem set -- one output
element per thread, a loop over keys holding the QK dot product (an inner
loop over d), the two-state online softmax (running max, rescaled sum) and
the V accumulation, then ``acc / sum`` written out (see
problems/a02_attention_128/k_matmul_softmax_reduce_6f0029.ir.txt of the
reference).  Q, K, V and the output are f16 [..., S, D] buffers (D = 64 or
128, S a multiple of 128); ``c`` comes from a one-element constant buffer at
run time.

Tuned body: one CTA per (head, QT query tiles of 128), QT = 2 when S allows
(384 threads), else 1 (224 threads):
  warps 0 .. 4QT-1  softmax, one warpgroup per query tile g; thread = query row,
            warp w reads TMEM lanes 32 (w % 4) ..;
  warp 4QT  TMA: K and V tiles of 128 keys through two-slot rings
            (128B-swizzled rows of 64 d); step j loads V(j) and K(j + 1) under
            one barrier, so the MMA warp waits once per key block;
  warp 4QT+1  tcgen05 issuer: S_g = Q_g K_i^T (SS form, M = 128 queries,
            N = 128 keys, K = D) and O_g += P_g V_i (TS form: A = P_g from
            TMEM, B = V as an MN-major shared operand), ordered PV_0, S_0(next),
            PV_1, S_1(next) so each group's softmax overlaps the other's MMAs,
            and one commit per block releases the ring step;
  warp 4QT+2  TMA: each query tile's Q_g once the previous tile's last S_g is
            done, and an L2 prefetch of the next tile's Q;
  with QT = 2 warp 11 completes the third warpgroup, which hands registers to
  the softmax warpgroups (setmaxnreg 168 -> 224 / 56).
The single-thread instructions (MMA, commit, TMA) are guarded by elect.sync.
TMEM (512 columns): O_g at 128 g, S_g at 256 + 128 g; P_g (f16 pairs) is
written over the first 64 columns of S_g.  Softmax per row and key block: the
128 scores in registers (four loads, one wait), a three-input max tree, O and
the running sum rescaled only when the max grew by more than 2^8 (P <= 256
stays exact in f16, the rescale is rare), P = 2^(s c' - m) with packed f32x2
FMAs and ex2.approx (one pair in 8 from a polynomial on the FMA pipe), packed
sums, f16 pairs stored back to TMEM.  Epilogue: O / l as f16 through each
warp's own 32-row staging box (128B-swizzled), one TMA store per box.
Scores run in the base-2 domain: c' = log2(e) / c, so exp(x) = 2^(x log2 e)
exactly as the IR's exp lowering.  All mbarrier waits are bounded
(thompiler.families.kit).
"""

from __future__ import annotations

import math

from thompiler import ir
from thompiler.families.base import TunedKernel
from thompiler.families.tuning import TUNING
from thompiler.families.kit import (TMAP_RING, TMAP_SETS, TMAP_TABLE, Kit, declare_tmap_ring, desc_hi, elect_one,
                                   idesc_f16, select_tmap_set, tmap_address)
from thompiler.lowering.types import F16, F32
from thompiler.load import KernelInfo

BM = BN = 128
SM_COUNT = 148
STAGES = 3                  # K and V rings each
LOG2E = math.log2(math.e)


def _var_tail(index: tuple, names: tuple) -> bool:
    return len(index) >= 2 and all(isinstance(e, ir.Var) and e.name == n for e, n in zip(index[-2:], names))


class TcAttention(TunedKernel):
    family = "tcgen05-attention"

    def __init__(self, kernel, q, k, v, out, scale, heads, Sq, Sk, D):
        super().__init__(kernel)
        self.pq, self.pk, self.pv, self.pout, self.pscale = q, k, v, out, scale
        self.heads, self.Sq, self.Sk, self.D = heads, Sq, Sk, D
        self.q_bytes = BM * D * 2
        self.kv_bytes = BN * D * 2
        # two 128-query tiles per CTA (two softmax warp groups sharing each K / V tile) when they fit
        self.qt = 2 if Sq % (2 * BM) == 0 else 1
        # warps 0 .. 4 qt - 1 softmax, one thread per query row (warp w reads TMEM lanes 32 (w % 4) ..),
        # then the K / V TMA warp, the MMA warp and the Q TMA warp; with two query tiles they fill one
        # more warpgroup (one warp idle) whose registers go to the softmax warpgroups through setmaxnreg
        sm_warps = 4 * self.qt
        self.sm_threads = 32 * sm_warps
        self.w_tma, self.w_mma, self.w_q = sm_warps, sm_warps + 1, sm_warps + 2
        self.threads = 32 * sm_warps + 128 if self.qt == 2 else 224
        # each of the SM's four sub-partitions holds 16384 registers and ceil(warps / 4) of the warps
        # (of the tuned CTA or of meta.json's, whichever is larger: the module serves both)
        warps = -(-max(self.threads, kernel.threads_per_cta) // 32)
        self.maxnreg = min(255, 16384 // (32 * -(-warps // 4)) // 8 * 8)
        if self.qt == 2:
            dec = 56
            inc = min(248, self.maxnreg + ((self.maxnreg - dec) * 128 // self.sm_threads) // 8 * 8)
            assert self.qt * inc + dec <= 512, "setmaxnreg split over one sub-partition's file"
            self.reg_split = (inc, dec)
        else:
            self.reg_split = None
        # K and V rings of equal depth: producer step j loads V(j) and K(j + 1) under one barrier
        self.ks = self.vs = 2 if D == 128 else STAGES
        # per softmax warp: a 32-row staging box for the output's TMA stores, 128 bytes wide
        # (128B swizzle), one thread per row
        self.box_bytes = 128
        self.stage_bytes = sm_warps * 32 * self.box_bytes
        self.smem = (self.qt * self.q_bytes + (self.ks + self.vs) * self.kv_bytes + self.stage_bytes
                     + 1024 + 256)
        self.tiles = heads * (Sq // (BM * self.qt))
        self.poly_pairs = TUNING.attention_poly_pairs
        assert 0 <= self.poly_pairs <= 8

    # ---- recognition -------------------------------------------------------------

    @classmethod
    def match(cls, kernel: KernelInfo):
        body = kernel.body
        if len(body) != 1 or not isinstance(body[0], ir.Tile):
            return None
        tile = body[0]
        if len(tile.axes) < 2:
            return None
        a0, a5 = tile.axes[-2].name, tile.axes[-1].name
        outer = [s for s in tile.body if isinstance(s, ir.Loop)]
        if len(outer) != 1:
            return None
        outer = outer[0]
        a1 = outer.axis.name
        inner = [s for s in outer.body if isinstance(s, ir.Loop)]
        if len(inner) != 1 or not outer.seed or not inner[0].seed:
            return None
        inner = inner[0]
        a2 = inner.axis.name
        loads = [s for s in ir.walk_stmts(tile.body) if isinstance(s, ir.Load)]
        qk = {}
        for s in inner.body:
            if isinstance(s, ir.Load):
                if _var_tail(s.index, (a0, a2)):
                    qk["q"] = s.input
                elif _var_tail(s.index, (a1, a2)):
                    qk["k"] = s.input
                else:
                    return None
        vl = [s for s in outer.body if isinstance(s, ir.Load)]
        if len(vl) != 1 or not _var_tail(vl[0].index, (a1, a5)):
            return None
        writes = [s for s in ir.walk_stmts(tile.body) if isinstance(s, ir.Write)]
        if len(writes) != 1 or not _var_tail(writes[0].index, (a0, a5)) or writes[0].atomic:
            return None
        consts = [s for s in loads if all(isinstance(x, ir.Literal) for x in s.index)]
        if len(consts) != 1 or set(qk) != {"q", "k"}:
            return None
        ops = [s.op.name for s in ir.walk_stmts(outer.body) if isinstance(s, ir.Assign)]
        accs = [(s.op.name, s.base is not None) for s in outer.body if isinstance(s, ir.Accum)]
        if ops.count("exp") != 2 or sorted(accs) != [("add", True), ("add", True), ("maximum", False)]:
            return None
        recips = [s for s in tile.body if isinstance(s, ir.Assign) and s.op.name == "reciprocal"]
        if len(recips) != 2:
            return None
        q, k = kernel.param(qk["q"]), kernel.param(qk["k"])
        v, out = kernel.param(vl[0].input), kernel.param(writes[0].output)
        scale = kernel.param(consts[0].input)
        if None in (q, k, v, out, scale) or len(kernel.params) != 5:
            return None
        if any(p.ty is not F16 for p in (q, k, v, out)) or scale.ty is not F32 or scale.nelems != 1:
            return None
        if not (q.shape == out.shape and k.shape == v.shape and q.shape[:-2] == k.shape[:-2]):
            return None
        Sq, D = q.shape[-2:]
        Sk = k.shape[-2]
        if k.shape[-1] != D or D not in (64, 128) or Sq % BM or Sk % BN:
            return None
        if tile.extents[-2:] != (Sq, D) or outer.axis.size != Sk or inner.axis.size != D:
            return None
        heads = 1
        for e in q.shape[:-2]:
            heads *= e
        if tuple(tile.extents[:-2]) != tuple(q.shape[:-2]):
            return None
        return cls(kernel, q, k, v, out, scale, heads, Sq, Sk, D)

    # ---- launch --------------------------------------------------------------------

    def sidecar(self) -> dict:
        D = self.D

        def tm(prm, rows, box=(64, 128), swizzle=3):
            return {"global": TMAP_RING, "param": prm.name, "dtype": "f16", "dims": [D, rows],
                    "strides": [D * 2], "box": list(box), "swizzle": swizzle}
        o_box = (self.box_bytes // 2, 32)                 # one warp's staging box of the output
        maps = [tm(self.pq, self.heads * self.Sq), tm(self.pk, self.heads * self.Sk),
                tm(self.pv, self.heads * self.Sk), tm(self.pout, self.heads * self.Sq, o_box, 3)]
        return {"grid": [min(self.tiles, SM_COUNT), 1, 1], "block": [self.threads, 1, 1], "smem_bytes": self.smem,
                "tmaps": maps, "tmap_ptrs": {"global": TMAP_TABLE, "params": [m["param"] for m in maps]},
                "tmap_sets": TMAP_SETS, "error_word": "thc_error", "tile": [BM * self.qt, BN, D],
                "stages": [self.ks, self.vs]}

    def guard(self, generic: str) -> None:
        em = self.em
        declare_tmap_ring(em, 4)
        em.module(".global .align 4 .u32 thc_error")
        em.module(".extern .shared .align 1024 .b8 smem_pool[]")
        # the softmax rows live in registers: cap them so the tuned CTA (and meta.json's) can launch
        em.entry_attrs.append(f".maxnreg {self.maxnreg}")
        p = em.tmp("pred")
        r = self.special("%ntid.x")
        em.ins(f"setp.ne.u32 {p}, {r}, {self.threads}")
        em.ins(f"@{p} bra {generic}")
        # the tensor-map set encoded for these buffers (else the generic lowering)
        self.tmap_set = select_tmap_set(em, [q.name for q in (self.pq, self.pk, self.pv, self.pout)], generic)

    # ---- the tuned body ----------------------------------------------------------------

    def emit_tuned(self) -> None:  # noqa: C901 - one kernel, in order
        em = self.em
        t, ins, place, lab = em.tmp, em.ins, em.place, em.label
        D, n_blk, QT = self.D, self.Sk // BN, self.qt
        dblk = D // 64
        qb, kvb = self.q_bytes, self.kv_bytes
        KS, VS = self.ks, self.vs
        commit = "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64"
        tma = "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        self.pdl_trigger()

        tid, warp, lane = t("b32"), t("b32"), t("b32")
        ins(f"mov.u32 {tid}, %tid.x")
        ins(f"shr.u32 {warp}, {tid}, 5")
        ins(f"and.b32 {lane}, {tid}, 31")
        base = t("b32")
        ins(f"mov.u32 {base}, smem_pool")
        ins(f"add.u32 {base}, {base}, 1023")
        ins(f"and.b32 {base}, {base}, -1024")
        # shared: Q tiles (QT of them) | K ring | V ring | output staging (one 32-row box per
        # softmax warp) | barriers
        q_s = base
        k0, v0, stage0, bars = t("b32"), t("b32"), t("b32"), t("b32")
        ins(f"add.u32 {k0}, {base}, {QT * qb}")
        ins(f"add.u32 {v0}, {base}, {QT * qb + KS * kvb}")
        ins(f"add.u32 {stage0}, {base}, {QT * qb + (KS + VS) * kvb}")
        ins(f"add.u32 {bars}, {stage0}, {self.stage_bytes}")
        nb = 0

        def bar() -> int:
            nonlocal nb
            nb += 1
            return (nb - 1) * 8
        q_full, q_free = [bar() for _ in range(QT)], [bar() for _ in range(QT)]
        k0_full = bar()                                   # K(0) of the CTA's first tile
        kv_full, kv_empty = [bar() for _ in range(KS)], [bar() for _ in range(KS)]   # V(j) + K(j + 1)
        s_full = [bar() for _ in range(QT)]
        p_full = [bar() for _ in range(QT)]              # P_g stored by group g's 128 softmax threads
        o_done = [bar() for _ in range(QT)]
        o_free = [bar() for _ in range(QT)]
        counts = {o: 1 for o in range(0, nb * 8, 8)}
        for o in p_full + o_free:
            counts[o] = 128
        slot_off = nb * 8
        assert slot_off + 8 <= 256, "barriers outgrow their shared-memory slot"
        p = t("pred")
        skip = lab("at_noinit")
        ins(f"setp.ne.u32 {p}, {tid}, 0")
        ins(f"@{p} bra {skip}")
        for o, c in counts.items():
            ins(f"mbarrier.init.shared::cta.b64 [{bars}+{o}], {c}")
        ins("fence.mbarrier_init.release.cluster")
        ins("fence.proxy.async.shared::cta")
        place(skip)
        noalloc = lab("at_noalloc")
        ins(f"setp.ne.u32 {p}, {warp}, {self.w_mma}")
        ins(f"@{p} bra {noalloc}")
        slot = t("b32")
        ins(f"add.u32 {slot}, {bars}, {slot_off}")
        ins(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{slot}], 512")
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
        # TMEM columns: O_g at 128 g, S_g at 256 + 128 g; P_g (f16 pairs) in the first 64 columns of S_g
        O_COL, S_COL = 0, 256
        errp = t("b64")
        ins(f"mov.u64 {errp}, thc_error")
        end = lab("at_end")
        kit = Kit(em, errp, end)
        tmaps = {n: tmap_address(em, self.tmap_set, 4, i) for i, n in enumerate(("q", "k", "v"))}
        # persistent: CTA c takes tiles c, c + nctaid, ...; nt of them, nt * n_blk key blocks in all
        cta, ncta = self.special("%ctaid.x"), self.special("%nctaid.x")
        nt, total = t("b32"), t("b32")
        ins(f"setp.ge.u32 {p}, {cta}, {self.tiles}")
        ins(f"@{p} bra {end}")
        ins(f"sub.u32 {nt}, {self.tiles - 1}, {cta}")
        ins(f"div.u32 {nt}, {nt}, {ncta}")
        ins(f"add.u32 {nt}, {nt}, 1")
        ins(f"mul.lo.u32 {total}, {nt}, {n_blk}")
        groups = self.Sq // (BM * QT)

        def tile_rows(tile: str) -> tuple[str, str]:
            """First query row and first key row of ``tile`` in the flattened [heads * S] views."""
            bh, qg, qrow, kvrow = t("b32"), t("b32"), t("b32"), t("b32")
            ins(f"div.u32 {bh}, {tile}, {groups}")
            ins(f"rem.u32 {qg}, {tile}, {groups}")
            ins(f"mul.lo.u32 {qrow}, {bh}, {self.Sq}")
            ins(f"mad.lo.u32 {qrow}, {qg}, {BM * QT}, {qrow}")
            ins(f"mul.lo.u32 {kvrow}, {bh}, {self.Sk}")
            return qrow, kvrow

        role_mma, role_sm = lab("at_mma"), lab("at_softmax")
        ins(f"setp.lt.u32 {p}, {warp}, {self.w_tma}")                # the softmax warps
        ins(f"@{p} bra {role_sm}")
        if self.reg_split:
            # the producer warpgroup hands registers to the softmax warpgroups (each warpgroup runs
            # its own setmaxnreg before its warps part): per sub-partition 2 inc + dec <= 512 per
            # thread, and over the CTA the split is exactly what it launched with
            ins(f"setmaxnreg.dec.sync.aligned.u32 {self.reg_split[1]}")
        ins(f"setp.eq.u32 {p}, {warp}, {self.w_mma}")
        ins(f"@{p} bra {role_mma}")
        role_q = lab("at_qload")
        ins(f"setp.eq.u32 {p}, {warp}, {self.w_q}")
        ins(f"@{p} bra {role_q}")
        ins(f"setp.ne.u32 {p}, {warp}, {self.w_tma}")
        ins(f"@{p} bra {end}")                           # the warpgroup's idle warp

        # ---------------- producer (one warp) ----------------
        is0 = t("pred")
        elect_one(em, is0)

        # step j (over all of the CTA's key blocks, tile after tile): V(j) and K(j + 1) -- the keys
        # of the next S, which may open the next tile -- into ring slots j % KS and (j + 1) % KS
        # under kv_full[j % KS].  Their previous occupants V(j - KS) and K(j + 1 - KS) are
        # consumed by the MMA warp's block j - KS, whose release goes to kv_empty[(j + 1) % KS]
        # (the S(0) that consumes K(0), loaded first, releases as block -1, into kv_empty[0])
        def load(mapname: str, sbase: str, slot: str, row: str, fb: str, pred: str) -> None:
            buf = t("b32")
            ins(f"mad.lo.u32 {buf}, {slot}, {kvb}, {sbase}")
            for db in range(dblk):
                ins(f"@{pred} {tma} [{buf}+{db * BN * 128}], [{tmaps[mapname]}, {{{db * 64}, {row}}}], [{fb}]")

        _, kvrow = tile_rows(cta)
        ins(f"@{is0} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{bars}+{k0_full}], {kvb}")
        slot0 = t("b32")
        ins(f"mov.u32 {slot0}, 0")
        k0_bar = t("b32")
        ins(f"add.u32 {k0_bar}, {bars}, {k0_full}")
        load("k", k0, slot0, kvrow, k0_bar, is0)                   # K(0) of the first tile, slot 0
        ti, tile, j, blk = t("b32"), t("b32"), t("b32"), t("b32")
        ins(f"mov.u32 {ti}, 0")
        ins(f"mov.u32 {tile}, {cta}")
        ins(f"mov.u32 {j}, 0")
        ptile, pblk = lab("at_prod_tile"), lab("at_prod_blk")
        place(ptile)
        _, kvrow = tile_rows(tile)
        nt_ = t("b32")
        ins(f"add.u32 {nt_}, {tile}, {ncta}")
        _, nkvrow = tile_rows(nt_)                       # the next tile's first key row (if it has one)
        ins(f"mov.u32 {blk}, 0")
        place(pblk)
        st, fb, eb, hask, lk, lv = t("b32"), t("b32"), t("b32"), t("pred"), t("pred"), t("pred")
        j1 = t("b32")
        ins(f"add.u32 {j1}, {j}, 1")
        ins(f"rem.u32 {eb}, {j1}, {KS}")
        ins(f"mad.lo.u32 {eb}, {eb}, 8, {bars}")
        ins(f"add.u32 {eb}, {eb}, {kv_empty[0]}")
        kit.wait(eb, kit.parity(j1, KS, flip=True), 0)
        ins(f"rem.u32 {st}, {j}, {KS}")
        ins(f"mad.lo.u32 {fb}, {st}, 8, {bars}")
        ins(f"add.u32 {fb}, {fb}, {kv_full[0]}")
        ins(f"setp.lt.u32 {hask}, {j1}, {total}")
        ins(f"and.pred {lk}, {is0}, {hask}")
        ins(f"not.pred {lv}, {hask}")
        ins(f"and.pred {lv}, {is0}, {lv}")
        ins(f"@{lk} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fb}], {2 * kvb}")
        ins(f"@{lv} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fb}], {kvb}")
        row = t("b32")
        ins(f"mad.lo.u32 {row}, {blk}, {BN}, {kvrow}")
        load("v", v0, st, row, fb, is0)
        krow, kst, opens = t("b32"), t("b32"), t("pred")
        ins(f"add.u32 {krow}, {row}, {BN}")
        ins(f"add.u32 {kst}, {blk}, 1")                             # K(j + 1)'s block in this tile ...
        ins(f"setp.ge.u32 {opens}, {kst}, {n_blk}")
        ins(f"selp.u32 {krow}, {nkvrow}, {krow}, {opens}")     # ... or the next tile's first
        ins(f"rem.u32 {kst}, {j1}, {KS}")
        load("k", k0, kst, krow, fb, lk)
        ins(f"mov.u32 {j}, {j1}")
        ins(f"add.u32 {blk}, {blk}, 1")
        ins(f"setp.lt.u32 {p}, {blk}, {n_blk}")
        ins(f"@{p} bra {pblk}")
        ins(f"add.u32 {ti}, {ti}, 1")
        ins(f"add.u32 {tile}, {tile}, {ncta}")
        ins(f"setp.lt.u32 {p}, {ti}, {nt}")
        ins(f"@{p} bra {ptile}")
        ins(f"bra {end}")

        # ---------------- Q loads (one warp) ----------------
        # Q_g of tile t + 1 goes into Q_g's buffer once the last S_g of tile t is done (q_free[g]),
        # each query tile on its own, and was prefetched into L2 while tile t ran: the load at the
        # tile change reads L2, under the softmax of the last key block
        place(role_q)
        isq = t("pred")
        elect_one(em, isq)
        qti, qtile = t("b32"), t("b32")
        ins(f"mov.u32 {qti}, 0")
        ins(f"mov.u32 {qtile}, {cta}")
        qtop = lab("at_q_tile")
        place(qtop)
        qrow, _ = tile_rows(qtile)
        for g in range(QT):
            first = lab("at_q_first")
            ins(f"setp.eq.u32 {p}, {qti}, 0")
            ins(f"@{p} bra {first}")
            qprev = t("b32")
            ins(f"sub.u32 {qprev}, {qti}, 1")
            kit.wait(f"{bars}+{q_free[g]}", kit.parity(qprev, 1), 0)     # tile t's last S_g is done
            place(first)
            ins(f"@{isq} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{bars}+{q_full[g]}], {qb}")
            qr = t("b32")
            ins(f"add.u32 {qr}, {qrow}, {g * BM}")
            for db in range(dblk):
                ins(f"@{isq} {tma} [{q_s}+{g * qb + db * BM * 128}], [{tmaps['q']}, {{{db * 64}, {qr}}}], "
                    f"[{bars}+{q_full[g]}]")
        ins(f"add.u32 {qti}, {qti}, 1")
        ins(f"add.u32 {qtile}, {qtile}, {ncta}")
        nopf = lab("at_q_nopf")
        ins(f"setp.ge.u32 {p}, {qti}, {nt}")
        ins(f"@{p} bra {nopf}")
        nrow, _ = tile_rows(qtile)
        for g in range(QT):
            qr = t("b32")
            ins(f"add.u32 {qr}, {nrow}, {g * BM}")
            for db in range(dblk):
                ins(f"@{isq} cp.async.bulk.prefetch.tensor.2d.L2.global [{tmaps['q']}, {{{db * 64}, {qr}}}]")
        place(nopf)
        ins(f"setp.lt.u32 {p}, {qti}, {nt}")
        ins(f"@{p} bra {qtop}")
        ins(f"bra {end}")

        # ---------------- MMA issuer (one warp) ----------------
        place(role_mma)
        ism = t("pred")
        elect_one(em, ism)
        zero = t("b32")
        ins(f"mov.u32 {zero}, 0")
        hi = t("b32")
        ins(f"mov.u32 {hi}, {desc_hi(1024)}")
        qdesc = [kit.desc_add(kit.desc(q_s, 16, hi), g * qb) for g in range(QT)]
        id_s = idesc_f16(BM, BN)
        id_o = idesc_f16(BM, D, b_mn_major=True)
        always, never = t("pred"), t("pred")
        ins(f"setp.eq.u32 {always}, {zero}, 0")
        ins(f"setp.ne.u32 {never}, {zero}, 0")

        def issue_s(g: int, ks_: str) -> None:
            """S_g = Q_g K^T for the K tile at ks_ (already waited for)."""
            kd = kit.desc(ks_, 16, hi)
            dcol = t("b32")
            ins(f"add.u32 {dcol}, {tmem}, {S_COL + 128 * g}")
            for kk in range(D // 16):
                a = kit.desc_add(qdesc[g], (kk // 4) * BM * 128 + (kk % 4) * 32)
                bb = kit.desc_add(kd, (kk // 4) * BN * 128 + (kk % 4) * 32)
                ins(f"@{ism} tcgen05.mma.cta_group::1.kind::f16 [{dcol}], {a}, {bb}, {id_s}, "
                    f"{never if kk == 0 else always}")
            ins(f"@{ism} {commit} [{bars}+{s_full[g]}]")

        def issue_pv(g: int, vs_: str, acc0: str, last: str) -> None:
            """O_g (+)= P_g V for the V tile at vs_, P_g read from TMEM (the TS form); acc0 false
            starts a tile.  o_done[g] is committed at a tile's last block only (the epilogue's
            wait): within a tile the softmax's view of S_g(j + 1) already covers PV_g(j), which
            the same thread issued before it."""
            vd = kit.desc(vs_, BN * 128, hi)
            dcol = t("b32")
            ins(f"add.u32 {dcol}, {tmem}, {O_COL + 128 * g}")
            for kk in range(BN // 16):
                a = t("b32")
                ins(f"add.u32 {a}, {tmem}, {S_COL + 128 * g + 8 * kk}")
                bb = kit.desc_add(vd, kk * 16 * 128)
                ins(f"@{ism} tcgen05.mma.cta_group::1.kind::f16 [{dcol}], [{a}], {bb}, {id_o}, "
                    f"{acc0 if kk == 0 else always}")
            ins(f"@{last} {commit} [{bars}+{o_done[g]}]")

        def q_released(g: int, jj: str) -> None:
            """After S_g of a tile's last key block: Q_g may be overwritten."""
            if n_blk == 1:
                ins(f"@{ism} {commit} [{bars}+{q_free[g]}]")
                return
            r_, skipq = t("b32"), lab("at_q_keep")
            ins(f"rem.u32 {r_}, {jj}, {n_blk}")
            ins(f"setp.ne.u32 {p}, {r_}, {n_blk - 1}")
            ins(f"@{p} bra {skipq}")
            ins(f"@{ism} {commit} [{bars}+{q_free[g]}]")
            place(skipq)

        # S_g(0) of the first tile; then per key block j: one wait for V(j) and K(j + 1), PV_g(j)
        # and S_g(j + 1) for each group in turn -- S_g(j + 1) may already belong to the next tile
        # (its Q_g is loaded once q_free[g] fires) -- and one release of the ring step
        kit.wait(f"{bars}+{k0_full}", zero, 1)
        for g in range(QT):
            kit.wait(f"{bars}+{q_full[g]}", zero, 1)
            ins("tcgen05.fence::after_thread_sync")
            issue_s(g, k0)
            q_released(g, zero)
        ins(f"@{ism} {commit} [{bars}+{kv_empty[0]}]")                # K(0) consumed (block -1)
        mj, mblk, mti = t("b32"), t("b32"), t("b32")
        ins(f"mov.u32 {mj}, 0")
        ins(f"mov.u32 {mblk}, 0")
        ins(f"mov.u32 {mti}, 0")
        mtop = lab("at_mma_k")
        place(mtop)
        nxt = t("b32")
        ins(f"add.u32 {nxt}, {mj}, 1")
        more, acc0, newtile, last = t("pred"), t("pred"), t("pred"), t("pred")
        ins(f"setp.lt.u32 {more}, {nxt}, {total}")
        ins(f"setp.ne.u32 {acc0}, {mblk}, 0")
        ins(f"setp.eq.u32 {newtile}, {mblk}, {n_blk - 1}")           # S(j + 1) opens the next tile
        ins(f"and.pred {last}, {ism}, {newtile}")
        st_, fb_, vs_, ks_ = t("b32"), t("b32"), t("b32"), t("b32")
        ins(f"rem.u32 {st_}, {mj}, {KS}")
        ins(f"mad.lo.u32 {fb_}, {st_}, 8, {bars}")
        ins(f"mad.lo.u32 {vs_}, {st_}, {kvb}, {v0}")
        kst = t("b32")
        ins(f"rem.u32 {kst}, {nxt}, {KS}")
        ins(f"mad.lo.u32 {ks_}, {kst}, {kvb}, {k0}")
        kf = t("b32")
        ins(f"add.u32 {kf}, {fb_}, {kv_full[0]}")
        kit.wait(kf, kit.parity(mj, KS), 1)                          # V(j) and K(j + 1) landed
        for g in range(QT):
            kit.wait(f"{bars}+{p_full[g]}", kit.parity(mj, 1), 1)
            nowait = lab("at_o_ready")
            ins(f"@{acc0} bra {nowait}")
            ins(f"setp.eq.u32 {p}, {mti}, 0")
            ins(f"@{p} bra {nowait}")
            pt = t("b32")
            ins(f"sub.u32 {pt}, {mti}, 1")
            kit.wait(f"{bars}+{o_free[g]}", kit.parity(pt, 1), 1)     # the previous tile's O_g was read
            place(nowait)
            ins("tcgen05.fence::after_thread_sync")
            issue_pv(g, vs_, acc0, last)
            skip_s = lab("at_nos")
            ins(f"@!{more} bra {skip_s}")
            sameq = lab("at_same_q")
            ins(f"@!{newtile} bra {sameq}")
            nq = t("b32")
            ins(f"add.u32 {nq}, {mti}, 1")
            kit.wait(f"{bars}+{q_full[g]}", kit.parity(nq, 1), 1)     # the next tile's Q_g landed
            ins("tcgen05.fence::after_thread_sync")
            place(sameq)
            issue_s(g, ks_)
            q_released(g, nxt)
            place(skip_s)
        ke = t("b32")
        ins(f"mad.lo.u32 {ke}, {kst}, 8, {bars}")
        ins(f"add.u32 {ke}, {ke}, {kv_empty[0]}")
        ins(f"@{ism} {commit} [{ke}]")                      # V(j) and K(j + 1) consumed: release j
        ins(f"mov.u32 {mj}, {nxt}")
        ins(f"add.u32 {mblk}, {mblk}, 1")
        ins(f"setp.eq.u32 {p}, {mblk}, {n_blk}")
        ins(f"@{p} add.u32 {mti}, {mti}, 1")
        ins(f"@{p} mov.u32 {mblk}, 0")
        ins(f"@{more} bra {mtop}")
        ins(f"bra {end}")

        # ---------------- softmax + epilogue (warps 0 .. 4 QT - 1) ----------------
        # warp w: query tile g = w / 4, TMEM lanes 32 (w % 4) .. (= the tile's rows of this thread)
        place(role_sm)
        if self.reg_split:
            ins(f"setmaxnreg.inc.sync.aligned.u32 {self.reg_split[0]}")
        grp, quarter, r = t("b32"), t("b32"), t("b32")
        ins(f"shr.u32 {grp}, {warp}, 2")
        ins(f"and.b32 {quarter}, {warp}, 3")
        ins(f"mad.lo.u32 {r}, {quarter}, 32, {lane}")
        trow = t("b32")
        ins(f"shl.b32 {trow}, {quarter}, 21")
        ins(f"add.u32 {trow}, {trow}, {tmem}")
        ocol, scol, gb8 = t("b32"), t("b32"), t("b32")
        ins(f"mad.lo.u32 {ocol}, {grp}, 128, {trow}")
        ins(f"add.u32 {scol}, {ocol}, {S_COL}")                  # the row's scores; P (key k in column k / 2)
        ins(f"add.u32 {ocol}, {ocol}, {O_COL}")
        ins(f"mad.lo.u32 {gb8}, {grp}, 8, {bars}")
        rowoff = t("b32")                                  # this thread's query row within the tile pair
        ins(f"mad.lo.u32 {rowoff}, {grp}, {BM}, {r}")
        wstage, srowa, r7 = t("b32"), t("b32"), t("b32")    # the warp's staging box and this row in it
        ins(f"mad.lo.u32 {wstage}, {warp}, {32 * self.box_bytes}, {stage0}")
        ins(f"mad.lo.u32 {srowa}, {lane}, {self.box_bytes}, {wstage}")
        ins(f"and.b32 {r7}, {lane}, 7")
        lead = t("pred")
        elect_one(em, lead)
        tmap_o = tmap_address(em, self.tmap_set, 4, 3)
        sc = t("f32")
        ins(f"ld.global.nc.f32 {sc}, [{em.buffer_reg(self.pscale.name)}]")
        ins(f"rcp.rn.f32 {sc}, {sc}")
        ins(f"mul.rn.f32 {sc}, {sc}, 0f{_f32bits(LOG2E)}")
        mref, mref8, l = t("f32"), t("f32"), t("f32")
        sti, stile, sj, blk2 = t("b32"), t("b32"), t("b32"), t("b32")
        ins(f"mov.u32 {sti}, 0")
        ins(f"mov.u32 {stile}, {cta}")
        ins(f"mov.u32 {sj}, 0")
        stile_top = lab("at_sm_tile")
        place(stile_top)
        ins(f"mov.f32 {mref}, 0fFF800000")
        ins(f"mov.f32 {mref8}, 0fFF800000")
        ins(f"mov.f32 {l}, 0f00000000")
        ins(f"mov.u32 {blk2}, 0")
        stop = lab("at_sm_blk")
        place(stop)
        kit.wait(f"{gb8}+{s_full[0]}", kit.parity(sj, 1), 2)
        ins("tcgen05.fence::after_thread_sync")
        # the row's 128 scores into registers: all loads in flight, one wait
        srow = [t("f32") for _ in range(BN)]
        for c in range(BN // 32):
            a = t("b32")
            ins(f"add.u32 {a}, {scol}, {32 * c}")
            ins(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(srow[32 * c:32 * c + 32])}}}, [{a}]")
        ins("tcgen05.wait::ld.sync.aligned")
        mx = _tree(em, "max.f32", srow, arity=3)
        mnew = t("f32")
        ins(f"mul.rn.f32 {mnew}, {mx}, {sc}")
        # a row rescales when its maximum grew by more than 2^8; the warp decides together (the
        # O rescale is warp-wide tcgen05 work): a lane whose row need not rescale takes alpha = 1
        norescale, noowait = lab("at_norescale"), lab("at_first")
        grew, anyg = t("pred"), t("pred")
        ins(f"setp.gt.f32 {grew}, {mnew}, {mref8}")
        ins(f"vote.sync.any.pred {anyg}, {grew}, -1")
        ins(f"@!{anyg} bra {norescale}")
        alpha, dm = t("f32"), t("f32")
        ins(f"sub.rn.f32 {dm}, {mref}, {mnew}")
        ins(f"ex2.approx.ftz.f32 {alpha}, {dm}")
        ins(f"selp.f32 {alpha}, {alpha}, 0f3F800000, {grew}")
        ins(f"mul.rn.f32 {l}, {l}, {alpha}")
        ins(f"setp.eq.u32 {p}, {blk2}, 0")
        ins(f"@{p} bra {noowait}")
        # PV_g(j - 1) is complete: the commit this thread waited for (S_g(j)) covers it
        rw = 16                             # columns at a time: the scores hold the registers
        for c in range(D // rw):
            ov = [t("f32") for _ in range(rw)]
            a = t("b32")
            ins(f"add.u32 {a}, {ocol}, {rw * c}")
            ins(f"tcgen05.ld.sync.aligned.32x32b.x{rw}.b32 {{{', '.join(ov)}}}, [{a}]")
            ins("tcgen05.wait::ld.sync.aligned")
            for x in ov:
                ins(f"mul.rn.f32 {x}, {x}, {alpha}")
            ins(f"tcgen05.st.sync.aligned.32x32b.x{rw}.b32 [{a}], {{{', '.join(ov)}}}")
        ins("tcgen05.wait::st.sync.aligned")
        place(noowait)
        m8 = t("f32")
        ins(f"add.rn.f32 {m8}, {mnew}, 0f41000000")
        ins(f"selp.f32 {mref}, {mnew}, {mref}, {grew}")
        ins(f"selp.f32 {mref8}, {m8}, {mref8}, {grew}")
        place(norescale)
        negm = t("f32")
        ins(f"neg.f32 {negm}, {mref}")
        # P = 2^(s c' - m), 16 scores at a time, written back as f16 pairs over S's first 64 columns
        # (every score of the row is already in registers, so the stores cannot overtake a load).
        # Pairs of scores go through the packed f32x2 FMA pipe.
        pair = t("b64"), t("b64")
        ins(f"mov.b64 {pair[0]}, {{{sc}, {sc}}}")
        ins(f"mov.b64 {pair[1]}, {{{negm}, {negm}}}")
        ex2 = _Exp2(em) if self.poly_pairs else None
        for c in range(BN // 16):
            sv = srow[16 * c:16 * c + 16]
            packs = []
            for k in range(8):
                x0, x1 = sv[2 * k], sv[2 * k + 1]
                d = t("b64")
                ins(f"mov.b64 {d}, {{{x0}, {x1}}}")
                ins(f"fma.rn.ftz.f32x2 {d}, {d}, {pair[0]}, {pair[1]}")
                if k < self.poly_pairs:
                    packs.append(ex2.pair(d, x0, x1))
                    continue
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
            ins(f"add.u32 {a2}, {scol}, {8 * c}")
            ins(f"tcgen05.st.sync.aligned.32x32b.x8.b32 [{a2}], {{{', '.join(hp)}}}")
        ins("tcgen05.wait::st.sync.aligned")
        ins("tcgen05.fence::before_thread_sync")
        ins(f"mbarrier.arrive.shared::cta.b64 _, [{gb8}+{p_full[0]}]")
        ins(f"add.u32 {sj}, {sj}, 1")
        ins(f"add.u32 {blk2}, {blk2}, 1")
        ins(f"setp.lt.u32 {p}, {blk2}, {n_blk}")
        ins(f"@{p} bra {stop}")
        # epilogue: O / l -> f16 -> this row of the output through the warp's staging box and TMA
        # stores; O_g's TMEM goes back to the MMA warp once read (the TMEM and shared memory go on
        # to the next tile), the box is reused only after the previous store has read it
        qrow_s, _ = tile_rows(stile)
        orow = t("b32")
        ins(f"add.u32 {orow}, {qrow_s}, {rowoff}")
        ins(f"sub.u32 {orow}, {orow}, {lane}")                    # the warp's first row
        kit.wait(f"{gb8}+{o_done[0]}", kit.parity(sti, 1), 3)           # the tile's last PV_g
        ins("tcgen05.fence::after_thread_sync")
        ov = [t("f32") for _ in range(D)]
        for c in range(D // 32):
            a = t("b32")
            ins(f"add.u32 {a}, {ocol}, {32 * c}")
            ins(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ov[32 * c:32 * c + 32])}}}, [{a}]")
        ins("tcgen05.wait::ld.sync.aligned")
        ins("tcgen05.fence::before_thread_sync")
        ins(f"mbarrier.arrive.shared::cta.b64 _, [{gb8}+{o_free[0]}]")
        inv = t("f32")
        ins(f"rcp.rn.f32 {inv}, {l}")
        # 64 columns at a time: this row's 128 bytes into the warp's 32 x 128 B box (16-byte chunk
        # c of row r at chunk c ^ (r % 8): the 128-byte swizzle, conflict-free)
        for hb in range(D // 64):
            ins(f"@{lead} cp.async.bulk.wait_group.read 0")
            ins("bar.warp.sync -1")
            for c in range(8):
                oh = [t("b32") for _ in range(4)]
                for k in range(4):
                    x0, x1 = ov[64 * hb + 8 * c + 2 * k], ov[64 * hb + 8 * c + 2 * k + 1]
                    ins(f"mul.rn.f32 {x0}, {x0}, {inv}")
                    ins(f"mul.rn.f32 {x1}, {x1}, {inv}")
                    ins(f"cvt.rn.f16x2.f32 {oh[k]}, {x1}, {x0}")
                ch = t("b32")
                ins(f"xor.b32 {ch}, {r7}, {c}")
                ins(f"mad.lo.u32 {ch}, {ch}, 16, {srowa}")
                ins(f"st.shared.v4.b32 [{ch}], {{{', '.join(oh)}}}")
            ins("fence.proxy.async.shared::cta")
            ins("bar.warp.sync -1")
            ins(f"@{lead} cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [{tmap_o}, "
                f"{{{64 * hb}, {orow}}}], [{wstage}]")
            ins(f"@{lead} cp.async.bulk.commit_group")
        ins(f"add.u32 {sti}, {sti}, 1")
        ins(f"add.u32 {stile}, {stile}, {ncta}")
        ins(f"setp.lt.u32 {p}, {sti}, {nt}")
        ins(f"@{p} bra {stile_top}")
        ins(f"@{lead} cp.async.bulk.wait_group 0")               # the output stores are complete

        # ---------------- common exit ----------------
        place(end)
        ins("barrier.sync 0")
        nod = lab("at_nodealloc")
        ins(f"setp.ne.u32 {p}, {warp}, {self.w_mma}")
        ins(f"@{p} bra {nod}")
        ins("tcgen05.fence::after_thread_sync")
        ins(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {tmem}, 512")
        place(nod)


def _f32bits(x: float) -> str:
    import struct
    return "%08X" % struct.unpack("<I", struct.pack("<f", x))[0]


class _Exp2:
    """2^x for a pair of f32 lanes on the FMA pipe (packed f32x2), in place of two ex2.approx.

    Range reduction in the Cody-Waite manner: x (clamped to >= -125, where 2^x already rounds to
    0 in the f16 P tile) is split as x = j + f, j = round(x) by adding and subtracting 1.5 * 2^23,
    |f| <= 1/2.  2^f comes from a degree-3 polynomial fitted for this kernel (least squares on
    Chebyshev nodes of [-1/2, 1/2], reweighted toward equal relative error: at most 7.5e-5
    relative, evaluated in f32, under the 2^-11 rounding of the f16 P), and j is added into the
    exponent field as an integer: the low bits of (x + 1.5 * 2^23) hold j, so (its bits << 23)
    is j << 23 modulo 2^32.
    """

    COEF = (0.9999280727914258, 0.6932609870112008, 0.24261113509452387, 0.055171666814684134)

    def __init__(self, em):
        self.em = em
        self.k = []
        for v in (12582912.0,) + self.COEF:
            r = em.tmp("b64")
            h = _f32bits(v)
            em.ins(f"mov.b64 {r}, 0x{h}{h}")
            self.k.append(r)

    def pair(self, d: str, x0: str, x1: str) -> str:
        em, ins = self.em, self.em.ins
        mag, c0, c1, c2, c3 = self.k
        ins(f"mov.b64 {{{x0}, {x1}}}, {d}")
        ins(f"max.f32 {x0}, {x0}, 0fC2FA0000")
        ins(f"max.f32 {x1}, {x1}, 0fC2FA0000")
        x, tj, f, p = em.tmp("b64"), em.tmp("b64"), em.tmp("b64"), em.tmp("b64")
        ins(f"mov.b64 {x}, {{{x0}, {x1}}}")
        ins(f"add.rn.f32x2 {tj}, {x}, {mag}")
        ins(f"sub.rn.f32x2 {f}, {tj}, {mag}")
        ins(f"sub.rn.f32x2 {f}, {x}, {f}")
        ins(f"fma.rn.f32x2 {p}, {f}, {c3}, {c2}")
        ins(f"fma.rn.f32x2 {p}, {p}, {f}, {c1}")
        ins(f"fma.rn.f32x2 {p}, {p}, {f}, {c0}")
        j0, j1, p0, p1 = (em.tmp("b32") for _ in range(4))
        ins(f"mov.b64 {{{j0}, {j1}}}, {tj}")
        ins(f"mov.b64 {{{p0}, {p1}}}, {p}")
        for j, q, x_ in ((j0, p0, x0), (j1, p1, x1)):
            ins(f"mad.lo.u32 {q}, {j}, {1 << 23}, {q}")
            ins(f"mov.b32 {x_}, {q}")
        r = em.tmp("b64")
        ins(f"mov.b64 {r}, {{{x0}, {x1}}}")
        return r


def _tree(em, op: str, regs: list[str], arity: int = 2, kind: str = "f32") -> str:
    """Reduction tree of ``regs`` with ``op`` (keeps the inputs); ``arity`` 3 uses
    the three-source form sm_100 has for max / min."""
    cur = list(regs)
    while len(cur) > 1:
        nxt, i = [], 0
        while i < len(cur):
            n = min(arity, len(cur) - i)
            if n == 1:
                nxt.append(cur[i])
            else:
                d = em.tmp(kind)
                em.ins(f"{op} {d}, {', '.join(cur[i:i + n])}")
                nxt.append(d)
            i += n
        cur = nxt
    return cur[0]


def recognise(kernel: KernelInfo):
    return TcAttention.match(kernel)
