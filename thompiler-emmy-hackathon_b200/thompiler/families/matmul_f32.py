"""Tuned family: f32 matmul on the FMA pipes (the m01 / m02 schedules).

Recognised IR: the reference problems' f32 matmul schedules (problems/m01_matmul_512,
problems/m02_matmul_rect) -- CpAsyncCopy of A and B tiles into two shared arrays, an unrolled
inner loop of Loads from them whose products are accumulated (``Accum add`` of ``Assign
multiply``), then the accumulators written to C; m02 adds 32 split-K partials into a zeroed C
with atomic Writes (``red.global.add``).  What is checked: three f32 2-D parameters, A [M, K]
and B [K, N] read only and C [M, N] written; each shared array filled from one of them; the
inner loop variable in the last index of A's tile loads and the first index of B's (both
operands row-major in shared memory); the Write rows / columns driven by the same thread
coordinates as A's rows / B's columns; products and sums only.  Atomic Writes are accepted when
meta.json zeroes C before every launch (then writing the full sum is the same result).

Tuned body: C = A B with every output's full K sum kept in a register of one thread -- no
split-K, no atomics.  A CTA of 256 threads (16 x 16) owns a BM x BN tile of C (64 x 64, each
thread 4 x 4 outputs, or 32 x 32 with 2 x 2 when that gives more CTAs to fill the SMs).  K goes
in steps of 16: the next step's A and B chunks are loaded (``ld.global.nc.v4``) into registers
while the current step's tiles in shared memory feed ``fma.rn.f32`` (A stored k-major, so a
thread's RM rows of one k are one vector load; B row-major, RN columns one vector load); the
two shared buffers alternate.  Sums run in ascending k, in f32 -- within rtol 1e-3 of the
reference's order (its 32 partials of 8 terms added in arrival order).  Why not the tensor
cores: kind::tf32 rounds the operands to 10 mantissa bits, which misses these problems' f32
tolerance at K = 512, and at m01's and m02's sizes (0.27 and 0.004 GFLOP) the launch, not the
FMA rate, bounds the time.

Guard: the tuned launch's block (256) and grid (the tile count), and 16-byte aligned A, B and C;
any other launch runs the generic lowering of the same IR.
"""

from __future__ import annotations

from thompiler import ir
from thompiler.families.base import TunedKernel
from thompiler.load import KernelInfo
from thompiler.lowering.types import F32

BK = 16
THREADS = 256
SM_COUNT = 148
TILES = ((64, 64), (32, 32))          # (BM, BN): A and B chunks per K step fill 512 / 256 threads


def _vars(e) -> set[str]:
    if isinstance(e, ir.Var):
        return {e.name}
    out: set[str] = set()
    for f in ("left", "right", "cond", "if_true", "if_false", "operand", "value"):
        x = getattr(e, f, None)
        if x is not None and not isinstance(x, (str, int, float)):
            out |= _vars(x)
    for x in getattr(e, "args", ()) or ():
        if not isinstance(x, (str, int, float)):
            out |= _vars(x)
    return out


class MatmulF32(TunedKernel):
    family = "simt-matmul-f32"

    def __init__(self, kernel: KernelInfo, a, b, c, M, N, K, bm, bn):
        super().__init__(kernel)
        self.a, self.b, self.c = a, b, c
        self.M, self.N, self.K = M, N, K
        self.BM, self.BN = bm, bn
        self.RM, self.RN = bm // 16, bn // 16
        self.tiles = (M // bm) * (N // bn)

    @classmethod
    def match(cls, kernel: KernelInfo):  # noqa: C901 - one recogniser, in order
        body = kernel.body
        if len(body) != 1 or not isinstance(body[0], ir.Tile) or len(kernel.params) != 3:
            return None
        tile = body[0]
        ok = (ir.Init, ir.Smem, ir.StridedLoop, ir.Loop, ir.CpAsyncCopy, ir.CpAsyncCommit, ir.CpAsyncWait,
              ir.Sync, ir.Load, ir.Assign, ir.Accum, ir.Write)
        stmts = list(ir.walk_stmts(tile.body))
        if not all(isinstance(s, ok) for s in stmts):
            return None
        if any(p.ty is not F32 or len(p.shape) != 2 for p in kernel.params):
            return None
        outs = [p for p in kernel.params if p.written]
        if len(outs) != 1:
            return None
        c = outs[0]
        smem = {s.name for s in stmts if isinstance(s, ir.Smem)}
        if len(smem) != 2:
            return None
        fill: dict[str, str] = {}
        for s in stmts:
            if isinstance(s, ir.CpAsyncCopy):
                src = kernel.param(s.src)
                if s.smem not in smem or src is None or src.written or fill.setdefault(s.smem, s.src) != s.src:
                    return None
        if set(fill) != smem or len(set(fill.values())) != 2:
            return None
        loads = {}
        for s in stmts:
            if isinstance(s, ir.Load):
                if s.input not in smem or len(s.names) != 1 or len(s.index) != 2:
                    return None
                loads[s.names[0]] = s
        products = {}
        for s in stmts:
            if isinstance(s, ir.Assign):
                if s.op.name != "multiply" or len(s.args) != 2 or not all(x in loads for x in s.args):
                    return None
                srcs = {loads[x].input for x in s.args}
                if srcs != smem:
                    return None
                products[s.name] = s
        accs = set()
        for s in stmts:
            if isinstance(s, ir.Accum):
                if s.op.name != "add" or s.base is not None or s.value not in products:
                    return None
                accs.add(s.name)
            elif isinstance(s, ir.Init) and s.identity != 0.0:
                return None
        writes = [s for s in stmts if isinstance(s, ir.Write)]
        if not writes or not accs or any(w.output != c.name or len(w.index) != 2 for w in writes):
            return None
        if any(v not in accs for w in writes for v in w.values):
            return None
        atomic = {w.atomic for w in writes}
        if len(atomic) != 1 or (atomic == {True} and c.name not in kernel.zero_outputs):
            return None
        # which shared array is A: the inner (Loop) variable is the last index of A's tile loads
        # and the first of B's; A's row and B's column are driven by the Write's row / column vars
        inner = {s.axis.name for s in stmts if isinstance(s, ir.Loop)}
        if len(inner) != 1:
            return None
        ki = inner.pop()
        row_v = set().union(*(_vars(w.index[0]) for w in writes)) - {ki}
        col_v = set().union(*(_vars(w.index[1]) for w in writes)) - {ki}
        role = {}
        for ld in loads.values():
            first, last = _vars(ld.index[0]), _vars(ld.index[1])
            if ki in last and ki not in first and first & row_v and not first & col_v:
                r = "a"
            elif ki in first and ki not in last and last & col_v and not last & row_v:
                r = "b"
            else:
                return None
            if role.setdefault(ld.input, r) != r:
                return None
        if sorted(role.values()) != ["a", "b"]:
            return None
        inv = {r: s for s, r in role.items()}
        a, b = kernel.param(fill[inv["a"]]), kernel.param(fill[inv["b"]])
        M, K = a.shape
        K2, N = b.shape
        if K2 != K or c.shape != (M, N) or K % BK or N % 4:
            return None
        for bm, bn in TILES:
            if M % bm == 0 and N % bn == 0 and (M // bm) * (N // bn) >= SM_COUNT:
                return cls(kernel, a, b, c, M, N, K, bm, bn)
        small = [(bm, bn) for bm, bn in TILES if M % bm == 0 and N % bn == 0]
        if not small:
            return None
        return cls(kernel, a, b, c, M, N, K, *small[-1])

    # ---- launch ---------------------------------------------------------------------

    def sidecar(self) -> dict:
        return {"grid": [self.tiles, 1, 1], "block": [THREADS, 1, 1], "smem_bytes": 0,
                "tile": [self.BM, self.BN, BK]}

    def guard(self, generic: str) -> None:
        em = self.em
        sa, sb = 2 * BK * (self.BM + 4) * 4, 2 * BK * self.BN * 4
        em.module(f".shared .align 16 .b8 mf_a[{sa}]")
        em.module(f".shared .align 16 .b8 mf_b[{sb}]")
        p = em.tmp("pred")
        for reg, want in (("%ntid.x", THREADS), ("%nctaid.x", self.tiles)):
            r = self.special(reg)
            em.ins(f"setp.ne.u32 {p}, {r}, {want}")
            em.ins(f"@{p} bra {generic}")
        for prm in (self.a, self.b, self.c):
            raw, low = em.tmp("b64"), em.tmp("b64")
            em.ins(f"ld.param.u64 {raw}, [p_{prm.name}]")
            em.ins(f"and.b64 {low}, {raw}, 15")
            em.ins(f"setp.ne.u64 {p}, {low}, 0")
            em.ins(f"@{p} bra {generic}")

    # ---- the tuned body ----------------------------------------------------------------

    def emit_tuned(self) -> None:
        em = self.em
        t, ins, place, lab = em.tmp, em.ins, em.place, em.label
        self.pdl_trigger()
        self.pdl_wait()
        M, N, K, BM, BN, RM, RN = self.M, self.N, self.K, self.BM, self.BN, self.RM, self.RN
        AS = BM + 4                          # k-major A rows, padded against bank conflicts
        a_buf, b_buf = BK * AS * 4, BK * BN * 4
        ach, bch = BM * BK // 4, BK * BN // 4      # 16-byte chunks of one K step
        ga, gb, gc = (em.buffer_reg(p.name) for p in (self.a, self.b, self.c))
        tid, tx, ty = t("b32"), t("b32"), t("b32")
        ins(f"mov.u32 {tid}, %tid.x")
        ins(f"and.b32 {tx}, {tid}, 15")
        ins(f"shr.u32 {ty}, {tid}, 4")
        bid, bm, bn = t("b32"), t("b32"), t("b32")
        ins(f"mov.u32 {bid}, %ctaid.x")
        ins(f"div.u32 {bm}, {bid}, {N // BN}")
        ins(f"rem.u32 {bn}, {bid}, {N // BN}")
        sa0, sb0 = t("b32"), t("b32")
        ins(f"mov.u32 {sa0}, mf_a")
        ins(f"mov.u32 {sb0}, mf_b")

        # this thread's chunks of each K step: ids tid + 256 r; ids below ach are A chunks
        assert (ach + bch) % THREADS == 0 and (ach % THREADS == 0 or ach + bch == THREADS)
        rounds = [r * THREADS for r in range((ach + bch) // THREADS)]

        # per round: the chunk id, whether it is an A chunk, the global address and shared offset
        plan = []
        for c0 in rounds:
            cid = t("b32")
            ins(f"add.u32 {cid}, {tid}, {c0}")
            is_a = t("pred")
            ins(f"setp.lt.u32 {is_a}, {cid}, {ach}")
            # A chunk c: row c / (BK / 4), k (c % (BK / 4)) * 4
            arow, ak, aoff = t("b32"), t("b32"), t("b64")
            ins(f"shr.u32 {arow}, {cid}, {(BK // 4).bit_length() - 1}")
            ins(f"and.b32 {ak}, {cid}, {BK // 4 - 1}")
            ins(f"shl.b32 {ak}, {ak}, 2")
            grow = t("b32")
            ins(f"mad.lo.u32 {grow}, {bm}, {BM}, {arow}")
            gidx = t("b64")
            ins(f"mul.wide.u32 {gidx}, {grow}, {K}")
            ak64 = t("b64")
            ins(f"cvt.u64.u32 {ak64}, {ak}")
            ins(f"add.u64 {gidx}, {gidx}, {ak64}")
            ins(f"shl.b64 {aoff}, {gidx}, 2")
            ins(f"add.u64 {aoff}, {aoff}, {ga}")
            # shared: A[k][row] at (k * AS + row) * 4
            asts = t("b32")
            ins(f"mad.lo.u32 {asts}, {ak}, {AS}, {arow}")
            ins(f"shl.b32 {asts}, {asts}, 2")
            # B chunk c' = c - ach: k c' / (BN / 4), column (c' % (BN / 4)) * 4
            bc, bk, bcol, boff = t("b32"), t("b32"), t("b32"), t("b64")
            ins(f"sub.u32 {bc}, {cid}, {ach}")
            ins(f"shr.u32 {bk}, {bc}, {(BN // 4).bit_length() - 1}")
            ins(f"and.b32 {bcol}, {bc}, {BN // 4 - 1}")
            ins(f"shl.b32 {bcol}, {bcol}, 2")
            gcol = t("b32")
            ins(f"mad.lo.u32 {gcol}, {bn}, {BN}, {bcol}")
            bidx = t("b64")
            ins(f"mul.wide.u32 {bidx}, {bk}, {N}")
            gcol64 = t("b64")
            ins(f"cvt.u64.u32 {gcol64}, {gcol}")
            ins(f"add.u64 {bidx}, {bidx}, {gcol64}")
            ins(f"shl.b64 {boff}, {bidx}, 2")
            ins(f"add.u64 {boff}, {boff}, {gb}")
            bsts = t("b32")
            ins(f"mad.lo.u32 {bsts}, {bk}, {BN}, {bcol}")
            ins(f"shl.b32 {bsts}, {bsts}, 2")
            plan.append((is_a, aoff, asts, ak, boff, bsts))

        regs = [[t("f32") for _ in range(4)] for _ in plan]

        def gload(step: str) -> None:
            """The chunks of K step ``step`` into registers."""
            for (is_a, aoff, _, _, boff, _), v in zip(plan, regs):
                ka, kb = t("b64"), t("b64")
                ins(f"mul.wide.u32 {ka}, {step}, {BK * 4}")
                ins(f"add.u64 {ka}, {ka}, {aoff}")
                ins(f"mul.wide.u32 {kb}, {step}, {BK * N * 4}")
                ins(f"add.u64 {kb}, {kb}, {boff}")
                ins(f"@{is_a} ld.global.nc.v4.f32 {{{', '.join(v)}}}, [{ka}]")
                ins(f"@!{is_a} ld.global.nc.v4.f32 {{{', '.join(v)}}}, [{kb}]")

        def sstore(buf: str) -> None:
            """The loaded chunks into shared buffer ``buf`` (0 / 1): A transposed, B as it is."""
            for (is_a, _, asts, _, _, bsts), v in zip(plan, regs):
                ab, bb = t("b32"), t("b32")
                ins(f"mad.lo.u32 {ab}, {buf}, {a_buf}, {asts}")
                ins(f"add.u32 {ab}, {ab}, {sa0}")
                ins(f"mad.lo.u32 {bb}, {buf}, {b_buf}, {bsts}")
                ins(f"add.u32 {bb}, {bb}, {sb0}")
                for i in range(4):
                    ins(f"@{is_a} st.shared.f32 [{ab}+{i * AS * 4}], {v[i]}")
                ins(f"@!{is_a} st.shared.v4.f32 [{bb}], {{{', '.join(v)}}}")

        acc = [[t("f32") for _ in range(RN)] for _ in range(RM)]
        for row in acc:
            for x in row:
                ins(f"mov.f32 {x}, 0f00000000")
        step, buf = t("b32"), t("b32")
        ins(f"mov.u32 {step}, 0")
        ins(f"mov.u32 {buf}, 0")
        gload(step)
        sstore(buf)
        ins("bar.sync 0")
        # this thread's reads: A rows ty * RM .., B columns tx * RN ..
        ra, rb = t("b32"), t("b32")
        ins(f"shl.b32 {ra}, {ty}, {(RM * 4).bit_length() - 1}")
        ins(f"add.u32 {ra}, {ra}, {sa0}")
        ins(f"shl.b32 {rb}, {tx}, {(RN * 4).bit_length() - 1}")
        ins(f"add.u32 {rb}, {rb}, {sb0}")
        nsteps = K // BK
        top, last = lab("mf_k"), lab("mf_last")
        more = t("pred")
        place(top)
        nxt = t("b32")
        ins(f"add.u32 {nxt}, {step}, 1")
        ins(f"setp.lt.u32 {more}, {nxt}, {nsteps}")
        skip = lab("mf_noload")
        ins(f"@!{more} bra {skip}")
        gload(nxt)                                   # next step's chunks in flight during the FMAs
        place(skip)
        pa, pb = t("b32"), t("b32")
        ins(f"mad.lo.u32 {pa}, {buf}, {a_buf}, {ra}")
        ins(f"mad.lo.u32 {pb}, {buf}, {b_buf}, {rb}")
        for kk in range(BK):
            av = [t("f32") for _ in range(RM)]
            bv = [t("f32") for _ in range(RN)]
            ins(f"ld.shared.v{RM}.f32 {{{', '.join(av)}}}, [{pa}+{kk * AS * 4}]")
            ins(f"ld.shared.v{RN}.f32 {{{', '.join(bv)}}}, [{pb}+{kk * BN * 4}]")
            for i in range(RM):
                for j in range(RN):
                    ins(f"fma.rn.f32 {acc[i][j]}, {av[i]}, {bv[j]}, {acc[i][j]}")
        ins(f"@!{more} bra {last}")
        ins(f"xor.b32 {buf}, {buf}, 1")
        sstore(buf)                                  # the other buffer: nobody reads it now
        ins("bar.sync 0")
        ins(f"mov.u32 {step}, {nxt}")
        ins(f"bra {top}")
        place(last)
        # C rows bm BM + ty RM + i, columns bn BN + tx RN ..
        crow, ccol = t("b32"), t("b32")
        ins(f"mad.lo.u32 {crow}, {bm}, {BM}, 0")
        ins(f"mad.lo.u32 {crow}, {ty}, {RM}, {crow}")
        ins(f"mul.lo.u32 {ccol}, {bn}, {BN}")
        ins(f"mad.lo.u32 {ccol}, {tx}, {RN}, {ccol}")
        for i in range(RM):
            r_, idx, ad = t("b32"), t("b64"), t("b64")
            ins(f"add.u32 {r_}, {crow}, {i}")
            ins(f"mul.wide.u32 {idx}, {r_}, {N}")
            c64 = t("b64")
            ins(f"cvt.u64.u32 {c64}, {ccol}")
            ins(f"add.u64 {idx}, {idx}, {c64}")
            ins(f"shl.b64 {ad}, {idx}, 2")
            ins(f"add.u64 {ad}, {ad}, {gc}")
            ins(f"st.global.v{RN}.f32 [{ad}], {{{', '.join(acc[i])}}}")


def recognise(kernel: KernelInfo):
    return MatmulF32.match(kernel)
