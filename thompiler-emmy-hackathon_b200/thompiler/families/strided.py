"""Tuned family: strided reductions -- full sums / means (r01, r02, r03) and
row reductions with an optional elementwise pass (r04 row sums, f01
RMSNorm, f02 softmax, f03 L2-normalise).

The IR shape it recognises (emmy's cooperative-reduce schedule, e.g. the
reference's problems/f01_rmsnorm/k_mean_cbd1de.ir.txt):

    Tile[rows..., co]            co: one thread per column slot, extent T = block
      pre:  constant loads / Assign / Let
      L1:   for v in co..C:T      (seed)  loads of x[rows..., v] / w[v] / constants,
                                          Assigns, Accums  -- no stores
      WarpShuffle(states, 32) ... Smem, Cond(lane == 0) store, Sync, TreeHalve(T/32)
      mid:  constant loads / Assign / Let
      tail: either  for v2 in co..C:T { loads, Assigns, one store out[rows..., v2] }   (row map)
            or      if co == 0 { ..., store out[rows...] }                             (reduce)

Row mode (rows present).  One row per CTA, as meta.json launches it (grid =
rows, block = T), rows strided by the grid so any grid is correct.  Each
thread owns C/T elements, loaded with 128-bit ``ld.global.nc.v4`` in
coalesced chunks (chunk j of thread t starts at element (j*T + t)*4) and
kept in registers, so x is read from HBM once and y written once with
128-bit stores -- the reference re-reads x in its second loop with scalar
loads (2 reads + 1 write, 4-byte accesses).  The IR's own Assign / Accum
statements are replayed per resident element, and its shuffle / tree
combine statements are lowered by the generic handlers.

Full mode (no row axes).  A grid-stride stream of v4 chunks over all CTAs
(4 chunks in flight per thread), the IR's combine per CTA, then a
deterministic second pass: each CTA stores its state to a module-scope
``.global`` partials array, and the CTA whose ``atom.inc`` arrives last
(the counter wraps to 0 by itself, ready for the next launch) folds the
partials in CTA order with the IR's ``combine_states`` and runs the IR's
epilogue.  Under meta.json's single-CTA launch the second pass is skipped.
The tuned launch (recorded in the sidecar) is ``ctas_per_sm`` CTAs of T
threads per SM.  A single f32 sum also carries an in-kernel combine across
GPUs (off unless the host binds the module to its peers): the finishing CTA
adds the other ranks' results over NVLink before the epilogue, replacing a
separate all-reduce of the per-GPU partials.
"""

from __future__ import annotations

from math import prod

from thompiler import ir
from thompiler.families.base import TunedKernel
from thompiler.handlers.blocks import seed_accumulators
from thompiler.lowering.types import F32, dtype_of
from thompiler.load import KernelInfo

MAX_RESIDENT = 64           # elements a thread keeps in registers (row mode)
MAX_PARTIALS = 8192         # CTAs the full-mode second pass supports
SM_COUNT = 148
CTAS_PER_SM = 8
UNROLL = 4                  # v4 chunks in flight per thread (full mode)
MAX_PEERS = 8               # GPUs the in-kernel combine of a sharded sum supports
PEER_WAIT_LIMIT = 1 << 20   # polling rounds before the peer combine gives up


def _is_var(e, name: str) -> bool:
    return isinstance(e, ir.Var) and e.name == name


def _lit(e):
    if isinstance(e, ir.Literal):
        return e.value
    if isinstance(e, int) and not isinstance(e, bool):
        return e
    return None


def _const_index(index: tuple) -> bool:
    return all(isinstance(i, ir.Literal) for i in index)


def _stmt_names(s) -> set[str]:
    """IR names an index, value or condition of statement ``s`` refers to."""
    out: set[str] = set()
    for f in ("index", "value", "cond", "start", "end", "step"):
        v = getattr(s, f, None)
        for e in (v if isinstance(v, tuple) else (v,)):
            out |= _names_in(e)
    return out


def _names_in(e) -> set[str]:
    if isinstance(e, ir.Var):
        return {e.name}
    if isinstance(e, ir.BinaryExpr):
        return _names_in(e.left) | _names_in(e.right)
    if isinstance(e, ir.TernaryExpr):
        return _names_in(e.cond) | _names_in(e.if_true) | _names_in(e.if_false)
    return set()


class StridedReduce(TunedKernel):
    family = "strided-reduce"

    def __init__(self, kernel: KernelInfo, tile, rows, co, C, T, pre, l1, combine, mid, tail, states):
        super().__init__(kernel)
        self.tile, self.rows, self.co, self.C, self.T = tile, rows, co, C, T
        self.pre, self.l1, self.combine, self.mid, self.tail = pre, l1, combine, mid, tail
        self.states = states
        self.row_mode = bool(rows)
        self.R = prod(a.size for a in rows) if rows else 1
        self.E = C // T
        self.V = next(v for v in (4, 2, 1) if self.E % v == 0) if self.row_mode else \
            next(v for v in (4, 2, 1) if C % v == 0)
        self.resident: dict[str, list[str]] = {}     # buffer -> register per owned element
        self.consts: dict[tuple, str] = {}           # (buffer, index) -> register
        self.elem: int | None = None                 # element being replayed
        self.outs: dict[int, str] = {}               # element -> value register (row map)

    # ---- recognition --------------------------------------------------------

    @classmethod
    def match(cls, kernel: KernelInfo):
        body = kernel.body
        if len(body) != 1 or not isinstance(body[0], ir.Tile):
            return None
        tile = body[0]
        T = kernel.threads_per_cta
        if not tile.axes or tile.aux_threads or kernel.block[1:] != (1, 1):
            return None
        co = tile.axes[-1]
        rows = tuple(tile.axes[:-1])
        if co.size != T or T % 32 or T > 1024:
            return None
        stmts = list(tile.body)
        i1 = next((i for i, s in enumerate(stmts) if isinstance(s, ir.StridedLoop)), None)
        if i1 is None:
            return None
        pre, l1 = stmts[:i1], stmts[i1]
        row_names = {a.name for a in rows}
        rshape = tuple(a.size for a in rows)
        if not cls._loop_ok(l1, co, T):
            return None
        C = l1.axis.size
        if (rows and C % T) or kernel.dynamic_smem_bytes:
            return None
        if not cls._simple(pre, kernel, allow_loads="const"):
            return None
        if not cls._body_ok(l1.body, l1.axis.name, rows, rshape, C, kernel, allow_write=False):
            return None
        if not l1.seed:
            return None
        accs = {s.name for s in l1.body if isinstance(s, ir.Accum)}
        rest = stmts[i1 + 1:]
        ish = next((i for i, s in enumerate(rest) if isinstance(s, ir.WarpShuffle)), None)
        itr = next((i for i, s in enumerate(rest) if isinstance(s, ir.TreeHalve)), None)
        if ish != 0 or itr is None:
            return None
        sh, tr = rest[0], rest[itr]
        states = tuple(sh.state)
        if int(sh.length) != 32 or set(states) != accs or tuple(tr.state) != states:
            return None
        if int(tr.length) != T // 32 or tr.tid_var != "warp" or tr.inner is not None:
            return None
        combine = rest[:itr + 1]
        for s in combine[1:-1]:
            if not isinstance(s, (ir.Smem, ir.Sync, ir.Cond)):
                return None
        after = rest[itr + 1:]
        if not after:
            return None
        tail, mid = after[-1], after[:-1]
        if not cls._simple(mid, kernel, allow_loads="const"):
            return None
        if isinstance(tail, ir.StridedLoop):
            if not rows or not cls._loop_ok(tail, co, T) or tail.axis.size != C:
                return None
            if not cls._body_ok(tail.body, tail.axis.name, rows, rshape, C, kernel, allow_write=True):
                return None
        elif isinstance(tail, ir.Cond):
            c = tail.cond
            if not (isinstance(c, ir.BinaryExpr) and c.op == "==" and _is_var(c.left, co.name)
                    and _lit(c.right) == 0) or tail.else_body:
                return None
            for s in ir.walk_stmts(tail.body):
                if isinstance(s, (ir.Loop, ir.StridedLoop, ir.Sync, ir.Tile)):
                    return None
        else:
            return None
        # the column axis may only appear where this family rewrites it
        if any(co.name in _stmt_names(x) for x in ir.walk_stmts(tuple(pre) + tuple(mid))):
            return None
        k = cls(kernel, tile, rows, co, C, T, pre, l1, combine, mid, tail, states)
        if k.row_mode and k.E > MAX_RESIDENT:
            return None
        return k

    @staticmethod
    def _loop_ok(loop, co, T) -> bool:
        return (isinstance(loop, ir.StridedLoop) and _is_var(loop.start, co.name) and _lit(loop.step) == T
                and loop.end is None and loop.axis.extent.is_static)

    @staticmethod
    def _simple(stmts, kernel, allow_loads) -> bool:
        for s in stmts:
            if isinstance(s, ir.Load):
                if not _const_index(s.index) or kernel.param(s.input) is None or len(s.names) != 1:
                    return False
            elif not isinstance(s, (ir.Assign, ir.Let)):
                return False
            if isinstance(s, ir.Let) and not isinstance(s.value, ir.Literal):
                return False
        return True

    @staticmethod
    def _body_ok(body, var, rows, rshape, C, kernel, allow_write) -> bool:
        writes = 0
        for s in body:
            if isinstance(s, ir.Load):
                p = kernel.param(s.input)
                if p is None or len(s.names) != 1 or p.written:
                    return False
                if _const_index(s.index):
                    continue
                idx = tuple(s.index)
                if idx == tuple(ir.Var(a.name) for a in rows) + (ir.Var(var),) and p.shape == rshape + (C,):
                    continue
                if idx == (ir.Var(var),) and p.shape == (C,):
                    continue
                return False
            elif isinstance(s, ir.Write):
                p = kernel.param(s.output)
                if (not allow_write or p is None or s.atomic or len(s.values) != 1
                        or tuple(s.index) != tuple(ir.Var(a.name) for a in rows) + (ir.Var(var),)
                        or p.shape != rshape + (C,)):
                    return False
                writes += 1
            elif isinstance(s, ir.Let):
                if not isinstance(s.value, ir.Literal):
                    return False
            elif isinstance(s, ir.Accum):
                if allow_write:
                    return False
            elif not isinstance(s, ir.Assign):
                return False
        return writes == (1 if allow_write else 0)

    # ---- launch --------------------------------------------------------------

    def guard(self, generic: str) -> None:
        em = self.em
        ntid = self.special("%ntid.x")
        p = em.tmp("pred")
        em.ins(f"setp.ne.u32 {p}, {ntid}, {self.T}")
        em.ins(f"@{p} bra {generic}")
        if not self.row_mode:
            self.nctaid = self.special("%nctaid.x")
            em.ins(f"setp.gt.u32 {p}, {self.nctaid}, {MAX_PARTIALS}")
            em.ins(f"@{p} bra {generic}")

    def sidecar(self) -> dict | None:
        if self.row_mode:
            return None
        chunks = -(-self.C // self.V)
        ctas = min(MAX_PARTIALS, SM_COUNT * CTAS_PER_SM, max(1, -(-chunks // (self.T * UNROLL))))
        side = {"grid": [ctas, 1, 1], "block": [self.T, 1, 1], "smem_bytes": 0}
        if self._peer_capable():
            side.update(error_word="thc_error",
                        peer={"table": "thc_peer_ptr", "world": "thc_world", "rank": "thc_rank",
                              "max_ranks": MAX_PEERS})
        return side

    # ---- hooks -------------------------------------------------------------------

    def _load_hook(self, w, load: ir.Load) -> bool:
        key = (load.input, tuple(l.value for l in load.index)) if _const_index(load.index) else None
        em = self.em
        if key is not None and key in self.consts:
            src = self.consts[key]
        elif key is None and load.input in self.resident:
            src = self.resident[load.input][self.elem]
        else:
            return False
        ty = self.k.param(load.input).ty
        em.ins(f"mov.{ty.mov} {em.value(load.names[0], ty.reg)}, {src}")
        return True

    def _write_hook(self, w, wr: ir.Write) -> bool:
        p = self.k.param(wr.output)
        r = self.em.tmp(p.ty.reg)
        self.em.ins(f"mov.{p.ty.mov} {r}, {self.em.get(wr.values[0])}")
        self.outs[self.elem] = r
        return True

    def _hoist_consts(self, stmts) -> None:
        em = self.em
        for s in ir.walk_stmts(tuple(stmts)):
            if isinstance(s, ir.Load) and _const_index(s.index):
                key = (s.input, tuple(l.value for l in s.index))
                if key in self.consts:
                    continue
                p = self.k.param(s.input)
                flat = 0
                for size, i in zip(p.shape, key[1]):
                    flat = flat * size + int(i)
                r = em.tmp(p.ty.reg)
                off = flat * p.ty.nbytes
                base = em.buffer_reg(p.name)
                em.ins(f"ld.global.nc.{p.ty.mov} {r}, [{base}{'+' + str(off) if off else ''}]")
                self.consts[key] = r

    # ---- emission ------------------------------------------------------------------

    def emit_tuned(self) -> None:
        w = self.w
        self.pdl_trigger()
        self.pdl_wait()              # the body reads its inputs from the first instruction on
        w.load_hook = self._load_hook
        self._hoist_consts(tuple(self.l1.body) + (tuple(self.tail.body) if self.row_mode else ()))
        if self.row_mode:
            self._emit_rows()
        else:
            self._emit_full()

    def _buffers(self, body, var) -> list[str]:
        out = []
        for s in body:
            if isinstance(s, ir.Load) and not _const_index(s.index) and s.input not in out:
                out.append(s.input)
        return out

    def _preload(self, buffers, row_off64: str | None, tid: str) -> None:
        """Load this thread's E elements of each buffer (row slice or 1-D) into registers."""
        em, T, V, E = self.em, self.T, self.V, self.E
        for b in buffers:
            if b in self.resident:
                continue
            p = self.k.param(b)
            base = em.buffer_reg(b)
            if len(p.shape) > 1:
                rb = em.tmp("b64")
                em.ins(f"mad.lo.s64 {rb}, {row_off64}, {p.ty.nbytes}, {base}")
                base = rb
            t0 = em.tmp("b64")
            em.ins(f"mul.wide.u32 {t0}, {tid}, {V * p.ty.nbytes}")
            addr = em.tmp("b64")
            em.ins(f"add.s64 {addr}, {base}, {t0}")
            regs = [em.tmp(p.ty.reg) for _ in range(E)]
            vt = f"v{V}." if V > 1 else ""
            for j in range(E // V):
                off = j * T * V * p.ty.nbytes
                grp = regs[j * V:(j + 1) * V]
                dst = f"{{{', '.join(grp)}}}" if V > 1 else grp[0]
                em.ins(f"ld.global.nc.{vt}{p.ty.mov} {dst}, [{addr}{'+' + str(off) if off else ''}]")
            self.resident[b] = regs

    def _emit_rows(self) -> None:
        em, w, T, V, E, C = self.em, self.w, self.T, self.V, self.E, self.C
        tid = self.special("%tid.x")
        em.ins(f"mov.u32 {em.value(self.co.name, 'b32')}, {tid}")
        row = em.tmp("b32")
        em.ins(f"mov.u32 {row}, %ctaid.x")
        nrow = self.special("%nctaid.x")
        top, done = em.label("row"), em.label("rows_done")
        p = em.tmp("pred")
        em.ins(f"setp.ge.u32 {p}, {row}, {self.R}")
        em.ins(f"@{p} bra {done}")
        em.place(top)
        # decode the row axes (row-major) from the row index
        ext = [a.size for a in self.rows]
        for i, a in enumerate(self.rows):
            stride = prod(ext[i + 1:])
            reg = em.value(a.name, "b32")
            if i == 0:
                em.ins(f"div.u32 {reg}, {row}, {stride}" if stride != 1 else f"mov.u32 {reg}, {row}")
            else:
                q = em.tmp("b32")
                em.ins(f"div.u32 {q}, {row}, {stride}")
                em.ins(f"rem.u32 {reg}, {q}, {ext[i]}")
        roff = em.tmp("b64")
        em.ins(f"mul.wide.u32 {roff}, {row}, {C}")
        self.resident = {}
        self._preload(self._buffers(self.l1.body, self.l1.axis.name), roff, tid)
        w.body(self.pre)
        seed_accumulators(w, self.l1.body)
        for e in range(E):
            self.elem = e
            w.body(self.l1.body)
        self.elem = None
        w.body(self.combine)
        w.body(self.mid)
        if isinstance(self.tail, ir.StridedLoop):
            self._preload(self._buffers(self.tail.body, self.tail.axis.name), roff, tid)
            w.write_hook = self._write_hook
            self.outs = {}
            for e in range(E):
                self.elem = e
                w.body(self.tail.body)
            self.elem = None
            w.write_hook = None
            wr = next(s for s in self.tail.body if isinstance(s, ir.Write))
            po = self.k.param(wr.output)
            ob = em.tmp("b64")
            em.ins(f"mad.lo.s64 {ob}, {roff}, {po.ty.nbytes}, {em.buffer_reg(po.name)}")
            t0 = em.tmp("b64")
            em.ins(f"mul.wide.u32 {t0}, {tid}, {V * po.ty.nbytes}")
            em.ins(f"add.s64 {ob}, {ob}, {t0}")
            vt = f"v{V}." if V > 1 else ""
            for j in range(E // V):
                off = j * T * V * po.ty.nbytes
                grp = [self.outs[j * V + i] for i in range(V)]
                src = f"{{{', '.join(grp)}}}" if V > 1 else grp[0]
                em.ins(f"st.global.{vt}{po.ty.mov} [{ob}{'+' + str(off) if off else ''}], {src}")
        else:
            w.body((self.tail,))
        em.ins("bar.sync 0")          # the next row reuses the combine's shared slots
        em.ins(f"add.u32 {row}, {row}, {nrow}")
        em.ins(f"setp.lt.u32 {p}, {row}, {self.R}")
        em.ins(f"@{p} bra {top}")
        em.place(done)

    def _emit_full(self) -> None:
        em, w, T, V, C = self.em, self.w, self.T, self.V, self.C
        x = self._buffers(self.l1.body, self.l1.axis.name)
        tid = self.special("%tid.x")
        cta = self.special("%ctaid.x")
        nct = self.nctaid
        em.ins(f"mov.u32 {em.value(self.co.name, 'b32')}, {tid}")
        w.body(self.pre)
        seed_accumulators(w, self.l1.body)
        nchunks = C // V
        c = em.tmp("b32")
        stride = em.tmp("b32")
        em.ins(f"mad.lo.u32 {c}, {cta}, {T}, {tid}")
        em.ins(f"mul.lo.u32 {stride}, {nct}, {T}")
        bases = {b: em.buffer_reg(b) for b in x}
        nbytes = {b: self.k.param(b).ty.nbytes for b in x}

        def load_chunks(cregs: list[str]) -> None:
            self.resident = {}
            for b in x:
                p = self.k.param(b)
                regs = []
                for ci in cregs:
                    a = em.tmp("b64")
                    em.ins(f"mad.wide.u32 {a}, {ci}, {V * nbytes[b]}, {bases[b]}")
                    grp = [em.tmp(p.ty.reg) for _ in range(V)]
                    vt = f"v{V}." if V > 1 else ""
                    dst = f"{{{', '.join(grp)}}}" if V > 1 else grp[0]
                    em.ins(f"ld.global.nc.{vt}{p.ty.mov} {dst}, [{a}]")
                    regs += grp
                self.resident[b] = regs

        def fold(n: int) -> None:
            for e in range(n):
                self.elem = e
                w.body(self.l1.body)
            self.elem = None

        main, tail, tail_top, done = em.label("stream"), em.label("stream_tail"), em.label("tail_top"), \
            em.label("stream_done")
        last = em.tmp("b32")
        p = em.tmp("pred")
        em.place(main)
        em.ins(f"mad.lo.u32 {last}, {stride}, {UNROLL - 1}, {c}")
        em.ins(f"setp.ge.u32 {p}, {last}, {nchunks}")
        em.ins(f"@{p} bra {tail}")
        cs = [c] + [em.tmp("b32") for _ in range(UNROLL - 1)]
        for i in range(1, UNROLL):
            em.ins(f"mad.lo.u32 {cs[i]}, {stride}, {i}, {c}")
        load_chunks(cs)
        fold(UNROLL * V)
        em.ins(f"mad.lo.u32 {c}, {stride}, {UNROLL}, {c}")
        em.ins(f"bra {main}")
        em.place(tail)
        em.ins(f"setp.ge.u32 {p}, {c}, {nchunks}")
        em.ins(f"@{p} bra {done}")
        em.place(tail_top)
        load_chunks([c])
        fold(V)
        em.ins(f"add.u32 {c}, {c}, {stride}")
        em.ins(f"setp.lt.u32 {p}, {c}, {nchunks}")
        em.ins(f"@{p} bra {tail_top}")
        em.place(done)
        w.body(self.combine)
        final = em.label("final")
        em.ins(f"setp.eq.u32 {p}, {nct}, 1")
        em.ins(f"@{p} bra {final}")
        self._second_pass(cta, tid, nct)
        em.place(final)
        if self._peer_capable():
            self._peer_combine(tid)
        w.body(self.mid)
        w.body((self.tail,))

    def _peer_capable(self) -> bool:
        """A plain f32 sum: one add state written out as it is (r01 / r02) -- the result the
        ranks of a sharded sum add up.  A mean (r03) divides by its count and is left alone."""
        accs = [s for s in self.l1.body if isinstance(s, ir.Accum)]
        if self.row_mode or len(self.states) != 1 or len(accs) != 1:
            return False
        if accs[0].op.name != "add" or dtype_of(accs[0].dtype, "Accum") is not F32:
            return False
        tail = self.tail.body if isinstance(self.tail, ir.Cond) else ()
        writes = [s for s in tail if isinstance(s, ir.Write)]
        return (not any(isinstance(s, ir.Assign) for s in tuple(self.mid) + tuple(tail))
                and len(writes) == 1 and tuple(writes[0].values) == (self.states[0],))

    def _peer_combine(self, tid: str) -> None:
        """Add the other GPUs' results to this one over peer memory, inside the kernel.

        Off unless the host sets ``thc_world`` > 1 (``thompiler.shard.PeerCombine``), which
        also fills ``thc_peer_ptr[r]`` with rank r's mailbox (8 slots of 8 bytes, CUDA IPC
        mapped) and ``thc_rank``.  Thread 0 of the finishing CTA bumps the module's launch
        counter ``thc_epoch``, publishes (epoch << 32 | f32 bits) into slot ``rank`` of every
        rank's mailbox -- one 64-bit store carries both, so relaxed system-scope stores and loads
        suffice (no release fence per peer) -- then polls all of its own mailbox's slots in one
        round until each carries this epoch and adds the values in rank order: every rank gets
        the same total.  The wait gives up after PEER_WAIT_LIMIT rounds (tens of nanoseconds
        apart), sets bit 0 of ``thc_error`` and adds only the values that arrived, so a rank that
        never arrives costs at most about a second and no hang.  The ranks run the same sequence
        of launches, so their epochs agree.
        """
        em = self.em
        em.module(f".global .align 8 .u64 thc_peer_ptr[{MAX_PEERS}]")
        em.module(".global .align 4 .u32 thc_world = 1")
        em.module(".global .align 4 .u32 thc_rank = 0")
        em.module(".global .align 4 .u32 thc_epoch = 0")
        em.module(".global .align 4 .u32 thc_error = 0")
        em.module(".shared .align 4 .f32 thc_peer_total")
        acc = em.get(self.states[0])
        p, q = em.tmp("pred"), em.tmp("pred")
        world, rank, e = em.tmp("b32"), em.tmp("b32"), em.tmp("b32")
        skip, bar = em.label("no_peer"), em.label("peer_bar")
        em.ins(f"ld.global.u32 {world}, [thc_world]")
        em.ins(f"setp.le.u32 {p}, {world}, 1")
        em.ins(f"@{p} bra {skip}")
        em.ins(f"setp.ne.u32 {p}, {tid}, 0")
        em.ins(f"@{p} bra {bar}")
        em.ins(f"ld.global.u32 {rank}, [thc_rank]")
        em.ins(f"ld.global.u32 {e}, [thc_epoch]")
        em.ins(f"add.u32 {e}, {e}, 1")
        em.ins(f"st.global.u32 [thc_epoch], {e}")
        vb, pack, off = em.tmp("b32"), em.tmp("b64"), em.tmp("b64")
        em.ins(f"mov.b32 {vb}, {acc}")
        em.ins(f"mov.b64 {pack}, {{{vb}, {e}}}")
        em.ins(f"mul.wide.u32 {off}, {rank}, 8")
        for r in range(MAX_PEERS):                        # publish into slot `rank` of every mailbox
            base = em.tmp("b64")
            em.ins(f"setp.gt.u32 {q}, {world}, {r}")
            em.ins(f"@{q} ld.global.u64 {base}, [thc_peer_ptr+{8 * r}]")
            em.ins(f"@{q} add.u64 {base}, {base}, {off}")
            em.ins(f"@{q} st.relaxed.sys.global.u64 [{base}], {pack}")
        own, tab = em.tmp("b64"), em.tmp("b64")
        em.ins(f"mov.u64 {tab}, thc_peer_ptr")
        em.ins(f"add.u64 {tab}, {tab}, {off}")
        em.ins(f"ld.global.u64 {own}, [{tab}]")
        total, n = em.tmp("f32"), em.tmp("b32")
        em.ins(f"mov.f32 {total}, 0f00000000")
        # poll every slot in one round until all carry this epoch, then add them in rank order
        top, done = em.label("peer_wait"), em.label("peer_done")
        live = [em.tmp("pred") for _ in range(MAX_PEERS)]
        got = [em.tmp("pred") for _ in range(MAX_PEERS)]
        los = [em.tmp("b32") for _ in range(MAX_PEERS)]
        for r in range(MAX_PEERS):
            em.ins(f"setp.gt.u32 {live[r]}, {world}, {r}")
        em.ins(f"mov.u32 {n}, 0")
        em.place(top)
        allin = em.tmp("pred")
        em.ins(f"setp.eq.u32 {allin}, {n}, {n}")
        for r in range(MAX_PEERS):
            x, hi = em.tmp("b64"), em.tmp("b32")
            em.ins(f"mov.u32 {hi}, {e}")
            em.ins(f"@{live[r]} ld.relaxed.sys.global.u64 {x}, [{own}+{8 * r}]")
            em.ins(f"@{live[r]} mov.b64 {{{los[r]}, {hi}}}, {x}")
            em.ins(f"setp.eq.u32 {got[r]}, {hi}, {e}")
            em.ins(f"and.pred {allin}, {allin}, {got[r]}")
        em.ins(f"@{allin} bra {done}")
        em.ins(f"add.u32 {n}, {n}, 1")
        em.ins(f"setp.lt.u32 {q}, {n}, {PEER_WAIT_LIMIT}")
        em.ins(f"@{q} nanosleep.u32 32")
        em.ins(f"@{q} bra {top}")
        em.ins(f"atom.global.or.b32 {em.tmp('b32')}, [thc_error], 1")   # gave up: add what arrived
        em.place(done)
        for r in range(MAX_PEERS):
            vf = em.tmp("f32")
            em.ins(f"and.pred {got[r]}, {got[r]}, {live[r]}")
            em.ins(f"mov.b32 {vf}, {los[r]}")
            em.ins(f"@{got[r]} add.rn.f32 {total}, {total}, {vf}")
        em.ins(f"st.shared.f32 [thc_peer_total], {total}")
        em.place(bar)
        em.ins("bar.sync 0")
        em.ins(f"ld.shared.f32 {acc}, [thc_peer_total]")
        em.place(skip)

    def _second_pass(self, cta: str, tid: str, nct: str) -> None:
        """Store the CTA's state; the last CTA to arrive folds all states in CTA order."""
        em, w, T = self.em, self.w, self.T
        S = len(self.states)
        tys = {s.name: dtype_of(s.dtype, "Accum") for s in self.l1.body if isinstance(s, ir.Accum)}
        ty = tys[self.states[0]]
        if any(tys[s] != ty for s in self.states):
            raise NotImplementedError("strided reduce with mixed state types")
        em.module(f".global .align 16 .b8 thc_partials[{MAX_PARTIALS * S * ty.nbytes}]")
        em.module(".global .align 4 .u32 thc_arrivals = 0")
        em.module(".shared .align 4 .u32 thc_is_last")
        parts, cnt = em.tmp("b64"), em.tmp("b64")
        em.ins(f"mov.u64 {parts}, thc_partials")
        em.ins(f"mov.u64 {cnt}, thc_arrivals")
        p = em.tmp("pred")
        skip = em.label("not_t0")
        em.ins(f"setp.ne.u32 {p}, {tid}, 0")
        em.ins(f"@{p} bra {skip}")
        slot = em.tmp("b64")
        em.ins(f"mad.wide.u32 {slot}, {cta}, {S * ty.nbytes}, {parts}")
        for i, s in enumerate(self.states):
            em.ins(f"st.global.cg.{ty.mov} [{slot}+{i * ty.nbytes}], {em.get(s)}")
        # the arrival is an acq_rel atomic: its release orders this thread's partial stores before
        # it, and the last CTA's acquire (then its barrier and fence) makes them visible to the fold
        old, lim, flag = em.tmp("b32"), em.tmp("b32"), em.tmp("b32")
        em.ins(f"sub.u32 {lim}, {nct}, 1")
        em.ins(f"atom.acq_rel.gpu.global.inc.u32 {old}, [{cnt}], {lim}")
        em.ins(f"setp.eq.u32 {p}, {old}, {lim}")
        em.ins(f"selp.u32 {flag}, 1, 0, {p}")
        em.ins(f"st.shared.u32 [thc_is_last], {flag}")
        em.place(skip)
        em.ins("bar.sync 0")
        em.ins(f"ld.shared.u32 {flag}, [thc_is_last]")
        em.ins(f"setp.eq.u32 {p}, {flag}, 0")
        em.ins(f"@{p} bra {self.exit}")
        em.ins("fence.acq_rel.gpu")
        # fold partials tid, tid+T, ... in order, starting from the identity
        idents = {s.name: s.op.identity for s in self.l1.body if isinstance(s, ir.Accum)}
        for s in self.states:
            em.ins(f"mov.{ty.mov} {em.get(s)}, {ty.imm(idents[s])}")
        sh = self.combine[0]
        i = em.tmp("b32")
        top, end = em.label("fold"), em.label("fold_end")
        em.ins(f"mov.u32 {i}, {tid}")
        em.ins(f"setp.ge.u32 {p}, {i}, {nct}")
        em.ins(f"@{p} bra {end}")
        em.place(top)
        a = em.tmp("b64")
        em.ins(f"mad.wide.u32 {a}, {i}, {S * ty.nbytes}, {parts}")
        for k, o in enumerate(sh.state_b):
            em.ins(f"ld.global.cg.{ty.mov} {em.value(o, ty.reg)}, [{a}+{k * ty.nbytes}]")
        for asg in sh.combine_states:
            w.stmt(asg)
        em.ins(f"add.u32 {i}, {i}, {T}")
        em.ins(f"setp.lt.u32 {p}, {i}, {nct}")
        em.ins(f"@{p} bra {top}")
        em.place(end)
        em.ins("bar.sync 0")           # shared slots of the first combine are reused
        w.body(self.combine)


def recognise(kernel: KernelInfo):
    return StridedReduce.match(kernel)
