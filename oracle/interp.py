"""Oracle: a CPU interpreter of Emmy Kernel IR (test infrastructure only).

It executes a KernelOp under a launch (grid x block threads) the way the
reference compiler's PTX executes it, vectorised over threads with numpy:
every statement runs for all threads in lock step under an active mask.
Lock-step execution is a valid schedule of these SPMD programs (their
cross-thread exchanges are barriers, shuffles and disjoint writes), so for
race-free kernels it computes what the GPU computes.

Semantics restated from the reference compiler (paths are the reference's):
  * Tile: gid = ctaid * ntid + tid, threads past N idle, row-major decode
    (thompiler/handlers/blocks.py:25-76);
  * loops seed their direct Accums with the op identity (blocks.py:132-145);
    StridedLoop runs start..end by step (blocks.py:92-108);
  * arithmetic in the value's IEEE type with round-to-nearest
    (lowering/ops.py:18-40); exp(x) = 2^(fl32(x * log2 e))
    (handlers/compute.py:77-83) -- ex2.approx is modelled by a correctly
    rounded exp2, within its 2-ulp bound; relu = max(x, 0);
  * WarpShuffle = XOR butterfly replaying combine_states (reduce.py:58-84);
    TreeHalve = shared tree with tid < step folding slot tid + step, then a
    broadcast read of the root (reduce.py:87-133);
  * cp.async / ldmatrix / mma.sync m16n8k16 / RegStore per the PTX ISA
    fragment layouts (handlers/cp_async.py, handlers/mma.py);
  * swizzle e ^ (((e >> s) & m) << 3) (lowering/address.py:115-150).

Every global and shared access is bounds-checked; an out-of-range access by
an active thread raises, which makes the interpreter a memory checker too.

The IR is read with the clean-room emmy stand-in in oracle/emmy_shim, not
with the product's reader, so a reader bug cannot hide on both sides.
"""

from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent / "emmy_shim"))

from emmy.compiler import _model as M  # noqa: E402

DT = {"f32": np.float32, "f16": np.float16, "f64": np.float64}
SMEM_DT = {"float": np.float32, "__half": np.float16, "double": np.float64}
LOG2_E32 = np.float32(math.log2(math.e))
SWZ = {"B128": (6, 7), "B64": (6, 3), "B32": (6, 1)}


class OracleError(RuntimeError):
    pass


def c_div(a, b):
    a = np.asarray(a, dtype=np.int64)
    b = np.asarray(b, dtype=np.int64)
    q = np.abs(a) // np.abs(b)
    return np.where((a >= 0) == (b >= 0), q, -q)


def swizzle(e, mode):
    if mode in (None, "NONE", ""):
        return e
    base, _, sh = mode.partition("@")
    shift, mask = SWZ[base]
    if sh:
        shift = int(sh)
    return e ^ (((e >> shift) & mask) << 3)


def _dtype_name(d):
    if d is None:
        return None
    return getattr(d, "name", d)


class Interp:
    def __init__(self, kernel_op, params: dict, grid: int, block: int, dyn_smem: int = 0):
        """params: buffer name -> numpy array (shape as in the IR); outputs are
        written in place."""
        self.k = kernel_op
        self.buf = params
        self.G, self.B = int(grid), int(block)
        self.T = self.G * self.B
        t = np.arange(self.T, dtype=np.int64)
        self.tid = t % self.B
        self.cta = t // self.B
        self.env: dict[str, np.ndarray] = {}
        self.consts: dict[str, int] = {}
        self.smem: dict[str, tuple[np.ndarray, tuple]] = {}
        self.frags: dict[str, dict] = {}
        self.env["lane"] = self.tid & 31
        self.env["warp"] = self.tid >> 5
        # lane index of each thread's XOR partner is computed per step
        self.base_of_warp = (t // 32) * 32

    # ---- values ----------------------------------------------------------

    def set(self, name, value, m):
        value = np.asarray(value)
        if value.shape == ():
            value = np.full(self.T, value, dtype=value.dtype)
        cur = self.env.get(name)
        if cur is None or cur.dtype != value.dtype:
            cur = np.zeros(self.T, dtype=value.dtype) if cur is None else cur.astype(value.dtype)
        cur = cur.copy()
        cur[m] = value[m]
        self.env[name] = cur

    def get(self, name):
        if name in self.consts:
            return np.full(self.T, self.consts[name], dtype=np.int64)
        if name not in self.env:
            raise OracleError(f"IR value {name!r} read before it is defined")
        return self.env[name]

    # ---- expressions -------------------------------------------------------

    def ival(self, e):
        if isinstance(e, (int, np.integer)) and not isinstance(e, bool):
            return np.full(self.T, int(e), dtype=np.int64)
        if isinstance(e, M.Var):
            return self.get(e.name).astype(np.int64)
        if isinstance(e, M.Literal):
            return np.full(self.T, int(e.value), dtype=np.int64)
        if isinstance(e, M.BinaryExpr):
            a, b = self.ival(e.left), self.ival(e.right)
            if e.op == "+":
                return a + b
            if e.op == "-":
                return a - b
            if e.op == "*":
                return a * b
            if e.op == "/":
                return c_div(a, np.where(b == 0, 1, b))
            if e.op == "%":
                bb = np.where(b == 0, 1, b)
                return a - c_div(a, bb) * bb
            raise OracleError(f"integer operator {e.op}")
        if isinstance(e, M.TernaryExpr):
            return np.where(self.pval(e.cond), self.ival(e.if_true), self.ival(e.if_false))
        raise OracleError(f"index expression {type(e).__name__}")

    def fval(self, e):
        if isinstance(e, M.Var):
            if e.name in self.consts or self.get(e.name).dtype.kind in "iu":
                return self.ival(e)
            return self.get(e.name)
        if isinstance(e, M.Literal):
            if e.dtype == "float":
                return np.full(self.T, float(e.value), dtype=np.float32)
            return np.full(self.T, int(e.value), dtype=np.int64)
        return self.ival(e)

    def pval(self, e):
        if isinstance(e, M.BinaryExpr) and e.op in ("&&", "||"):
            a, b = self.pval(e.left), self.pval(e.right)
            return (a & b) if e.op == "&&" else (a | b)
        if isinstance(e, M.BinaryExpr):
            a, b = self.fval(e.left), self.fval(e.right)
            return {"==": np.equal, "!=": np.not_equal, "<": np.less, "<=": np.less_equal,
                    ">": np.greater, ">=": np.greater_equal}[e.op](a, b)
        raise OracleError(f"condition {e!r}")

    # ---- memory -------------------------------------------------------------

    def flat(self, shape, index, m, what):
        if len(index) != len(shape):
            raise OracleError(f"{what}: {len(index)} indices for shape {shape}")
        f = np.zeros(self.T, dtype=np.int64)
        for size, e in zip(shape, index):
            i = self.ival(e)
            if np.any(m & ((i < 0) | (i >= size))):
                raise OracleError(f"{what}: index out of range for extent {size}")
            f = f * size + i
        return f

    def gather(self, name, index, width, m, swz="NONE"):
        if name in self.buf:
            arr = self.buf[name]
            flat = self.flat(arr.shape, index, m, name) if arr.ndim else np.zeros(self.T, np.int64)
            src = arr.reshape(-1)
            outs = []
            for k in range(width):
                i = flat + k
                if np.any(m & (i >= src.size)):
                    raise OracleError(f"load past the end of {name}")
                outs.append(src[np.where(m, i, 0)])
            return outs
        if name in self.smem:
            arr, ext = self.smem[name]
            flat = self.flat(ext, index, m, name)
            outs = []
            for k in range(width):
                i = swizzle(flat + k, swz)
                if np.any(m & (i >= arr.shape[1])):
                    raise OracleError(f"shared load past the end of {name}")
                outs.append(arr[self.cta, np.where(m, i, 0)])
            return outs
        raise OracleError(f"{name!r} is neither a parameter nor an Smem array")

    def scatter(self, name, index, values, m, atomic=False, swz="NONE"):
        if name in self.buf:
            arr = self.buf[name]
            flat = self.flat(arr.shape, index, m, name) if arr.ndim else np.zeros(self.T, np.int64)
            dst = arr.reshape(-1)
            for k, v in enumerate(values):
                i = (flat + k)[m]
                if np.any(i >= dst.size):
                    raise OracleError(f"store past the end of {name}")
                if atomic:
                    np.add.at(dst, i, v[m].astype(dst.dtype))
                else:
                    dst[i] = v[m].astype(dst.dtype)
            return
        if name in self.smem:
            arr, ext = self.smem[name]
            flat = self.flat(ext, index, m, name)
            for k, v in enumerate(values):
                i = swizzle(flat + k, swz)[m]
                if np.any(i >= arr.shape[1]):
                    raise OracleError(f"shared store past the end of {name}")
                arr[self.cta[m], i] = v[m].astype(arr.dtype)
            return
        raise OracleError(f"{name!r} is neither a parameter nor an Smem array")

    # ---- arithmetic ----------------------------------------------------------

    def apply(self, op, args, dtype):
        x = args[0]
        dt = np.dtype(dtype)
        if op == "copy":
            return x.astype(dt)
        if dt == np.float16 and op not in ("copy",):
            # f16 arithmetic through f32 (one rounding back)
            return self.apply(op, [a.astype(np.float32) for a in args], np.float32).astype(np.float16)
        with np.errstate(all="ignore"):
            if op == "add":
                return (args[0] + args[1]).astype(dt)
            if op == "subtract":
                return (args[0] - args[1]).astype(dt)
            if op == "multiply":
                return (args[0] * args[1]).astype(dt)
            if op == "divide":
                return (args[0] / args[1]).astype(dt)
            if op == "maximum":
                return np.fmax(args[0], args[1]).astype(dt)
            if op == "minimum":
                return np.fmin(args[0], args[1]).astype(dt)
            if op == "relu":
                return np.fmax(x, dt.type(0)).astype(dt)
            if op == "sqrt":
                return np.sqrt(x).astype(dt)
            if op == "reciprocal":
                return (dt.type(1) / x).astype(dt)
            if op == "negative":
                return (-x).astype(dt)
            if op == "abs":
                return np.abs(x).astype(dt)
            if op == "exp":
                if dt != np.float32:
                    raise OracleError("exp on non-f32 values")
                t = (x * LOG2_E32).astype(np.float32)
                return np.exp2(t.astype(np.float64)).astype(np.float32)
            if op == "rsqrt":
                return (1.0 / np.sqrt(x.astype(np.float64))).astype(dt)
            if op in ("tanh", "sin", "cos"):
                return getattr(np, op)(x.astype(np.float64)).astype(dt)
        raise OracleError(f"operation {op!r}")

    # ---- statements ------------------------------------------------------------

    def run(self):
        m = np.ones(self.T, dtype=bool)
        self.body(self.k.body, m)

    def body(self, stmts, m):
        for s in stmts:
            getattr(self, "s_" + type(s).__name__)(s, m)

    def s_Tile(self, s, m):
        if s.aux_threads:
            raise OracleError("aux_threads")
        gid = self.cta * self.B + self.tid
        n = s.n_elements
        m = m & (gid < n)
        ext = s.extents
        for i, ax in enumerate(s.axes):
            stride = math.prod(ext[i + 1:])
            v = gid // stride
            if i:
                v = v % ext[i]
            self.set(ax.name, v, m)
        self.body(s.body, m)

    def _seed(self, body, m):
        for st in body:
            if isinstance(st, M.Accum):
                dt = DT[_dtype_name(st.dtype) or "f32"]
                self.set(st.name, np.full(self.T, st.op.identity, dtype=dt), m)

    def _frag_loop(self, var, body):
        return _indexes_fragment(var, body)

    def s_Loop(self, s, m):
        if s.seed:
            self._seed(s.body, m)
        n = s.axis.extent.as_static()
        unroll = self._frag_loop(s.axis.name, s.body)
        for v in range(n):
            if unroll:
                self.consts[s.axis.name] = v
            else:
                self.set(s.axis.name, np.full(self.T, v, np.int64), m)
            self.body(s.body, m)
        self.consts.pop(s.axis.name, None)

    def s_StridedLoop(self, s, m):
        if s.seed:
            self._seed(s.body, m)
        start = self.ival(s.start)
        end = self.ival(s.end) if s.end is not None else np.full(self.T, s.axis.extent.as_static(), np.int64)
        step = self.ival(s.step) if not isinstance(s.step, int) else np.full(self.T, s.step, np.int64)
        unroll = self._frag_loop(s.axis.name, s.body)
        if unroll:
            a, b, c = int(start[0]), int(end[0]), int(step[0])
            for v in range(a, b, c):
                self.consts[s.axis.name] = v
                self.body(s.body, m)
            self.consts.pop(s.axis.name, None)
            return
        var = start.copy()
        while True:
            act = m & (var < end)
            if not act.any():
                break
            self.set(s.axis.name, var, act)
            self.body(s.body, act)
            var = var + step

    def s_Cond(self, s, m):
        p = self.pval(s.cond)
        self.body(s.body, m & p)
        if s.else_body:
            self.body(s.else_body, m & ~p)

    def s_Load(self, s, m):
        vals = self.gather(s.input, s.index, len(s.names), m)
        for n, v in zip(s.names, vals):
            self.set(n, v, m)

    def s_Assign(self, s, m):
        args = [self.get(a) for a in s.args]
        dt = DT[_dtype_name(s.dtype)] if s.dtype is not None else args[0].dtype
        if s.op.name == "copy" or np.dtype(dt) == args[0].dtype:
            val = self.apply(s.op.name, args, dt)
        else:
            raise OracleError(f"{s.op.name} changes dtype")
        self.set(s.name, val, m)

    def s_Let(self, s, m):
        if isinstance(s.value, M.Literal) and s.value.dtype == "float":
            dt = DT[_dtype_name(s.dtype) or "f32"]
            self.set(s.name, np.full(self.T, float(s.value.value), dtype=dt), m)
        else:
            self.set(s.name, self.ival(s.value), m)

    def s_Accum(self, s, m):
        base = self.get(s.base) if s.base is not None else self.get(s.name)
        val = self.get(s.value)
        self.set(s.name, self.apply(s.op.name, [base, val], base.dtype), m)

    def s_Init(self, s, m):
        dt = DT[_dtype_name(s.dtype) or "f32"]
        self.set(s.name, np.full(self.T, s.identity, dtype=dt), m)

    def s_Write(self, s, m):
        vals = [self.get(v) for v in s.values]
        self.scatter(s.output, s.index, vals, m, atomic=s.atomic, swz=s.swizzle)

    def _combine(self, states, partners, combine, partner_idx, m):
        for st, o in zip(states, partners):
            v = self.get(st)
            self.set(o, v[partner_idx], m)
        for a in combine:
            self.s_Assign(a, m)

    def s_WarpShuffle(self, s, m):
        step = int(s.length) // 2
        t = np.arange(self.T)
        while step:
            self._combine(s.state, s.state_b, s.combine_states, self.base_of_warp + ((t & 31) ^ step), m)
            step //= 2

    def s_TreeHalve(self, s, m):
        tid = self.get(s.tid_var).astype(np.int64)

        def slot(i):
            if s.inner is None:
                return i
            var, scale = s.inner
            return i * int(scale) + self.get(var).astype(np.int64)

        step = int(s.length) // 2
        while step:
            act = m & (tid < step)
            for buf, st, o in zip(s.bufs, s.state, s.state_b):
                arr, _ = self.smem[buf]
                self.set(st, arr[self.cta, np.where(act, slot(tid), 0)], act)
                self.set(o, arr[self.cta, np.where(act, slot(tid + step), 0)], act)
            for a in s.combine_states:
                self.s_Assign(a, act)
            for buf, st in zip(s.bufs, s.state):
                arr, _ = self.smem[buf]
                arr[self.cta[act], slot(tid)[act]] = self.get(st)[act]
            step //= 2
        root = self.get(s.inner[0]).astype(np.int64) if s.inner is not None else np.zeros(self.T, np.int64)
        for buf, st in zip(s.bufs, s.state):
            arr, _ = self.smem[buf]
            self.set(st, arr[self.cta, root], m)

    def s_Smem(self, s, m):
        if s.name in self.smem:
            return
        ext = tuple(int(e) for e in s.extents)
        self.smem[s.name] = (np.zeros((self.G, math.prod(ext)), dtype=SMEM_DT[s.dtype]), ext)

    def s_Sync(self, s, m):
        pass

    def s_CpAsyncCommit(self, s, m):
        pass

    def s_CpAsyncWait(self, s, m):
        pass

    def s_CpAsyncCopy(self, s, m):
        arr, ext = self.smem[s.smem]
        src = self.buf[s.src]
        n = int(s.nbytes) // src.dtype.itemsize
        e = self.flat(ext, s.smem_index, m, s.smem)
        if s.lane_index is not None:
            r, c = s.lane_index
            e = e + self.ival(r) * ext[-1] + self.ival(c)
        g = self.flat(src.shape, s.src_index, m, s.src)
        flat_src = src.reshape(-1)
        for k in range(n):
            d = swizzle(e + k, s.swizzle)
            arr[self.cta[m], d[m]] = flat_src[(g + k)[m]]

    # ---- tensor-core fragments -------------------------------------------------

    def s_RegFragment(self, s, m):
        dt = _dtype_name(s.dtype)
        mm, nn, kk = s.shape
        if s.role == "a":
            nregs = mm * kk // 64
        elif s.role == "b":
            nregs = kk * nn // 64
        else:
            nregs = mm * nn // (64 if dt == "f16" else 32)
        self.frags[s.name] = dict(role=s.role, dtype=dt, regs=np.zeros((int(s.count), self.T, nregs),
                                  dtype=np.float32 if (s.role == "c" and dt == "f32") else np.uint32))

    def _frag(self, ref):
        name, _, idx = ref.partition("[")
        f = self.frags[name]
        member = 0
        if idx:
            member = int(eval(idx.rstrip("]"), {"__builtins__": {}}, dict(self.consts)))  # noqa: S307
        return f, member

    @staticmethod
    def _pack(lo, hi):
        return (lo.astype(np.float16).view(np.uint16).astype(np.uint32)
                | (hi.astype(np.float16).view(np.uint16).astype(np.uint32) << 16))

    @staticmethod
    def _unpack(r):
        lo = (r & 0xFFFF).astype(np.uint16).view(np.float16)
        hi = (r >> 16).astype(np.uint16).view(np.float16)
        return lo, hi

    def s_LdmatrixLoad(self, s, m):
        arr, ext = self.smem[s.src_buffer]
        f, mem = self._frag(s.frag)
        regs = [(f, mem, i) for i in range(f["regs"].shape[2])]
        if s.pair_frag is not None:
            f2, mem2 = self._frag(s.pair_frag)
            regs += [(f2, mem2, i) for i in range(f2["regs"].shape[2])]
        ldm = int(s.ldm) or ext[-1]
        lane = self.tid & 31
        pair = s.pair_frag is not None
        if s.role == "a" or not s.b_trans:
            row = lane % 16
        elif pair:
            row = lane % 8 + (lane // 16) * 8
        else:
            row = lane % 8
        if s.role == "a" or (pair and not s.b_trans):
            col = (lane // 16) * 8
        elif s.b_trans:
            col = ((lane // 8) % 2) * 8
        else:
            col = 0
        nmat = 4 if (s.role == "a" or pair) else 2
        trans = s.role == "b" and not s.b_trans
        base = self.flat(ext, s.src_index, m, s.src_buffer)
        rowstart = swizzle(base + row * ldm + col, s.swizzle)      # per lane: start of its 8-element row
        # matrix i, row r (0..7) comes from lane 8i + r of the same warp
        t = np.arange(self.T)
        wb = self.base_of_warp
        for i in range(nmat):
            # element (r, c) of matrix i for this thread's requested slots
            g, q = (t & 31) // 4, (t & 31) % 4
            if not trans:
                src_lane = wb + 8 * i + g
                e0 = rowstart[src_lane] + 2 * q
                vals = (arr[self.cta, e0], arr[self.cta, e0 + 1])
            else:
                s0 = wb + 8 * i + 2 * q
                s1 = s0 + 1
                vals = (arr[self.cta, rowstart[s0] + g], arr[self.cta, rowstart[s1] + g])
            ff, mm_, ri = regs[i]
            packed = self._pack(vals[0], vals[1])
            ff["regs"][mm_, m, ri] = packed[m]

    def s_MmaSyncPtx(self, s, m):
        fc, mc = self._frag(s.c_frag)
        fa, ma = self._frag(s.a_frag)
        fb, mb = self._frag(s.b_frag)
        W = self.T // 32
        lane = np.arange(32)
        g, q = lane // 4, lane % 4
        ar = fa["regs"][ma].reshape(W, 32, 4)
        br = fb["regs"][mb].reshape(W, 32, 2)
        A = np.zeros((W, 16, 16), np.float64)
        Bm = np.zeros((W, 16, 8), np.float64)
        for r in range(4):
            lo, hi = self._unpack(ar[:, :, r])
            rr = g + (8 if r % 2 else 0)
            cc = 2 * q + (8 if r >= 2 else 0)
            A[:, rr, cc] = lo
            A[:, rr, cc + 1] = hi
        for r in range(2):
            lo, hi = self._unpack(br[:, :, r])
            kk = 2 * q + (8 if r else 0)
            Bm[:, kk, g] = lo
            Bm[:, kk + 1, g] = hi
        if fc["dtype"] == "f32":
            cr = fc["regs"][mc].reshape(W, 32, 4)
            C = np.zeros((W, 16, 8), np.float64)
            for r in range(4):
                rr = g + (8 if r >= 2 else 0)
                C[:, rr, 2 * q + (r % 2)] = cr[:, :, r]
            D = (C + np.einsum("wmk,wkn->wmn", A, Bm)).astype(np.float32)
            out = np.zeros((W, 32, 4), np.float32)
            for r in range(4):
                rr = g + (8 if r >= 2 else 0)
                out[:, :, r] = D[:, rr, 2 * q + (r % 2)]
            flat = out.reshape(self.T, 4)
            fc["regs"][mc][m] = flat[m]
        else:
            raise OracleError("f16 accumulator fragments")

    def s_RegStore(self, s, m):
        """C registers 0, 1 at row g, columns 2q, 2q + 1 and 2, 3 at row g + 8 (g = lane / 4,
        q = lane % 4), stored from the fragment's origin ``dst_index``.  The fused forms of the
        IR reference (TASK.md:157-160): an ``epilogue`` Lambda applied per element, its leading
        parameters bound to the element of ``frag`` and of each of ``extra_frags``, two more
        (when declared) to the element's destination row and column, its one result stored in
        the buffer's type; ``m_guard`` / ``n_guard`` exclusive bounds on that row and column;
        ``atomic`` adds instead of storing."""
        if (s.fragment_layout not in (None, "m16n8k16") or s.volta_interleaved
                or s.swizzle not in (None, "NONE")):
            raise OracleError("RegStore layout")
        f, mem = self._frag(s.frag)
        extra = [self._frag(r) for r in (s.extra_frags or ())]
        dst = self.buf[s.dst_buffer]
        index = list(s.dst_index)
        rd = len(index) - 2 if s.row_dim is None else int(s.row_dim)
        cd = len(index) - 1 if s.col_dim is None else int(s.col_dim)
        lane = self.tid & 31
        g, q = lane // 4, lane % 4
        regs = f["regs"][mem]
        d = dst.reshape(-1)
        for dr, pair in ((0, (0, 1)), (8, (2, 3))):
            for j, reg in enumerate(pair):
                idx = [self.ival(e) for e in index]
                row, col = idx[rd] + g + dr, idx[cd] + 2 * q + j
                idx[rd], idx[cd] = row, col
                v = regs[:, reg]
                if s.epilogue is not None:
                    v = self._epilogue(s.epilogue, [v] + [ef["regs"][em][:, reg] for ef, em in extra], row, col, m)
                ok = m.copy()
                if s.m_guard is not None:
                    ok &= row < self.ival(s.m_guard)
                if s.n_guard is not None:
                    ok &= col < self.ival(s.n_guard)
                flat = np.zeros(self.T, np.int64)
                for size, i in zip(dst.shape, idx):
                    if np.any(ok & ((i < 0) | (i >= size))):
                        raise OracleError(f"RegStore to {s.dst_buffer}: index out of range for extent {size}")
                    flat = flat * size + i
                if s.atomic:
                    np.add.at(d, flat[ok], v[ok].astype(dst.dtype))
                else:
                    d[flat[ok]] = v[ok].astype(dst.dtype)

    def _epilogue(self, lam, elems, row, col, m):
        params = [p.name if isinstance(p, M.Var) else p for p in lam.params]
        if len(params) not in (len(elems), len(elems) + 2):
            raise OracleError(f"epilogue of {len(params)} parameters for {len(elems)} fragments")
        for name, v in zip(params, elems):
            self.set(name, v.astype(np.float32), m)
        if len(params) == len(elems) + 2:
            self.set(params[-2], row, m)
            self.set(params[-1], col, m)
        self.body(lam.body, m)
        (res,) = lam.results
        return self.get(res).copy()

    def s_Select(self, s, m):
        """``name`` = the value of the first branch whose predicate holds, else the last's."""
        def value(v):
            if isinstance(v, str):
                return self.get(v)
            return self.fval(v)
        arms = [(value(b.value), None if b.select is None else self.pval(b.select)) for b in s.branches]
        out = arms[-1][0]
        for v, p in reversed(arms[:-1]):
            out = v if p is None else np.where(p, v, out)
        self.set(s.name, out, m)


def _indexes_fragment(var, node):
    import re
    if isinstance(node, str):
        mm = re.match(r"^(\w+)\[([^\]]+)\]$", node)
        return bool(mm and re.search(rf"\b{re.escape(var)}\b", mm.group(2)))
    if isinstance(node, tuple):
        return any(_indexes_fragment(var, x) for x in node)
    if hasattr(node, "__dataclass_fields__"):
        return any(_indexes_fragment(var, getattr(node, f)) for f in node.__dataclass_fields__)
    return False


# ---------------------------------------------------------------------------
# problem packages


def seeded(shape, seed, dtype):
    """The runner's seeded input: default_rng(seed).standard_normal (docs/API.md:46)."""
    return np.random.default_rng(seed).standard_normal(list(shape) or [1]).astype(DT[dtype])


def run_package(pdir: Path, inputs: dict | None = None) -> dict:
    """Interpret every kernel of a problem package in meta.json order; returns
    every buffer produced (outputs and intermediates) as numpy arrays."""
    pdir = Path(pdir)
    meta = json.loads((pdir / "meta.json").read_text())
    produced: dict[str, np.ndarray] = {}
    for k in meta["kernels"]:
        graph = M.Graph.from_dict(json.loads((pdir / f"{k['entry']}.ir.json").read_text()))
        kop = next(n.op for n in graph.nodes.values() if isinstance(n.op, M.KernelOp))
        params = {}
        for a in k["args"]:
            t = graph.buffer(a["name"])
            shape = tuple(d.as_static() for d in t.shape)
            dt = DT[a["dtype"]]
            if a.get("output"):
                params[a["name"]] = np.zeros(shape, dtype=dt)
            elif a.get("intermediate"):
                params[a["name"]] = produced[a["name"]].reshape(shape).astype(dt)
            elif "data" in a:
                params[a["name"]] = np.asarray(a["data"], dtype=dt).reshape(shape)
            else:
                if inputs is not None and a["name"] in inputs:
                    params[a["name"]] = np.asarray(inputs[a["name"]], dtype=dt).reshape(shape)
                elif "init" in a:
                    ini = a["init"]
                    rng = np.random.default_rng(ini.get("seed", a.get("seed", 0)))
                    if ini["dist"] == "uniform":
                        v = rng.uniform(ini.get("low", 0.0), ini.get("high", 1.0), list(shape) or [1])
                    elif ini["dist"] == "integers":        # low..high inclusive
                        v = rng.integers(ini.get("low", -2), ini.get("high", 2) + 1, list(shape) or [1])
                    else:
                        v = rng.standard_normal(list(shape) or [1]) * ini.get("std", 1.0) + ini.get("mean", 0.0)
                    params[a["name"]] = v.astype(dt).reshape(shape)
                else:
                    params[a["name"]] = seeded(shape, a["seed"], a["dtype"]).reshape(shape)
        for name in k.get("zero_outputs", []):
            params[name][...] = 0
        Interp(kop, params, int(np.prod(k["grid"])), int(np.prod(k["block"])), k.get("smem_bytes", 0)).run()
        for a in k["args"]:
            if a.get("output"):
                produced[a["name"]] = params[a["name"]]
    return produced
