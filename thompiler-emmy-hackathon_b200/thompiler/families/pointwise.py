"""Tuned family: pointwise kernels (p00-p03, x01, x02) with 128-bit loads and stores.

Recognised IR: one Tile whose body is straight-line Load / Assign / Let / Write over 1-D
buffers, each thread handling U consecutive elements -- the reference problems' unrolled
schedule, e.g. problems/p01_vector_add: ``x0[a0 * 2 + 0]``, ``x0[a0 * 2 + 1]`` loaded by two
statements, the sums written by one.  The generic lowering issues one 4-byte access per
statement; here the single-element Loads of a read-only buffer at ``X + 0 .. X + U-1`` become
one vector load (``ld.global.nc.v{V}``, V = min(U, 16 / element bytes), so a warp moves
whole 128-byte lines per instruction) issued at the first of them, and single-value Writes at
``X + 0 .. X + U-1`` one vector store issued at the last of them (every value is computed by
then).  The values, their order of computation and the IR's arithmetic are unchanged, so the
results are bit-identical to the generic lowering.

X must be ``a * m`` with m a multiple of V (so element X + jV sits on a V-element boundary);
the guard also checks at run time that every vectorised buffer's base pointer is aligned to
V elements, else the generic lowering of the same IR runs (a caller may pass an offset view).
"""

from __future__ import annotations

from thompiler import ir
from thompiler.families.base import TunedKernel
from thompiler.load import KernelInfo


def _split(index: tuple):
    """(X, k) for a 1-D index X + k (k a literal), X given as a hashable repr; else None."""
    if len(index) != 1:
        return None
    e = index[0]
    if isinstance(e, ir.BinaryExpr) and e.op == "+" and isinstance(e.right, ir.Literal) \
            and isinstance(e.right.value, int):
        return e.left, int(e.right.value)
    return e, 0


def _multiple_of(x, v: int) -> bool:
    """Is the index expression x always a multiple of v?"""
    if isinstance(x, ir.Literal) and isinstance(x.value, int):
        return x.value % v == 0
    if isinstance(x, ir.BinaryExpr) and x.op == "*":
        for a, b in ((x.left, x.right), (x.right, x.left)):
            if isinstance(b, ir.Literal) and isinstance(b.value, int) and b.value % v == 0:
                return True
    return False


class Pointwise(TunedKernel):
    family = "pointwise-vector"

    def __init__(self, kernel: KernelInfo, loads: dict, writes: dict, params: dict):
        super().__init__(kernel)
        self.loads, self.writes, self.vparams = loads, writes, params

    @classmethod
    def match(cls, kernel: KernelInfo):
        body = kernel.body
        if len(body) != 1 or not isinstance(body[0], ir.Tile) or len(body[0].axes) != 1:
            return None
        stmts = body[0].body
        if not all(isinstance(s, (ir.Load, ir.Assign, ir.Let, ir.Write)) for s in stmts):
            return None
        lgroups: dict = {}
        wgroups: dict = {}
        for i, s in enumerate(stmts):
            if isinstance(s, ir.Load) and len(s.names) == 1:
                p = kernel.param(s.input)
                xk = _split(s.index)
                if p is not None and not p.written and xk is not None:
                    lgroups.setdefault((s.input, repr(xk[0])), (xk[0], p, []))[2].append((xk[1], i, s))
            elif isinstance(s, ir.Write) and len(s.values) == 1 and not s.atomic:
                p = kernel.param(s.output)
                xk = _split(s.index)
                if p is not None and xk is not None:
                    wgroups.setdefault((s.output, repr(xk[0])), (xk[0], p, []))[2].append((xk[1], i, s))
        read = {s.input for s in stmts if isinstance(s, ir.Load)}
        wgroups = {key: g for key, g in wgroups.items() if key[0] not in read}   # no deferred store is re-read
        loads, writes, params = {}, {}, {}

        def plan(groups, out, first: bool) -> None:
            for (buf, _), (x, p, members) in groups.items():
                ks = sorted(k for k, _, _ in members)
                U = len(ks)
                V = min(U, 16 // p.ty.nbytes)
                if U < 2 or ks != list(range(U)) or U % V or V < 2 or not _multiple_of(x, V):
                    continue
                byk = {k: (i, s) for k, i, s in members}
                for j in range(0, U, V):
                    part = [byk[k] for k in range(j, j + V)]
                    at = min(i for i, _ in part) if first else max(i for i, _ in part)
                    out[at] = (p, x, j, [s for _, s in part])
                    for i, _ in part:
                        out.setdefault(i, None)          # a member served by the vector access
                params[p.name] = max(params.get(p.name, 1), V * p.ty.nbytes)

        plan(lgroups, loads, True)
        plan(wgroups, writes, False)
        if not params:
            return None
        k = cls(kernel, loads, writes, params)
        k.stmts = stmts
        return k

    def guard(self, generic: str) -> None:
        em = self.em
        p = em.tmp("pred")
        for name, align in sorted(self.vparams.items()):
            raw, low = em.tmp("b64"), em.tmp("b64")
            em.ins(f"ld.param.u64 {raw}, [p_{name}]")
            em.ins(f"and.b64 {low}, {raw}, {align - 1}")
            em.ins(f"setp.ne.u64 {p}, {low}, 0")
            em.ins(f"@{p} bra {generic}")

    def emit_tuned(self) -> None:
        from thompiler.lowering import address
        em, w = self.em, self.w
        self.pdl_trigger()
        self.pdl_wait()
        pos = {id(s): i for i, s in enumerate(self.stmts)}

        def load_hook(w_, load) -> bool:
            i = pos.get(id(load))
            if i is None or i not in self.loads:
                return False
            g = self.loads[i]
            if g is None:
                return True                              # loaded with its group
            p, x, j, members = g
            idx = (ir.BinaryExpr("+", x, ir.Literal(j, "int")),) if j else (x,)
            _, addr, ty, _ = address.access(w_, p.name, idx)
            regs = [em.value(s.names[0], ty.reg) for s in members]
            em.ins(f"ld.global.nc.v{len(regs)}.{ty.mov} {{{', '.join(regs)}}}, [{addr}]")
            return True

        def write_hook(w_, wr) -> bool:
            i = pos.get(id(wr))
            if i is None or i not in self.writes:
                return False
            g = self.writes[i]
            if g is None:
                return True                              # stored with its group
            p, x, j, members = g
            idx = (ir.BinaryExpr("+", x, ir.Literal(j, "int")),) if j else (x,)
            _, addr, ty, _ = address.access(w_, p.name, idx)
            vals = [em.get(s.values[0]) for s in members]
            em.ins(f"st.global.v{len(vals)}.{ty.mov} [{addr}], {{{', '.join(vals)}}}")
            return True

        w.load_hook, w.write_hook = load_hook, write_hook
        w.body(self.k.body)
        w.load_hook = w.write_hook = None


def recognise(kernel: KernelInfo):
    return Pointwise.match(kernel)
