"""Emmy Kernel IR, read without emmy.

A Kernel IR file stores each KernelOp body as the Python ``repr`` of emmy's
statement dataclasses, e.g. ``Tile(axes=(Axis(name='a0', extent=Dim(64),
window=None),), body=(...), block_threads=128, ...)``.  emmy-ml is not a
dependency of this compiler, so this module gives every constructor of that
vocabulary a frozen dataclass of its own and rebuilds the tree from the
string with ``ast`` -- never ``eval``: only whitelisted constructor names,
literals, tuples and lists are accepted.

A constructor this module does not know becomes an ``Opaque`` node that keeps
its name and fields, so reading never fails on new vocabulary; the walker
rejects it with ``NotImplementedError`` when it reaches it, which is where
the reference compiler fails too (thompiler/walk.py:48-52 of the reference).

Field names and meanings follow the IR reference table in the reference's
TASK.md:89-185; the reader itself is this project's own.
"""

from __future__ import annotations

import ast
import dataclasses
from dataclasses import dataclass, field
from typing import Any


# ---------------------------------------------------------------------------
# leaf values


@dataclass(frozen=True)
class DataType:
    """An element type: ``name`` is the IR dtype ("f32", "f16", "f64", ...)."""
    name: str
    np: Any = None
    nbytes: int = 0


@dataclass(frozen=True)
class Dim:
    value: Any

    @property
    def is_static(self) -> bool:
        return isinstance(self.value, int)

    def as_static(self) -> int:
        if not self.is_static:
            raise NotImplementedError(f"dimension {self.value!r} is not static")
        return int(self.value)


@dataclass(frozen=True)
class Window:
    parent: Any = None
    base: Any = None
    bound: Any = None
    partition: bool = False


@dataclass(frozen=True)
class Axis:
    name: str
    extent: Dim
    window: Window | None = None

    @property
    def size(self) -> int:
        return self.extent.as_static()


# Elementwise operation name -> (arity, identity of the fold, or None).
# Identities are the accumulator seeds: 0 for add, 1 for multiply, and the
# finite -1e30 / 1e30 for maximum / minimum (emmy's generated CUDA seeds a
# max with -1e+30f, problems/f02_row_softmax/k_softmax_05263d.ref.cu:9), so
# online-softmax rescales exp(seed - x) to 0 instead of exp(-inf + inf) = NaN.
ELEMENTWISE: dict[str, tuple[int, float | None]] = {
    "add": (2, 0.0), "subtract": (2, None), "multiply": (2, 1.0), "divide": (2, None),
    "maximum": (2, -1e30), "minimum": (2, 1e30), "mod": (2, None),
    "copy": (1, None), "exp": (1, None), "reciprocal": (1, None), "relu": (1, None),
    "sqrt": (1, None), "rsqrt": (1, None), "negative": (1, None), "abs": (1, None),
    "tanh": (1, None), "sin": (1, None), "cos": (1, None), "log": (1, None),
    "sigmoid": (1, None),
}


@dataclass(frozen=True)
class ElementwiseImpl:
    name: str

    @property
    def arity(self) -> int:
        if self.name not in ELEMENTWISE:
            raise NotImplementedError(f"elementwise operation {self.name!r}")
        return ELEMENTWISE[self.name][0]

    @property
    def identity(self) -> float | None:
        return ELEMENTWISE.get(self.name, (0, None))[1]


# ---------------------------------------------------------------------------
# expressions


class Expr:
    def pretty(self) -> str:  # pragma: no cover - overridden
        return repr(self)


@dataclass(frozen=True)
class Var(Expr):
    name: str

    def pretty(self) -> str:
        return self.name


@dataclass(frozen=True)
class Literal(Expr):
    value: Any
    dtype: str = "int"

    def pretty(self) -> str:
        return repr(self.value)


@dataclass(frozen=True)
class BinaryExpr(Expr):
    op: str
    left: Any
    right: Any

    def pretty(self) -> str:
        return f"({pretty(self.left)} {self.op} {pretty(self.right)})"


@dataclass(frozen=True)
class TernaryExpr(Expr):
    cond: Any
    if_true: Any
    if_false: Any

    def pretty(self) -> str:
        return f"({pretty(self.cond)} ? {pretty(self.if_true)} : {pretty(self.if_false)})"


@dataclass(frozen=True)
class Builtin(Expr):
    name: str


@dataclass(frozen=True)
class FuncCallExpr(Expr):
    name: str
    args: tuple = ()


@dataclass(frozen=True)
class CastExpr(Expr):
    dtype: Any
    expr: Any


@dataclass(frozen=True)
class FlatIndex(Expr):
    buffer: str
    index: tuple = ()


def pretty(e: Any) -> str:
    """A short one-line text of an expression or value (for PTX comments)."""
    if isinstance(e, Expr):
        return e.pretty()
    if isinstance(e, tuple):
        return ", ".join(pretty(x) for x in e)
    return str(e)


# ---------------------------------------------------------------------------
# statements


class Stmt:
    """Base of every statement; ``pretty`` is a one-line summary for comments."""

    def pretty(self) -> str:
        names = [f.name for f in dataclasses.fields(self)][:3]  # type: ignore[arg-type]
        return f"{type(self).__name__}(" + ", ".join(
            f"{n}={_short(getattr(self, n))}" for n in names) + ")"


def _short(v: Any) -> str:
    text = pretty(v) if not isinstance(v, (str, int, float)) else repr(v)
    return text if len(text) < 60 else text[:57] + "..."


@dataclass(frozen=True)
class Tile(Stmt):
    axes: tuple
    body: tuple
    block_threads: int = 0
    aux_threads: int = 0
    raster_axes: Any = None
    raster_group: Any = None
    raster_orient: str = "m"

    @property
    def extents(self) -> tuple[int, ...]:
        return tuple(a.size for a in self.axes)

    @property
    def n_elements(self) -> int:
        n = 1
        for e in self.extents:
            n *= e
        return n

    def pretty(self) -> str:
        return f"Tile[{', '.join(a.name for a in self.axes)}] (N={self.n_elements})"


@dataclass(frozen=True)
class Loop(Stmt):
    axis: Axis
    body: tuple
    unroll: Any = False
    seed: bool = False
    carries: tuple = ()

    def pretty(self) -> str:
        return f"for {self.axis.name} in 0..{pretty(self.axis.extent.value)}"


@dataclass(frozen=True)
class StridedLoop(Stmt):
    axis: Axis
    start: Any
    step: Any
    body: tuple
    unroll: Any = False
    end: Any = None
    seed: bool = False

    def pretty(self) -> str:
        end = pretty(self.end) if self.end is not None else pretty(self.axis.extent.value)
        return f"for {self.axis.name} in {pretty(self.start)}..{end}:{pretty(self.step)}"


@dataclass(frozen=True)
class Cond(Stmt):
    cond: Any
    body: tuple
    else_body: tuple = ()

    def pretty(self) -> str:
        return f"if {pretty(self.cond)}"


@dataclass(frozen=True)
class Load(Stmt):
    names: tuple
    input: str
    index: tuple
    dtype: Any = None

    def pretty(self) -> str:
        return f"{', '.join(self.names)} = load {self.input}[{pretty(self.index)}]"


@dataclass(frozen=True)
class Assign(Stmt):
    name: str
    op: ElementwiseImpl
    args: tuple
    dtype: Any = None

    def pretty(self) -> str:
        return f"{self.name} = {self.op.name}({', '.join(self.args)})"


@dataclass(frozen=True)
class Let(Stmt):
    name: str
    value: Any
    dtype: Any = None

    def pretty(self) -> str:
        return f"{self.name} = {pretty(self.value)}"


@dataclass(frozen=True)
class Accum(Stmt):
    name: str
    value: str
    op: ElementwiseImpl
    dtype: Any = None
    axes: tuple = ()
    base: Any = None

    def pretty(self) -> str:
        return f"{self.name} <- {self.op.name}({self.base or self.name}, {self.value})"


@dataclass(frozen=True)
class Init(Stmt):
    name: str
    identity: Any
    dtype: Any = None

    def pretty(self) -> str:
        return f"Init({self.name} = {self.identity})"


@dataclass(frozen=True)
class Write(Stmt):
    output: str
    index: tuple
    values: tuple
    value_dtype: Any = None
    atomic: bool = False
    swizzle: str = "NONE"

    def pretty(self) -> str:
        op = "+=" if self.atomic else "="
        return f"{self.output}[{pretty(self.index)}] {op} ({', '.join(self.values)})"


@dataclass(frozen=True)
class WarpShuffle(Stmt):
    state: tuple
    state_b: tuple
    combine_states: tuple
    length: int = 32
    dtype: Any = None

    def pretty(self) -> str:
        return f"WarpShuffle({', '.join(self.state)}, length={self.length})"


@dataclass(frozen=True)
class TreeHalve(Stmt):
    bufs: tuple
    state: tuple
    state_b: tuple
    combine_states: tuple
    length: int
    tid_var: str
    dtype: Any = None
    barrier_id: int = 0
    barrier_count: Any = None
    inner: Any = None

    def pretty(self) -> str:
        return f"TreeHalve({', '.join(self.state)}, length={self.length}, tid={self.tid_var})"


@dataclass(frozen=True)
class Smem(Stmt):
    name: str
    extents: tuple
    dtype: str
    align: int = 0

    def pretty(self) -> str:
        dims = "".join(f"[{e}]" for e in self.extents)
        return f"Smem {self.dtype} {self.name}{dims} align={self.align}"


@dataclass(frozen=True)
class Sync(Stmt):
    barrier_id: int = 0
    count: Any = None
    warp: bool = False

    def pretty(self) -> str:
        return "SyncWarp" if self.warp else f"Sync(id={self.barrier_id}, count={self.count})"


@dataclass(frozen=True)
class CpAsyncCopy(Stmt):
    smem: str
    smem_index: tuple
    src: str
    src_index: tuple
    nbytes: int
    swizzle: str = "NONE"
    lane_index: Any = None
    lane_rows: Any = None

    def pretty(self) -> str:
        return f"cp.async[{self.nbytes}B] {self.smem}[{pretty(self.smem_index)}] <- {self.src}[...]"


@dataclass(frozen=True)
class CpAsyncCommit(Stmt):
    pass


@dataclass(frozen=True)
class CpAsyncWait(Stmt):
    group: int = 0


@dataclass(frozen=True)
class RegFragment(Stmt):
    name: str
    role: str
    shape: tuple
    dtype: Any
    count: int = 1
    nregs: Any = None


@dataclass(frozen=True)
class LdmatrixLoad(Stmt):
    frag: str
    src_buffer: str
    src_index: tuple
    role: str
    ldm: int = 0
    swizzle: str = "NONE"
    staged: bool = True
    gmem_guard: Any = None
    k_zero: Any = None
    b_trans: bool = False
    pair_frag: Any = None
    byte_slab: bool = False
    scale_buffer: Any = None
    scale_index: tuple = ()
    scale_ldm: int = 0
    fragment_layout: str = "m16n8k16"
    fragment_index: Any = None


@dataclass(frozen=True)
class MmaSyncPtx(Stmt):
    c_frag: str
    a_frag: str
    b_frag: str
    shape: tuple
    ab_dtype: str
    c_dtype: str
    b_row_major: bool = False
    sfa_frag: Any = None
    sfb_frag: Any = None

    @property
    def block_scaled(self) -> bool:
        return self.sfa_frag is not None


@dataclass(frozen=True)
class RegStore(Stmt):
    dst_buffer: str
    dst_index: tuple
    frag: str
    shape: tuple
    ldm: int = 0
    epilogue: Any = None
    extra_frags: tuple = ()
    m_guard: Any = None
    n_guard: Any = None
    atomic: bool = False
    fragment_layout: str = "m16n8k16"
    volta_interleaved: bool = False
    fragment_index: Any = None
    swizzle: str = "NONE"
    row_dim: Any = None
    col_dim: Any = None


# Statements of the IR reference that the reference compiler does not lower (the entries marked
# * in its TASK.md:95-180) and no shipped kernel uses.  Field names follow that table; the
# handlers in thompiler/handlers/async_copy.py and compute.py lower the TMA / mbarrier /
# register-budget subset, Select and ZeroPrologue onto sm_100a, handlers/wgmma.py the
# warpgroup tensor-core statements (Wgmma*) onto tcgen05, handlers/fragments.py the register
# fragment operations (Fragment*).


@dataclass(frozen=True)
class Branch:
    """One arm of a Select: ``value`` when ``select`` (a coordinate predicate; None = otherwise)."""
    value: Any
    select: Any = None


@dataclass(frozen=True)
class Select(Stmt):
    name: str
    branches: tuple = ()


@dataclass(frozen=True)
class Pre(Stmt):
    name: str
    carrier: str = ""
    index: tuple = ()


@dataclass(frozen=True)
class Carry(Stmt):
    name: str
    value: Any = None
    index: tuple = ()
    seed: Any = None
    dtype: Any = None


@dataclass(frozen=True)
class ZeroPrologue(Stmt):
    dst: str
    words: Any = 0


@dataclass(frozen=True)
class TmaDescriptor(Stmt):
    name: str
    src_buf: str = ""
    src_shape: tuple = ()
    box_extents: tuple = ()
    swizzle: Any = None
    dtype: Any = None


@dataclass(frozen=True)
class TmaLoad(Stmt):
    smem: str
    smem_index: tuple = ()
    desc: str = ""
    coords: tuple = ()
    mbar: str = ""
    mbar_slot: Any = None


@dataclass(frozen=True)
class MbarrierInit(Stmt):
    mbar: str
    count: Any = 1
    slot: Any = None


@dataclass(frozen=True)
class MbarrierArriveExpectTx(Stmt):
    mbar: str
    bytes_: Any = 0
    slot: Any = None


@dataclass(frozen=True)
class MbarrierArrive(Stmt):
    mbar: str
    slot: Any = None


@dataclass(frozen=True)
class MbarrierWait(Stmt):
    mbar: str
    phase: Any = 0
    slot: Any = None


@dataclass(frozen=True)
class SetMaxNReg(Stmt):
    count: int
    direction: Any = "inc"


@dataclass(frozen=True)
class FragLayout:
    """Per-atom geometry of a C fragment: element count, the row (0 top, 1 bottom) of each
    element, the lane xors that combine a row's lanes, and text the IR's renderer uses."""
    n_elems: int = 4
    elem_row: tuple = ()
    reduce_xors: tuple = ()
    lane_decl: Any = None
    lane_names: tuple = ()
    row_off: Any = None
    col_off: Any = None


@dataclass(frozen=True)
class Lambda:
    """A pure per-element function (a RegStore epilogue): ``params`` are bound on entry,
    ``body`` (Load / Assign / Let / Select statements) is evaluated, ``results`` name the
    values it returns."""
    params: tuple = ()
    body: tuple = ()
    results: tuple = ()


@dataclass(frozen=True)
class FragmentPromote(Stmt):
    dst: str
    src: str = ""


@dataclass(frozen=True)
class FragmentApply(Stmt):
    out: str
    op: Any = None
    args: tuple = ()
    kinds: tuple = ()
    in_place: bool = False
    layout: Any = None
    post: Any = None
    row_base: Any = None
    col_base: Any = None


@dataclass(frozen=True)
class FragmentRowReduce(Stmt):
    top: str
    bot: str = ""
    frags: tuple = ()
    op: Any = None
    layout: Any = None
    dtype: Any = None


@dataclass(frozen=True)
class FragmentRepack(Stmt):
    frag: str
    srcs: tuple = ()
    ab_dtype: str = "f16"
    fragment_layout: str = "m16n8k16"
    part: Any = None


@dataclass(frozen=True)
class WgmmaDescriptor(Stmt):
    name: str
    smem: str = ""
    smem_index: tuple = ()
    swizzle: Any = None
    lbo_bytes: Any = 0
    sbo_bytes: Any = 0


@dataclass(frozen=True)
class WgmmaMma(Stmt):
    c_frags: tuple
    b_desc: str = ""
    shape: tuple = ()
    ab_dtype: str = "f16"
    a_desc: Any = None
    a_frag: Any = None
    scale_d: Any = 1
    trans_a: bool = False
    trans_b: bool = False


@dataclass(frozen=True)
class WgmmaFence(Stmt):
    pass


@dataclass(frozen=True)
class WgmmaCommit(Stmt):
    pass


@dataclass(frozen=True)
class WgmmaWait(Stmt):
    group: Any = 0


@dataclass(frozen=True)
class Opaque(Stmt):
    """A constructor this reader does not model; kept so the walker can name
    it when it fails (BlockScaleLoad appears in the IR reference but in no
    shipped kernel)."""
    kind: str
    fields: tuple = field(default=())

    def pretty(self) -> str:
        return f"{self.kind}(...)"


# ---------------------------------------------------------------------------
# the reader

_CONSTRUCTORS: dict[str, type] = {
    c.__name__: c for c in (
        DataType, Dim, Window, Axis, ElementwiseImpl, Var, Literal, BinaryExpr, TernaryExpr,
        Builtin, FuncCallExpr, CastExpr, FlatIndex, Tile, Loop, StridedLoop, Cond, Load,
        Assign, Let, Accum, Init, Write, WarpShuffle, TreeHalve, Smem, Sync, CpAsyncCopy,
        CpAsyncCommit, CpAsyncWait, RegFragment, LdmatrixLoad, MmaSyncPtx, RegStore,
        Branch, Select, Pre, Carry, ZeroPrologue, TmaDescriptor, TmaLoad, MbarrierInit,
        MbarrierArriveExpectTx, MbarrierArrive, MbarrierWait, SetMaxNReg, WgmmaDescriptor, WgmmaMma,
        WgmmaFence, WgmmaCommit, WgmmaWait, FragLayout, Lambda, FragmentPromote, FragmentApply, FragmentRowReduce,
        FragmentRepack)
}


class IRSyntaxError(ValueError):
    pass


def _value(node: ast.AST) -> Any:
    if isinstance(node, ast.Constant):
        return node.value
    if isinstance(node, (ast.Tuple, ast.List)):
        return tuple(_value(e) for e in node.elts)
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, ast.USub):
        v = _value(node.operand)
        if isinstance(v, (int, float)):
            return -v
    if isinstance(node, ast.Name) and node.id in ("inf", "nan"):
        return float(node.id)
    if isinstance(node, ast.Call) and isinstance(node.func, ast.Name):
        name = node.func.id
        args = [_value(a) for a in node.args]
        kwargs = {k.arg: _value(k.value) for k in node.keywords}
        if name == "dtype":            # numpy dtype('float32') inside DataType(np=...)
            return args[0] if args else kwargs.get("dtype")
        cls = _CONSTRUCTORS.get(name)
        if cls is None:
            return Opaque(name, tuple(sorted(kwargs.items())) + tuple(enumerate(args)))
        try:
            return cls(*args, **kwargs)
        except TypeError as exc:
            raise IRSyntaxError(f"{name}: {exc}") from None
    raise IRSyntaxError(f"unsupported IR syntax: {ast.dump(node)[:120]}")


def parse_stmt(text: str) -> Any:
    """One statement (or expression) from its repr text."""
    try:
        tree = ast.parse(text, mode="eval")
    except SyntaxError as exc:
        raise IRSyntaxError(f"IR body is not a constructor expression: {exc}") from None
    return _value(tree.body)


def parse_body(body: list[str] | tuple[str, ...] | str) -> tuple:
    """A KernelOp body: a list of statement reprs -> tuple of statements."""
    if isinstance(body, str):
        body = [body]
    return tuple(parse_stmt(s) for s in body)


# ---------------------------------------------------------------------------
# graph level


@dataclass(frozen=True)
class TensorInfo:
    name: str
    shape: tuple
    dtype: str


@dataclass(frozen=True)
class KernelNode:
    """The one KernelOp node of an IR file."""
    node: str
    name: str
    body: tuple
    zero_delegated: tuple
    serial: tuple
    inputs: tuple


@dataclass(frozen=True)
class Graph:
    inputs: tuple
    outputs: tuple
    nodes: dict            # node id -> raw dict (op, op_fields, inputs, outputs)
    tensors: dict          # buffer name -> TensorInfo
    kernels: tuple         # KernelNode, in file order

    @classmethod
    def from_dict(cls, data: dict) -> "Graph":
        tensors: dict[str, TensorInfo] = {}
        kernels = []
        for nid, node in data["nodes"].items():
            for t in node.get("outputs", []):
                tensors[t["name"]] = TensorInfo(t["name"], tuple(t["shape"]), t["dtype"])
            if node.get("op") == "KernelOp":
                of = node["op_fields"]
                kernels.append(KernelNode(nid, of.get("name") or nid, parse_body(of["body"]),
                                          tuple(of.get("zero_delegated", ())),
                                          tuple(of.get("serial", ())),
                                          tuple(node.get("inputs", ()))))
        return cls(tuple(data.get("inputs", ())), tuple(data.get("outputs", ())),
                   dict(data["nodes"]), tensors, tuple(kernels))

    def buffer(self, name: str) -> TensorInfo | None:
        return self.tensors.get(name)


def walk_stmts(stmts: Any):
    """Every statement under ``stmts`` (pre-order), descending into bodies."""
    for s in stmts:
        yield s
        for attr in ("body", "else_body"):
            sub = getattr(s, attr, None)
            if isinstance(sub, tuple):
                yield from walk_stmts(sub)
