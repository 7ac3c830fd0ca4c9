"""Emmy Kernel IR, read without emmy.

A Kernel IR file stores each KernelOp body as the Python ``repr`` of emmy's
statement dataclasses, e.g. ``Tile(axes=(Axis(name='a0', extent=Dim(64),
window=None),), body=(...), block_threads=128, ...)``.  emmy-ml is not a
dependency of this compiler, so this module gives every constructor of that
vocabulary a frozen record class of its own and rebuilds the tree from the
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
from dataclasses import field
from typing import Any


# ---------------------------------------------------------------------------
# frozen records
#
# The IR's node classes are frozen records with the behaviour of frozen dataclasses (keyword or
# positional construction with defaults, field-wise equality and hash, the dataclass repr), but
# their methods are shared functions installed on each class rather than source generated and
# compiled per class: a frozen dataclass costs about a millisecond to create, and this module
# defines some sixty, which every ``compile.py`` process would pay on start-up.


def _rec_init(self, *args, **kwargs) -> None:
    cls = type(self)
    names = cls._fields
    if len(args) > len(names):
        raise TypeError(f"{cls.__name__}.__init__() takes {len(names)} positional arguments but "
                        f"{len(args)} were given")
    d = self.__dict__
    for k, v in zip(names, args):
        d[k] = v
    for k, v in kwargs.items():
        if k not in cls._defaults and k not in names:
            raise TypeError(f"{cls.__name__}.__init__() got an unexpected keyword argument '{k}'")
        if k in d:
            raise TypeError(f"{cls.__name__}.__init__() got multiple values for argument '{k}'")
        d[k] = v
    if len(d) < len(names):
        for k in names:
            if k not in d:
                if k not in cls._defaults:
                    raise TypeError(f"{cls.__name__}.__init__() missing 1 required positional argument: '{k}'")
                d[k] = cls._defaults[k]


def _rec_values(self) -> tuple:
    return tuple(getattr(self, k) for k in self._fields)


def _rec_eq(self, other) -> bool:
    if other.__class__ is not self.__class__:
        return NotImplemented
    return _rec_values(self) == _rec_values(other)


def _rec_hash(self) -> int:
    return hash(_rec_values(self))


def _rec_repr(self) -> str:
    return f"{type(self).__qualname__}(" + ", ".join(f"{k}={getattr(self, k)!r}" for k in self._fields) + ")"


def _rec_setattr(self, name, value) -> None:
    raise dataclasses.FrozenInstanceError(f"cannot assign to field '{name}'")


def _rec_delattr(self, name) -> None:
    raise dataclasses.FrozenInstanceError(f"cannot delete field '{name}'")


def record(cls):
    """Make ``cls`` a frozen record: its fields are its annotations after its bases' fields, their
    defaults the class attributes of those names (a ``dataclasses.field(default=...)`` too)."""
    names: list[str] = []
    defaults: dict[str, Any] = {}
    for base in reversed(cls.__mro__[1:]):
        for k in getattr(base, "_fields", ()):
            if k not in names:
                names.append(k)
        defaults.update(getattr(base, "_defaults", {}))
    for k in cls.__dict__.get("__annotations__", {}):
        if k not in names:
            names.append(k)
        if k in cls.__dict__:
            v = cls.__dict__[k]
            defaults[k] = v.default if isinstance(v, dataclasses.Field) else v
            delattr(cls, k)
    cls._fields, cls._defaults = tuple(names), defaults
    cls.__init__, cls.__eq__, cls.__hash__ = _rec_init, _rec_eq, _rec_hash
    cls.__setattr__, cls.__delattr__ = _rec_setattr, _rec_delattr
    if "__repr__" not in cls.__dict__:
        cls.__repr__ = _rec_repr
    return cls


def is_record(o) -> bool:
    """An IR node (an instance of a record class)?"""
    return hasattr(o, "_fields") and not isinstance(o, type)


def field_names(o) -> tuple:
    """The field names of a record (or of a dataclass instance)."""
    if is_record(o):
        return o._fields
    return tuple(f.name for f in dataclasses.fields(o))


# ---------------------------------------------------------------------------
# leaf values


@record
class DataType:
    """An element type: ``name`` is the IR dtype ("f32", "f16", "f64", ...)."""
    name: str
    np: Any = None
    nbytes: int = 0


@record
class Dim:
    value: Any

    @property
    def is_static(self) -> bool:
        return isinstance(self.value, int)

    def as_static(self) -> int:
        if not self.is_static:
            raise NotImplementedError(f"dimension {self.value!r} is not static")
        return int(self.value)


@record
class Window:
    parent: Any = None
    base: Any = None
    bound: Any = None
    partition: bool = False


@record
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


@record
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


@record
class Var(Expr):
    name: str

    def pretty(self) -> str:
        return self.name


@record
class Literal(Expr):
    value: Any
    dtype: str = "int"

    def pretty(self) -> str:
        return repr(self.value)


@record
class BinaryExpr(Expr):
    op: str
    left: Any
    right: Any

    def pretty(self) -> str:
        return f"({pretty(self.left)} {self.op} {pretty(self.right)})"


@record
class TernaryExpr(Expr):
    cond: Any
    if_true: Any
    if_false: Any

    def pretty(self) -> str:
        return f"({pretty(self.cond)} ? {pretty(self.if_true)} : {pretty(self.if_false)})"


@record
class Builtin(Expr):
    name: str


@record
class FuncCallExpr(Expr):
    name: str
    args: tuple = ()


@record
class CastExpr(Expr):
    dtype: Any
    expr: Any


@record
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
        names = list(field_names(self))[:3]
        return f"{type(self).__name__}(" + ", ".join(
            f"{n}={_short(getattr(self, n))}" for n in names) + ")"


def _short(v: Any) -> str:
    text = pretty(v) if not isinstance(v, (str, int, float)) else repr(v)
    return text if len(text) < 60 else text[:57] + "..."


@record
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


@record
class Loop(Stmt):
    axis: Axis
    body: tuple
    unroll: Any = False
    seed: bool = False
    carries: tuple = ()

    def pretty(self) -> str:
        return f"for {self.axis.name} in 0..{pretty(self.axis.extent.value)}"


@record
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


@record
class Cond(Stmt):
    cond: Any
    body: tuple
    else_body: tuple = ()

    def pretty(self) -> str:
        return f"if {pretty(self.cond)}"


@record
class Load(Stmt):
    names: tuple
    input: str
    index: tuple
    dtype: Any = None

    def pretty(self) -> str:
        return f"{', '.join(self.names)} = load {self.input}[{pretty(self.index)}]"


@record
class Assign(Stmt):
    name: str
    op: ElementwiseImpl
    args: tuple
    dtype: Any = None

    def pretty(self) -> str:
        return f"{self.name} = {self.op.name}({', '.join(self.args)})"


@record
class Let(Stmt):
    name: str
    value: Any
    dtype: Any = None

    def pretty(self) -> str:
        return f"{self.name} = {pretty(self.value)}"


@record
class Accum(Stmt):
    name: str
    value: str
    op: ElementwiseImpl
    dtype: Any = None
    axes: tuple = ()
    base: Any = None

    def pretty(self) -> str:
        return f"{self.name} <- {self.op.name}({self.base or self.name}, {self.value})"


@record
class Init(Stmt):
    name: str
    identity: Any
    dtype: Any = None

    def pretty(self) -> str:
        return f"Init({self.name} = {self.identity})"


@record
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


@record
class WarpShuffle(Stmt):
    state: tuple
    state_b: tuple
    combine_states: tuple
    length: int = 32
    dtype: Any = None

    def pretty(self) -> str:
        return f"WarpShuffle({', '.join(self.state)}, length={self.length})"


@record
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


@record
class Smem(Stmt):
    name: str
    extents: tuple
    dtype: str
    align: int = 0

    def pretty(self) -> str:
        dims = "".join(f"[{e}]" for e in self.extents)
        return f"Smem {self.dtype} {self.name}{dims} align={self.align}"


@record
class Sync(Stmt):
    barrier_id: int = 0
    count: Any = None
    warp: bool = False

    def pretty(self) -> str:
        return "SyncWarp" if self.warp else f"Sync(id={self.barrier_id}, count={self.count})"


@record
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


@record
class CpAsyncCommit(Stmt):
    pass


@record
class CpAsyncWait(Stmt):
    group: int = 0


@record
class RegFragment(Stmt):
    name: str
    role: str
    shape: tuple
    dtype: Any
    count: int = 1
    nregs: Any = None


@record
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


@record
class BlockScaleLoad(Stmt):
    frag: str
    src_buffer: str
    src_index: tuple = ()
    role: str = "a"
    ldm: int = 0


@record
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


@record
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


@record
class Branch:
    """One arm of a Select: ``value`` when ``select`` (a coordinate predicate; None = otherwise)."""
    value: Any
    select: Any = None


@record
class Select(Stmt):
    name: str
    branches: tuple = ()


@record
class Pre(Stmt):
    name: str
    carrier: str = ""
    index: tuple = ()


@record
class Carry(Stmt):
    name: str
    value: Any = None
    index: tuple = ()
    seed: Any = None
    dtype: Any = None


@record
class ZeroPrologue(Stmt):
    dst: str
    words: Any = 0


@record
class TmaDescriptor(Stmt):
    name: str
    src_buf: str = ""
    src_shape: tuple = ()
    box_extents: tuple = ()
    swizzle: Any = None
    dtype: Any = None


@record
class TmaLoad(Stmt):
    smem: str
    smem_index: tuple = ()
    desc: str = ""
    coords: tuple = ()
    mbar: str = ""
    mbar_slot: Any = None


@record
class MbarrierInit(Stmt):
    mbar: str
    count: Any = 1
    slot: Any = None


@record
class MbarrierArriveExpectTx(Stmt):
    mbar: str
    bytes_: Any = 0
    slot: Any = None


@record
class MbarrierArrive(Stmt):
    mbar: str
    slot: Any = None


@record
class MbarrierWait(Stmt):
    mbar: str
    phase: Any = 0
    slot: Any = None


@record
class SetMaxNReg(Stmt):
    count: int
    direction: Any = "inc"


@record
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


@record
class Lambda:
    """A pure per-element function (a RegStore epilogue): ``params`` are bound on entry,
    ``body`` (Load / Assign / Let / Select statements) is evaluated, ``results`` name the
    values it returns."""
    params: tuple = ()
    body: tuple = ()
    results: tuple = ()


@record
class FragmentPromote(Stmt):
    dst: str
    src: str = ""


@record
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


@record
class FragmentRowReduce(Stmt):
    top: str
    bot: str = ""
    frags: tuple = ()
    op: Any = None
    layout: Any = None
    dtype: Any = None


@record
class FragmentRepack(Stmt):
    frag: str
    srcs: tuple = ()
    ab_dtype: str = "f16"
    fragment_layout: str = "m16n8k16"
    part: Any = None


@record
class WgmmaDescriptor(Stmt):
    name: str
    smem: str = ""
    smem_index: tuple = ()
    swizzle: Any = None
    lbo_bytes: Any = 0
    sbo_bytes: Any = 0


@record
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


@record
class WgmmaFence(Stmt):
    pass


@record
class WgmmaCommit(Stmt):
    pass


@record
class WgmmaWait(Stmt):
    group: Any = 0


@record
class Opaque(Stmt):
    """A constructor this reader does not model; kept so the walker can name
    it when it fails."""
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
        CpAsyncCommit, CpAsyncWait, RegFragment, LdmatrixLoad, BlockScaleLoad, MmaSyncPtx, RegStore,
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


@record
class TensorInfo:
    name: str
    shape: tuple
    dtype: str


@record
class KernelNode:
    """The one KernelOp node of an IR file."""
    node: str
    name: str
    body: tuple
    zero_delegated: tuple
    serial: tuple
    inputs: tuple


@record
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
