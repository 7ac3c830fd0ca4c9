"""A clean-room stand-in for the parts of emmy-ml 0.3.11 that the reference
compiler imports (test infrastructure only -- never imported by the product).

emmy-ml is not installed and cannot be; this module gives the reference's
``compile.py`` the classes, attribute names and ``Graph.from_dict`` it uses
(reference thompiler/load.py:15-18, walk.py:11-17 and the handlers), so the
reference compiler runs unmodified here and prints its own PTX.  The IR
bodies are rebuilt from their repr text with ``ast`` and a whitelist of
constructor names; no ``eval``.
"""

from __future__ import annotations

import ast
from dataclasses import dataclass, field, fields
from typing import Any

_IDENT = {"add": (2, 0.0), "multiply": (2, 1.0), "maximum": (2, -1e30), "minimum": (2, 1e30)}
_ARITY1 = {"copy", "exp", "reciprocal", "relu", "sqrt", "rsqrt", "negative", "abs", "tanh", "sin", "cos"}


@dataclass
class DataType:
    name: str
    np: Any = None
    nbytes: int = 0


@dataclass
class Dim:
    value: Any

    @property
    def is_static(self):
        return isinstance(self.value, int)

    def as_static(self):
        return int(self.value)


@dataclass
class Window:
    parent: Any = None
    base: Any = None
    bound: Any = None
    partition: bool = False


@dataclass
class Axis:
    name: str
    extent: Dim
    window: Any = None


class ElementwiseImpl:
    def __init__(self, name):
        self.name = name

    @property
    def arity(self):
        return 1 if self.name in _ARITY1 else 2

    @property
    def identity(self):
        return _IDENT.get(self.name, (0, None))[1]

    def __repr__(self):
        return f"ElementwiseImpl({self.name!r})"


class Expr:
    def pretty(self):
        return _text(self)


class Stmt:
    def pretty(self, indent=""):
        return [indent + _text(self)]


def _text(o):
    if isinstance(o, Var):
        return o.name
    if isinstance(o, Literal):
        return repr(o.value)
    if isinstance(o, BinaryExpr):
        return f"({_text(o.left)} {o.op} {_text(o.right)})"
    if isinstance(o, TernaryExpr):
        return f"({_text(o.cond)} ? {_text(o.if_true)} : {_text(o.if_false)})"
    if isinstance(o, tuple):
        return ", ".join(_text(x) for x in o)
    if hasattr(o, "__dataclass_fields__"):
        head = [f.name for f in fields(o)][:2]
        return f"{type(o).__name__}(" + ", ".join(
            f"{n}={_text(getattr(o, n)) if not isinstance(getattr(o, n), (str, int, float)) else getattr(o, n)}"
            for n in head if not isinstance(getattr(o, n), tuple) or n != "body") + ")"
    return str(o)


@dataclass
class Var(Expr):
    name: str


@dataclass
class Literal(Expr):
    value: Any
    dtype: str = "int"


@dataclass
class BinaryExpr(Expr):
    op: str
    left: Any
    right: Any


@dataclass
class TernaryExpr(Expr):
    cond: Any
    if_true: Any
    if_false: Any


@dataclass
class FlatIndex(Expr):
    buffer: str = ""
    index: tuple = ()


def _stmt(name, spec):
    """A statement dataclass ``name`` with fields ``spec`` [(field, default|REQ)]."""
    ns = {"__annotations__": {}}
    for fname, default in spec:
        ns["__annotations__"][fname] = Any
        if default is not REQ:
            ns[fname] = field(default=default)
    return dataclass(type(name, (Stmt,), ns))


REQ = object()

Tile = _stmt("Tile", [("axes", REQ), ("body", REQ), ("block_threads", 0), ("aux_threads", 0),
                      ("raster_axes", None), ("raster_group", None), ("raster_orient", "m")])
Tile.extents = property(lambda self: tuple(a.extent.as_static() for a in self.axes))
Tile.n_elements = property(lambda self: __import__("math").prod(self.extents))
Loop = _stmt("Loop", [("axis", REQ), ("body", REQ), ("unroll", False), ("seed", False)])
Loop.carries = property(lambda self: ())
StridedLoop = _stmt("StridedLoop", [("axis", REQ), ("start", REQ), ("step", REQ), ("body", REQ),
                                    ("unroll", False), ("end", None), ("seed", False)])
Cond = _stmt("Cond", [("cond", REQ), ("body", REQ), ("else_body", ())])
Load = _stmt("Load", [("names", REQ), ("input", REQ), ("index", REQ), ("dtype", None)])
Assign = _stmt("Assign", [("name", REQ), ("op", REQ), ("args", REQ), ("dtype", None)])
Let = _stmt("Let", [("name", REQ), ("value", REQ), ("dtype", None)])
Accum = _stmt("Accum", [("name", REQ), ("value", REQ), ("op", REQ), ("dtype", None), ("axes", ()),
                        ("base", None)])
Init = _stmt("Init", [("name", REQ), ("identity", REQ), ("dtype", None)])
Write = _stmt("Write", [("output", REQ), ("index", REQ), ("values", REQ), ("value_dtype", None),
                        ("atomic", False), ("swizzle", "NONE")])
WarpShuffle = _stmt("WarpShuffle", [("state", REQ), ("state_b", REQ), ("combine_states", REQ),
                                    ("length", 32), ("dtype", None)])
TreeHalve = _stmt("TreeHalve", [("bufs", REQ), ("state", REQ), ("state_b", REQ), ("combine_states", REQ),
                                ("length", REQ), ("tid_var", REQ), ("dtype", None), ("barrier_id", 0),
                                ("barrier_count", None), ("inner", None)])
Smem = _stmt("Smem", [("name", REQ), ("extents", REQ), ("dtype", REQ), ("align", 0)])
Sync = _stmt("Sync", [("barrier_id", 0), ("count", None), ("warp", False)])
CpAsyncCopy = _stmt("CpAsyncCopy", [("smem", REQ), ("smem_index", REQ), ("src", REQ), ("src_index", REQ),
                                    ("nbytes", REQ), ("swizzle", "NONE"), ("lane_index", None),
                                    ("lane_rows", None)])
CpAsyncCommit = _stmt("CpAsyncCommit", [])
CpAsyncWait = _stmt("CpAsyncWait", [("group", 0)])
RegFragment = _stmt("RegFragment", [("name", REQ), ("role", REQ), ("shape", REQ), ("dtype", REQ),
                                    ("count", 1), ("nregs", None)])
LdmatrixLoad = _stmt("LdmatrixLoad", [(n, None) for n in (
    "frag", "src_buffer", "src_index", "role", "ldm", "swizzle", "staged", "gmem_guard", "k_zero",
    "b_trans", "pair_frag", "byte_slab", "scale_buffer", "scale_index", "scale_ldm", "fragment_layout",
    "fragment_index")])
MmaSyncPtx = _stmt("MmaSyncPtx", [(n, None) for n in (
    "c_frag", "a_frag", "b_frag", "shape", "ab_dtype", "c_dtype", "b_row_major", "sfa_frag", "sfb_frag")])
MmaSyncPtx.block_scaled = property(lambda self: self.sfa_frag is not None)
RegStore = _stmt("RegStore", [(n, None) for n in (
    "dst_buffer", "dst_index", "frag", "shape", "ldm", "epilogue", "extra_frags", "m_guard", "n_guard",
    "atomic", "fragment_layout", "volta_interleaved", "fragment_index", "swizzle", "row_dim", "col_dim")])

# The sm_90 vocabulary's Select (TASK.md:120-135 of the reference) and the RegStore epilogue
# Lambda (TASK.md:159): plain records, interpreted by oracle/interp.py.
Select = _stmt("Select", [("name", REQ), ("branches", ())])


@dataclass
class Branch:
    value: Any = None
    select: Any = None


@dataclass
class Lambda:
    params: tuple = ()
    body: tuple = ()
    results: tuple = ()


_CTORS = {c.__name__: c for c in (
    DataType, Dim, Window, Axis, ElementwiseImpl, Var, Literal, BinaryExpr, TernaryExpr, FlatIndex,
    Tile, Loop, StridedLoop, Cond, Load, Assign, Let, Accum, Init, Write, WarpShuffle, TreeHalve, Smem,
    Sync, CpAsyncCopy, CpAsyncCommit, CpAsyncWait, RegFragment, LdmatrixLoad, MmaSyncPtx, RegStore,
    Select, Branch, Lambda)}


def _build(node):
    if isinstance(node, ast.Constant):
        return node.value
    if isinstance(node, (ast.Tuple, ast.List)):
        return tuple(_build(e) for e in node.elts)
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, ast.USub):
        return -_build(node.operand)
    if isinstance(node, ast.Call) and isinstance(node.func, ast.Name):
        args = [_build(a) for a in node.args]
        kw = {k.arg: _build(k.value) for k in node.keywords}
        if node.func.id == "dtype":
            return args[0]
        return _CTORS[node.func.id](*args, **kw)
    raise ValueError(f"unsupported IR syntax {ast.dump(node)[:80]}")


class KernelOp:
    def __init__(self, name, body, zero_delegated=(), serial=()):
        self.name, self.body = name, body
        self.zero_delegated, self.serial = tuple(zero_delegated), tuple(serial)


class InputOp:
    pass


class ConstantOp:
    def __init__(self, value=None):
        self.value = value


@dataclass
class Tensor:
    name: str
    shape: tuple
    dtype: DataType


@dataclass
class Node:
    op: Any
    inputs: tuple
    outputs: tuple


class Graph:
    def __init__(self, inputs, outputs, nodes):
        self.inputs, self.outputs, self.nodes = inputs, outputs, nodes
        self._buffers = {t.name: t for n in nodes.values() for t in n.outputs}

    @classmethod
    def from_dict(cls, d):
        nodes = {}
        for nid, raw in d["nodes"].items():
            of = raw.get("op_fields", {})
            if raw["op"] == "KernelOp":
                body = tuple(_build(ast.parse(b, mode="eval").body) for b in of["body"])
                op = KernelOp(of.get("name") or nid, body, of.get("zero_delegated", ()), of.get("serial", ()))
            elif raw["op"] == "ConstantOp":
                op = ConstantOp(of.get("value"))
            else:
                op = InputOp()
            outs = tuple(Tensor(t["name"], tuple(Dim(int(x)) for x in t["shape"]), DataType(t["dtype"]))
                         for t in raw.get("outputs", []))
            nodes[nid] = Node(op, tuple(raw.get("inputs", ())), outs)
        return cls(tuple(d.get("inputs", ())), tuple(d.get("outputs", ())), nodes)

    def buffer(self, name):
        return self._buffers.get(name)
