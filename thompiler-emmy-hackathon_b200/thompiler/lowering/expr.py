"""IR expressions -> PTX operands.

``int_operand`` / ``pred_operand`` emit whatever instructions an expression
needs and return the operand that holds its value: a register, or an
immediate when the value is known at compile time (literals, variables of
unrolled loops, and arithmetic between them, folded with C's truncating
``/`` and ``%`` as in the reference's thompiler/lowering/expr.py:143-152).

Integer expressions are signed 32-bit, like emmy's C ``int`` indices.  The
address code widens to 64 bits where a buffer needs it (address.py).
"""

from __future__ import annotations

from typing import TYPE_CHECKING

from thompiler import ir
from thompiler.lowering import ops
from thompiler.lowering.types import F32, I32, LITERAL_TYPES, REG_VALUE_TYPE, Ty

if TYPE_CHECKING:
    from thompiler.walk import Walker


def is_imm(operand: str) -> bool:
    return not operand.startswith("%")


def c_div(a: int, b: int) -> int:
    if b == 0:
        raise ZeroDivisionError("integer division by zero in an index expression")
    q = abs(a) // abs(b)
    return q if (a >= 0) == (b >= 0) else -q


def fold(op: str, a: int, b: int) -> int:
    if op == "+":
        return a + b
    if op == "-":
        return a - b
    if op == "*":
        return a * b
    if op == "/":
        return c_div(a, b)
    if op == "%":
        return a - c_div(a, b) * b
    raise NotImplementedError(f"no integer lowering for {op!r}")


def int_operand(w: "Walker", e: object) -> str:
    em = w.em
    if isinstance(e, ir.Var):
        if e.name in w.consts:
            return str(w.consts[e.name])
        reg = em.get(e.name)
        if em.named[reg] != "b32":
            raise TypeError(f"{e.name} is a .{em.named[reg]} value used as an integer index")
        return reg
    if isinstance(e, ir.Literal):
        if LITERAL_TYPES.get(e.dtype) is not I32 or not isinstance(e.value, int):
            raise TypeError(f"literal {e.value!r} ({e.dtype}) in an integer expression")
        return str(int(e.value))
    if isinstance(e, int) and not isinstance(e, bool):
        return str(e)
    if isinstance(e, ir.BinaryExpr):
        if e.op not in ops.INDEX_OPS:
            raise NotImplementedError(f"no integer lowering for {e.op!r}")
        a, b = int_operand(w, e.left), int_operand(w, e.right)
        if is_imm(a) and is_imm(b):
            return str(fold(e.op, int(a), int(b)))
        # identities that need no instruction
        if e.op in ("+", "-") and b == "0":
            return a
        if e.op == "+" and a == "0":
            return b
        if e.op in ("*", "/") and b == "1":
            return a
        if e.op == "*" and a == "1":
            return b
        out = em.tmp("b32")
        em.ins(f"{ops.instruction(ops.BINARY, ops.INDEX_OPS[e.op], I32)} {out}, {a}, {b}")
        return out
    if isinstance(e, ir.TernaryExpr):
        p = pred_operand(w, e.cond)
        a, b = int_operand(w, e.if_true), int_operand(w, e.if_false)
        out = em.tmp("b32")
        em.ins(f"selp.s32 {out}, {a}, {b}, {p}")
        return out
    if isinstance(e, ir.Builtin):
        sreg = BUILTINS.get(e.name)
        if sreg is None:
            raise NotImplementedError(f"built-in variable {e.name!r}")
        out = em.tmp("b32")
        em.ins(f"mov.u32 {out}, {sreg}")
        return out
    if isinstance(e, ir.CastExpr):
        name = getattr(e.dtype, "name", e.dtype)
        if name not in INT_NAMES:
            raise NotImplementedError(f"cast to {name!r} in an integer expression")
        inner = e.expr
        if isinstance(inner, ir.Var) and inner.name not in w.consts and em.cls_of(inner.name) in ("f32", "f64"):
            out = em.tmp("b32")             # C's float -> int conversion truncates toward zero
            em.ins(f"cvt.rzi.s32.{em.cls_of(inner.name)} {out}, {em.get(inner.name)}")
            return out
        return int_operand(w, inner)
    if isinstance(e, ir.FuncCallExpr):
        fn = INT_FUNCS.get(e.name)
        if fn is None or len(e.args) != fn[1]:
            raise NotImplementedError(f"integer function {e.name}({len(e.args)} args)")
        args = [int_operand(w, a) for a in e.args]
        if all(is_imm(a) for a in args):
            return str(fn[2](*[int(a) for a in args]))
        out = em.tmp("b32")
        em.ins(f"{fn[0]} {out}, {', '.join(args)}")
        return out
    raise NotImplementedError(f"index expression {type(e).__name__}")


# Builtin names (CUDA spelling) -> PTX special registers
BUILTINS = {f"{v}.{c}": f"%{r}.{c}" for v, r in (("threadIdx", "tid"), ("blockIdx", "ctaid"),
                                                 ("blockDim", "ntid"), ("gridDim", "nctaid")) for c in "xyz"}
BUILTINS.update({"laneid": "%laneid", "warpid": "%warpid", "smid": "%smid"})
INT_NAMES = ("int", "int32", "i32", "s32")
# integer functions of index expressions: PTX instruction, arity, compile-time value
INT_FUNCS = {"min": ("min.s32", 2, min), "minimum": ("min.s32", 2, min), "max": ("max.s32", 2, max),
             "maximum": ("max.s32", 2, max), "abs": ("abs.s32", 1, abs)}


WIDE_OPS = {"+": "add.s64", "-": "sub.s64", "*": "mul.lo.s64", "/": "div.s64", "%": "rem.s64"}


def int_operand_wide(w: "Walker", e: object) -> str:
    """An index expression evaluated in signed 64-bit arithmetic (b64 register or immediate):
    the form an offset into a buffer of 2^31 or more elements needs, where an intermediate
    such as ``a0 * 4`` may pass 2^31 although every axis value fits in 32 bits."""
    em = w.em
    if isinstance(e, ir.BinaryExpr):
        if e.op not in WIDE_OPS:
            raise NotImplementedError(f"no integer lowering for {e.op!r}")
        a, b = int_operand_wide(w, e.left), int_operand_wide(w, e.right)
        if is_imm(a) and is_imm(b):
            return str(fold(e.op, int(a), int(b)))
        if e.op in ("+", "-") and b == "0":
            return a
        if e.op == "+" and a == "0":
            return b
        if e.op in ("*", "/") and b == "1":
            return a
        out = em.tmp("b64")
        em.ins(f"{WIDE_OPS[e.op]} {out}, {a}, {b}")
        return out
    if isinstance(e, ir.TernaryExpr):
        p = pred_operand(w, e.cond)
        a, b = int_operand_wide(w, e.if_true), int_operand_wide(w, e.if_false)
        out = em.tmp("b64")
        em.ins(f"selp.b64 {out}, {a}, {b}, {p}")
        return out
    v = int_operand(w, e)                 # a variable or a literal: a 32-bit value
    if is_imm(v):
        return v
    out = em.tmp("b64")
    em.ins(f"cvt.s64.s32 {out}, {v}")
    return out


def value_type(w: "Walker", e: object) -> Ty:
    """Type of an expression (I32 for indices, the register's type for
    IR values, F32 for float literals)."""
    if isinstance(e, ir.Var):
        if e.name in w.consts:
            return I32
        return REG_VALUE_TYPE[w.em.cls_of(e.name)]
    if isinstance(e, ir.Literal):
        ty = LITERAL_TYPES.get(e.dtype)
        if ty is None:
            raise NotImplementedError(f"literal of dtype {e.dtype!r}")
        return ty
    if isinstance(e, ir.BinaryExpr) and e.op in ops.INDEX_OPS:
        a, b = value_type(w, e.left), value_type(w, e.right)
        if a != b:
            raise TypeError(f"operands of different types in {e.pretty()}")
        return a
    if isinstance(e, ir.TernaryExpr):
        a, b = value_type(w, e.if_true), value_type(w, e.if_false)
        if a != b:
            raise TypeError(f"the two arms of {e.pretty()} differ in type")
        return a
    if isinstance(e, (ir.Builtin, ir.FuncCallExpr)):
        return I32
    if isinstance(e, ir.CastExpr) and getattr(e.dtype, "name", e.dtype) in INT_NAMES:
        return I32
    raise NotImplementedError(f"expression {type(e).__name__}")


def float_operand(w: "Walker", e: object, ty: Ty) -> str:
    """A float Var or Literal as an operand of type ``ty`` (conditions only
    compare values; they do no float arithmetic)."""
    if isinstance(e, ir.Var):
        return w.em.get(e.name)
    if isinstance(e, ir.Literal):
        return ty.imm(float(e.value))
    raise NotImplementedError(f"{ty.name} expression {type(e).__name__} in a condition")


def pred_operand(w: "Walker", e: object) -> str:
    em = w.em
    if isinstance(e, ir.BinaryExpr) and e.op in ops.COMPARE:
        lt, rt = value_type(w, e.left), value_type(w, e.right)
        if lt != rt:
            # a float value against an int literal compares as float
            if lt.is_float and isinstance(e.right, ir.Literal):
                rt = lt
            elif rt.is_float and isinstance(e.left, ir.Literal):
                lt = rt
            else:
                raise TypeError(f"comparison of mixed types: {e.pretty()}")
        ty = lt
        cmp = ops.COMPARE[e.op]["float" if ty.is_float else "int"]
        if ty.is_float:
            a, b = float_operand(w, e.left, ty), float_operand(w, e.right, ty)
        else:
            a, b = int_operand(w, e.left), int_operand(w, e.right)
        out = em.tmp("pred")
        em.ins(f"setp.{cmp}.{ty.ptx} {out}, {a}, {b}")
        return out
    if isinstance(e, ir.BinaryExpr) and e.op in ops.LOGIC:
        a, b = pred_operand(w, e.left), pred_operand(w, e.right)
        out = em.tmp("pred")
        em.ins(f"{ops.LOGIC[e.op]} {out}, {a}, {b}")
        return out
    raise NotImplementedError(f"condition {ir.pretty(e)}")


def add_ints(w: "Walker", a: str, b: str) -> str:
    if is_imm(a) and is_imm(b):
        return str(int(a) + int(b))
    if b == "0":
        return a
    if a == "0":
        return b
    out = w.em.tmp("b32")
    w.em.ins(f"add.s32 {out}, {a}, {b}")
    return out
