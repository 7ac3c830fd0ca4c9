"""Elementwise operations -> PTX instructions.

Every rounding float operation is IEEE round-to-nearest (``.rn``) so that
pointwise results are bit-identical to numpy / torch on the CPU: an
explicit rounding mode also stops ptxas from contracting a mul and an add
into one fma (which rounds once instead of twice).  The transcendental
ops map to the SFU ``.approx`` forms, as in the reference compiler
(thompiler/lowering/ops.py:18-99 of the reference); exp is lowered by the
caller as 2^(x*log2 e).

f16 values compute natively (sm_53 and later have .rn f16 add / mul /
fma and min / max); there is no f16 division, square root or
transcendental instruction, so those go through f32 in the compute
handler.
"""

from __future__ import annotations

from thompiler.lowering.types import F16, Ty

# op -> {type kind or exact type name -> template}; {t} = arithmetic suffix.
UNARY: dict[str, dict[str, str]] = {
    "copy": {"float": "mov.{m}", "int": "mov.{m}"},
    "negative": {"float": "neg.{t}", "int": "neg.{t}"},
    "abs": {"float": "abs.{t}", "int": "abs.{t}"},
    "sqrt": {"f32": "sqrt.rn.f32", "f64": "sqrt.rn.f64"},
    "reciprocal": {"f32": "rcp.rn.f32", "f64": "rcp.rn.f64"},
    "rsqrt": {"f32": "rsqrt.approx.f32", "f64": "rsqrt.approx.f64"},
    "tanh": {"f32": "tanh.approx.f32"},
    "sin": {"f32": "sin.approx.f32"},
    "cos": {"f32": "cos.approx.f32"},
}

BINARY: dict[str, dict[str, str]] = {
    "add": {"float": "add.rn.{t}", "int": "add.{t}"},
    "subtract": {"float": "sub.rn.{t}", "int": "sub.{t}"},
    "multiply": {"float": "mul.rn.{t}", "int": "mul.lo.{t}"},
    "divide": {"f32": "div.rn.f32", "f64": "div.rn.f64", "int": "div.{t}"},
    "mod": {"int": "rem.{t}"},
    "maximum": {"float": "max.{t}", "int": "max.{t}"},
    "minimum": {"float": "min.{t}", "int": "min.{t}"},
}

# Folds an Accum may use.
ACCUM_OPS = ("add", "multiply", "maximum", "minimum")

# Index-expression operator -> BINARY op (integer only).
INDEX_OPS: dict[str, str] = {"+": "add", "-": "subtract", "*": "multiply", "/": "divide", "%": "mod"}

# Comparisons.  For floats, C's != is true when an operand is NaN, which is
# PTX's unordered ``neu``; the other five are the ordered forms, as in C.
COMPARE: dict[str, dict[str, str]] = {
    "==": {"float": "eq", "int": "eq"},
    "!=": {"float": "neu", "int": "ne"},
    "<": {"float": "lt", "int": "lt"},
    "<=": {"float": "le", "int": "le"},
    ">": {"float": "gt", "int": "gt"},
    ">=": {"float": "ge", "int": "ge"},
}

LOGIC: dict[str, str] = {"&&": "and.pred", "||": "or.pred"}


def lookup(table: dict[str, dict[str, str]], op: str, ty: Ty) -> str | None:
    forms = table.get(op)
    if forms is None:
        return None
    form = forms.get(ty.name) or forms.get(ty.kind)
    if form is None:
        return None
    return form.format(t=ty.ptx, m=ty.mov)


def instruction(table: dict[str, dict[str, str]], op: str, ty: Ty) -> str:
    form = lookup(table, op, ty)
    if form is None:
        raise NotImplementedError(f"operation {op!r} on {ty.name} values")
    return form


def f16_native(op: str) -> bool:
    """Ops whose f16 form is a native instruction (others widen to f32)."""
    return op in ("copy", "negative", "abs", "add", "subtract", "multiply", "maximum", "minimum")


# (from, to) -> cvt.  Narrowing needs a rounding mode (.rn); widening is exact.
CONVERT: dict[tuple[str, str], str] = {
    ("f32", "f16"): "cvt.rn.f16.f32",
    ("f64", "f16"): "cvt.rn.f16.f64",
    ("f64", "f32"): "cvt.rn.f32.f64",
    ("f16", "f32"): "cvt.f32.f16",
    ("f16", "f64"): "cvt.f64.f16",
    ("f32", "f64"): "cvt.f64.f32",
}


def convert(src: Ty, dst: Ty) -> str:
    form = CONVERT.get((src.name, dst.name))
    if form is None:
        raise NotImplementedError(f"conversion from {src.name} to {dst.name}")
    return form


__all__ = ["UNARY", "BINARY", "ACCUM_OPS", "INDEX_OPS", "COMPARE", "LOGIC", "instruction",
           "lookup", "convert", "f16_native", "F16"]
