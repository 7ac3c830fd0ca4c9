"""The IR synthesizer against the reference's shipped IR.

``thompiler.synth`` writes packages at any size in the shipped schedules: the
benchmark shapes have no shipped IR, so the synthesizer is what the benchmark
and most family tests compile.  Here it is pinned to the shipped packages it
generalises: at the shipped sizes it must reproduce each KernelOp body (the
statement tree's text, names included) byte for byte, and the package's
argument order and launch geometry.  Shipped IR: reference
problems/{r01_array_sum,r02_big_sum,r03_mean,r04_row_sum,f01_rmsnorm,
f02_row_softmax,f03_l2norm}/*.ir.json (the golden copies under
tests/golden/packages).
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest

from thompiler import synth

GOLDEN = Path(__file__).parent / "golden" / "packages"


def _kernel(d: Path) -> tuple[list, dict]:
    meta = json.loads((d / "meta.json").read_text())
    k = meta["kernels"][0]
    g = json.loads((d / f"{k['entry']}.ir.json").read_text())
    body = [n for n in g["nodes"].values() if n["op"] == "KernelOp"][0]["op_fields"]["body"]
    return body, k


CASES = {
    "r01_array_sum": lambda d: synth.sum_package(d, 1024),
    "r02_big_sum": lambda d: synth.sum_package(d, 65536),
    "r03_mean": lambda d: synth.sum_package(d, 32768, kind="mean"),
    "r04_row_sum": lambda d: synth.row_package(d, "rowsum", 64, 512),
    "f01_rmsnorm": lambda d: synth.row_package(d, "rmsnorm", 64, 1024),
    "f02_row_softmax": lambda d: synth.row_package(d, "softmax", 64, 256),
    "f03_l2norm": lambda d: synth.row_package(d, "l2norm", 64, 512),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_synth_reproduces_shipped_body(tmp_path, name):
    want, wk = _kernel(GOLDEN / name)
    got, gk = _kernel(CASES[name](tmp_path / name))
    assert got == want
    assert gk["grid"] == wk["grid"] and gk["block"] == wk["block"]
    assert sorted(gk["arg_order"]) == sorted(wk["arg_order"])
    assert {a["name"]: a["shape"] for a in gk["args"]} == {a["name"]: a["shape"] for a in wk["args"]}


@pytest.mark.parametrize("name", ["f01_rmsnorm", "f02_row_softmax", "f03_l2norm", "r04_row_sum"])
def test_synth_scales_only_the_extents(tmp_path, name):
    """At the benchmark's [8192, 4096] the body differs from the shipped one only in the
    extents: every statement, name and operator is the same."""
    import re
    kind = {"f01_rmsnorm": "rmsnorm", "f02_row_softmax": "softmax", "f03_l2norm": "l2norm",
            "r04_row_sum": "rowsum"}[name]
    want, wk = _kernel(GOLDEN / name)
    got, _ = _kernel(synth.row_package(tmp_path / kind, kind, 8192, 4096))
    rows, cols = next(a["shape"] for a in wk["args"] if a["name"] == "x")
    strip = lambda s, r, c: re.sub(rf"Dim\({c}\)", "Dim(C)", re.sub(rf"Dim\({r}\)", "Dim(R)", s))  # noqa: E731
    assert strip(got[0], 8192, 4096) == strip(want[0], rows, cols)
