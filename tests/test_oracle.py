"""The oracle is pinned: the IR interpreter reproduces the reference's own
golden outputs (expected.npz, reference tools/expressions_open.py etc.) for
every shipped problem within the problem's tolerance, bit-exactly for the
tolerance-0 pointwise problems; and the committed oracle.npz fixtures are
what the interpreter computes."""

import json

import numpy as np
import pytest

from conftest import GOLDEN, PACKAGES
from oracle.interp import Interp, OracleError, run_package


@pytest.mark.parametrize("name", PACKAGES)
def test_interpreter_matches_expected(name):
    d = GOLDEN / name
    meta = json.loads((d / "meta.json").read_text())
    produced = run_package(d)
    for out, want in dict(np.load(d / "expected.npz")).items():
        got = produced[out].reshape(want.shape)
        assert got.dtype == want.dtype
        if meta["rtol"] == 0 and meta["atol"] == 0:
            assert np.array_equal(got, want)
        assert np.allclose(got, want, rtol=meta["rtol"], atol=meta["atol"])
    fixture = dict(np.load(d / "oracle.npz"))
    for out, arr in fixture.items():
        assert np.array_equal(produced[out], arr), out


def test_interpreter_checks_bounds():
    from emmy.compiler import _model as M
    body = M.Tile(axes=(M.Axis("a0", M.Dim(8)),),
                  body=(M.Load(names=("v",), input="x", index=(M.BinaryExpr("+", M.Var("a0"), M.Literal(1, "int")),),
                               dtype=M.DataType("f32")),), block_threads=8)
    k = M.KernelOp("k", (body,))
    with pytest.raises(OracleError):
        Interp(k, {"x": np.zeros(8, np.float32)}, 1, 8).run()
