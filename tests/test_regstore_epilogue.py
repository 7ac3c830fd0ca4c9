"""The fused RegStore forms on the CPU: an epilogue Lambda (bound to the element, the extra
fragments' elements and optionally the element's row and column), ``m_guard`` / ``n_guard``
and ``atomic``.  The kernels of tests/sm90_ir.py that use them parse from the IR's repr, lower
to PTX that ptxas accepts for sm_100a without spills, emit the store forms the geometry asks
for, and the malformed forms are refused at compile time."""

import re
import shutil
import subprocess

import pytest

from sm90_ir import EPILOGUE_FORMS, epilogue_matmul_package, wgmma_gemm_package
from thompiler import ir, load, synth
from thompiler.compiler import compile_kernel


def _ir(d):
    return next(d.glob("*.ir.json"))


def _ptx(d):
    return compile_kernel(load.load(str(_ir(d))))


def _lines(ptx):
    return [ln.strip() for ln in ptx.splitlines() if ln.startswith("\t") and not ln.strip().startswith("//")]


def _ptxas(ptx, tmp_path):
    if shutil.which("ptxas") is None:
        pytest.skip("ptxas not on PATH")
    f = tmp_path / "k.ptx"
    f.write_text(ptx)
    r = subprocess.run(["ptxas", "-arch=sm_100a", "-v", str(f), "-o", str(tmp_path / "k.cubin")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "0 bytes spill stores" in r.stderr, r.stderr


def _regstores(d):
    kernel = load.load(str(_ir(d)))
    return [s for s in ir.walk_stmts(kernel.body) if isinstance(s, ir.RegStore)]


def test_lambda_parses_from_repr(tmp_path):
    lam = ir.Lambda(("v", "row", "col"), (ir.Load(("b",), "bias", (synth.V("col"),), synth.F32T),
                                          synth.assign("o", "add", "v", "b")), ("o",))
    assert ir.parse_stmt(synth.to_repr(lam)) == lam
    (st,) = _regstores(epilogue_matmul_package(tmp_path / "e", "bias_relu_mask"))
    assert isinstance(st.epilogue, ir.Lambda) and st.epilogue.results == ("ov",)


@pytest.mark.parametrize("form", EPILOGUE_FORMS)
def test_forms_lower(tmp_path, form):
    ptx = _ptx(epilogue_matmul_package(tmp_path / form, form))
    assert "// family:" not in ptx
    body = _lines(ptx)
    count = lambda pat: sum(bool(re.match(pat, ln)) for ln in body)   # noqa: E731
    # eight m16n8 accumulators per thread: 16 register pairs, 32 elements
    if form == "bias_relu_mask":
        assert count(r"cvt\.rn\.f16x2\.f32 %r\d+, %f\d+, %f\d+;") == 16          # hi, lo of each pair
        assert count(r"st\.global\.b32 \[%rd\d+\], %r\d+;") == 16
        assert count(r"ld\.global\.nc\.f32 %n_bv, ") == 32                       # bias[col] per element
        assert count(r"setp\.le\.s32 %p\d+, %n_col, %n_row;") == 32
    elif form == "guarded":
        assert count(r"@%p\d+ st\.global\.f32 \[%rd\d+(\+4)?\], %fr_c_\d_\d;") == 32
        assert count(r"setp\.lt\.s32 %p\d+, %r\d+, 100;") == 16                   # one row test per pair
        assert count(r"setp\.lt\.s32 %p\d+, %r\d+, 90;") == 32
        assert "st.global.v2" not in ptx
    elif form == "atomic":
        assert count(r"red\.global\.add\.f32 \[%rd\d+(\+4)?\], %fr_c_\d_\d;") == 32
        assert "st.global.v2" not in ptx
    else:
        assert count(r"mul\.rn\.f32 %n_pv, %n_v, %n_w;") == 32
        assert count(r"mov\.f32 %n_w, %fr_d_\d_\d;") == 32
        assert count(r"st\.global\.v2\.f32 \[%rd\d+\], \{%f\d+, %f\d+\};") == 16
    _ptxas(ptx, tmp_path)


def test_wgmma_epilogue_lowers(tmp_path):
    """The m64nN warpgroup accumulator through an epilogue into an f16 buffer: 64 registers per
    thread at BN = 128, so 32 scaled pairs, each one f16x2 store."""
    ptx = _ptx(wgmma_gemm_package(tmp_path / "w", 256, 512, 512, out_scale=0.25))
    body = _lines(ptx)
    assert sum(ln.startswith("mul.rn.f32 %n_o, %n_v, %n_sc") for ln in body) == 64
    assert sum(bool(re.match(r"cvt\.rn\.f16x2\.f32 %r\d+, %f\d+, %f\d+;", ln)) for ln in body) == 32
    assert sum(bool(re.match(r"st\.global\.b32 \[%rd\d+\], %r\d+;", ln)) for ln in body) == 32
    _ptxas(ptx, tmp_path)


def _edit(d, old, new):
    f = _ir(d)
    text = f.read_text()
    assert old in text, old
    f.write_text(text.replace(old, new))


def test_refusals(tmp_path):
    d = epilogue_matmul_package(tmp_path / "a", "extra")
    _edit(d, "params=('v', 'w')", "params=('v',)")
    with pytest.raises(ValueError, match="takes 1 parameters for 2 fragments"):
        _ptx(d)

    d = epilogue_matmul_package(tmp_path / "b", "extra")
    _edit(d, "results=('pv',)", "results=('pv', 'v')")
    with pytest.raises(NotImplementedError, match="with 2 results"):
        _ptx(d)

    d = epilogue_matmul_package(tmp_path / "c", "bias_relu_mask")
    _edit(d, "Let(name='half'", "Write(output='y', index=(Var(name='col'),), values=('v',), value_dtype=None, "
             "atomic=False, swizzle='NONE'), Let(name='half'")
    with pytest.raises(NotImplementedError, match="epilogue statement Write"):
        _ptx(d)

    d = epilogue_matmul_package(tmp_path / "d", "guarded")
    _edit(d, "extra_frags=()", "extra_frags=('c[_s]',)")
    with pytest.raises(ValueError, match="extra_frags without an epilogue"):
        _ptx(d)

    d = epilogue_matmul_package(tmp_path / "e", "guarded")
    _edit(d, "epilogue=None", "epilogue=Opaque(kind='x')")
    with pytest.raises(NotImplementedError):
        _ptx(d)


@pytest.mark.parametrize("form", EPILOGUE_FORMS)
def test_oracle_interprets_fused_forms(tmp_path, form):
    """The oracle interpreter's restatement of the fused forms (epilogue Lambda with a bias load,
    relu and a coordinate Select; edge guards; atomic K slices; an extra fragment) gives the
    numpy expression of each kernel on the same inputs -- the same expectation the GPU tests
    check the compiled kernels against.  Integer inputs make every form but the f16 one exact."""
    import numpy as np
    from oracle.interp import run_package as oracle_run
    from thompiler import problems
    d = epilogue_matmul_package(tmp_path / form, form, 128, 128, 256)
    x = problems.make_inputs(problems.load_package(d))
    got = oracle_run(d)["y"]
    acc = x["x0"].astype(np.int64) @ x["x1"].astype(np.int64).T
    if form == "bias_relu_mask":
        t = np.float32(0.5) * acc.astype(np.float32) + x["bias"].astype(np.float32)
        rows, cols = np.indices(t.shape)
        want = np.where(cols <= rows, np.maximum(t, np.float32(0)), np.float32(0)).astype(np.float16)
        assert got.dtype == np.float16
        np.testing.assert_array_equal(got, want)
    elif form == "guarded":
        np.testing.assert_array_equal(got, acc[:-28, :-38].astype(np.float32))
    elif form == "atomic":
        np.testing.assert_array_equal(got, acc.astype(np.float32))
    else:
        dd = x["x0"].astype(np.int64) @ x["x2"].astype(np.int64).T
        np.testing.assert_array_equal(got, (acc * dd).astype(np.float32))
