"""The register-fragment statements (FragmentPromote / FragmentRowReduce / FragmentApply /
FragmentRepack) on the CPU: they parse from the IR's repr, the two kernels of tests/sm90_ir.py
that use them (an mma.sync flash attention and an f16-accumulate GEMM promoted into f32) lower
through the generic path to PTX that ptxas accepts for sm_100a, the emitted code follows the
accumulator geometry, and the forms outside it are refused at compile time."""

import re
import shutil
import subprocess

import pytest

from sm90_ir import (FRAGMENT_ATTENTION_EXTRAS, blockscaled_matmul_package, chained_matmul_package,
                     fragment_attention_package, promote_matmul_package)
from thompiler import ir, load, synth
from thompiler.compiler import compile_kernel

LAYOUT = ir.FragLayout(4, (0, 0, 1, 1), (1, 2), None, (), None, None)


def _ir(d):
    return next(d.glob("*.ir.json"))


def _ptx(d):
    return compile_kernel(load.load(str(_ir(d))))


def _ptxas(ptx, tmp_path):
    if shutil.which("ptxas") is None:
        pytest.skip("ptxas not on PATH")
    f = tmp_path / "k.ptx"
    f.write_text(ptx)
    r = subprocess.run(["ptxas", "-arch=sm_100a", "-v", str(f), "-o", str(tmp_path / "k.cubin")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "0 bytes spill stores" in r.stderr, r.stderr


def _lines(ptx):
    return [ln.strip() for ln in ptx.splitlines() if ln.startswith("\t") and not ln.strip().startswith("//")]


def test_statements_parse_from_repr():
    stmts = [ir.FragmentPromote("c[0]", "c16[0]"),
             ir.FragmentApply("s[_e]", synth.E("subtract"), ("s[_e]", ("mt", "mb")), ("frag", "row"), False, LAYOUT,
                              synth.E("exp"), None, None),
             ir.FragmentRowReduce("mt", "mb", ("s[0]", "s[1]"), synth.E("maximum"), LAYOUT, synth.F32T),
             ir.FragmentRepack("pa[_p]", ("s[0]", "s[1]"), "f16", "m16n8k16", synth.V("_p"))]
    for s in stmts:
        assert ir.parse_stmt(synth.to_repr(s)) == s


def test_fragment_attention_lowers(tmp_path):
    ptx = _ptx(fragment_attention_package(tmp_path / "a"))
    assert "// family:" not in ptx
    body = _lines(ptx)
    # per key block: two row reductions (max, sum) of two rows each over the quad (xor 1, 2)
    assert sum(ln.startswith("shfl.sync.bfly.b32") for ln in body) == 8
    assert sum(bool(re.match(r"shfl\.sync\.bfly\.b32 %f\d+, %f\d+, [12], 31, -1;", ln)) for ln in body) == 8
    # P as four A fragments of four f16x2 words, each from a C register pair (hi, lo)
    reps = [ln for ln in body if ln.startswith("cvt.rn.f16x2.f32 %fr_pa_")]
    assert len(reps) == 16
    assert "cvt.rn.f16x2.f32 %fr_pa_0_0, %fr_s_0_1, %fr_s_0_0;" in reps
    assert "cvt.rn.f16x2.f32 %fr_pa_1_3, %fr_s_3_3, %fr_s_3_2;" in reps
    # probabilities: exp of the score minus its own row's maximum (top registers 0, 1; bottom 2, 3)
    assert "sub.rn.f32" in ptx and re.search(r"sub\.rn\.f32 %f\d+, %fr_s_3_2, %n_mn_b;", ptx)
    assert re.search(r"sub\.rn\.f32 %f\d+, %fr_s_3_1, %n_mn_t;", ptx)
    # the output strip is divided by the row sums before it is stored
    assert re.search(r"div\.rn\.f32 %f\d+, %fr_o_7_3, %n_l_b;", ptx)
    _ptxas(ptx, tmp_path)


def test_promote_lowers(tmp_path):
    ptx = _ptx(promote_matmul_package(tmp_path / "p"))
    assert "// family:" not in ptx
    body = _lines(ptx)
    assert sum(ln.startswith("mma.sync.aligned.m16n8k16.row.col.f16.f16.f16.f16") for ln in body) == 32
    # eight f16 accumulators of two words: 16 splits, 32 exact widenings and f32 adds, 16 clears
    # (plus the 16 zero fills of their RegFragment)
    assert sum(ln.startswith("mov.b32 {%h") for ln in body) == 16
    assert sum(ln.startswith("cvt.f32.f16") for ln in body) == 32
    assert sum(bool(re.match(r"add\.rn\.f32 %fr_c_\d_\d, %fr_c_\d_\d, %f\d+;", ln)) for ln in body) == 32
    assert sum(bool(re.match(r"mov\.b32 %fr_c16_\d_\d, 0;", ln)) for ln in body) == 16 + 16
    _ptxas(ptx, tmp_path)


def _edit(d, old, new):
    f = _ir(d)
    text = f.read_text()
    assert old in text, old
    f.write_text(text.replace(old, new))


def test_refusals(tmp_path):
    d = fragment_attention_package(tmp_path / "a")
    _edit(d, "kinds=('frag', 'row'), in_place=False, layout=None", "kinds=('frag', 'mask'), in_place=False, layout=None")
    with pytest.raises(ValueError, match="needs row_base and col_base"):
        _ptx(d)

    d = fragment_attention_package(tmp_path / "a2")
    _edit(d, "kinds=('frag', 'row'), in_place=False, layout=None", "kinds=('frag', 'halo'), in_place=False, layout=None")
    with pytest.raises(NotImplementedError, match="kind 'halo'"):
        _ptx(d)

    d = fragment_attention_package(tmp_path / "b")
    _edit(d, "elem_row=(0, 0, 1, 1), reduce_xors=(1, 2)", "elem_row=(0, 1, 0, 1), reduce_xors=(1, 2)")
    with pytest.raises(NotImplementedError, match="element rows"):
        _ptx(d)

    d = fragment_attention_package(tmp_path / "c")
    _edit(d, "op=ElementwiseImpl('maximum'), layout=None", "op=ElementwiseImpl('multiply'), layout=None")
    with pytest.raises(NotImplementedError, match="FragmentRowReduce with multiply"):
        _ptx(d)

    d = fragment_attention_package(tmp_path / "d")
    _edit(d, "FragmentRepack(frag='pa[_p]'", "FragmentRepack(frag='qa[_p]'")   # fine: qa is an A fragment
    _ptx(d)
    _edit(d, "FragmentRepack(frag='qa[_p]'", "FragmentRepack(frag='o[_p]'")
    with pytest.raises(ValueError, match="not a 16-bit m16n8k16 A fragment"):
        _ptx(d)

    d = promote_matmul_package(tmp_path / "e")
    _edit(d, "FragmentPromote(dst='c[_q]', src='c16[_q]')", "FragmentPromote(dst='c[_q]', src='c[_q]')")
    with pytest.raises(ValueError, match="not the packed f16 shadow"):
        _ptx(d)


@pytest.mark.parametrize("extra", FRAGMENT_ATTENTION_EXTRAS)
def test_fragment_apply_coordinate_arguments(tmp_path, extra):
    """FragmentApply mask and bias arguments: each score's coordinates are row_base + the element's
    row (lane / 4, + 8 for the bottom registers) and col_base + its column (8 i + 2 (lane % 4) +
    j), and the argument is evaluated per element at them -- a Lambda (a Select of 0 / -1e30), a
    predicate (selp 1 / 0), a global load at (row, col) or at (col) of a 1-d buffer."""
    ptx = _ptx(fragment_attention_package(tmp_path / "a", 256, 64, extra))
    body = ptx.splitlines()
    if extra == "causal":
        assert sum("selp.f32" in ln and "0fF149F2CA" in ln for ln in body) == 8 * 4   # -1e30 where masked
    elif extra == "causal_pred":
        assert sum(ln.strip().startswith("selp.f32") and "0f3F800000, 0f00000000" in ln for ln in body) == 8 * 4
    else:
        loads = [ln for ln in body if "ld.global.nc.f32" in ln]
        assert len(loads) == 8 * 4                          # one per score element
    _ptxas(ptx, tmp_path)


def test_blockscaled_fp4_lowering(tmp_path):
    """The block-scaled fp4 statements: fp4 LdmatrixLoad (x4 for A, x2 for B, from byte Smem
    arrays), BlockScaleLoad (four scale bytes for A, two for B, from u8 buffers), and the
    m16n8k64 e2m1 MmaSyncPtx emulated per warp on the FMA pipes (64 x 4 FMAs per lane through a
    per-warp shared scratch, decoded through a 16-entry e2m1 table)."""
    ptx = _ptx(blockscaled_matmul_package(tmp_path / "b", 128, 128, 128))
    body = ptx.splitlines()
    assert sum("ldmatrix.sync.aligned.m8n8.x4.shared.b16" in ln for ln in body) == 2
    assert sum("ldmatrix.sync.aligned.m8n8.x2.shared.b16" in ln for ln in body) == 2 * 8
    assert sum("ld.global.nc.u8" in ln for ln in body) == 2 * (4 + 8 * 2)
    assert sum(ln.strip().startswith("fma.rn.f32") for ln in body) == 2 * 8 * 64 * 4
    assert ".const .align 4 .b32 thc_e2m1[16] = {0x00000000, 0x3F000000" in ptx
    assert "mma.sync" not in ptx                               # sm_100a has no block-scaled mma.sync
    _ptxas(ptx, tmp_path)


def test_fp4_decode_table():
    from thompiler.handlers.blockscale import e2m1_value
    assert [e2m1_value(n) for n in range(8)] == [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    assert [e2m1_value(n) for n in range(8, 16)] == [-0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]


def test_regstore_into_swizzled_shared_memory(tmp_path):
    """RegStore into a shared array with the 128-byte swizzle: each register pair of the first
    product becomes one f16x2 store at the swizzled element (row 16 w + g (+ 8), column 8 s + 2 t),
    which the second product's ldmatrix reads back under the same swizzle.  A swizzle on a
    global output and the Volta layout stay refused."""
    d = chained_matmul_package(tmp_path / "c")
    ptx = _ptx(d)
    body = ptx.splitlines()
    assert sum("st.shared.b32" in ln for ln in body) == 8 * 2
    assert sum(ln.strip().startswith("cvt.rn.f16x2.f32") for ln in body) == 8 * 2
    _ptxas(ptx, tmp_path)
    _edit(d, "swizzle='NONE', row_dim=None, col_dim=None)", "swizzle='B128', row_dim=None, col_dim=None)")
    with pytest.raises(NotImplementedError, match="into global memory"):
        _ptx(d)
    d = chained_matmul_package(tmp_path / "v")
    _edit(d, "volta_interleaved=False, fragment_index=None, swizzle='NONE'",
          "volta_interleaved=True, fragment_index=None, swizzle='NONE'")
    with pytest.raises(NotImplementedError, match="Volta"):
        _ptx(d)
