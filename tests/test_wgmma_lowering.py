"""The warpgroup tensor-core statements (WgmmaDescriptor / WgmmaFence / WgmmaMma / WgmmaCommit /
WgmmaWait) on the CPU: the sm_90-style GEMM kernels of tests/sm90_ir.py lower through the
generic path onto tcgen05 (tensor-memory accumulators, single-thread M = 64 MMAs, bounded
mbarrier waits), ptxas accepts them for sm_100a, and the forms tcgen05 cannot run are refused
at compile time."""

import json
import re
import shutil
import subprocess

import pytest

from sm90_ir import wgmma_gemm_package
from thompiler import load
from thompiler.compiler import compile_kernel
from thompiler.handlers import wgmma

VARIANTS = [({}, 4, 128), ({"n_wg": 2}, 4, 256), ({"trans_b": True}, 4, 128), ({"tail_overwrite": True}, 5, 128),
            ({"BN": 64}, 4, 64), ({"BN": 256}, 4, 256)]


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


@pytest.mark.parametrize("kw,mmas,cols", VARIANTS, ids=[",".join(f"{k}={v}" for k, v in kw.items()) or "base"
                                                         for kw, _, _ in VARIANTS])
def test_wgmma_gemm_lowers_onto_tcgen05(tmp_path, kw, mmas, cols):
    d = wgmma_gemm_package(tmp_path / "w", 256, 256, 256, **kw)
    ptx = _ptx(d)
    assert "// family:" not in ptx                   # the generic lowering, not a tuned family
    body = [ln.strip() for ln in ptx.splitlines() if ln.startswith("\t") and not ln.strip().startswith("//")]
    assert not any(ln.startswith("wgmma") for ln in body)
    assert sum("tcgen05.mma.cta_group::1.kind::f16" in ln for ln in body) == mmas
    assert f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [thc_wg_tmem], {cols};" in body
    assert f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 %wg_base, {cols};" in body
    assert any(ln.startswith("tcgen05.st.sync.aligned.16x256b") for ln in body)
    assert any(ln.startswith("tcgen05.ld.sync.aligned.16x256b") for ln in body)
    # every mbarrier wait is bounded
    waits = [ln for ln in body if ln.startswith("mbarrier.try_wait")]
    assert waits and len(re.findall(r"setp\.lt\.u32 %p\d+, %r\d+, 262144", ptx)) >= len(waits)
    _ptxas(ptx, tmp_path)


def test_descriptor_words(tmp_path):
    """The 128-byte-swizzle K-major descriptors: LBO 16 >> 4 in bits 16-29 of the low word; high
    word SBO 1024 >> 4, version 1 (bit 46), layout 2 (bits 61-63); the M = 64, N = 128 f16
    instruction descriptor."""
    ptx = _ptx(wgmma_gemm_package(tmp_path / "w", 256, 256, 256))
    hi = (1024 >> 4) | (1 << 14) | (2 << 29)
    assert re.search(rf"mov\.u32 %r\d+, {hi};", ptx)
    assert re.search(r"or\.b32 %r\d+, %r\d+, 65536;", ptx)
    idesc = (1 << 4) | ((128 >> 3) << 17) | ((64 >> 4) << 24)
    assert idesc == 0x4200010 and f", {idesc}, %p" in ptx
    assert wgmma._idesc(128, "f16", False, True) == idesc | (1 << 16)
    assert wgmma._idesc(64, "bf16", True, False) == (1 << 4) | (1 << 7) | (1 << 10) | (1 << 15) | (8 << 17) | (4 << 24)


def test_plan_and_chunks(tmp_path):
    p = wgmma.plan(load.load(str(_ir(wgmma_gemm_package(tmp_path / "w", 256, 256, 256, n_wg=2)))))
    assert (p.cols_per_wg, p.n_wg, p.ncols) == (128, 2, 256) and p.frags == {"acc": (0, 128, 1)}
    assert list(wgmma._chunks(16)) == [(0, 16)]
    assert list(wgmma._chunks(12)) == [(0, 8), (8, 4)]
    assert list(wgmma._chunks(3)) == [(0, 2), (2, 1)]
    assert wgmma._pow2_at_least(24) == 32 and wgmma._pow2_at_least(96) == 128


def test_operand_extents():
    """Bytes one k16 step reads from a descriptor's start: K-major 128-byte swizzle, 64 rows:
    seven 1024-byte row groups, seven 128-byte rows and the 32-byte slice; MN-major with the
    swizzle, 128 columns: two 64-column atoms LBO apart and two 8-row groups SBO apart."""
    k_major = wgmma.Desc("d", None, "0", 2, 16, 1024)
    assert wgmma._extent(k_major, 64, False, "A") == 7 * 1024 + 7 * 128 + 32
    mn_major = wgmma.Desc("d", None, "0", 2, 8192, 1024)
    assert wgmma._extent(mn_major, 128, True, "B") == 8192 + 1024 + 1024
    plain = wgmma.Desc("d", None, "0", 0, 128, 256)
    assert wgmma._extent(plain, 64, False, "A") == 7 * 256 + 128 + 128
    with pytest.raises(NotImplementedError, match="MN-major operand without swizzle"):
        wgmma._extent(plain, 64, True, "B")


def _edit(d, old, new, count=None):
    f = _ir(d)
    text = f.read_text()
    assert old in text, old
    f.write_text(text.replace(old, new) if count is None else text.replace(old, new, count))


def test_refusals(tmp_path):
    d = wgmma_gemm_package(tmp_path / "a", 256, 256, 256)
    _edit(d, "a_desc='ad', a_frag=None", "a_desc=None, a_frag='af'")
    with pytest.raises(NotImplementedError, match="A in registers"):
        _ptx(d)

    d = wgmma_gemm_package(tmp_path / "b", 256, 256, 256)
    _edit(d, "RegFragment(name='acc', role='c', shape=(64, 128, 16), dtype=DataType(name='f32', np=dtype('float32'), "
             "nbytes=4)", "RegFragment(name='acc', role='c', shape=(64, 128, 16), dtype=DataType(name='f16', "
                          "np=dtype('float16'), nbytes=2)")
    with pytest.raises(NotImplementedError, match="only f32 accumulators"):
        _ptx(d)

    d = wgmma_gemm_package(tmp_path / "c", 256, 256, 256)
    _edit(d, "sbo_bytes=Literal(value=1024, dtype='int')", "sbo_bytes=Literal(value=2048, dtype='int')")
    with pytest.raises(ValueError, match="operand A.*do not fit a_s"):
        _ptx(d)

    d = wgmma_gemm_package(tmp_path / "e", 256, 256, 256)
    _edit(d, "lbo_bytes=Literal(value=16, dtype='int')", "lbo_bytes=Literal(value=24, dtype='int')")
    with pytest.raises(ValueError, match="leading byte offset 24"):
        _ptx(d)

    d = wgmma_gemm_package(tmp_path / "f", 256, 256, 256)
    meta = json.loads((d / "meta.json").read_text())
    meta["kernels"][0]["grid"] = [16, 1, 1]          # twice the CTAs the Tile has cells for
    (d / "meta.json").write_text(json.dumps(meta))
    with pytest.raises(NotImplementedError, match="fill the launch exactly"):
        _ptx(d)


def test_runtime_operand_checks(tmp_path):
    """A descriptor at a run-time offset (the warpgroup's rows of A) is checked before the MMA:
    16-byte alignment and the last start byte the operand fits from (8192 - 8096 = 96 for a
    64 x 64 A slab); a failure skips the MMA and sets bit 2 of the error word."""
    ptx = _ptx(wgmma_gemm_package(tmp_path / "w", 256, 256, 256))
    assert re.search(r"setp\.gt\.s32 %p\d+, %r\d+, 96;", ptx)
    assert re.search(r"red\.global\.or\.b32 \[%rd\d+\], 4;", ptx)
