"""The tuned families' launch plans, on the CPU: which family a package gets, its tuned launch,
its shared-memory layout and the work split -- the numbers the GPU kernels are built around."""

import re

import pytest

from conftest import GOLDEN
from thompiler import load, synth
from thompiler.families import recognise
from thompiler.families.attention import TcAttention
from thompiler.families.matmul import TcMatmul
from thompiler.families.pointwise import Pointwise
from thompiler.families.strided import StridedReduce
from thompiler.families.tuning import TUNING


def _kernel(path):
    return load.load(str(path))


def _ir(d):
    return next(d.glob("*.ir.json"))


@pytest.mark.parametrize("M,N,K,rem,parts", [(4096, 4096, 4096, 68, 2), (8192, 3072, 1024, 0, 1),
                                            (2048, 2560, 2048, 12, 2), (256, 256, 512, 0, 1)])
def test_matmul_split_tail_plan(tmp_path, monkeypatch, M, N, K, rem, parts):
    monkeypatch.setattr(TUNING, "matmul_pair", False)
    fam = recognise(_kernel(_ir(synth.matmul_package(tmp_path / "mm", M, N, K))))
    assert isinstance(fam, TcMatmul)
    assert (fam.rem, fam.parts) == (rem, parts)
    assert fam.units == fam.tiles - rem + rem * parts
    assert fam.units - (fam.tiles - rem) <= 148                 # the split tail is one round at most
    # shared memory: stages | staging | barriers, all inside the dynamic allocation
    assert fam.stages * (fam.a_bytes + fam.b_bytes) + fam.staging + 1024 + 256 == fam.smem <= 227 * 1024


def test_attention_plan_benchmark_shape(tmp_path, monkeypatch):
    fam = recognise(_kernel(_ir(synth.attention_package(tmp_path / "a", 8, 16, 2048, 128))))
    assert isinstance(fam, TcAttention)
    assert (fam.qt, fam.threads, fam.ks, fam.vs, fam.tiles) == (2, 384, 2, 2, 1024)
    assert (fam.maxnreg, fam.reg_split) == (168, (224, 56))
    # per sub-partition: 2 softmax warps at 224 + 1 producer warp at 56 registers <= 512 per thread,
    # and the split hands over exactly what the launch holds (168 per thread)
    assert 2 * 224 + 56 <= 512 and 256 * 224 + 128 * 56 == 384 * 168
    assert fam.smem == 2 * 32768 + 4 * 32768 + fam.stage_bytes + 1024 + 256 <= 227 * 1024
    ptx = fam.emit()
    assert ".maxnreg 168" in ptx and "setmaxnreg.inc.sync.aligned.u32 224" in ptx
    # P handed over and O released by the 128 softmax threads of a group: four barriers of 128
    inits = re.findall(r"mbarrier\.init\.shared::cta\.b64 \[[^\]]+\], (\d+);", ptx)
    assert inits.count("128") == 2 + 2
    # one-lane instructions under elect.sync (K / V producer, MMA issuer, Q loader, epilogue);
    # each query tile's Q loaded on its own, the next tile's prefetched into L2
    assert ptx.count("elect.sync") == 4
    assert "cp.async.bulk.prefetch.tensor.2d.L2.global" in ptx


@pytest.mark.parametrize("shape,qt,threads", [((1, 1, 128, 64), 1, 224), ((2, 2, 384, 64), 1, 224),
                                              ((2, 2, 512, 64), 2, 384), ((1, 3, 512, 128), 2, 384)])
def test_attention_plan_small(tmp_path, shape, qt, threads):
    fam = recognise(_kernel(_ir(synth.attention_package(tmp_path / "a", *shape))))
    assert (fam.qt, fam.threads) == (qt, threads)
    assert fam.smem <= 227 * 1024
    assert (fam.reg_split is not None) == (qt == 2)


def test_pointwise_plan_on_shipped_packages():
    for name, align in (("p01_vector_add", 8), ("p03_relu_mul", 16), ("x01_f64_relu_mul_add", 16)):
        fam = recognise(_kernel(_ir(GOLDEN / name)))
        assert isinstance(fam, Pointwise), name
        assert set(fam.vparams.values()) == {align}, (name, fam.vparams)
        ptx = fam.emit()
        assert "and.b64" in ptx and re.search(r"ld\.global\.nc\.v[24]\.", ptx)


def test_strided_sum_plans():
    r01 = recognise(_kernel(_ir(GOLDEN / "r01_array_sum")))
    assert isinstance(r01, StridedReduce) and not r01.row_mode
    side = r01.sidecar()
    assert side["peer"]["max_ranks"] == 8 and side["error_word"] == "thc_error"
    f02 = recognise(_kernel(_ir(GOLDEN / "f02_row_softmax")))
    assert isinstance(f02, StridedReduce) and f02.row_mode and f02.sidecar() is None
    r03 = recognise(_kernel(_ir(GOLDEN / "r03_mean")))
    assert "peer" not in (r03.sidecar() or {})                 # a mean is not combined across GPUs


@pytest.mark.parametrize("M,N,K,lay,bn,want_bn,tiles,stages,rem,parts", [
    (4096, 4096, 4096, "col", 0, 256, 256, 6, 0, 1), (8192, 3072, 1024, "col", 0, 256, 384, 6, 0, 1),
    (8192, 3072, 1024, "col", 192, 192, 512, 6, 0, 1), (8192, 3072, 1024, "row", 0, 256, 384, 6, 0, 1),
    (6400, 768, 1024, "col", 0, 192, 100, 6, 0, 1),
    (2048, 2560, 2048, "col", 0, 256, 80, 6, 0, 1), (256, 128, 256, "row", 0, 128, 1, 8, 0, 1),
    (512, 256, 256, "col", 128, 128, 4, 8, 0, 1)])
def test_matmul_pair_plan(tmp_path, monkeypatch, M, N, K, lay, bn, want_bn, tiles, stages, rem, parts):
    """The CTA-pair matmul (the default where it applies): 256 x BN pair tiles, each CTA's stage A 128 x 64 plus half
    of B; one pair per two SMs; a cluster launch of an even grid; shared memory (with the
    generic path's static arrays) inside one SM's 227 KB.  The width scores wave efficiency times
    the width's own (192: 0.8 of 256, measured): 8192 x 3072 x 1024 keeps 256 (5.19 waves of 74
    pairs; 192's 6.92 waves do not make up for it), 6400 x 768 x 1024 takes 192 (75 tiles at 256
    fill 1.01 waves of pairs, 100 at 192 fill 1.35); 192 needs K-major B."""
    from thompiler.families.matmul_pair import TcMatmulPair
    d = synth.matmul_package(tmp_path / "mm", M, N, K, b_layout=lay)
    monkeypatch.setattr(TUNING, "matmul_pair", False)
    assert not isinstance(recognise(_kernel(_ir(d))), TcMatmulPair)
    monkeypatch.setattr(TUNING, "matmul_pair", True)                           # on by default
    if bn:
        monkeypatch.setattr(TUNING, "matmul_bn", bn)
    fam = recognise(_kernel(_ir(d)))
    assert isinstance(fam, TcMatmulPair)
    assert (fam.tiles, fam.stages, fam.BN) == (tiles, stages, want_bn)
    assert fam.b_bytes == fam.BN // 2 * 64 * 2 and fam.a_bytes == 128 * 64 * 2
    assert (fam.rem, fam.parts) == (rem, parts)                  # the last wave cut along K
    # or, where its tiles halved fit one wave (K-major B, 256 wide), along N into 256 x 128 units
    hrem = {(8192, 3072, 1024): 14, (4096, 4096, 4096): 34, (2048, 2560, 2048): 6}.get((M, N, K), 0) \
        if (lay, want_bn) == ("col", 256) else 0
    assert fam.hrem == hrem
    assert fam.units == tiles - rem - hrem + rem * parts + 2 * hrem
    assert fam.ctas == 2 * min(fam.units, 74)
    side = fam.sidecar()
    assert side["cluster"] == [2, 1, 1] and side["grid"] == [fam.ctas, 1, 1]
    assert fam.smem + fam.static_smem <= 227 * 1024
    if lay == "col":
        assert side["tmaps"][1]["box"] == [64, fam.BN // 2]
    ptx = fam.emit()
    assert ".reqnctapercluster 2, 1, 1" in ptx and "tcgen05.mma.cta_group::2.kind::f16" in ptx
    assert ptx.count("elect.sync") == 3                          # producer, MMA issuer, epilogue
    assert "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global" in ptx   # each CTA's own loads
    assert not re.search(r"cp\.async\.bulk[^\n]*multicast", ptx)     # no load is multicast
    assert ("thc_tail_ws" in ptx) == bool(rem)


def test_matmul_pair_declines_odd_generic_grid(tmp_path, monkeypatch):
    """A cluster launch needs an even grid under meta.json's launch too: a package whose generic
    grid is odd keeps the single-CTA kernel."""
    import json
    from thompiler.families.matmul_pair import TcMatmulPair
    monkeypatch.setattr(TUNING, "matmul_pair", True)
    d = synth.matmul_package(tmp_path / "mm", 256, 256, 256)        # generic grid 4 x 4 = 16: even
    assert isinstance(recognise(_kernel(_ir(d))), TcMatmulPair)
    meta = json.loads((d / "meta.json").read_text())
    meta["kernels"][0]["grid"] = [11, 1, 1]
    (d / "meta.json").write_text(json.dumps(meta))
    fam = recognise(_kernel(_ir(d)))
    assert isinstance(fam, TcMatmul) and not isinstance(fam, TcMatmulPair)


@pytest.mark.parametrize("name,tile,grid", [("m01_matmul_512", [32, 32, 16], 256), ("m02_matmul_rect", [32, 32, 16], 8)])
def test_matmul_f32_plan(name, tile, grid):
    """The reference's f32 matmul schedules (m01: 512^3 in 32 x 32 cp.async tiles; m02: 128 x 64 x
    256 as 32 split-K slices added atomically into a zeroed C) compile to the FMA-pipe family:
    one thread per 2 x 2 outputs with the full K sum in registers, no atomics."""
    from thompiler.families.matmul_f32 import MatmulF32
    fam = recognise(_kernel(_ir(GOLDEN / name)))
    assert isinstance(fam, MatmulF32)
    side = fam.sidecar()
    assert side["tile"] == tile and side["grid"] == [grid, 1, 1] and side["block"] == [256, 1, 1]
    ptx = fam.emit()
    tuned = ptx[:ptx.index("generic lowering")]
    assert "fma.rn.f32" in tuned and "red.global" not in tuned and "atom." not in tuned
    assert (fam.a.name, fam.b.name, fam.c.name) == ("x0", "x1", "matmul")


def test_matmul_f32_declines_an_accumulating_output(tmp_path):
    """Atomic Writes into an output meta.json does not zero mean C += A B: the full-sum body would
    drop C's old value, so the family declines and the generic lowering runs."""
    import json
    import shutil
    d = tmp_path / "m02"
    shutil.copytree(GOLDEN / "m02_matmul_rect", d)
    meta = json.loads((d / "meta.json").read_text())
    meta["kernels"][0]["zero_outputs"] = []
    (d / "meta.json").write_text(json.dumps(meta))
    assert recognise(_kernel(_ir(d))) is None


@pytest.mark.parametrize("M,N,K,rem,parts", [(4096, 4096, 4096, 34, 2), (2048, 2560, 2048, 6, 2),
                                            (8192, 3072, 1024, 0, 1)])
def test_matmul_pair_k_split_plan(tmp_path, monkeypatch, M, N, K, rem, parts):
    """With the half tail off the pair kernel cuts a partial last wave along K, where K holds at
    least two parts of 16 blocks (the rectangle's 16 blocks do not: it keeps whole tiles)."""
    from thompiler.families.matmul_pair import TcMatmulPair
    monkeypatch.setattr(TUNING, "matmul_pair", True)
    monkeypatch.setattr(TUNING, "matmul_half_tail", False)
    fam = recognise(_kernel(_ir(synth.matmul_package(tmp_path / "mm", M, N, K))))
    assert isinstance(fam, TcMatmulPair)
    assert (fam.rem, fam.parts, fam.hrem) == (rem, parts, 0)
    assert ("thc_tail_ws" in fam.emit()) == bool(rem)
