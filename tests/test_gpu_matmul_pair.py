"""GPU parity of the CTA-pair tcgen05 matmul (``tcgen05-matmul-pair``: cta_group::2 MMAs of
256 x BN over two SMs, each CTA loading its own A rows and half of B).

* small shapes through the host-buffer run against the oracle interpreter on the same seeded
  inputs (both B layouts, f32 and f16 out, BN 256 and 128), and the same module under
  meta.json's launch (its generic mma.sync lowering);
* the benchmark shapes against the generic lowering and a float64 row checksum, twice (the
  second launch must give the same bits);
* a persistent grid of two pairs over many tiles, so accumulator and stage phases carry over.
Every tuned launch checks the kernel's wait-time-out word stays 0.  Tolerances as for the
single-CTA kernel: rtol 2e-2 / atol 2e-3 against the oracle, 1e-4 absolute for f32 out.
"""

import numpy as np
import pytest

from oracle.interp import run_package as oracle_run
from thompiler import problems, runner, synth
from thompiler.device import DeviceKernel
from thompiler.families.tuning import TUNING

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3
FAMILY = "family: tcgen05-matmul-pair"


@pytest.fixture(autouse=True)
def _pair(monkeypatch):
    monkeypatch.setattr(TUNING, "matmul_pair", True)                    # on by default


@pytest.mark.parametrize("M,N,K,lay,out,bn", [(256, 256, 512, "col", "f32", 0), (256, 128, 256, "row", "f32", 0),
                                              (512, 512, 256, "col", "f16", 0), (256, 256, 320, "row", "f16", 0),
                                              (512, 256, 256, "col", "f32", 128), (512, 384, 256, "col", "f32", 192),
                                              (768, 576, 320, "col", "f16", 192)])
def test_pair_small_vs_oracle(tmp_path, monkeypatch, M, N, K, lay, out, bn):
    if bn:
        monkeypatch.setattr(TUNING, "matmul_bn", bn)
    d = synth.matmul_package(tmp_path / "mm", M, N, K, b_layout=lay, out_dtype=out)
    pkg = problems.load_package(d)
    ptx = problems.compile_package(pkg)
    assert FAMILY in ptx["k_matmul_f16"] and "tcgen05.mma.cta_group::2" in ptx["k_matmul_f16"]
    tuned = problems.run_package(pkg, ptx)
    assert tuned["launch"]["k_matmul_f16"].tmaps
    meta = problems.run_package(pkg, ptx, honour_meta=True)
    want = oracle_run(d)["matmul"]
    for res in (tuned, meta):
        got = res["outputs"]["matmul"].astype(np.float64)
        np.testing.assert_allclose(got, want.astype(np.float64), rtol=RTOL, atol=ATOL)
    if out == "f32":
        x = problems.make_inputs(pkg)
        b = x["x1"].astype(np.float64)
        ref = x["x0"].astype(np.float64) @ (b.T if lay == "col" else b)
        assert np.max(np.abs(tuned["outputs"]["matmul"] - ref)) < 1e-3


def _run_twice(k, a, b, M, N, s):
    import torch
    outs = []
    for _ in range(2):
        c = torch.full((M, N), float("nan"), device="cuda")
        k({"x0": a.data_ptr(), "x1": b.data_ptr(), "matmul": c.data_ptr()}, s)
        torch.cuda.synchronize()
        outs.append(c)
    assert runner.read_error_word(k.module, k.plan) == 0
    assert not torch.isnan(outs[0]).any()
    assert torch.equal(outs[0], outs[1])
    return outs[0]


@pytest.mark.parametrize("M,N,K,grid", [(4096, 4096, 4096, 0), (8192, 3072, 1024, 0), (1024, 1024, 512, 4)])
def test_pair_large(tmp_path, M, N, K, grid):
    import torch
    d = synth.matmul_package(tmp_path / "mm", M, N, K, b_layout="col", out_dtype="f32")
    ir = d / "k_matmul_f16.ir.json"
    tuned = DeviceKernel(ir)
    assert tuned.family == "tcgen05-matmul-pair"
    if grid:
        tuned.plan.grid = (grid, 1, 1)
    g = torch.Generator(device="cuda").manual_seed(3)
    a = (torch.randn(M, K, device="cuda", generator=g) * 0.02).half()
    b = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    s = torch.cuda.current_stream().cuda_stream
    c1 = _run_twice(tuned, a, b, M, N, s)
    generic = DeviceKernel(ir, tuned=False)
    c2 = torch.full((M, N), float("nan"), device="cuda")
    generic({"x0": a.data_ptr(), "x1": b.data_ptr(), "matmul": c2.data_ptr()}, s)
    torch.cuda.synchronize()
    err = (c1.double() - c2.double()).abs().max().item()
    assert err < 1e-4, err
    ones_ref = a.double() @ b.double().sum(0)
    assert torch.allclose(c1.double().sum(1), ones_ref, rtol=1e-4, atol=1e-3)
    # every element against an independent float64 product, at the f16-input tolerance
    ref = a.double() @ b.double().t()
    assert torch.allclose(c1.double(), ref, rtol=2e-2, atol=2e-3)
    err64 = (c1.double() - ref).abs().max().item()
    print(f"{M}x{N}x{K}: max |C - C_f64| = {err64:.3e}")
    assert err64 < 1e-4, err64                           # exact f16 products summed in f32
    tuned.close()
    generic.close()


@pytest.mark.parametrize("grid", [0, 10])
def test_pair_split_tail(tmp_path, monkeypatch, grid):
    """More pair tiles than pairs with a partial last wave (2048 x 2560 x 2048: 80 tiles of
    256 x 256 on 74 pairs, 6 left over), with the half tail switched off: those are cut along K
    into two parts whose partials
    meet in the module's workspace per tile and CTA rank, the last part to arrive adding them in
    part order.  grid 10 (5 pairs) puts several whole tiles and several parts on each pair."""
    import torch
    M, N, K = 2048, 2560, 2048
    monkeypatch.setattr(TUNING, "matmul_half_tail", False)          # the K split (else the half tail)
    d = synth.matmul_package(tmp_path / "mm", M, N, K, b_layout="col", out_dtype="f32")
    k = DeviceKernel(d / "k_matmul_f16.ir.json")
    assert k.family == "tcgen05-matmul-pair" and "thc_tail_ws" in k.ptx
    if grid:
        k.plan.grid = (grid, 1, 1)
    g = torch.Generator(device="cuda").manual_seed(4)
    a = (torch.randn(M, K, device="cuda", generator=g) * 0.02).half()
    b = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    c = _run_twice(k, a, b, M, N, torch.cuda.current_stream().cuda_stream)   # the part order fixes the rounding
    ref = a.double() @ b.double().t()
    assert (c.double() - ref).abs().max().item() < 1e-4
    k.close()


@pytest.mark.parametrize("grid", [0, 10])
def test_pair_half_tail(tmp_path, grid):
    """A partial last wave whose K is too short to cut (2048 x 2560 x 1024: 80 pair tiles on 74
    pairs, 16 K blocks): its 6 tiles run as 12 units of 256 x 128 over the full K, N = 128 MMAs
    on the same B boxes loaded at the half's column offset, no workspace.  grid 10 (5 pairs)
    puts whole tiles and halves on each pair; the last tile column's second half reads rows
    past N as the tensor map's zero fill."""
    import torch
    M, N, K = 2048, 2560, 1024
    d = synth.matmul_package(tmp_path / "mm", M, N, K, b_layout="col", out_dtype="f32")
    k = DeviceKernel(d / "k_matmul_f16.ir.json")
    assert k.family == "tcgen05-matmul-pair" and "thc_tail_ws" not in k.ptx
    if grid:
        k.plan.grid = (grid, 1, 1)
    g = torch.Generator(device="cuda").manual_seed(5)
    a = (torch.randn(M, K, device="cuda", generator=g) * 0.02).half()
    b = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    c = _run_twice(k, a, b, M, N, torch.cuda.current_stream().cuda_stream)
    ref = a.double() @ b.double().t()
    assert (c.double() - ref).abs().max().item() < 1e-4
    k.close()
