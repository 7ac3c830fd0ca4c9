"""GPU parity of the tcgen05 attention family.

* small shapes: the tuned kernel and the same module under meta.json's
  launch (the generic lowering of the a02-style IR) against the oracle
  interpreter on the same seeded inputs;
* the benchmark shape [8, 16, 2048, 128]: against a plain float32 PyTorch
  evaluation of softmax(Q K^T / sqrt(d)) V on the GPU (all 128 heads), and
  against the float64 numpy expression on the CPU for two heads;
* the kernel's wait-time-out word stays 0.
Tolerance for f16-input attention: rtol 2e-2 / atol 2e-3.
"""

import numpy as np
import pytest

from oracle.interp import run_package as oracle_run
from thompiler import problems, runner, synth
from thompiler.device import DeviceKernel

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3


def _sdpa64(q, k, v):
    q, k, v = (x.astype(np.float64) for x in (q, k, v))
    s = q @ np.swapaxes(k, -1, -2) / np.sqrt(q.shape[-1])
    p = np.exp(s - s.max(-1, keepdims=True))
    return (p / p.sum(-1, keepdims=True)) @ v


@pytest.mark.parametrize("shape", [(1, 1, 128, 64), (1, 1, 256, 128)])
def test_attention_small_vs_oracle(tmp_path, shape):
    d = synth.attention_package(tmp_path / "att", *shape)
    pkg = problems.load_package(d)
    ptx = problems.compile_package(pkg)
    assert "tcgen05.mma" in ptx["k_attention"]
    tuned = problems.run_package(pkg, ptx)
    assert tuned["launch"]["k_attention"].tmaps
    meta = problems.run_package(pkg, ptx, honour_meta=True)
    want = oracle_run(d)["attn"].astype(np.float64)
    for res in (tuned, meta):
        np.testing.assert_allclose(res["outputs"]["attn"].astype(np.float64), want, rtol=RTOL, atol=ATOL)
    x = problems.make_inputs(pkg)
    ref = _sdpa64(x["q"], x["k"], x["v"])
    assert np.max(np.abs(tuned["outputs"]["attn"] - ref)) < 5e-3


@pytest.mark.parametrize("shape", [(2, 2, 384, 64), (1, 3, 512, 128), (2, 2, 512, 64)])
def test_attention_medium_vs_expression(tmp_path, shape):
    d = synth.attention_package(tmp_path / "att", *shape)
    pkg = problems.load_package(d)
    res = problems.run_package(pkg, problems.compile_package(pkg))
    x = problems.make_inputs(pkg)
    np.testing.assert_allclose(res["outputs"]["attn"].astype(np.float64), _sdpa64(x["q"], x["k"], x["v"]),
                               rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("poly", [0, 2, 8])
def test_attention_exponential_paths(tmp_path, monkeypatch, poly):
    """P from the exponential unit alone (0), or with 2 or all 8 of every 8 score pairs from the
    polynomial 2^x on the FMA pipe (the default takes 1): all within the f16 tolerance."""
    from thompiler.families.tuning import TUNING
    monkeypatch.setattr(TUNING, "attention_poly_pairs", poly)
    d = synth.attention_package(tmp_path / "att", 1, 3, 512, 128)
    pkg = problems.load_package(d)
    ptx = problems.compile_package(pkg)
    assert ("0x4B4000004B400000" in ptx["k_attention"]) == (poly > 0)     # 1.5 * 2^23, the rounding constant
    res = problems.run_package(pkg, ptx)
    x = problems.make_inputs(pkg)
    np.testing.assert_allclose(res["outputs"]["attn"].astype(np.float64), _sdpa64(x["q"], x["k"], x["v"]),
                               rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("shape,grid", [((2, 3, 512, 128), 1), ((2, 3, 512, 128), 5), ((1, 2, 384, 64), 4)])
def test_attention_persistent_tiles(tmp_path, shape, grid):
    """Fewer CTAs than (head, query-tile) tiles: each CTA walks several tiles, carrying its
    K / V rings, barrier phases and TMEM accumulators from one tile to the next."""
    import torch
    d = synth.attention_package(tmp_path / "att", *shape)
    k = DeviceKernel(d / "k_attention.ir.json")
    k.plan.grid = (grid, 1, 1)
    g = torch.Generator(device="cuda").manual_seed(11)
    q, kk, v = (torch.randn(*shape, device="cuda", generator=g).half() for _ in range(3))
    c = torch.tensor([shape[-1] ** 0.5], device="cuda")
    o = torch.full(shape, float("nan"), device="cuda", dtype=torch.float16)
    for _ in range(2):                                 # a second launch starts from the first's phases
        k({"div_c1": c.data_ptr(), "q": q.data_ptr(), "k": kk.data_ptr(), "v": v.data_ptr(),
           "attn": o.data_ptr()}, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert runner.read_error_word(k.module, k.plan) == 0
    ref = _sdpa64(q.cpu().numpy(), kk.cpu().numpy(), v.cpu().numpy())
    np.testing.assert_allclose(o.float().cpu().numpy(), ref, rtol=RTOL, atol=ATOL)
    k.close()


def test_attention_benchmark_shape(tmp_path):
    import torch
    B, H, S, D = 8, 16, 2048, 128
    k = DeviceKernel(synth.attention_package(tmp_path / "att", B, H, S, D) / "k_attention.ir.json")
    assert k.plan.tmaps and "tcgen05.mma" in k.ptx
    g = torch.Generator(device="cuda").manual_seed(9)
    q, kk, v = (torch.randn(B, H, S, D, device="cuda", generator=g).half() for _ in range(3))
    c = torch.tensor([D ** 0.5], device="cuda")
    o = torch.full((B, H, S, D), float("nan"), device="cuda", dtype=torch.float16)
    k({"div_c1": c.data_ptr(), "q": q.data_ptr(), "k": kk.data_ptr(), "v": v.data_ptr(), "attn": o.data_ptr()},
      torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert runner.read_error_word(k.module, k.plan) == 0
    assert not torch.isnan(o).any()
    worst = 0.0
    for b in range(B):
        s = (q[b].float() @ kk[b].float().transpose(-1, -2)) / D ** 0.5
        ref = torch.softmax(s, -1) @ v[b].float()
        assert torch.allclose(o[b].float(), ref, rtol=RTOL, atol=ATOL)
        worst = max(worst, (o[b].float() - ref).abs().max().item())
    assert worst < 5e-3, worst
    ref64 = _sdpa64(q[0, :2].cpu().numpy(), kk[0, :2].cpu().numpy(), v[0, :2].cpu().numpy())
    np.testing.assert_allclose(o[0, :2].float().cpu().numpy(), ref64, rtol=RTOL, atol=ATOL)
    k.close()


@pytest.mark.parametrize("grid", [None, 3])
def test_attention_rescale_in_part_of_a_warp(tmp_path, grid):
    """Rows whose running maximum jumps in a later key block rescale O and the running sum; here
    the lanes of a warp disagree: keys 400-403 of each head are set to 1.2 q_r for query rows r =
    0, 5, 17 and 31 (scores about 13.6 there against about N(0, 1) elsewhere), so in key block 3
    only those rows of warp 0 grow by more than 2^8.  The warp takes the rescale path together
    (the other lanes with a factor of 1) and every row matches the float64 expression."""
    import torch
    shape = (1, 2, 1024, 128)
    d = synth.attention_package(tmp_path / "att", *shape)
    k = DeviceKernel(d / "k_attention.ir.json")
    if grid:
        k.plan.grid = (grid, 1, 1)
    g = torch.Generator(device="cuda").manual_seed(19)
    q, kk, v = (torch.randn(*shape, device="cuda", generator=g) for _ in range(3))
    for i, r in enumerate((0, 5, 17, 31)):
        kk[0, :, 400 + i] = 1.2 * q[0, :, r]
    q, kk, v = q.half(), kk.half(), v.half()
    c = torch.tensor([shape[-1] ** 0.5], device="cuda")
    o = torch.full(shape, float("nan"), device="cuda", dtype=torch.float16)
    k({"div_c1": c.data_ptr(), "q": q.data_ptr(), "k": kk.data_ptr(), "v": v.data_ptr(), "attn": o.data_ptr()},
      torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert k.error_word() == 0
    ref = _sdpa64(q.cpu().numpy(), kk.cpu().numpy(), v.cpu().numpy())
    np.testing.assert_allclose(o.float().cpu().numpy(), ref, rtol=RTOL, atol=ATOL)
    k.close()


@pytest.mark.parametrize("units", [16, 32, 64])
def test_attention_shard_shapes(tmp_path, units):
    """The kernels the ranks of a 8-, 4- and 2-GPU run compile for their share of the benchmark's
    128 (batch, head) units: [units, 1, 2048, 128], i.e. 128, 256 and 512 tiles of 256 queries
    over the 148 SMs (one partial wave; one full wave and a partial one; three and a partial
    one).  Every unit against float32 PyTorch; the error word stays 0."""
    import torch
    shape = (units, 1, 2048, 128)
    k = DeviceKernel(synth.attention_package(tmp_path / "att", *shape) / "k_attention.ir.json")
    g = torch.Generator(device="cuda").manual_seed(53 + units)
    q, kk, v = (torch.randn(*shape, device="cuda", generator=g).half() for _ in range(3))
    c = torch.tensor([shape[-1] ** 0.5], device="cuda")
    o = torch.full(shape, float("nan"), device="cuda", dtype=torch.float16)
    k({"div_c1": c.data_ptr(), "q": q.data_ptr(), "k": kk.data_ptr(), "v": v.data_ptr(), "attn": o.data_ptr()},
      torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert k.error_word() == 0 and not torch.isnan(o).any()
    s = (q[:, 0].float() @ kk[:, 0].float().transpose(-1, -2)) / shape[-1] ** 0.5
    ref = torch.softmax(s, -1) @ v[:, 0].float()
    assert torch.allclose(o[:, 0].float(), ref, rtol=RTOL, atol=ATOL), (o[:, 0].float() - ref).abs().max()
    k.close()
