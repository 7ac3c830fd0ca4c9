"""GPU parity of the tuned families on synthesized packages.

Small sizes are checked against the oracle interpreter on the same seeded
inputs; the benchmark sizes ([8192, 4096] row ops, 2^20 and 2^30 sums) are
checked against the problem's torch/numpy expression evaluated on the CPU
in float64, and through size-independent properties (softmax rows sum to 1,
L2-normalised rows have unit norm, a sum is linear in its halves).  Each
tuned kernel is also run under meta.json's launch (the generic path of the
same module) and must agree with its tuned launch.
"""

import json

import numpy as np
import pytest

from oracle.interp import run_package as oracle_run
from thompiler import problems, synth

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


def run(pdir, honour_meta=False, inputs=None):
    pkg = problems.load_package(pdir)
    ptx = problems.compile_package(pkg)
    assert all("family: strided-reduce" in p for p in ptx.values())
    return pkg, problems.run_package(pkg, ptx, inputs=inputs, honour_meta=honour_meta)


@pytest.mark.parametrize("kind", ["softmax", "rmsnorm", "l2norm", "rowsum"])
@pytest.mark.parametrize("shape", [(64, 4096), (33, 512), (16, 8192)])
def test_row_ops_vs_oracle(tmp_path, kind, shape):
    d = synth.row_package(tmp_path / kind, kind, *shape)
    pkg, res = run(d)
    _, meta_res = run(d, honour_meta=True)
    want = oracle_run(d)
    out = pkg.meta["graph_outputs"][0]
    got = res["outputs"][out].reshape(want[out].shape)
    if kind == "rowsum":
        # a sum's rounding error scales with its summands, not with the (cancelling) result:
        # |got - want| <= rtol * ||row||_2, the scale of a sum of random-sign terms
        x = problems.make_inputs(pkg)["x"].astype(np.float64)
        scale = np.sqrt((x * x).sum(-1))
        assert np.all(np.abs(got.astype(np.float64) - want[out]) <= RTOL * scale + ATOL)
        assert np.all(np.abs(meta_res["outputs"][out].reshape(got.shape) - got) <= RTOL * scale + ATOL)
        return
    np.testing.assert_allclose(got, want[out], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(meta_res["outputs"][out].reshape(got.shape), got, rtol=RTOL, atol=ATOL)


def _expr(kind, x, w, eps):
    x = x.astype(np.float64)
    if kind == "softmax":
        e = np.exp(x - x.max(-1, keepdims=True))
        return e / e.sum(-1, keepdims=True)
    if kind == "rmsnorm":
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * w
    if kind == "l2norm":
        return x / np.sqrt((x * x).sum(-1, keepdims=True))
    return x.sum(-1)


@pytest.mark.parametrize("kind", ["softmax", "rmsnorm", "l2norm"])
def test_row_ops_full_size(tmp_path, kind):
    rows, cols, eps = 8192, 4096, 1e-6
    d = synth.row_package(tmp_path / kind, kind, rows, cols, eps=eps,
                          w_init={"dist": "uniform", "low": 0.5, "high": 1.5, "seed": 1})
    pkg, res = run(d)
    inputs = problems.make_inputs(pkg)
    out = pkg.meta["graph_outputs"][0]
    got = res["outputs"][out].astype(np.float64)
    want = _expr(kind, inputs["x"], inputs.get("w"), eps)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    if kind == "softmax":
        np.testing.assert_allclose(got.sum(-1), 1.0, rtol=0, atol=1e-5)
    if kind == "l2norm":
        np.testing.assert_allclose(np.sqrt((got ** 2).sum(-1)), 1.0, rtol=0, atol=1e-5)


@pytest.mark.parametrize("n,kind", [(1 << 20, "sum"), (1 << 20, "mean"), (1000 * 1024 + 4, "sum"),
                                    (4096 * 3 + 2, "sum")])
def test_full_sum_vs_oracle(tmp_path, n, kind):
    d = synth.sum_package(tmp_path / kind, n, kind=kind, init={"dist": "uniform", "low": -1, "high": 1, "seed": 0})
    pkg, res = run(d)
    _, meta_res = run(d, honour_meta=True)
    want = oracle_run(d)
    out = pkg.meta["graph_outputs"][0]
    plan = res["launch"][pkg.meta["kernels"][0]["entry"]]
    assert plan.tuned and plan.grid[0] > 1          # the multi-CTA second pass ran
    # against the exact (float64) sum: the tuned kernel's error is far inside rtol 1e-5
    x = problems.make_inputs(pkg)["x"].astype(np.float64)
    ref = x.sum() if kind == "sum" else x.mean()
    np.testing.assert_allclose(float(res["outputs"][out][0]), ref, rtol=RTOL, atol=ATOL)
    # against the oracle, whose 128 threads each fold n/128 values in f32 in sequence, the
    # difference is that sequential fold's own rounding error (about sqrt(n/128) ulps per thread)
    bound = 1e-3 if kind == "sum" else 1e-8
    np.testing.assert_allclose(res["outputs"][out].reshape(()), want[out].reshape(()), rtol=2 * RTOL, atol=bound)
    np.testing.assert_allclose(meta_res["outputs"][out].reshape(()), want[out].reshape(()), rtol=2 * RTOL,
                               atol=bound)


def test_repeated_launches_reuse_the_arrival_counter(tmp_path):
    """The self-resetting counter: many launches in a row all produce the full sum."""
    d = synth.sum_package(tmp_path / "s", 1 << 22, init={"dist": "uniform", "low": -1, "high": 1, "seed": 3})
    pkg = problems.load_package(d)
    res = problems.run_package(pkg, problems.compile_package(pkg), warmup=7, iters=13)
    x = problems.make_inputs(pkg)["x"].astype(np.float64)
    np.testing.assert_allclose(float(res["outputs"]["sum_1"][0]), x.sum(), rtol=RTOL, atol=1e-3)


def test_big_sum_2_30(tmp_path):
    """The full benchmark size: 2^30 f32 elements (4 GiB), against a float64 CPU sum,
    and linear in its halves (each half summed by its own launch).  The bound is rtol 1e-5
    relative to the data's l2 norm, the scale of an f32 sum's rounding error: the sum of
    2^30 values uniform in [-1, 1) cancels to about the norm itself (~1.9e4), so a bound
    relative to the result alone would ask for less than the f32 rounding of the terms."""
    import torch

    from thompiler.device import DeviceKernel
    n = 1 << 30
    k = DeviceKernel(synth.sum_package(tmp_path / "big", n) / "k_sum_1_reduce.ir.json")
    h = DeviceKernel(synth.sum_package(tmp_path / "half", n // 2) / "k_sum_1_reduce.ir.json")
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.rand(n, device="cuda", generator=g) * 2 - 1
    out = torch.zeros(3, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    k({"x": x.data_ptr(), "sum_1": out.data_ptr()}, s)
    h({"x": x.data_ptr(), "sum_1": out.data_ptr() + 4}, s)
    h({"x": x.data_ptr() + 4 * (n // 2), "sum_1": out.data_ptr() + 8}, s)
    torch.cuda.synchronize()
    ref = float(x.double().sum())
    l2 = float(x.double().norm())
    got = out.cpu().numpy().astype(np.float64)
    print(f"2^30 sum: |got - ref| = {abs(got[0] - ref):.3e}, l2 = {l2:.4e}")
    assert abs(got[0] - ref) <= 1e-5 * l2, (got[0], ref)
    assert abs(got[1] + got[2] - got[0]) <= 1e-5 * l2, (got[1], got[2], got[0])
    for kk in (k, h):
        kk.close()


@pytest.mark.parametrize("kind", ["add", "relu_mul"])
def test_pointwise_vectorised(tmp_path, kind):
    """The pointwise family's 128-bit accesses give the generic lowering's bits: bit-exact
    against numpy (f32, tolerance 0) at 2^22 elements, and inputs passed at a 4-byte offset
    (not 16-byte aligned) take the generic path of the same module, still bit-exact.  (The
    output stays aligned: the IR's own Write of 4 values is a 16-byte store in every lowering.)"""
    import torch
    from thompiler.device import DeviceKernel
    n = 1 << 22
    d = synth.pointwise_package(tmp_path / "pw", n, kind)
    meta = json.loads((d / "meta.json").read_text())
    k = DeviceKernel(d / f"{meta['kernels'][0]['entry']}.ir.json")
    assert "family: pointwise-vector" in k.ptx and "ld.global.nc.v4.f32" in k.ptx
    g = torch.Generator(device="cuda").manual_seed(21)
    x = torch.randn(2, n + 4, device="cuda", generator=g)
    out = "mul" if kind == "relu_mul" else "add"
    for off in (0, 1):                                   # aligned views, then 4-byte-offset views
        x0, x1 = x[0, off:off + n], x[1, off:off + n]
        y = torch.full((n,), float("nan"), device="cuda")
        k({"x0": x0.data_ptr(), "x1": x1.data_ptr(), out: y.data_ptr()}, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        a, b = x0.cpu().numpy(), x1.cpu().numpy()
        want = np.maximum(a, 0) * b if kind == "relu_mul" else a + b
        assert np.array_equal(y.cpu().numpy(), want.astype(np.float32)), off
    k.close()


def test_past_2_31_elements(tmp_path):
    """Buffers longer than 2^31 elements (8.6 GB of f32 each): the pointwise family's 64-bit
    addressing (bit-exact at the far end of the range) and the full-mode sum's chunk indexing
    (within 1e-4 of the data's l2 norm of the float64 sum)."""
    import torch
    from thompiler.device import DeviceKernel
    n = (1 << 31) + (1 << 20)
    d = synth.pointwise_package(tmp_path / "pw", n, "relu_mul")
    k = DeviceKernel(d / "k_mul_pointwise.ir.json")
    g = torch.Generator(device="cuda").manual_seed(31)
    x0 = torch.randn(n, device="cuda", generator=g)
    x1 = torch.randn(n, device="cuda", generator=g)
    y = torch.full((n,), float("nan"), device="cuda")
    k({"x0": x0.data_ptr(), "x1": x1.data_ptr(), "mul": y.data_ptr()}, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    for lo in (0, (1 << 31) - 4096, n - 4096):
        want = torch.relu(x0[lo:lo + 4096]) * x1[lo:lo + 4096]
        assert torch.equal(y[lo:lo + 4096], want), lo
    assert not torch.isnan(y).any()
    k.close()
    del x1, y
    d2 = synth.sum_package(tmp_path / "s", n)
    ks = DeviceKernel(d2 / "k_sum_1_reduce.ir.json")
    out = torch.zeros(1, device="cuda")
    ks({"x": x0.data_ptr(), "sum_1": out.data_ptr()}, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    want = float(x0.double().sum())
    l2 = float(x0.double().norm())                       # f32 summation error scales with it
    assert abs(float(out.item()) - want) <= 1e-4 * l2, (float(out.item()), want)
    ks.close()
