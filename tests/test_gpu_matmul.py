"""GPU parity of the tcgen05 matmul family.

* small shapes: the tuned kernel (tuned launch, TMA + tcgen05) and the same
  module under meta.json's launch (generic mma.sync lowering) against the
  oracle interpreter on the same seeded inputs;
* the benchmark shapes (4096^3 and M=8192, N=3072, K=1024, f16 in, f32 out,
  B column-major): against the reference compiler's own PTX for the same IR
  (mma.sync, committed nowhere: the emmy stand-in that generates it needs the
  reference checkout, absent where the GPU tests run, so the generic lowering -- which is
  bit-identical to the reference PTX on every shipped package -- stands in),
  and against a float64 checksum: C @ 1 == A @ (B^T @ 1) row by row.
Every tuned launch also checks the kernel's wait-time-out word stays 0.
Tolerance for f16-input tensor-core results: rtol 2e-2 / atol 2e-3.
"""

import numpy as np
import pytest

from oracle.interp import run_package as oracle_run
from thompiler import problems, runner, synth
from thompiler.device import DeviceKernel
from thompiler.families.tuning import TUNING

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3


@pytest.mark.parametrize("M,N,K,lay,out", [(128, 64, 256, "col", "f32"), (256, 256, 512, "col", "f32"),
                                           (256, 128, 256, "row", "f32"), (128, 128, 128, "row", "f16"),
                                           (384, 192, 320, "col", "f16")])
def test_matmul_small_vs_oracle(tmp_path, M, N, K, lay, out):
    d = synth.matmul_package(tmp_path / "mm", M, N, K, b_layout=lay, out_dtype=out)
    pkg = problems.load_package(d)
    ptx = problems.compile_package(pkg)
    assert "tcgen05.mma" in ptx["k_matmul_f16"]
    tuned = problems.run_package(pkg, ptx)
    assert tuned["launch"]["k_matmul_f16"].tmaps
    meta = problems.run_package(pkg, ptx, honour_meta=True)
    want = oracle_run(d)["matmul"]
    for res in (tuned, meta):
        got = res["outputs"]["matmul"].astype(np.float64)
        np.testing.assert_allclose(got, want.astype(np.float64), rtol=RTOL, atol=ATOL)
    # f32 outputs: the tensor cores sum exact f16 products in f32 -- far inside the bar
    if out == "f32":
        x = problems.make_inputs(pkg)
        b = x["x1"].astype(np.float64)
        ref = x["x0"].astype(np.float64) @ (b.T if lay == "col" else b)
        assert np.max(np.abs(tuned["outputs"]["matmul"] - ref)) < 1e-3


@pytest.mark.parametrize("M,N,K", [(4096, 4096, 4096), (8192, 3072, 1024)])
def test_matmul_benchmark_shapes(tmp_path, M, N, K):
    import torch
    d = synth.matmul_package(tmp_path / "mm", M, N, K, b_layout="col", out_dtype="f32")
    ir = d / "k_matmul_f16.ir.json"
    tuned = DeviceKernel(ir)
    generic = DeviceKernel(ir, tuned=False)
    assert tuned.plan.tmaps and "tcgen05.mma" in tuned.ptx
    g = torch.Generator(device="cuda").manual_seed(3)
    a = (torch.randn(M, K, device="cuda", generator=g) * 0.02).half()
    b = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    c1 = torch.full((M, N), float("nan"), device="cuda")
    c2 = torch.full((M, N), float("nan"), device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    tuned({"x0": a.data_ptr(), "x1": b.data_ptr(), "matmul": c1.data_ptr()}, s)
    generic({"x0": a.data_ptr(), "x1": b.data_ptr(), "matmul": c2.data_ptr()}, s)
    torch.cuda.synchronize()
    assert runner.read_error_word(tuned.module, tuned.plan) == 0
    assert not torch.isnan(c1).any()
    assert torch.allclose(c1, c2, rtol=RTOL, atol=ATOL)
    err = (c1.double() - c2.double()).abs().max().item()
    assert err < 1e-4, err
    # checksum: every row of C sums to the row of A times the column sums of B^T
    ones_ref = a.double() @ b.double().sum(0)
    assert torch.allclose(c1.double().sum(1), ones_ref, rtol=1e-4, atol=1e-3)
    # every element against an independent float64 product, at the f16-input tolerance
    ref = a.double() @ b.double().t()
    assert torch.allclose(c1.double(), ref, rtol=RTOL, atol=ATOL)
    err64 = (c1.double() - ref).abs().max().item()
    print(f"{M}x{N}x{K}: max |C - C_f64| = {err64:.3e}")
    assert err64 < 1e-4, err64                           # exact f16 products summed in f32
    # a second launch (tensor maps already in place) gives the same bits
    c1b = torch.empty_like(c1)
    tuned({"x0": a.data_ptr(), "x1": b.data_ptr(), "matmul": c1b.data_ptr()}, s)
    torch.cuda.synchronize()
    assert torch.equal(c1, c1b)
    tuned.close()
    generic.close()


@pytest.mark.parametrize("grid", [0, 5])
def test_matmul_split_tail(tmp_path, monkeypatch, grid):
    """More tiles than SMs with a partial last wave (2048 x 2560 x 2048: 160 tiles of 128 x 256,
    12 left over): those are cut along K into parts whose partials meet in the module's
    workspace, the last part to arrive adding them in part order.  grid 5 puts several whole
    tiles and several parts on each CTA (the arrival barriers' phases carry over)."""
    import torch
    monkeypatch.setattr(TUNING, "matmul_pair", False)     # this split tail belongs to the single-CTA kernel
    M, N, K = 2048, 2560, 2048
    d = synth.matmul_package(tmp_path / "mm", M, N, K, b_layout="col", out_dtype="f32")
    k = DeviceKernel(d / "k_matmul_f16.ir.json")
    assert "thc_tail_ws" in k.ptx
    if grid:
        k.plan.grid = (grid, 1, 1)
    g = torch.Generator(device="cuda").manual_seed(4)
    a = (torch.randn(M, K, device="cuda", generator=g) * 0.02).half()
    b = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    outs = []
    for _ in range(2):
        c = torch.full((M, N), float("nan"), device="cuda")
        k({"x0": a.data_ptr(), "x1": b.data_ptr(), "matmul": c.data_ptr()}, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        outs.append(c)
    assert runner.read_error_word(k.module, k.plan) == 0
    ref = a.double() @ b.double().t()
    assert (outs[0].double() - ref).abs().max().item() < 1e-4
    assert torch.equal(outs[0], outs[1])                 # the part order fixes the rounding
    k.close()


def test_split_tail_counters_cleared_after_a_give_up(tmp_path, monkeypatch):
    """A bounded wait that gives up can leave a split-tail (tile, rank) counter part-way through
    its count.  The failure is made on the host: the counter of tail tile 0 is set to 1 (one of
    its two parts arrived) and the error word to the wait's code, as a give-up would leave them.
    The counter then stays off by one launch after launch (each launch's first part to arrive
    takes itself for the last and may add a partial the other part has not written yet), until
    ``clear_error`` zeroes the error word and the counters; then every launch leaves them at 0."""
    import ctypes

    import torch
    monkeypatch.setattr(TUNING, "matmul_pair", False)
    M, N, K = 2048, 2560, 2048
    d = synth.matmul_package(tmp_path / "mm", M, N, K, b_layout="col", out_dtype="f32")
    k = DeviceKernel(d / "k_matmul_f16.ir.json")
    assert k.plan.counters == ["thc_tile_arrivals"]
    g = torch.Generator(device="cuda").manual_seed(6)
    a = (torch.randn(M, K, device="cuda", generator=g) * 0.02).half()
    b = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    c = torch.empty(M, N, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    lib = runner.library()
    cnt_ptr, cnt_bytes = k.module.global_ptr("thc_tile_arrivals")

    def run():
        c.fill_(float("nan"))
        k({"x0": a.data_ptr(), "x1": b.data_ptr(), "matmul": c.data_ptr()}, s)
        torch.cuda.synchronize()
        return (c.double() - a.double() @ b.double().t()).abs().max().item()

    def counters():
        buf = (ctypes.c_uint32 * (cnt_bytes // 4))()
        runner.check(lib.thr_memcpy_dtoh(buf, cnt_ptr, cnt_bytes), "read counters")
        return list(buf)

    from thompiler.families.kit import TMAP_SETS
    assert cnt_bytes // 4 == 12 * TMAP_SETS                # 12 tail tiles, one counter each, per set
    # the first launch binds tensor-map set 0: its counters are the first 12
    assert run() < 1e-4 and k.error_word() == 0 and set(counters()) == {0}
    for name, val in (("thc_tile_arrivals", 1), ("thc_error", 1 << 2)):
        dst, _ = k.module.global_ptr(name)
        v = ctypes.c_uint32(val)
        runner.check(lib.thr_memcpy_htod(dst, ctypes.byref(v), 4, 0), name)
    runner.check(lib.thr_synchronize(), "sync")
    run()
    assert counters()[0] == 1 and set(counters()[1:]) == {0}    # still part-way: the hazard persists
    k.clear_error()
    assert k.error_word() == 0 and set(counters()) == {0}
    assert run() < 1e-4 and set(counters()) == {0}
    k.close()
