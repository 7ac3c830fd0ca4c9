"""The allocation-free sum entry point (thr_sum_f32_noalloc) against the
existing path for the same reduction.

Callers that cannot call cudaMalloc -- their device memory belongs to their
own allocator or pool, or they sit on a path where cudaMalloc / cudaFree
would block or synchronise the device -- use thr_sum_f32_noalloc, whose only
scratch is a static device array inside the library.  This test calls it
through the C ABI twice in a row on the same input (the second call must
not be disturbed by what the first left in the shared array) and checks
both results against the compiled two-pass sum kernel launched through
thr_launch, within the f32 reduction tolerance (rtol 1e-5).  The file sorts
last so a stop-at-first-failure run has run every other test first.
"""

import ctypes

import numpy as np
import pytest

from thompiler import runner, synth
from thompiler.device import DeviceKernel

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def entry():
    lib = runner.library()
    f = lib.thr_sum_f32_noalloc
    f.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64]
    f.restype = ctypes.c_int
    return f


@pytest.mark.parametrize("n", [1 << 22, (1 << 20) + 3])
def test_noalloc_sum_matches_the_compiled_kernel(tmp_path, n):
    import torch
    runner.init(0)
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.rand(n, device="cuda", generator=g) * 2 - 1
    ref_out = torch.zeros(1, device="cuda")
    out = torch.full((2,), float("nan"), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    k = DeviceKernel(synth.sum_package(tmp_path / "sum", n) / "k_sum_1_reduce.ir.json")
    k({"x": x.data_ptr(), "sum_1": ref_out.data_ptr()}, stream)
    f = entry()
    for i in range(2):
        st = f(x.data_ptr(), n, out.data_ptr() + 4 * i, 0, stream)
        assert st == 0, runner.last_error()
    torch.cuda.synchronize()
    want = float(ref_out.item())
    got = out.cpu().numpy()
    for v in got:
        assert abs(float(v) - want) <= RTOL * max(1.0, abs(want)), (got, want)
    exact = np.sum(x.cpu().numpy(), dtype=np.float64)
    assert abs(float(got[1]) - exact) <= RTOL * max(1.0, abs(exact))
    k.close()


@pytest.mark.parametrize("n,ctas", [(1 << 24, 4096), (3, 1), (1, 1), (4097, 4096)])
def test_noalloc_explicit_cta_counts(n, ctas):
    """Explicit CTA counts, twice each: 4096 fills the whole partials array (the last CTA folds 16
    partials per thread); one CTA with fewer than 4 elements is all tail; 4096 CTAs over 4097
    elements leave most CTAs without a chunk.  Against the float64 sum of the same f32 data."""
    import torch
    runner.init(0)
    g = torch.Generator(device="cuda").manual_seed(n + ctas)
    x = torch.rand(n, device="cuda", generator=g) * 2 - 1
    out = torch.full((2,), float("nan"), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    f = entry()
    for i in range(2):
        st = f(x.data_ptr(), n, out.data_ptr() + 4 * i, ctas, stream)
        assert st == 0, runner.last_error()
    torch.cuda.synchronize()
    exact = float(np.sum(x.cpu().numpy(), dtype=np.float64))
    l2 = float(np.linalg.norm(x.cpu().numpy().astype(np.float64)))
    for v in out.cpu().numpy():
        assert abs(float(v) - exact) <= RTOL * max(1.0, l2), (v, exact)


def test_noalloc_rejects_unaligned_pointers():
    import torch
    runner.init(0)
    x = torch.zeros(1024, device="cuda")
    out = torch.zeros(2, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert entry()(x.data_ptr() + 4, 1000, out.data_ptr(), 0, s) == 4 and "16-byte" in runner.last_error()
    assert entry()(x.data_ptr(), 1024, out.data_ptr() + 2, 0, s) == 4 and "4-byte" in runner.last_error()


def test_noalloc_rejects_more_ctas_than_its_scratch():
    import torch
    runner.init(0)
    x = torch.zeros(1024, device="cuda")
    out = torch.zeros(1, device="cuda")
    st = entry()(x.data_ptr(), 1024, out.data_ptr(), 4097, torch.cuda.current_stream().cuda_stream)
    assert st == 4 and "at most 4096" in runner.last_error()
