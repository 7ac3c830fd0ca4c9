"""Launches of one compiled module on different buffers in flight together.

A tuned module keeps its tensor maps as a ring of sets, one per set of buffers, and its kernel
uses the set whose recorded addresses equal its parameters (thr_tmap_bind); the matmul split
tail keeps its partials and arrival counters per set too.  So launches of one module on
different buffers may overlap on several streams, and thr_run_batch takes several requests of
one module.  Checked against float64 products / attention on the same f16 inputs (rtol 2e-2,
atol 2e-3, the f16 tensor-core tolerance).
"""

import numpy as np
import pytest

from thompiler import runner, synth
from thompiler.device import DeviceKernel
from thompiler.families.kit import TMAP_SETS

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3


def _mm_check(a, b, c):
    ref = a.double() @ b.double().t()
    assert (c.double() - ref).abs().max().item() < 1e-4


def _att_ref(q, k, v):
    import torch
    s = (q.float() @ k.float().transpose(-1, -2)) / q.shape[-1] ** 0.5
    return torch.softmax(s, -1) @ v.float()


def test_two_modules_on_two_streams(tmp_path, monkeypatch):
    """One attention module and one matmul module (a K-split tail shape, the half tail switched
    off so the per-set partials and counters are exercised), each launched on six buffer sets --
    more than the module's tensor-map sets -- alternating between two streams, interleaved;
    every output against float64 / float32 references."""
    import torch
    from thompiler.families.tuning import TUNING
    monkeypatch.setattr(TUNING, "matmul_half_tail", False)
    M, N, K = 2048, 2560, 2048                      # 80 pair tiles on 74 pairs: a split tail
    mm = DeviceKernel(synth.matmul_package(tmp_path / "mm", M, N, K) / "k_matmul_f16.ir.json")
    assert mm.plan.counters == ["thc_tile_arrivals"] and mm.module.sidecar["tmap_sets"] == TMAP_SETS
    shape = (2, 4, 1024, 128)
    att = DeviceKernel(synth.attention_package(tmp_path / "att", *shape) / "k_attention.ir.json")
    g = torch.Generator(device="cuda").manual_seed(23)
    sets = 6
    mb = [((torch.randn(M, K, device="cuda", generator=g) * 0.02).half(),
           (torch.randn(N, K, device="cuda", generator=g) * 0.02).half(),
           torch.full((M, N), float("nan"), device="cuda")) for _ in range(sets)]
    ab = [tuple(torch.randn(*shape, device="cuda", generator=g).half() for _ in range(3))
          + (torch.full(shape, float("nan"), device="cuda", dtype=torch.float16),) for _ in range(sets)]
    c = torch.tensor([shape[-1] ** 0.5], device="cuda")
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    torch.cuda.synchronize()
    for rnd in range(2):
        for i in range(sets):
            s = streams[(i + rnd) % 2].cuda_stream
            a, b, cc = mb[i]
            mm({"x0": a.data_ptr(), "x1": b.data_ptr(), "matmul": cc.data_ptr()}, s)
            q, k, v, o = ab[i]
            att({"div_c1": c.data_ptr(), "q": q.data_ptr(), "k": k.data_ptr(), "v": v.data_ptr(),
                 "attn": o.data_ptr()}, s)
    torch.cuda.synchronize()
    assert mm.error_word() == 0 and att.error_word() == 0
    for i in range(sets):
        _mm_check(*mb[i])
        q, k, v, o = ab[i]
        assert torch.allclose(o.float(), _att_ref(q, k, v), rtol=RTOL, atol=ATOL), i
    mm.close()
    att.close()


def test_split_tail_concurrent_launches(tmp_path, monkeypatch):
    """The single-CTA kernel's split tail (12 tail tiles cut in two K parts): two launches on
    different buffers, on two streams at once, each with its own partials and counters."""
    import torch

    from thompiler.families.tuning import TUNING
    monkeypatch.setattr(TUNING, "matmul_pair", False)
    M, N, K = 2048, 2560, 2048
    mm = DeviceKernel(synth.matmul_package(tmp_path / "mm", M, N, K) / "k_matmul_f16.ir.json")
    assert "thc_tail_ws" in mm.ptx
    g = torch.Generator(device="cuda").manual_seed(29)
    bufs = [((torch.randn(M, K, device="cuda", generator=g) * 0.02).half(),
             (torch.randn(N, K, device="cuda", generator=g) * 0.02).half(),
             torch.full((M, N), float("nan"), device="cuda")) for _ in range(2)]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    torch.cuda.synchronize()
    for _ in range(5):
        for (a, b, cc), s in zip(bufs, streams):
            mm({"x0": a.data_ptr(), "x1": b.data_ptr(), "matmul": cc.data_ptr()}, s.cuda_stream)
    torch.cuda.synchronize()
    assert mm.error_word() == 0
    for a, b, cc in bufs:
        _mm_check(a, b, cc)
    mm.close()


def test_run_batch_requests_of_one_module(tmp_path):
    """thr_run_batch with six requests of one tensor-map module (host buffers): each request
    binds its own set; past the module's sets a set's re-encoding waits for its earlier reader."""
    M, N, K = 512, 512, 256
    d = synth.matmul_package(tmp_path / "mm", M, N, K)
    k = DeviceKernel(d / "k_matmul_f16.ir.json")
    rng = np.random.default_rng(3)
    reqs, host = [], []
    for _ in range(6):
        a = (rng.standard_normal((M, K)) * 0.02).astype(np.float16)
        b = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
        c = np.full((M, N), np.nan, dtype=np.float32)
        arrs = {"x0": a, "x1": b, "matmul": c}
        reqs.append((k.fn, k.plan, [{"array": arrs[n], "output": n == "matmul"} for n in k.arg_order], k.arg_order))
        host.append((a, b, c))
    for _ in range(2):
        r = runner.run_batch(reqs)
        assert r["ok"], r
        for a, b, c in host:
            ref = a.astype(np.float64) @ b.astype(np.float64).T
            assert np.max(np.abs(c - ref)) < 1e-4
            c[...] = np.nan
    runner.release()
    k.close()


def test_captured_launches_on_two_buffer_sets(tmp_path):
    """A CUDA graph holding launches of one module on two buffer sets (bound before the capture:
    those sets are then kept for the graph), replayed twice on fresh inputs."""
    import torch
    M, N, K = 1024, 1024, 512
    k = DeviceKernel(synth.matmul_package(tmp_path / "mm", M, N, K) / "k_matmul_f16.ir.json")
    g = torch.Generator(device="cuda").manual_seed(31)
    bufs = [(torch.empty(M, K, device="cuda", dtype=torch.float16),
             torch.empty(N, K, device="cuda", dtype=torch.float16), torch.empty(M, N, device="cuda"))
            for _ in range(2)]
    s = torch.cuda.current_stream().cuda_stream
    for a, b, c in bufs:                           # bind outside the capture
        k({"x0": a.data_ptr(), "x1": b.data_ptr(), "matmul": c.data_ptr()}, s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        cs = torch.cuda.current_stream().cuda_stream
        for a, b, c in bufs:
            k({"x0": a.data_ptr(), "x1": b.data_ptr(), "matmul": c.data_ptr()}, cs)
    for _ in range(2):
        for a, b, c in bufs:
            a.copy_(torch.randn(M, K, device="cuda", generator=g) * 0.02)
            b.copy_(torch.randn(N, K, device="cuda", generator=g) * 0.02)
            c.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        for a, b, c in bufs:
            _mm_check(a, b, c)
    del graph
    k.close()
