"""A wider sweep of the tcgen05 families' shapes against float64 references on the GPU: every
tile width the matmul picker can choose (N = 256 / 192 / 128 / 64), both B layouts, f16 and f32
outputs, a split tail; attention with one and two query tiles per CTA, d = 64 and 128, more
tiles than SMs.  Each launch's wait-time-out word stays 0.
Tolerances: f32-out matmul 1e-3 absolute (f16 products summed in f32); f16-out and attention
rtol 2e-2 / atol 2e-3."""

import pytest

from thompiler import runner, synth
from thompiler.device import DeviceKernel

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,lay,out", [
    (1024, 1536, 512, "col", "f32"), (768, 640, 1024, "row", "f16"), (2048, 1536, 256, "col", "f16"),
    (4096, 384, 2048, "row", "f32"), (640, 320, 192, "col", "f32"), (8192, 256, 512, "col", "f32"),
    (3072, 4096, 1024, "col", "f32")])
@pytest.mark.parametrize("pair", ["0", "1"], ids=["single", "pair"])
def test_matmul_shape_sweep(tmp_path, monkeypatch, M, N, K, lay, out, pair):
    """Both matmul kernels: the single-CTA one (pair off) and, where M is a multiple of 256 and
    N of 128, the CTA-pair one (the default there)."""
    import torch
    from thompiler.families.tuning import TUNING
    monkeypatch.setattr(TUNING, "matmul_pair", pair == "1")
    d = synth.matmul_package(tmp_path / "mm", M, N, K, b_layout=lay, out_dtype=out)
    k = DeviceKernel(d / "k_matmul_f16.ir.json")
    paired = pair == "1" and M % 256 == 0 and N % 128 == 0
    assert k.family == ("tcgen05-matmul-pair" if paired else "tcgen05-matmul")
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = (torch.randn(M, K, device="cuda", generator=g) * 0.02).half()
    b = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half() if lay == "col" else \
        (torch.randn(K, N, device="cuda", generator=g) * 0.02).half()
    c = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float32 if out == "f32" else torch.float16)
    k({"x0": a.data_ptr(), "x1": b.data_ptr(), "matmul": c.data_ptr()}, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert runner.read_error_word(k.module, k.plan) == 0
    ref = a.double() @ (b.double().t() if lay == "col" else b.double())
    if out == "f32":
        assert (c.double() - ref).abs().max().item() < 1e-3
    else:
        assert torch.allclose(c.double(), ref, rtol=2e-2, atol=2e-3)
    k.close()


@pytest.mark.parametrize("shape", [(2, 4, 768, 64), (1, 8, 1024, 128), (3, 2, 640, 128), (4, 40, 512, 128)])
def test_attention_shape_sweep(tmp_path, shape):
    import torch
    B, H, S, D = shape
    k = DeviceKernel(synth.attention_package(tmp_path / "a", B, H, S, D) / "k_attention.ir.json")
    assert k.family == "tcgen05-attention"
    g = torch.Generator(device="cuda").manual_seed(S + H)
    q, kk, v = (torch.randn(*shape, device="cuda", generator=g).half() for _ in range(3))
    c = torch.tensor([D ** 0.5], device="cuda")
    o = torch.full(shape, float("nan"), device="cuda", dtype=torch.float16)
    k({"div_c1": c.data_ptr(), "q": q.data_ptr(), "k": kk.data_ptr(), "v": v.data_ptr(), "attn": o.data_ptr()},
      torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert runner.read_error_word(k.module, k.plan) == 0
    s = (q.double() @ kk.double().transpose(-1, -2)) / D ** 0.5
    ref = torch.softmax(s, -1) @ v.double()
    assert torch.allclose(o.double(), ref, rtol=2e-2, atol=2e-3)
    k.close()
