"""Programmatic dependent launch on the GPU: kernels launched to overlap the stream's previous
kernel (``LaunchPlan.pdl``) must still see everything that kernel wrote.  A pointwise kernel
writes y = relu(x0) * x1 and a full-sum kernel, launched right behind it, reads y; a row
softmax then reads the pointwise output of the next round.  Every round gets fresh inputs from
torch kernels (ordinary launches), and the chain runs both eagerly and inside a CUDA graph
(where the launches become programmatic edges).  Results against torch on the same data:
the sum within the f32 reduction bound (relative to the l2 norm), the softmax to rtol 1e-5."""

import pytest

from thompiler import synth
from thompiler.device import DeviceKernel

pytestmark = pytest.mark.gpu

N = 1 << 22
ROWS, COLS = 1024, 4096


def _kernels(tmp_path):
    pw = DeviceKernel(synth.pointwise_package(tmp_path / "pw", N, "relu_mul") / "k_mul_pointwise.ir.json")
    sm = DeviceKernel(synth.sum_package(tmp_path / "s", N) / "k_sum_1_reduce.ir.json")
    rs = DeviceKernel(synth.row_package(tmp_path / "r", "softmax", ROWS, COLS) / "k_softmax_rows.ir.json")
    for k in (pw, sm, rs):
        assert k.plan.pdl, k.family
    return pw, sm, rs


def _round(pw, sm, rs, x0, x1, y, out, z, stream):
    pw({"x0": x0.data_ptr(), "x1": x1.data_ptr(), "mul": y.data_ptr()}, stream)
    sm({"x": y.data_ptr(), "sum_1": out.data_ptr()}, stream)
    rs({"x": y.data_ptr(), "softmax": z.data_ptr()}, stream)


def _check(x0, x1, out, z):
    import torch
    y = torch.relu(x0) * x1
    want = y.double().sum().item()
    assert abs(out.item() - want) <= 1e-5 * y.double().norm().item() + 1e-6, (out.item(), want)
    ref = torch.softmax(y[:ROWS * COLS].view(ROWS, COLS).double(), -1)
    assert torch.allclose(z.double(), ref, rtol=1e-5, atol=1e-8)


def test_overlapped_launches_see_the_previous_kernels_writes(tmp_path):
    import torch
    pw, sm, rs = _kernels(tmp_path)
    g = torch.Generator(device="cuda").manual_seed(5)
    x0, x1 = torch.empty(N, device="cuda"), torch.empty(N, device="cuda")
    y, out = torch.empty(N, device="cuda"), torch.zeros(1, device="cuda")
    z = torch.empty(ROWS, COLS, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(20):
        x0.normal_(generator=g)
        x1.normal_(generator=g)
        _round(pw, sm, rs, x0, x1, y, out, z, s)
        torch.cuda.synchronize()
        _check(x0, x1, out, z)
    for k in (pw, sm, rs):
        k.close()


def test_overlapped_launches_in_a_cuda_graph(tmp_path):
    import torch
    pw, sm, rs = _kernels(tmp_path)
    g = torch.Generator(device="cuda").manual_seed(7)
    x0, x1 = torch.randn(N, device="cuda", generator=g), torch.randn(N, device="cuda", generator=g)
    y, out = torch.empty(N, device="cuda"), torch.zeros(1, device="cuda")
    z = torch.empty(ROWS, COLS, device="cuda")
    _round(pw, sm, rs, x0, x1, y, out, z, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        cs = torch.cuda.current_stream().cuda_stream
        for _ in range(3):                      # the same chain three times back to back
            _round(pw, sm, rs, x0, x1, y, out, z, cs)
    for _ in range(10):
        x0.normal_(generator=g)
        x1.normal_(generator=g)
        graph.replay()
        torch.cuda.synchronize()
        _check(x0, x1, out, z)
    del graph
    for k in (pw, sm, rs):
        k.close()


def test_tensor_core_kernels_read_what_the_previous_kernel_wrote(tmp_path):
    """The tcgen05 families under programmatic dependent launch: an attention kernel writes O
    (f16 [1, 2, 512, 128]) and a matmul launched right behind it reads O as its A operand through
    TMA ([1024, 128] @ B^T, B [256, 128]); fresh Q, K, V every round, eagerly and in a CUDA graph.
    C against the float64 product of the O the attention wrote, O against float32 attention."""
    import torch
    shape = (1, 2, 512, 128)
    M, N, K = 1024, 256, 128
    att = DeviceKernel(synth.attention_package(tmp_path / "att", *shape) / "k_attention.ir.json")
    mm = DeviceKernel(synth.matmul_package(tmp_path / "mm", M, N, K) / "k_matmul_f16.ir.json")
    assert att.plan.pdl and mm.plan.pdl and att.plan.tmaps and mm.plan.tmaps
    g = torch.Generator(device="cuda").manual_seed(61)
    q, k, v = (torch.empty(*shape, device="cuda", dtype=torch.float16) for _ in range(3))
    c = torch.tensor([shape[-1] ** 0.5], device="cuda")
    o = torch.empty(*shape, device="cuda", dtype=torch.float16)
    b = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
    out = torch.empty(M, N, device="cuda")

    def chain(stream):
        att({"div_c1": c.data_ptr(), "q": q.data_ptr(), "k": k.data_ptr(), "v": v.data_ptr(),
             "attn": o.data_ptr()}, stream)
        mm({"x0": o.data_ptr(), "x1": b.data_ptr(), "matmul": out.data_ptr()}, stream)

    def refill():
        for x in (q, k, v):
            x.copy_(torch.randn(*shape, device="cuda", generator=g))
        o.fill_(float("nan"))
        out.fill_(float("nan"))

    def check():
        s = (q[0].float() @ k[0].float().transpose(-1, -2)) / shape[-1] ** 0.5
        ref_o = torch.softmax(s, -1) @ v[0].float()
        assert torch.allclose(o[0].float(), ref_o, rtol=2e-2, atol=2e-3)
        ref_c = o.view(M, K).double() @ b.double().t()
        assert (out.double() - ref_c).abs().max().item() < 1e-4
        assert att.error_word() == 0 and mm.error_word() == 0

    for _ in range(4):
        refill()
        chain(torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        check()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        chain(torch.cuda.current_stream().cuda_stream)
    for _ in range(4):
        refill()
        graph.replay()
        torch.cuda.synchronize()
        check()
    del graph
    att.close()
    mm.close()
