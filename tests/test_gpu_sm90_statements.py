"""GPU checks of the IR statements the reference compiler does not lower (TMA box copies with
mbarriers, Select, ZeroPrologue, built-in / call / cast index expressions, FlatIndex): the
kernels of tests/sm90_ir.py against numpy, through the device-pointer launch (tensor maps
encoded from the launch's pointers) and the host-buffer C-ABI run (tensor maps per request).
The reference has no lowering of these statements to compare with, so numpy is the check."""

import numpy as np
import pytest

from sm90_ir import (COLS, EPILOGUE_FORMS, FRAGMENT_ATTENTION_EXTRAS, M, N, ROWS, blockscaled_matmul_package,
                     chained_matmul_package, dequant_fp4, epilogue_matmul_package, fragment_attention_package, promote_matmul_package,
                     scan_package, select_package, stuck_wait_package, tma_transpose_package, wgmma_gemm_package,
                     window_package)
from thompiler import problems, runner
from thompiler.device import DeviceKernel

pytestmark = pytest.mark.gpu


def test_tma_transpose_device_pointers(tmp_path):
    import torch
    d = tma_transpose_package(tmp_path / "t")
    k = DeviceKernel(d / "k_tma_transpose.ir.json")
    assert k.plan.tmaps and not k.plan.tuned
    x = torch.randn(N, N, device="cuda")
    for trial in range(2):                          # new pointers: the tensor map is re-encoded
        x = x + trial
        y = torch.full((N, N), float("nan"), device="cuda")
        k({"x": x.data_ptr(), "y": y.data_ptr()}, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert runner.read_error_word(k.module, k.plan) == 0
        assert torch.equal(y, x.t())
    k.close()


def test_tma_transpose_host_buffers(tmp_path):
    pkg = problems.load_package(tma_transpose_package(tmp_path / "t"))
    res = problems.run_package(pkg, problems.compile_package(pkg))
    x = problems.make_inputs(pkg)["x"]
    np.testing.assert_array_equal(res["outputs"]["y"], x.T)


def test_select_zero_prologue(tmp_path):
    import torch
    d = select_package(tmp_path / "s")
    k = DeviceKernel(d / "k_select.ir.json")
    x = torch.randn(M, device="cuda")
    z = torch.ones(M, device="cuda")
    y = torch.full((M,), float("nan"), device="cuda")
    k({"x": x.data_ptr(), "z": z.data_ptr(), "y": y.data_ptr()}, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    i = torch.arange(M, device="cuda")
    want = torch.where(i < 100, x[torch.clamp(i, max=99)], x * x)
    assert torch.equal(y, want)
    assert torch.all(z[:64] == 0) and torch.all(z[64:] == 1)
    k.close()


def test_wait_that_never_completes_gives_up(tmp_path):
    """A wait on an mbarrier nothing arrives on: every thread's bounded wait runs out (2^18
    polls, about a second), sets bit 1 of the kernel's error word and carries on, so the launch
    finishes and the statements after the wait still run -- the failure is reported, the GPU
    never hangs."""
    import time

    import torch
    d = stuck_wait_package(tmp_path / "w")
    k = DeviceKernel(d / "k_stuck_wait.ir.json")
    x = torch.randn(64, device="cuda")
    y = torch.zeros(64, device="cuda")
    t0 = time.perf_counter()
    k({"x": x.data_ptr(), "y": y.data_ptr()}, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert runner.read_error_word(k.module, k.plan) == 2
    assert torch.equal(y, x)
    assert elapsed < 10, elapsed
    print(f"bounded wait gave up after {elapsed:.2f} s")
    k.close()


def test_carried_state_scan(tmp_path):
    """Carry / Pre on the GPU: a per-row prefix sum (sequential f32 adds, so bit-exact against
    numpy's float32 cumsum), its total after the loop, and the Fibonacci carrier whose step reads
    cell 0 after setting it -- F(COLS + 1) only if that read sees the previous state."""
    pkg = problems.load_package(scan_package(tmp_path / "c"))
    res = problems.run_package(pkg, problems.compile_package(pkg))
    x = problems.make_inputs(pkg)["x"]
    want = np.cumsum(x, axis=1, dtype=np.float32)
    np.testing.assert_array_equal(res["outputs"]["y"], want)
    np.testing.assert_array_equal(res["outputs"]["t"].reshape(ROWS), want[:, -1])
    fib = [0, 1]
    for _ in range(COLS):
        fib = [fib[1], fib[0] + fib[1]]
    assert np.all(res["outputs"]["f"] == fib[1]) and fib[1] == 75025


WGMMA_CASES = [{}, {"n_wg": 2}, {"trans_b": True}, {"tail_overwrite": True}, {"BN": 64}, {"BN": 256},
               {"out_scale": 0.25}]


@pytest.mark.parametrize("kw", WGMMA_CASES, ids=[",".join(f"{k}={v}" for k, v in c.items()) or "base"
                                                  for c in WGMMA_CASES])
def test_wgmma_gemm(tmp_path, kw):
    """The sm_90-style GEMM (Wgmma* statements, m64 accumulator fragments) on tcgen05: y = x0 @ B
    against float64 numpy on the same f16 inputs, through the host-buffer run (TMA maps encoded
    per request; a non-zero error word -- a wait that gave up, a skipped copy or MMA -- fails the
    run).  The tolerance covers f32 accumulation over K = 512 products of N(0, 1) halves (|y| ~ 23);
    with ``out_scale`` the result leaves through a RegStore epilogue as f16, whose rounding (half
    an f16 ulp, 2.4e-4 relative) the same tolerance covers."""
    M_, N_, K_ = 256, 512, 512
    pkg = problems.load_package(wgmma_gemm_package(tmp_path / "g", M_, N_, K_, **kw))
    res = problems.run_package(pkg, problems.compile_package(pkg))
    x = problems.make_inputs(pkg)
    a = x["x0"].astype(np.float64)
    b = x["x1"].astype(np.float64)
    bk = b if kw.get("trans_b") else b.T                      # [K, N]
    if kw.get("tail_overwrite"):
        a, bk = a[:, K_ - 16:], bk[K_ - 16:, :]
    want = a @ bk * kw.get("out_scale", 1.0)
    got = res["outputs"]["y"]
    assert got.dtype == (np.float16 if "out_scale" in kw else np.float32)
    np.testing.assert_allclose(got.astype(np.float64), want, rtol=1e-3, atol=2e-3)


def test_fragment_attention(tmp_path):
    """Flash attention in register fragments (FragmentApply / FragmentRowReduce / FragmentRepack on
    mma.sync): one head, S = 256 keys in four blocks of 64, against float64 numpy softmax attention
    on the same f16 inputs.  The probabilities are rounded to f16 before P V, as any f16 flash
    attention does; the tolerance is the attention one (rtol 2e-2, atol 2e-3)."""
    pkg = problems.load_package(fragment_attention_package(tmp_path / "a", 256, 64))
    res = problems.run_package(pkg, problems.compile_package(pkg))
    x = problems.make_inputs(pkg)
    q, k, v = (x[n].astype(np.float64) for n in ("q", "k", "v"))
    sc = q @ k.T / 8.0
    p = np.exp(sc - sc.max(axis=1, keepdims=True))
    want = (p / p.sum(axis=1, keepdims=True)) @ v
    np.testing.assert_allclose(res["outputs"]["o"], want, rtol=2e-2, atol=2e-3)


@pytest.mark.parametrize("extra", FRAGMENT_ATTENTION_EXTRAS)
def test_fragment_attention_mask_and_bias(tmp_path, extra):
    """FragmentApply mask and bias arguments on the register-fragment flash attention (one head,
    S = 256): a causal mask as a Lambda added to the scores, the same mask as a predicate
    multiplying the probabilities, an [S, S] f32 bias at (query, key) by buffer name and by an
    explicit index, and a per-key [S] bias -- each against the float64 numpy expression."""
    pkg = problems.load_package(fragment_attention_package(tmp_path / "a", 256, 64, extra))
    res = problems.run_package(pkg, problems.compile_package(pkg))
    x = problems.make_inputs(pkg)
    q, k, v = (x[n].astype(np.float64) for n in ("q", "k", "v"))
    sc = q @ k.T / 8.0
    if extra in ("causal", "causal_pred"):
        sc = np.where(np.arange(256)[None, :] <= np.arange(256)[:, None], sc, -np.inf)
    elif extra in ("bias", "bias_index"):
        sc = sc + x["bias"].astype(np.float64)
    else:
        sc = sc + x["kbias"].astype(np.float64)[None, :]
    p = np.exp(sc - sc.max(axis=1, keepdims=True))
    want = (p / p.sum(axis=1, keepdims=True)) @ v
    np.testing.assert_allclose(res["outputs"]["o"], want, rtol=2e-2, atol=2e-3)


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (64, 192, 256)])
def test_blockscaled_fp4_matmul(tmp_path, M, N, K):
    """Block-scaled fp4 (e2m1 codes, ue8m0 scales per 32 k) through fp4 LdmatrixLoad,
    BlockScaleLoad and the m16n8k64 MmaSyncPtx, against the float64 numpy product of the
    dequantised operands (every dequantised value and product is exact in f32; only the f32
    sums round)."""
    pkg = problems.load_package(blockscaled_matmul_package(tmp_path / "b", M, N, K))
    res = problems.run_package(pkg, problems.compile_package(pkg))
    x = problems.make_inputs(pkg)
    want = dequant_fp4(x["xa"], x["sa"]) @ dequant_fp4(x["xb"], x["sb"]).T
    got = res["outputs"]["y"].astype(np.float64)
    assert np.max(np.abs(got - want)) <= 1e-5 * np.max(np.abs(want)), np.max(np.abs(got - want))


def test_regstore_into_swizzled_shared_memory(tmp_path):
    """A product's C fragments staged in shared memory with the 128-byte swizzle (RegStore, f16)
    and read back by ldmatrix under the same swizzle as the A operand of a second product:
    y = f16(x0 @ x1^T) @ x2^T against float64 numpy with the intermediate rounded to f16."""
    pkg = problems.load_package(chained_matmul_package(tmp_path / "c"))
    res = problems.run_package(pkg, problems.compile_package(pkg))
    x = problems.make_inputs(pkg)
    p = (x["x0"].astype(np.float64) @ x["x1"].astype(np.float64).T).astype(np.float16).astype(np.float64)
    want = p @ x["x2"].astype(np.float64).T
    np.testing.assert_allclose(res["outputs"]["y"], want, rtol=2e-2, atol=2e-3)


def test_carried_state_run_time_cells(tmp_path):
    """A carrier indexed at run time (cell j % 4 of a 4-cell ring, .local arrays): y[r, j] =
    x[r, j] - x[r, j - 4] (x[r, j] for j < 4, the seed 0) and the last step's cell read after
    the loop -- bit-exact against numpy float32."""
    pkg = problems.load_package(window_package(tmp_path / "w", 4))
    res = problems.run_package(pkg, problems.compile_package(pkg))
    x = problems.make_inputs(pkg)["x"]
    want = x.copy()
    want[:, 4:] = x[:, 4:] - x[:, :-4]
    np.testing.assert_array_equal(res["outputs"]["y"], want)
    np.testing.assert_array_equal(res["outputs"]["t"].reshape(-1), x[:, -1])


def test_promote_matmul_exact(tmp_path):
    """f16 accumulation per K block of 64, promoted into f32 (FragmentPromote): with integer inputs
    in -2..2 every partial is exact, so the result is the integer product bit for bit."""
    pkg = problems.load_package(promote_matmul_package(tmp_path / "p", 128, 128, 512))
    res = problems.run_package(pkg, problems.compile_package(pkg))
    x = problems.make_inputs(pkg)
    want = (x["x0"].astype(np.int64) @ x["x1"].astype(np.int64).T).astype(np.float32)
    np.testing.assert_array_equal(res["outputs"]["y"], want)


@pytest.mark.parametrize("form", EPILOGUE_FORMS)
def test_regstore_fused_forms(tmp_path, form):
    """The fused RegStore forms on an mma.sync GEMM of integer inputs in -2..2 (every accumulator an
    exact integer): an epilogue with the bias load, relu and a coordinate mask into f16; edge
    guards into a buffer smaller than the tile grid (a store past them would land outside it);
    four K slices added atomically into a zeroed buffer; an extra accumulator multiplied in.
    The integer forms are exact; the f16 one is within one f16 rounding of the float32 numpy
    expression.  The oracle interpreter's restatement of the forms agrees to the same bar."""
    from oracle.interp import run_package as oracle_run
    d = epilogue_matmul_package(tmp_path / form, form)
    pkg = problems.load_package(d)
    res = problems.run_package(pkg, problems.compile_package(pkg))
    x = problems.make_inputs(pkg)
    acc = x["x0"].astype(np.int64) @ x["x1"].astype(np.int64).T
    got = res["outputs"]["y"]
    np.testing.assert_allclose(got.astype(np.float64).reshape(-1), oracle_run(d)["y"].astype(np.float64).reshape(-1),
                               rtol=1e-3, atol=1e-3)
    if form == "bias_relu_mask":
        t = np.float32(0.5) * acc.astype(np.float32) + x["bias"].astype(np.float32)
        rows, cols = np.indices(t.shape)
        want = np.where(cols <= rows, np.maximum(t, np.float32(0)), np.float32(0)).astype(np.float16)
        assert got.dtype == np.float16
        np.testing.assert_allclose(got.astype(np.float32), want.astype(np.float32), rtol=1e-3, atol=1e-3)
    elif form == "guarded":
        np.testing.assert_array_equal(got.reshape(acc.shape[0] - 28, acc.shape[1] - 38),
                                      acc[:-28, :-38].astype(np.float32))
    elif form == "atomic":
        np.testing.assert_array_equal(got, acc.astype(np.float32))
    else:
        d = x["x0"].astype(np.int64) @ x["x2"].astype(np.int64).T
        np.testing.assert_array_equal(got, (acc * d).astype(np.float32))
