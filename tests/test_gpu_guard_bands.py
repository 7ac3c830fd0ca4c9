"""Out-of-bounds writes, caught with guard bands (no memory-checking tool runs beside these
tests): every buffer of a package is placed between two 64 KiB bands of a known byte
pattern, the package's kernels run through their tuned launches on the interior pointers
(device-pointer path, tensor maps encoded for those pointers), and afterwards every band
must be intact and the outputs must match the oracle."""

import numpy as np
import pytest

from conftest import GOLDEN, PACKAGES
from thompiler import problems, runner, synth
from thompiler.device import DeviceKernel

pytestmark = pytest.mark.gpu

GUARD = 64 * 1024
PATTERN = 0xA5
ESIZE = {"f16": 2, "f32": 4, "f64": 8}


def _alloc(shape, dtype):
    import torch
    nbytes = int(np.prod(shape, dtype=np.int64)) * ESIZE[dtype] if shape else ESIZE[dtype]
    span = GUARD + (nbytes + 255) // 256 * 256 + GUARD
    t = torch.full((span,), PATTERN, dtype=torch.uint8, device="cuda")
    return t, nbytes


def _check_bands(name, t, nbytes):
    assert bool((t[:GUARD] == PATTERN).all()), f"{name}: bytes written below the buffer"
    assert bool((t[GUARD + nbytes:] == PATTERN).all()), f"{name}: bytes written past the buffer"


def _run_guarded(pkg, inputs):
    import torch
    bufs = {}
    for k in pkg.meta["kernels"]:
        for a in k["args"]:
            if a["name"] not in bufs:
                bufs[a["name"]] = (*_alloc(a["shape"], a["dtype"]), a)
    for name, (t, nbytes, a) in bufs.items():
        inner = t[GUARD:GUARD + nbytes]
        if name in inputs:
            inner.copy_(torch.from_numpy(np.ascontiguousarray(inputs[name]).view(np.uint8).reshape(-1)).cuda())
        else:
            inner.zero_()
    ptrs = {n: t.data_ptr() + GUARD for n, (t, _, _) in bufs.items()}
    for k in pkg.meta["kernels"]:
        dk = DeviceKernel(pkg.ir_path(k["entry"]))
        for z in k.get("zero_outputs", []):
            t, nbytes, _ = bufs[z]
            t[GUARD:GUARD + nbytes].zero_()
        dk({n: ptrs[n] for n in k["arg_order"]}, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert runner.read_error_word(dk.module, dk.plan) == 0
        dk.close()
    out = {}
    for name, (t, nbytes, a) in bufs.items():
        _check_bands(name, t, nbytes)
        raw = t[GUARD:GUARD + nbytes].cpu().numpy()
        out[name] = raw.view(problems.NP_DTYPES[a["dtype"]]).reshape(a["shape"])
    return out


@pytest.mark.parametrize("name", PACKAGES)
def test_package_writes_stay_in_bounds(name):
    from test_gpu_packages import assert_close, oracle, tol
    pkg = problems.load_package(GOLDEN / name)
    out = _run_guarded(pkg, problems.make_inputs(pkg))
    rtol, atol = tol(name)
    for o, want in oracle(name).items():
        if o in out:
            assert_close(out[o], want, rtol, atol, f"{name}/{o} (guarded)")


@pytest.mark.parametrize("builder,args", [(synth.attention_package, (1, 2, 256, 128)),
                                          (synth.attention_package, (1, 3, 384, 64)),
                                          (synth.matmul_package, (384, 320, 512)),
                                          (synth.matmul_package, (512, 384, 256)),
                                          (synth.pointwise_package, (1 << 20, "relu_mul")),
                                          (synth.sum_package, (1 << 20,))])
def test_tuned_family_writes_stay_in_bounds(tmp_path, builder, args):
    """The tuned families at sizes whose last tile is partial or whose tile count is not a
    multiple of the SM count, against the oracle interpreter (exact expression for attention).
    The matmul cases take the single-CTA kernel (M = 384) and the CTA-pair one (M = 512,
    N = 384: three 256 x 128 pair tiles per row band)."""
    pkg = problems.load_package(builder(tmp_path / "p", *args))
    inputs = problems.make_inputs(pkg)
    out = _run_guarded(pkg, inputs)
    (k,) = pkg.meta["kernels"]
    final = k["arg_order"][-1]
    if builder is synth.attention_package:
        q, kk, v = (inputs[n].astype(np.float64) for n in ("q", "k", "v"))
        s = q @ np.swapaxes(kk, -1, -2) / np.sqrt(q.shape[-1])
        p = np.exp(s - s.max(-1, keepdims=True))
        want = (p / p.sum(-1, keepdims=True)) @ v
        np.testing.assert_allclose(out[final].astype(np.float64), want, rtol=2e-2, atol=2e-3)
    else:
        from oracle.interp import run_package as oracle_run
        want = oracle_run(pkg.dir)[final]
        rtol, atol = {synth.matmul_package: (2e-2, 2e-3), synth.pointwise_package: (0, 0),
                      synth.sum_package: (1e-5, 1e-6)}[builder]
        np.testing.assert_allclose(out[final].astype(np.float64), np.asarray(want, np.float64), rtol=rtol,
                                   atol=atol)
