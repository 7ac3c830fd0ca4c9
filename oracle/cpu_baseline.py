"""CPU baselines: the reference's CPU path for each benchmark workload.

Test infrastructure (used only by tests and by bench.py's cpu_baseline /
reference leg).  The reference's semantics for a problem is the torch
expression it was generated from, evaluated on the CPU (reference
tools/expressions_open.py:33-105, tests/expressions_mma.py:12-21 and the
``code`` field of every meta.json); these functions restate those
expressions for the benchmark shapes and time them on the host's cores
over a bounded sample of the workload.
"""

from __future__ import annotations

import os
import time

import torch


def threads() -> int:
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def softmax_rows(x):
    return torch.softmax(x, dim=-1)


def rmsnorm_rows(x, w, eps):
    return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps) * w


def l2norm_rows(x):
    return x / torch.sqrt((x * x).sum(-1, keepdim=True))


def matmul_f16(a, b_col_major):
    """C = A @ B with f16 inputs and an f32 result; B stored [N, K]."""
    return (a @ b_col_major.t()).float()


def attention_f16(q, k, v):
    s = (q.float() @ k.float().transpose(-1, -2)) / (q.shape[-1] ** 0.5)
    return (torch.softmax(s, dim=-1) @ v.float()).half()


def time_call(fn, reps: int = 3) -> float:
    fn()
    best = float("inf")
    for _ in range(reps):
        t = time.perf_counter()
        fn()
        best = min(best, time.perf_counter() - t)
    return best


def rowops_sample(rows: int, cols: int, eps: float = 1e-6, seed: int = 0) -> dict:
    """Seconds for softmax + RMSNorm + L2-normalise over a [rows, cols] f32 sample."""
    n = threads()
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g)
    w = torch.rand(cols, generator=g) + 0.5
    sec = time_call(lambda: (softmax_rows(x), rmsnorm_rows(x, w, eps), l2norm_rows(x)))
    return {"seconds": sec, "rows": rows, "cols": cols, "cores": n}


def sum_sample(n_elems: int, seed: int = 0) -> dict:
    n = threads()
    x = torch.rand(n_elems, generator=torch.Generator().manual_seed(seed)) * 2 - 1
    sec = time_call(lambda: torch.sum(x))
    return {"seconds": sec, "elements": n_elems, "cores": n}


def pointwise_sample(n_elems: int, seed: int = 0) -> dict:
    """relu(x0) * x1 (problems/p03_relu_mul's expression) on f32[n_elems]."""
    c = threads()
    g = torch.Generator().manual_seed(seed)
    x0, x1 = torch.randn(n_elems, generator=g), torch.randn(n_elems, generator=g)
    sec = time_call(lambda: torch.relu(x0) * x1)
    return {"seconds": sec, "elements": n_elems, "cores": c}


def matmul_sample(m: int, n: int, k: int, seed: int = 0) -> dict:
    c = threads()
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(m, k, generator=g) * 0.02).half()
    b = (torch.randn(n, k, generator=g) * 0.02).half()
    sec = time_call(lambda: matmul_f16(a, b), reps=1)
    return {"seconds": sec, "m": m, "n": n, "k": k, "cores": c}


def attention_sample(bh: int, s: int, d: int, seed: int = 0) -> dict:
    c = threads()
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(bh, s, d, generator=g).half() for _ in range(3))
    sec = time_call(lambda: attention_f16(q, k, v), reps=1)
    return {"seconds": sec, "heads": bh, "seq": s, "d": d, "cores": c}
