"""Host-side logic of the multi-GPU paths, on the CPU.

* ``slice_bounds`` / ``unit_range`` cover every element exactly once, in rank
  order, with aligned starts, for ragged sizes and more ranks than chunks;
* two and three ``gloo`` ranks (processes, 127.0.0.1) run the big-sum plan --
  slice, per-rank partial, one all-reduce -- and the attention plan -- a
  contiguous run of (batch, head) units per rank, no collective until the
  test gathers the pieces -- against the single-process result.  The per-rank
  partials come from the numpy expressions the problems were generated from
  (the GPU kernels are covered by the ``-m gpu`` tests).
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from thompiler.shard import combine_partials, slice_bounds, unit_range


@pytest.mark.parametrize("n", [0, 1, 3, 4, 5, 17, 1000, 1 << 20, (1 << 20) + 7])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_slices_cover_once(n, world):
    bounds = [slice_bounds(n, r, world) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == n
    for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
        assert a1 == b0
    for a0, a1 in bounds:
        assert 0 <= a0 <= a1 <= n
        assert a0 % 4 == 0 or a0 == n
    sizes = [b - a for a, b in bounds]
    assert max(sizes) - min(sizes) < 2 * 4      # one aligned chunk, plus the short last one


def test_units_even_split():
    assert [unit_range(128, r, 8) for r in range(8)] == [(16 * r, 16 * r + 16) for r in range(8)]
    assert [unit_range(128, r, 3) for r in range(3)] == [(0, 43), (43, 86), (86, 128)]
    with pytest.raises(ValueError):
        slice_bounds(10, 2, 2)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _sdpa(q, k, v):
    s = q @ np.swapaxes(k, -1, -2) / np.sqrt(q.shape[-1])
    p = np.exp(s - s.max(-1, keepdims=True))
    return (p / p.sum(-1, keepdims=True)) @ v


def _worker(rank, world, port, n, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # big sum: this rank's slice -> f32 partial -> all-reduce
        x = np.random.default_rng(0).uniform(-1, 1, n).astype(np.float32)
        a, b = slice_bounds(n, rank, world)
        part = torch.tensor([float(np.sum(x[a:b], dtype=np.float64))], dtype=torch.float32)
        total = combine_partials(part)
        # attention: (batch, head) units split over the ranks, gathered for the check
        B, H, S, D = 2, 5, 16, 8                # 10 units: 5 + 5 on two ranks, 4 + 3 + 3 on three
        g = np.random.default_rng(1)
        q, k, v = (g.standard_normal((B * H, S, D)) for _ in range(3))
        u0, u1 = unit_range(B * H, rank, world)
        mine = torch.from_numpy(_sdpa(q[u0:u1], k[u0:u1], v[u0:u1]).reshape(-1))
        sizes = [unit_range(B * H, r, world)[1] - unit_range(B * H, r, world)[0] for r in range(world)]
        bufs = [torch.zeros(s * S * D, dtype=torch.float64) for s in sizes]
        if len(set(sizes)) == 1:
            dist.all_gather(bufs, mine)
        else:                                   # ragged runs: gather through rank 0 one by one
            for r in range(1, world):
                if rank == r:
                    dist.send(mine, 0)
                elif rank == 0:
                    dist.recv(bufs[r], r)
            bufs[0] = mine
        if rank == 0:
            att = torch.cat(bufs).numpy().reshape(B * H, S, D)
            np.save(os.path.join(out_dir, "sum.npy"), np.array([float(total[0])]))
            np.save(os.path.join(out_dir, "att.npy"), att)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_ranks_match_single_process(tmp_path, world):
    n = 100_003
    mp.spawn(_worker, args=(world, _free_port(), n, str(tmp_path)), nprocs=world, join=True)
    x = np.random.default_rng(0).uniform(-1, 1, n).astype(np.float32)
    got = float(np.load(tmp_path / "sum.npy")[0])
    want = float(np.sum(x, dtype=np.float64))
    assert abs(got - want) <= 1e-5 * max(1.0, abs(want)) + 1e-6 * n ** 0.5
    B, H, S, D = 2, 5, 16, 8
    g = np.random.default_rng(1)
    q, k, v = (g.standard_normal((B * H, S, D)) for _ in range(3))
    np.testing.assert_allclose(np.load(tmp_path / "att.npy"), _sdpa(q, k, v), rtol=1e-12, atol=1e-12)
