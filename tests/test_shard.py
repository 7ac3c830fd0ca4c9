"""Host-side logic of the multi-GPU paths, on the CPU.

* ``slice_bounds`` / ``unit_range`` cover every element exactly once, in rank
  order, with aligned starts, for ragged sizes and more ranks than chunks;
* two and three ``gloo`` ranks (processes, 127.0.0.1) run the big-sum plan --
  slice, per-rank partial, one all-reduce -- and the attention plan -- a
  contiguous run of (batch, head) units per rank, no collective until the
  test gathers the pieces -- against the single-process result.  The per-rank
  partials come from the numpy expressions the problems were generated from
  (the GPU kernels are covered by the ``-m gpu`` tests);
* failure detection on the host: a rank that raises or stops is named by the
  others' ``StepMonitor`` before the next step's collective, and a collective a
  rank skips ends with the process group's time-out error.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from thompiler.shard import RankFailure, StepMonitor, combine_partials, slice_bounds, unit_range


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


# ---- failure detection on the host (gloo ranks; nothing runs on a GPU) --------------------

def _failing_worker(rank, world, port, mode, out_dir, timeout_s):
    """Rank 1 misbehaves (``mode``): raises before the step, or stays alive but stops posting
    steps, or skips the collective; rank 0 records what it saw."""
    import json
    import time
    from datetime import timedelta
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))
    mon = StepMonitor(store, rank, world, timeout_s=timeout_s)
    seen = {"steps": 0, "error": None, "missing": None}
    t0 = time.monotonic()
    try:
        for step in range(3):
            if rank == 1 and step == 1:
                if mode == "raise":
                    raise RuntimeError("rank 1 fails between steps")
                if mode == "stall":
                    time.sleep(timeout_s + 3)          # alive, but never reaches step 1
                    return
            mon.step(step)
            if rank == 1 and step == 1 and mode == "skip_collective":
                time.sleep(timeout_s + 3)              # reached the step, skips its all-reduce
                return
            combine_partials(torch.ones(1))
            seen["steps"] += 1
    except RankFailure as e:
        seen["error"], seen["missing"] = "RankFailure", e.missing
    except Exception as e:                             # the collective's own error or time-out
        seen["error"] = type(e).__name__
    finally:
        seen["elapsed"] = time.monotonic() - t0
        if rank == 0:
            with open(os.path.join(out_dir, "rank0.json"), "w") as f:
                json.dump(seen, f)


def _run_failing(tmp_path, mode, timeout_s=3.0):
    import json
    ctx = mp.get_context("spawn")
    port = _free_port()
    ps = [ctx.Process(target=_failing_worker, args=(r, 2, port, mode, str(tmp_path), timeout_s)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=60)
    for p in ps:
        if p.is_alive():
            p.kill()
            p.join()
    return json.loads((tmp_path / "rank0.json").read_text())


@pytest.mark.parametrize("mode", ["raise", "stall"])
def test_rank_that_leaves_is_named_before_the_next_step(tmp_path, mode):
    """A rank that raises (its process exits) or stops reaching steps: the survivor's monitor
    names it within the time limit, after the one step they completed together, and never
    enters the next step's collective."""
    seen = _run_failing(tmp_path, mode)
    assert seen["error"] == "RankFailure" and seen["missing"] == [1], seen
    assert seen["steps"] == 1 and seen["elapsed"] < 3.0 + 5, seen


def test_collective_left_waiting_times_out(tmp_path):
    """A rank that reached the step but skips its collective: the survivor's all-reduce ends with
    the process group's time-out error instead of waiting for good."""
    seen = _run_failing(tmp_path, "skip_collective")
    assert seen["error"] is not None and seen["error"] != "RankFailure", seen
    assert seen["steps"] == 1 and seen["elapsed"] < 3.0 + 10, seen


def test_step_monitor_single_process():
    store = dist.HashStore()
    mon = StepMonitor(store, 0, 1, timeout_s=0.5)
    mon.step(0)
    mon.step(1)
    other = StepMonitor(store, 0, 2, timeout_s=0.2)      # a world of two with rank 1 absent
    other.arrive(5)
    with pytest.raises(RankFailure) as e:
        other.wait_all(5)
    assert e.value.missing == [1]
    with pytest.raises(ValueError):
        StepMonitor(store, 2, 2)
