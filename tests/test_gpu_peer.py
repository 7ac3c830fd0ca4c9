"""In-kernel combine of a sharded sum over peer memory (families.strided, thompiler.shard).

* one GPU: a module told it has two ranks whose second mailbox slot nobody writes gives up
  after its bounded wait, sets bit 0 of its error word, returns, and the context stays usable
  (the next launch with the combine off is correct);
* two GPUs (skipped with fewer): each process reduces its contiguous slice, the kernels add
  their results over NVLink, and both ranks hold the full-array sum after every launch --
  several launches, so the epochs advance in step.  NVLS is off (``NCCL_NVLS_ENABLE=0``); the
  mailboxes are plain CUDA IPC memory.
Tolerance for the f32 sums: relative 1e-5 of the float64 sum (plus 1e-3 absolute).
"""

import ctypes
import os
import socket

import numpy as np
import pytest

from thompiler import runner, synth
from thompiler.device import DeviceKernel
from thompiler.shard import PeerCombine, peer_table, slice_bounds

pytestmark = pytest.mark.gpu


def _sum_kernel(tmp, n, device=0):
    k = DeviceKernel(synth.sum_package(tmp / f"sum_{n}", n) / "k_sum_1_reduce.ir.json", device=device)
    assert k.module.sidecar.get("peer"), "the full-sum module should carry the peer combine"
    return k


def _reset_error(k):
    dst, _ = k.module.global_ptr("thc_error")
    z = ctypes.c_uint32(0)
    runner.check(runner.library().thr_memcpy_htod(dst, ctypes.byref(z), 4, 0), "clear error word")
    runner.check(runner.library().thr_synchronize(), "sync")


def test_peer_wait_gives_up_and_context_survives(tmp_path):
    import torch
    n = 1 << 20
    k = _sum_kernel(tmp_path, n)
    x = torch.rand(n, device="cuda", generator=torch.Generator(device="cuda").manual_seed(5)) * 2 - 1
    out = torch.zeros(1, device="cuda")
    lib = runner.library()
    mine, h = ctypes.c_uint64(), ctypes.create_string_buffer(64)
    runner.check(lib.thr_peer_alloc(64, ctypes.byref(mine), h), "mailbox")
    try:
        _reset_error(k)
        peer_table(k.module, 0, 2, [mine.value, mine.value])     # "rank 1" never publishes
        k({"x": x.data_ptr(), "sum_1": out.data_ptr()}, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert runner.read_error_word(k.module, k.plan) & 1
        want = float(x.double().sum())
        assert abs(float(out.item()) - want) <= 1e-5 * max(1.0, abs(want)) + 1e-3   # own value only
        peer_table(k.module, 0, 1, [mine.value])
        _reset_error(k)
        out.zero_()
        k({"x": x.data_ptr(), "sum_1": out.data_ptr()}, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert runner.read_error_word(k.module, k.plan) == 0
        assert abs(float(out.item()) - want) <= 1e-5 * max(1.0, abs(want)) + 1e-3
    finally:
        lib.thr_peer_free(mine.value)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, n, out_dir):
    import pathlib
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    runner.init(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device(f"cuda:{rank}"))
    try:
        a, b = slice_bounds(n, rank, world)
        k = _sum_kernel(pathlib.Path(out_dir) / f"r{rank}", b - a, device=rank)
        pc = PeerCombine(k.module, rank, world)
        got = []
        for launch in range(3):
            full = torch.rand(n, generator=torch.Generator().manual_seed(100 + launch)) * 2 - 1
            x = full[a:b].to(f"cuda:{rank}")
            out = torch.zeros(1, device=f"cuda:{rank}")
            k({"x": x.data_ptr(), "sum_1": out.data_ptr()}, torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            got.append((float(out.item()), float(full.double().sum())))
        err = runner.read_error_word(k.module, k.plan)
        pc.close()
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.array([[g, w, err] for g, w in got]))
    finally:
        dist.destroy_process_group()


def test_peer_combine_two_gpus(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    n = (1 << 22) + 12
    mp.spawn(_rank, args=(2, _free_port(), n, str(tmp_path)), nprocs=2, join=True)
    res = [np.load(tmp_path / f"rank{r}.npy") for r in range(2)]
    for r in res:
        assert (r[:, 2] == 0).all(), "a peer wait gave up"
        for got, want, _ in r:
            assert abs(got - want) <= 1e-5 * max(1.0, abs(want)) + 1e-3, (got, want)
    assert (res[0][:, 0] == res[1][:, 0]).all(), "ranks disagree"
