"""Splitting the naturally sharded workloads over the GPUs of one node.

One process per GPU (torchrun-style ``RANK`` / ``WORLD_SIZE``); the plumbing
is ``torch.distributed``:

* the big sum: the f32 array is cut into contiguous slices, one per rank
  (``slice_bounds``); each GPU reduces its slice with the compiled two-pass
  kernel and the f32 partials are combined by one all-reduce
  (``combine_partials``: NCCL on GPUs, gloo in the CPU tests);
* batched attention: the (batch, head) units are independent, so each rank
  takes a contiguous run of them (``unit_range``) and no collective is needed.

Slices start on ``align``-element boundaries so every rank's base address
keeps the 16-byte alignment the vectorised loads want; the last rank takes
the ragged end.  An empty slice (more ranks than aligned chunks) is legal and
contributes 0 to the sum.
"""

from __future__ import annotations


def slice_bounds(n: int, rank: int, world: int, align: int = 4) -> tuple[int, int]:
    """[start, end) of rank ``rank``'s contiguous slice of ``n`` elements."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if n < 0 or align < 1:
        raise ValueError(f"n={n}, align={align}")
    chunks = -(-n // align)                       # aligned chunks, the last one may be short
    per, extra = divmod(chunks, world)
    c0 = rank * per + min(rank, extra)
    c1 = c0 + per + (1 if rank < extra else 0)
    return min(n, c0 * align), min(n, c1 * align)


def unit_range(units: int, rank: int, world: int) -> tuple[int, int]:
    """[first, last) of rank ``rank``'s contiguous run of independent units."""
    return slice_bounds(units, rank, world, align=1)


def combine_partials(partial, group=None):
    """Sum the ranks' partial results in place (one all-reduce) and return the tensor."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial


def peer_table(module, rank: int, world: int, pointers: list[int]) -> None:
    """Write a full-sum module's peer globals: ``thc_peer_ptr[r]`` = rank r's mailbox (as this
    process addresses it), ``thc_rank``, ``thc_world`` (1 switches the combine off)."""
    import ctypes
    from thompiler import runner
    side = module.sidecar or {}
    peer = side.get("peer")
    if peer is None:
        raise ValueError("this module has no in-kernel peer combine")
    if not 1 <= world <= peer["max_ranks"] or len(pointers) != world:
        raise ValueError(f"world {world} with {len(pointers)} mailboxes (at most {peer['max_ranks']})")
    lib = runner.library()
    tab = (ctypes.c_uint64 * peer["max_ranks"])(*(pointers + [0] * (peer["max_ranks"] - world)))
    for name, buf in ((peer["table"], tab), (peer["rank"], ctypes.c_uint32(rank)),
                      (peer["world"], ctypes.c_uint32(world))):
        dst, size = module.global_ptr(name)
        runner.check(lib.thr_memcpy_htod(dst, ctypes.byref(buf), ctypes.sizeof(buf), 0), f"write {name}")
    runner.check(lib.thr_synchronize(), "synchronise")


class PeerCombine:
    """Bind a compiled full-sum module to the other ranks' copies of it, so its finishing CTA
    adds the per-GPU results over NVLink (see ``families.strided``) -- the sharded sum's
    exchange step without a separate collective launch.

    Every rank allocates a zeroed mailbox (CUDA IPC-exportable), the handles travel once through
    ``torch.distributed.all_gather_object``, and each rank maps the others' mailboxes.  Call
    ``close`` on every rank (it switches the combine off and unmaps)."""

    SLOT_BYTES = 8

    def __init__(self, module, rank: int, world: int, group=None):
        import ctypes
        import torch.distributed as dist
        from thompiler import runner
        self.module, self.rank, self.world = module, rank, world
        lib = runner.library()
        mine, handle = ctypes.c_uint64(), ctypes.create_string_buffer(64)
        slots = (module.sidecar or {}).get("peer", {}).get("max_ranks", 8)
        runner.check(lib.thr_peer_alloc(slots * self.SLOT_BYTES, ctypes.byref(mine), handle), "mailbox")
        self.mine, self.opened = mine.value, []
        handles = [None] * world
        dist.all_gather_object(handles, handle.raw, group=group)
        pointers = []
        for r, h in enumerate(handles):
            if r == rank:
                pointers.append(self.mine)
                continue
            q = ctypes.c_uint64()
            runner.check(lib.thr_peer_open(h, ctypes.byref(q)), f"map rank {r}'s mailbox")
            self.opened.append(q.value)
            pointers.append(q.value)
        peer_table(module, rank, world, pointers)
        dist.barrier(group=group)            # every rank's table is in place before any launch

    def close(self, group=None) -> None:
        """Switch the combine off, then unmap and free -- after every rank's kernels have
        finished (device synchronise + barrier), so no rank still writes into a mailbox."""
        import torch.distributed as dist
        from thompiler import runner
        lib = runner.library()
        runner.check(lib.thr_synchronize(), "synchronise")
        dist.barrier(group=group)
        peer_table(self.module, 0, 1, [self.mine])
        for q in self.opened:
            lib.thr_peer_close(q)
        lib.thr_peer_free(self.mine)
        self.opened = []


class RankFailure(RuntimeError):
    """Some ranks did not reach a step in time: ``missing`` lists them."""

    def __init__(self, step: int, missing: list[int], timeout_s: float):
        super().__init__(f"ranks {missing} did not reach step {step} within {timeout_s:.1f} s")
        self.step, self.missing = step, missing


class StepMonitor:
    """Host-side failure detection between steps: before launching step ``s`` (its kernels and
    collectives), each rank posts ``s`` to a shared key-value store (a ``torch.distributed``
    Store) and waits, with a time limit, for every other rank's post.  A rank that raised,
    exited or stopped is named in a ``RankFailure`` on the others before they launch anything
    that would wait for it -- no kernel or collective is left waiting on a rank that is gone.
    Keys are namespaced by ``tag`` so several monitors can share one store."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0, tag: str = "step"):
        if world < 1 or not 0 <= rank < world:
            raise ValueError(f"rank {rank} of world {world}")
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.tag = float(timeout_s), tag

    def _key(self, step: int, rank: int) -> str:
        return f"{self.tag}/{step}/{rank}"

    def arrive(self, step: int) -> None:
        self.store.set(self._key(step, self.rank), "1")

    def wait_all(self, step: int) -> None:
        import time
        from datetime import timedelta
        deadline = time.monotonic() + self.timeout_s
        missing = []
        for r in range(self.world):
            left = max(0.0, deadline - time.monotonic())
            try:
                self.store.wait([self._key(step, r)], timedelta(seconds=max(left, 0.001)))
            except Exception:                  # the store's timeout (a RuntimeError / DistStoreError)
                missing.append(r)
        if missing:
            raise RankFailure(step, missing, self.timeout_s)

    def step(self, step: int) -> None:
        """Post this rank's arrival at ``step`` and wait for all the others'."""
        self.arrive(step)
        self.wait_all(step)
