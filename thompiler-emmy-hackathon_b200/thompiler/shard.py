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
