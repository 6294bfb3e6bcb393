"""Host-side plumbing of the data-parallel step (one process per GPU).

The exchange itself (gradient sum, SyncBN statistics) runs inside the C
library on its own NCCL communicator; this module holds what the launcher
needs around it, over any torch.distributed backend (NCCL on GPUs, gloo in
the CPU tests):

* ``shard(global_batch, world, rank)``: rank r takes images
  [r*B/n, (r+1)*B/n) of the global batch;
* ``share_unique_id(make)``: rank 0 creates the NCCL unique id, every rank
  receives the same bytes;
* ``max_over_ranks(values)``: the timing rule (max of per-rank device times).
"""
from __future__ import annotations

from typing import Callable, Sequence


def shard(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """(first image, count) of this rank's shard; the batch must divide evenly."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if global_batch % world:
        raise ValueError(f"global batch {global_batch} does not divide over {world} ranks")
    per = global_batch // world
    return rank * per, per


def share_unique_id(make: Callable[[], bytes]) -> bytes:
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size() == 1:
        return make()
    box = [make() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(box, src=0)
    uid = box[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise RuntimeError("NCCL unique id broadcast failed")
    return bytes(uid)


def max_over_ranks(values: Sequence[float], device=None) -> list[float]:
    import torch
    import torch.distributed as dist

    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()
