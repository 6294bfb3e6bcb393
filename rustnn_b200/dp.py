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


class Comm:
    """The library's own NCCL communicator (rnn_comm_*): the gradient sum of
    the batch-sharded step and the host watchdog that detects a rank that
    never joins a collective (rnn_comm_wait aborts the communicator and
    raises).  ``Comm.of(net)`` wraps a data-parallel network's communicator."""

    def __init__(self, rank: int, world: int, uid: bytes, device: int | None = None, _handle=None):
        import ctypes as C

        import torch

        from ._lib import call

        self.device = torch.cuda.current_device() if device is None else device
        self.owned = _handle is None
        if _handle is None:
            h = C.c_void_p()
            buf = (C.c_ubyte * len(uid)).from_buffer_copy(uid)
            call("rnn_comm_init", C.byref(h), self.device, rank, world, C.cast(buf, C.c_void_p))
            self.h = h
        else:
            self.h = _handle

    @classmethod
    def of(cls, net):
        import ctypes as C

        from ._lib import call

        h = C.c_void_p()
        call("rnn_resnet_comm", net.h, C.byref(h))
        return cls(0, 1, b"", device=net.device, _handle=h)

    def allreduce(self, ctx, grads, average: bool = False):
        import ctypes as C

        from ._lib import call

        call("rnn_allreduce_grads", ctx.bind(), self.h, C.c_void_p(grads.data_ptr()), grads.numel(), int(average))

    def wait(self, ctx, timeout_ms: int):
        """Waits for the context's stream; on a communicator error or after
        timeout_ms aborts the communicator and raises RnnError."""
        from ._lib import call

        call("rnn_comm_wait", ctx.bind(), self.h, int(timeout_ms))

    def check(self):
        from ._lib import call

        call("rnn_comm_check", self.h)

    def abort(self):
        from ._lib import call

        call("rnn_comm_abort", self.h)

    def close(self):
        from ._lib import lib

        if self.owned and self.h:
            lib().rnn_comm_destroy(self.h)
        self.h = None
