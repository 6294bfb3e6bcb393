"""Tier-2 runtime entries of the C ABI on one GPU: device memory and copies
on a context's stream (rnn_alloc / rnn_memcpy_* / rnn_free), and the
communicator's gradient sum and watchdog on a world of one rank."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_alloc_copy_round_trip():
    from rustnn_b200 import _lib, ops

    L = _lib.lib()
    ctx = ops.default_context()
    host = np.arange(1 << 20, dtype=np.float32) * np.float32(0.5)
    back = np.zeros_like(host)
    p = C.c_void_p()
    assert L.rnn_alloc(ctx.bind(), host.nbytes, C.byref(p)) == 0, L.rnn_last_error()
    assert L.rnn_memcpy_h2d(ctx.bind(), p, C.c_void_p(host.ctypes.data), host.nbytes) == 0
    assert L.rnn_memcpy_d2h(ctx.bind(), C.c_void_p(back.ctypes.data), p, host.nbytes) == 0
    assert L.rnn_ctx_synchronize(ctx.bind()) == 0
    assert np.array_equal(back, host)
    assert L.rnn_free(ctx.bind(), p) == 0
    # a copy past the end of an allocation is refused on the host
    q = C.c_void_p()
    assert L.rnn_alloc(ctx.bind(), 256, C.byref(q)) == 0
    assert L.rnn_memcpy_h2d(ctx.bind(), q, C.c_void_p(host.ctypes.data), host.nbytes) == -1
    assert L.rnn_free(ctx.bind(), q) == 0


def test_comm_world_of_one():
    from rustnn_b200 import dp, model, ops

    ctx = ops.default_context()
    comm = dp.Comm(0, 1, model.dp_unique_id())
    g = torch.arange(1000, dtype=torch.float32, device="cuda")
    want = g.clone()
    comm.allreduce(ctx, g)
    comm.allreduce(ctx, g, average=True)
    comm.wait(ctx, 10_000)
    comm.check()
    assert torch.equal(g, want)
    comm.close()
