"""The SyncBN peer exchange (rnn_batchnorm_stats_peer_dev) on one GPU: two
mailboxes in this device's memory stand for rank 0's and rank 1's, the test
plays rank 1 by writing its mailbox from the host.  Covers the arithmetic
(own sums + the peer's slot, in rank order) and the bounded wait: a peer that
never raises its flag makes the kernel give up after wait_ms and report
RNN_ERR_DEVICE through rnn_ctx_synchronize, and the context stays usable."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HEADER = 128  # mailbox layout: u64 flag, then two slots of [cmax][2] f64 from byte 128


def _slot(mb, cmax, s):
    """Slot s of a mailbox (a uint8 CUDA tensor) as a [cmax, 2] f64 view."""
    off = HEADER + s * cmax * 2 * 8
    return mb[off : off + cmax * 2 * 8].view(torch.float64).view(cmax, 2)


def _flag(mb):
    return mb[:8].view(torch.int64)


def test_peer_exchange_sums_and_timeout():
    from rustnn_b200 import _lib, ops

    L = _lib.lib()
    ctx = ops.default_context()
    n, c, hw, cmax = 8, 24, 64, 32
    nbytes = L.rnn_peer_mailbox_bytes(cmax)
    assert nbytes == HEADER + 2 * cmax * 2 * 8
    g = torch.Generator().manual_seed(7)
    y = (torch.randn(n, c, hw, generator=g) * 3 + 1).cuda()
    mb = [torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(2)]
    mail = torch.tensor([m.data_ptr() for m in mb], dtype=torch.int64, device="cuda")
    seq = torch.zeros(1, dtype=torch.int64, device="cuda")
    sums = torch.zeros(c, 2, dtype=torch.float64, device="cuda")
    torch.cuda.synchronize()

    def call(wait_ms):
        rc = L.rnn_batchnorm_stats_peer_dev(
            ctx.bind(), C.c_void_p(y.data_ptr()), n, c, hw, 0, 2, C.c_void_p(mail.data_ptr()),
            C.c_void_p(seq.data_ptr()), cmax, wait_ms, C.c_void_p(sums.data_ptr()))
        assert rc == 0, L.rnn_last_error()
        return L.rnn_ctx_synchronize(ctx.bind())

    yd = y.double().cpu()
    want = torch.stack([yd.sum(dim=(0, 2)), (yd * yd).sum(dim=(0, 2))], dim=1)

    # rank 1 never publishes exchange 1: the wait gives up after 300 ms,
    # the error word is reported once, and the sums are this rank's own plus
    # rank 1's stale (zero) slot
    rc = call(300)
    assert rc == -4, rc
    assert "peer" in L.rnn_last_error().decode()
    own = sums.cpu().clone()
    torch.testing.assert_close(own, want, rtol=1e-12, atol=1e-9)
    assert int(_flag(mb[0]).item()) == 1  # this rank published exchange 1 ...
    assert torch.equal(_slot(mb[0], cmax, 1)[:c].cpu(), own)  # ... in slot 1
    assert L.rnn_ctx_synchronize(ctx.bind()) == 0  # reported once, then cleared

    # exchange 2 (slot 0): rank 1 has published before this rank arrives
    peer = torch.randn(c, 2, generator=g, dtype=torch.float64) * 100
    _slot(mb[1], cmax, 0)[:c].copy_(peer)
    _flag(mb[1]).fill_(2)
    torch.cuda.synchronize()
    assert call(2000) == 0, L.rnn_last_error()
    assert int(seq.item()) == 2 and int(_flag(mb[0]).item()) == 2
    # rank order: 0.0 + own + peer, in f64, bit for bit
    assert torch.equal(sums.cpu(), (own + peer))
    assert torch.equal(_slot(mb[0], cmax, 0)[:c].cpu(), own)


def test_peer_exchange_rejects_bad_arguments():
    from rustnn_b200 import _lib, ops

    L = _lib.lib()
    ctx = ops.default_context()
    y = torch.zeros(2, 8, 16, device="cuda")
    mb = torch.zeros(L.rnn_peer_mailbox_bytes(8), dtype=torch.uint8, device="cuda")
    mail = torch.tensor([mb.data_ptr()], dtype=torch.int64, device="cuda")
    seq = torch.zeros(1, dtype=torch.int64, device="cuda")
    sums = torch.zeros(8, 2, dtype=torch.float64, device="cuda")

    def rc(c, cmax, rank, world, wait_ms, hw=16):
        return L.rnn_batchnorm_stats_peer_dev(
            ctx.bind(), C.c_void_p(y.data_ptr()), 2, c, hw, rank, world, C.c_void_p(mail.data_ptr()),
            C.c_void_p(seq.data_ptr()), cmax, wait_ms, C.c_void_p(sums.data_ptr()))

    assert rc(8, 4, 0, 1, 100) == -1  # c > cmax
    assert rc(8, 8, 1, 1, 100) == -1  # rank outside the world
    assert rc(8, 8, 0, 1, 0) == -1  # no wait bound
    assert rc(8, 8, 0, 1, 100, hw=6) == -1  # hw % 4 != 0
    # a world of one: plain statistics, no exchange
    assert rc(8, 8, 0, 1, 100) == 0
    assert L.rnn_ctx_synchronize(ctx.bind()) == 0
    assert int(seq.item()) == 0
