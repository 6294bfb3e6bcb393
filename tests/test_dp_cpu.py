"""World-size-2 gloo tests (CPU) of the data-parallel host plumbing:
sharding, the NCCL-id broadcast and the max-over-ranks timing rule, plus the
data-parallel gradient semantics on the CPU oracle: two ranks that each take
half a batch and average their gradients reproduce the whole-batch gradient
of every parameter that BatchNorm statistics do not couple (the classifier),
which is what the library's 1/world-scaled allreduce relies on."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as tmp

from rustnn_b200 import dp


def test_shard_partitions_the_batch():
    got = [dp.shard(1024, 8, r) for r in range(8)]
    assert got == [(128 * r, 128) for r in range(8)]
    with pytest.raises(ValueError):
        dp.shard(1000, 3, 0)
    with pytest.raises(ValueError):
        dp.shard(16, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        uid = dp.share_unique_id(lambda: bytes(range(128)) if rank == 0 else b"x")
        t = dp.max_over_ranks([float(rank + 1), 10.0 - rank])
        # data-parallel gradient semantics on the oracle classifier (nn.rs:501-563)
        from oracle import oracle as O

        rs = np.random.default_rng(0)
        n, fin, fout = 8, 6, 5
        x = rs.standard_normal((n, fin)).astype(np.float32)
        w = rs.standard_normal((fout, fin)).astype(np.float32)
        labels = rs.integers(0, fout, n).astype(np.uint32)
        lo, cnt = dp.shard(n, world, rank)
        xs = np.ascontiguousarray(x[lo:lo + cnt])
        logits = np.empty(cnt * fout, np.float32)
        b = np.zeros(fout, np.float32)
        O.lib().orc_fc_fwd(xs.ravel(), cnt, fin, fout, w.ravel(), b, logits)
        _, d, _ = O.softmax_ce(logits, labels[lo:lo + cnt], fout, 0.1)
        dw, db, dx = np.zeros(fout * fin, np.float32), np.zeros(fout, np.float32), np.zeros(cnt * fin, np.float32)
        O.lib().orc_fc_bwd(xs.ravel(), d, cnt, fin, fout, w.ravel(), dw, db, dx)
        g = torch.from_numpy(dw)
        dist.all_reduce(g)  # sum over ranks, then 1/world as in the SGD kernel
        g = (g / world).numpy()
        # whole batch in one process
        logits_f = np.empty(n * fout, np.float32)
        O.lib().orc_fc_fwd(x.ravel(), n, fin, fout, w.ravel(), b, logits_f)
        _, df, _ = O.softmax_ce(logits_f, labels, fout, 0.1)
        dwf, dbf, dxf = np.zeros(fout * fin, np.float32), np.zeros(fout, np.float32), np.zeros(n * fin, np.float32)
        O.lib().orc_fc_bwd(x.ravel(), df, n, fin, fout, w.ravel(), dwf, dbf, dxf)
        err = float(np.abs(g - dwf).max() / np.abs(dwf).max())
        out.put((rank, uid, t, err))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_plumbing_and_gradient_mean():
    ctx = tmp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, uid, t, err = q.get(timeout=120)
            res[rank] = (uid, t, err)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert res[0][0] == res[1][0] == bytes(range(128))
    assert res[0][1] == res[1][1] == [2.0, 10.0]
    assert res[0][2] < 1e-5 and res[1][2] < 1e-5
