"""Data-parallel ResNet step on 2 GPUs (one process per GPU, NCCL).

With SyncBN, two ranks that each take half of a batch must reproduce the
single-process step on the whole batch (the reference's semantics: one
process, whole-batch BatchNorm statistics, loss averaged over the batch).
The ranks run as spawned child processes with a short NCCL setup; the
parent compares their parameters with the CPU oracle on the full batch.
Skipped when fewer than two GPUs are visible.
"""
import multiprocessing as mp
import os

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

N_FULL, DEPTH, WIDTH, NCLASS, SEED, STEPS = 16, 1, 16, 100, 0, 2


def batch(step):
    rs = np.random.default_rng(1000 + step)
    u = rs.integers(0, 256, size=(N_FULL, 3, 32, 32)).astype(np.float32)
    x = ((u - 127.5) / 73.9).astype(np.float32)
    labels = rs.integers(0, NCLASS, size=N_FULL).astype(np.uint32)
    return x, labels


def _rank_main(rank, world, uid, sync_bn, q):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        import torch as T

        from rustnn_b200 import model

        T.cuda.set_device(rank)
        net = model.ResNet(DEPTH, WIDTH, NCLASS, SEED)
        net.dp_init(rank, world, uid, sync_bn=sync_bn)
        per = N_FULL // world
        for step in range(STEPS):
            x, labels = batch(step)
            xs = T.from_numpy(np.ascontiguousarray(x[rank * per:(rank + 1) * per]).ravel()).cuda()
            ls = T.from_numpy(labels[rank * per:(rank + 1) * per].astype(np.int32)).cuda()
            net.train_step(xs, ls)
        T.cuda.synchronize()
        net.ctx.synchronize()
        q.put((rank, net.params(), net.buffers()))
        net.close()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None))


def _run(world, sync_bn):
    from rustnn_b200 import model

    uid = model.dp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, uid, sync_bn, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, params, bufs = q.get(timeout=300)
            out[rank] = (params, bufs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return out


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_dp2_syncbn_matches_single_process_full_batch():
    out = _run(2, True)
    for r in (0, 1):
        assert not isinstance(out[r][0], str), out[r][0]
    o = O.ResNet(DEPTH, WIDTH, NCLASS, SEED)
    for step in range(STEPS):
        x, labels = batch(step)
        o.train_step(x.ravel(), labels)
    p0, p1 = out[0][0], out[1][0]
    assert np.array_equal(p0, p1), "ranks diverged"
    assert rel(p0, o.params()) < 1e-4
    assert rel(out[0][1], o.buffers()) < 1e-4
