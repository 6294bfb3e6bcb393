"""Data-parallel ResNet step on 2 and 4 GPUs (one process per GPU, NCCL).

With SyncBN, ranks that each take a slice of a batch must reproduce the
single-process step on the whole batch (the reference's semantics: one
process, whole-batch BatchNorm statistics, loss averaged over the batch).
The ranks run as spawned child processes with a short NCCL setup; the
parent compares their parameters with the CPU oracle on the full batch.
Each case is skipped when fewer GPUs than its ranks are visible.
"""
import multiprocessing as mp
import os

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

CASES = {
    # name: (world, depth_n, width, global batch, steps, CUDA graph)
    "dp2-resnet8-w16": (2, 1, 16, 16, 2, False),
    # BASELINE config 5's network through bench.py's code path: graph replay
    # (eager, capture, replay), SyncBN over peer memory with the statistics
    # exchanged from the conv epilogue
    "dp2-resnet56-w64": (2, 9, 64, 16, 3, True),
    "dp4-resnet56-w64": (4, 9, 64, 32, 3, True),
}
NCLASS, SEED = 100, 0


def batch(n_full, step):
    rs = np.random.default_rng(1000 + step)
    u = rs.integers(0, 256, size=(n_full, 3, 32, 32)).astype(np.float32)
    x = ((u - 127.5) / 73.9).astype(np.float32)
    labels = rs.integers(0, NCLASS, size=n_full).astype(np.uint32)
    return x, labels


def _rank_main(rank, world, uid, sync_bn, case, q):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        import torch as T

        from rustnn_b200 import model

        _, depth, width, n_full, steps, graph = CASES[case]
        T.cuda.set_device(rank)
        net = model.ResNet(depth, width, NCLASS, SEED)
        if graph:
            net.use_graph(True)
        net.dp_init(rank, world, uid, sync_bn=sync_bn)
        per = n_full // world
        for step in range(steps):
            x, labels = batch(n_full, step)
            xs = T.from_numpy(np.ascontiguousarray(x[rank * per:(rank + 1) * per]).ravel()).cuda()
            ls = T.from_numpy(labels[rank * per:(rank + 1) * per].astype(np.int32)).cuda()
            net.train_step(xs, ls)
        T.cuda.synchronize()
        net.ctx.synchronize()
        q.put((rank, net.params(), net.buffers()))
        net.close()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None))


def _run(world, sync_bn, case):
    from rustnn_b200 import model

    uid = model.dp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, uid, sync_bn, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, params, bufs = q.get(timeout=600)
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


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("case", sorted(CASES))
def test_dp_syncbn_matches_single_process_full_batch(case):
    world, depth, width, n_full, steps, _ = CASES[case]
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    out = _run(world, True, case)
    for r in range(world):
        assert not isinstance(out[r][0], str), out[r][0]
    o = O.ResNet(depth, width, NCLASS, SEED)
    for step in range(steps):
        x, labels = batch(n_full, step)
        o.train_step(x.ravel(), labels)
    p0 = out[0][0]
    for r in range(1, world):
        assert np.array_equal(p0, out[r][0]), f"rank {r} diverged"
    assert rel(p0, o.params()) < 1e-4
    assert rel(out[0][1], o.buffers()) < 1e-4


# ------------------------------------------------------------------ communicator


def _comm_rank(rank, world, uid, mode, q, ev):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        import torch as T

        from rustnn_b200 import dp, ops
        from rustnn_b200._lib import RnnError

        T.cuda.set_device(rank)
        ctx = ops.default_context(rank)
        comm = dp.Comm(rank, world, uid, device=rank)
        g = T.full((1 << 20,), float(rank + 1), device=f"cuda:{rank}")
        comm.allreduce(ctx, g)
        comm.wait(ctx, 30_000)
        total = float(g[0].item())
        comm.allreduce(ctx, g, average=True)
        comm.wait(ctx, 30_000)
        mean = float(g[0].item())
        if mode == "ok":
            q.put((rank, total, mean, None))
            comm.close()
            return
        # a rank that stays alive but never joins the next collective: the
        # other rank's watchdog must end its wait with an error, not hang
        if rank == 0:
            comm.allreduce(ctx, g)
            try:
                comm.wait(ctx, 2_000)
                q.put((rank, total, mean, "no error"))
            except RnnError as e:
                q.put((rank, total, mean, str(e)))
            ev.set()
        else:
            ev.wait(120)
            comm.abort()
            q.put((rank, total, mean, "abstained"))
        comm.close()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, None, repr(e)))


def _run_comm(world, mode):
    from rustnn_b200 import model

    uid = model.dp_unique_id()
    ctx = mp.get_context("spawn")
    q, ev = ctx.Queue(), ctx.Event()
    procs = [ctx.Process(target=_comm_rank, args=(r, world, uid, mode, q, ev)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, total, mean, note = q.get(timeout=300)
            out[rank] = (total, mean, note)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return out


def test_comm_allreduce_grads_two_ranks():
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    out = _run_comm(2, "ok")
    for r in (0, 1):
        assert out[r][2] is None, out[r]
        assert out[r][0] == 3.0 and out[r][1] == 3.0  # 1 + 2 summed, then the mean of (3, 3)


def test_comm_watchdog_detects_a_rank_that_never_joins():
    """Rank 1 stays alive between collectives and skips the next one; rank
    0's rnn_comm_wait gives up after 2 s, aborts the communicator and
    reports RNN_ERR_NCCL instead of waiting forever (NVLS off)."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    out = _run_comm(2, "fail")
    assert out[1][2] == "abstained", out[1]
    assert "aborted" in out[0][2], out[0]
