"""Data-parallel rustvit step (rnn_rustvit_dp_attach): one process per GPU,
each rank runs its own shard of the batch, and the step averages the flat
gradient (before clip_) and the BatchNorm running statistics over the ranks
on the library's NCCL communicator.

On one GPU a one-rank communicator must leave the step bit-identical to the
plain step (the averages are identities).  On two GPUs the ranks, fed
different shards and drop seeds, must end every step with bit-identical
parameters, moments, EMA and buffers, different from what either shard
alone produces, and within 1e-4 (relative Frobenius) of the CPU oracle's
restatement of the sharded step (oracle.rustvit.dp_step).  The two-rank
case is skipped when fewer GPUs are visible.
"""
import multiprocessing as mp
import os

import numpy as np
import pytest

from oracle import oracle as O
from oracle import rustvit as RV

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TINY = dict(width=4, cmid=6, dim=8, heads=2, depth3=2, dim4=12, heads4=2, depth4=1, mem_at=[1], droppath=0.2,
            img=16)
TINY_PARENT = np.array([0, 0, 1, 1, 2, 2], np.uint32)
TOL = 1e-4


def rel(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    den = np.linalg.norm(want)
    return float(np.linalg.norm(got - want) / (den if den > 0 else 1.0))


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _shard(rank, n, step):
    rng = O.Rng(1000 + 17 * rank + step)
    x = rng.rand_vec(n * 3 * 16 * 16)
    labels = np.array([rng.below(6) for _ in range(n)], np.uint32)
    return x, labels


def _steps(net, rank, device, n=3, steps=2):
    from rustnn_b200 import vit

    out = []
    for step in range(steps):
        x, labels = _shard(rank, n, step)
        tf, tc, coarse = vit.targets(labels, TINY_PARENT, 3)
        dv = lambda a, dt=np.float32: torch.from_numpy(np.ascontiguousarray(a, dt)).to(device)
        st = net.train_step(dv(x), dv(tf), dv(tc), dv(labels.astype(np.int32), np.int32),
                            dv(coarse.astype(np.int32), np.int32), drop_seed=50 + 7 * rank + step)
        out.append(st)
    return out


def _state(net):
    m, v2 = net.moments()
    return net.params(), m, v2, net.ema(), net.buffers()


def test_one_rank_communicator_is_the_plain_step():
    from rustnn_b200 import dp, model, vit

    a = vit.RustViT(vit.VitCfg(**TINY), TINY_PARENT, 3, 8)
    b = vit.RustViT(vit.VitCfg(**TINY), TINY_PARENT, 3, 8)
    comm = dp.Comm(0, 1, model.dp_unique_id(), device=torch.cuda.current_device())
    try:
        a.dp_attach(comm)
        sa = _steps(a, 0, "cuda")
        sb = _steps(b, 0, "cuda")
        assert sa == sb
        for u, v in zip(_state(a), _state(b)):
            assert np.array_equal(u, v)
        a.dp_attach(None)
    finally:
        a.close()
        b.close()
        comm.close()


def _vit_rank(rank, world, uid, q):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        import torch as T

        from rustnn_b200 import dp, vit

        T.cuda.set_device(rank)
        net = vit.RustViT(vit.VitCfg(**TINY), TINY_PARENT, 3, 8)
        alone = vit.RustViT(vit.VitCfg(**TINY), TINY_PARENT, 3, 8)
        comm = dp.Comm(rank, world, uid, device=rank)
        net.dp_attach(comm)
        _steps(net, rank, f"cuda:{rank}")
        _steps(alone, rank, f"cuda:{rank}")
        q.put((rank, [np.asarray(s) for s in _state(net)], alone.params(), None))
        net.close()
        alone.close()
        comm.close()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, None, repr(e)))


def test_two_ranks_end_each_step_identical():
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    from rustnn_b200 import model

    uid = model.dp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_vit_rank, args=(r, 2, uid, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(2):
            rank, state, alone, err = q.get(timeout=300)
            out[rank] = (state, alone, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in (0, 1):
        assert out[r][2] is None, out[r][2]
    for u, v in zip(out[0][0], out[1][0]):
        assert np.array_equal(u, v)
    # the shards differ, so the shared parameters are neither rank's own
    assert not np.array_equal(out[0][0][0], out[0][1])
    assert not np.array_equal(out[0][0][0], out[1][1])
    # the oracle's sharded step on the same shards and seeds
    trs = [RV.Trainer(RV.RustViT(RV.Cfg(**TINY), TINY_PARENT, 3, 8)) for _ in range(2)]
    for step in range(2):
        shards = []
        for r in range(2):
            x, labels = _shard(r, 3, step)
            shards.append((x, labels, 3))
        RV.dp_step(trs, shards, 6e-4, 0.06, [50 + 7 * r + step for r in range(2)])
    o = trs[0]
    want = (o.net.V, o.net.M, o.net.V2, o.ema.w, o.net.buffer_vec())
    for name, got, w in zip(("params", "m", "v2", "ema", "buffers"), out[0][0], want):
        assert rel(got, w) < TOL, name
