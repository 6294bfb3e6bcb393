"""Pins the rustvit composition of the oracle (oracle/rustvit.py) to the
reference's own checks: the published parameter and MAC counts
(README.md:142-143), the block gradcheck (check.rs:359-394) and the
whole-network gradcheck over every parameter at once (check.rs:397-455)."""
import numpy as np

from oracle import oracle as O
from oracle import rustvit as RV

TOL = 5e-3  # check.rs:42-44
EPS = 3e-4  # check.rs:55-60


def dircheck(base, grad, eps, rng, lossf):
    """check.rs:19-40."""
    base = np.asarray(base, np.float32)
    v = rng.rand_vec(base.size)
    lp = lossf((base + np.float32(eps) * v).astype(np.float32))
    lm = lossf((base - np.float32(eps) * v).astype(np.float32))
    num = (lp - lm) / (2.0 * eps)
    ana = float(np.dot(np.asarray(grad, np.float64), v.astype(np.float64)))
    return abs(num - ana) / (abs(num) + abs(ana) + 1e-6)


def test_rustvit_counts():
    net = RV.RustViT(RV.Cfg(), RV.cifar_parent(), 20, 1234)
    assert round(net.num_params() / 1e6, 2) == 6.37  # README.md:142-143
    assert round(net.macs() / 1e6, 1) == 318.6
    assert sum(1 for p in net.plist if p.rows > 0 and min(p.rows, p.cols) > 1) == 39
    # for_each_param covers every parameter exactly once
    assert sum(p.v.size for p in net.plist) == net.V.size


class _Flat:
    """A parameter list viewed as one vector (the check_params! macro, check.rs:74-101)."""

    def __init__(self, params):
        self.ps = list(params)

    def get(self, attr):
        return np.concatenate([getattr(p, attr) for p in self.ps]).astype(np.float32)

    def set_v(self, vec):
        off = 0
        for p in self.ps:
            p.v[:] = vec[off:off + p.v.size]
            off += p.v.size

    def zero_g(self):
        for p in self.ps:
            p.g[:] = 0.0


def _wrap_params(obj):
    """Standalone layers own separate arrays; nothing to flatten."""
    return _Flat(obj.params())


def test_block_gradcheck():
    """check.rs:359-394: a reader block with memory and a fixed DropPath seed."""
    rng = O.Rng(1234 ^ 0x1234)
    n, t, c = 3, 9, 8
    x = rng.rand_vec(n * t * c)
    r = rng.rand_vec(n * t * c)
    mh = mw = 6
    blk = RV.Block(c, 2, 3, 3, (mh, mw), 2, 0.2, 7, 0.3, rng)
    fl = _wrap_params(blk)
    for p in fl.ps:
        p.v[:] = (p.v + np.float32(0.2) * rng.rand_vec(p.v.size)).astype(np.float32)
    mem = rng.rand_vec(n * mh * mw * 2 * c)
    dmem = np.zeros_like(mem)
    blk.forward(x, mem, n, True, 99)
    dx = blk.backward(r.copy(), mem, dmem)
    # the seeded masks must drop something for this check to cover DropPath
    assert blk.dp1.mask is not None
    e = dircheck(x, dx, EPS, rng, lambda v: float(np.dot(blk.forward(v, mem, n, True, 99), r)))
    assert e < TOL, f"block dx {e}"
    e = dircheck(mem, dmem, EPS, rng, lambda v: float(np.dot(blk.forward(x, v, n, True, 99), r)))
    assert e < TOL, f"block dmem {e}"
    fl.zero_g()
    blk.forward(x, mem, n, True, 99)
    blk.backward(r.copy(), mem, np.zeros_like(mem))
    base, grad = fl.get("v"), fl.get("g")

    def loss(v):
        fl.set_v(v)
        return float(np.dot(blk.forward(x, mem, n, True, 99), r))

    e = dircheck(base, grad, EPS, rng, loss)
    fl.set_v(base)
    assert e < TOL, f"block dparams {e}"


def _tiny_net(rng):
    """The network of check.rs:397-433 with its parameters perturbed."""
    parent = np.array([0, 0, 1, 1, 2, 2], np.uint32)
    cfg = RV.Cfg(width=4, cmid=6, dim=8, heads=2, depth3=2, dim4=12, heads4=2, depth4=1, mem_at=[1],
                 droppath=0.2, img=16)
    net = RV.RustViT(cfg, parent, 3, 1234 ^ 0xBEEF)
    net.drop_seed = 4242
    net.V[:] = (net.V + np.float32(0.15) * rng.rand_vec(net.V.size)).astype(np.float32)
    return net


class _Span:
    def __init__(self, ps):
        self.ps = ps

    def params(self):
        return iter(self.ps)


def test_rustvit_netcheck():
    """check.rs:397-455: the tiny network with the loss the linear form
    <outputs, g>, so dL/doutput = g exactly; every head, both hints and the
    memory path are exercised.  The directional check runs per component
    group (stem+C1+C2, memory/token convs, S3 blocks, merge, S4 blocks, heads):
    one direction over all 6.4k parameters at once crosses enough ReLU kinks
    of the convolutional stem that the f32 central difference is off by a few
    percent at this seed, while every group alone agrees to < 5e-3."""
    rng = O.Rng(1234 ^ 0x1234)
    net = _tiny_net(rng)
    nf, bs = 6, 3
    x = rng.rand_vec(bs * 3 * 16 * 16)
    g = dict(logits=rng.rand_vec(bs * nf), coarse=rng.rand_vec(bs * 3), e1=rng.rand_vec(bs * nf),
             e2=rng.rand_vec(bs * nf), h1=rng.rand_vec(bs * 12), h2=rng.rand_vec(bs * 12),
             hfinal=rng.rand_vec(bs * 12))

    def lin(o):
        return float(sum(np.dot(o[k].astype(np.float64), g[k].astype(np.float64))
                         for k in ("logits", "coarse", "e1", "e2", "h1", "h2")) +
                     np.dot(o["feat"].astype(np.float64), g["hfinal"].astype(np.float64)))

    net.forward(x, bs, True)
    net.backward(g)
    base, grad = net.V.copy(), net.G.copy()
    groups = {
        "stem+C1+C2": [_Span([net.stem.w]), net.stem_bn, net.c1, net.c2],
        "memory/token convs": [_Span([net.memconv.w]), net.memln, _Span([net.tokconv.w]), net.tok_bn],
        "S3 blocks": net.blocks3,
        "merge": [net.mergeln, net.merge],
        "S4 blocks": net.blocks4,
        "heads and exits": [net.headln, net.pool, net.head, net.e1, net.pool2, net.e2],
    }
    offs, off = {}, 0
    for p in net.plist:
        offs[id(p)] = (off, p.v.size)
        off += p.v.size
    covered = 0
    for name, objs in groups.items():
        idx = np.concatenate([np.arange(*[offs[id(p)][0], offs[id(p)][0] + offs[id(p)][1]])
                              for o in objs for p in o.params()])
        covered += idx.size

        def loss(vals, idx=idx):
            net.V[:] = base
            net.V[idx] = vals
            return lin(net.forward(x, bs, True))

        e = dircheck(base[idx], grad[idx], EPS, rng, loss)
        net.V[:] = base
        assert e < TOL, f"{name}: {e}"
    assert covered == net.V.size


def test_targets_sum_to_one():
    """loss.rs:11-34: the soft targets are distributions."""
    parent = RV.cifar_parent()
    tf, tc, coarse = RV.targets(np.array([0, 17, 99], np.uint32), parent, 20, RV.LossCfg())
    assert np.allclose(tf.reshape(3, 100).sum(1), 1.0, atol=1e-5)
    assert np.allclose(tc.reshape(3, 20).sum(1), 1.0, atol=1e-5)
    assert list(coarse) == [0, 3, 19]
    # the four siblings of class 17 share eps * sib
    row = tf.reshape(3, 100)[1]
    assert np.isclose(row[15:20].sum() - row[17], 0.1 * 0.7, atol=1e-6)


def test_trainer_step_runs():
    """train.rs:346-387 on the default configuration at batch 2: finite loss
    near the uniform-prediction value, every parameter group moves."""
    net = RV.RustViT(RV.Cfg(), RV.cifar_parent(), 20, 7)
    tr = RV.Trainer(net)
    rng = O.Rng(3)
    n = 2
    x = rng.rand_vec(n * 3 * 32 * 32)
    labels = np.array([rng.below(100) for _ in range(n)], np.uint32)
    v0 = net.V.copy()
    total, ce, correct = tr.step(x, labels, n, 6e-4, 0.06, 11)
    assert np.isfinite(total) and 3.0 < ce < 6.5
    assert 0 <= correct <= n
    moved = np.abs(net.V - v0) > 0
    assert moved.mean() > 0.9
    assert not np.any(net.G)  # the optimiser zeroes every gradient


TINY = dict(width=4, cmid=6, dim=8, heads=2, depth3=2, dim4=12, heads4=2, depth4=1, mem_at=[1], droppath=0.2,
            img=16)
TINY_PARENT = np.array([0, 0, 1, 1, 2, 2], np.uint32)


def _tiny_shard(rank, n, step):
    rng = O.Rng(1000 + 17 * rank + step)
    x = rng.rand_vec(n * 3 * 16 * 16)
    labels = np.array([rng.below(6) for _ in range(n)], np.uint32)
    return x, labels, n


def test_dp_step_one_rank_is_the_trainer_step():
    """The batch-sharded step's restatement (rnn_rustvit_dp_attach's
    semantics) at one rank is Trainer.step, bit for bit."""
    a = RV.Trainer(RV.RustViT(RV.Cfg(**TINY), TINY_PARENT, 3, 8))
    b = RV.Trainer(RV.RustViT(RV.Cfg(**TINY), TINY_PARENT, 3, 8))
    for step in range(2):
        x, labels, n = _tiny_shard(0, 3, step)
        sa = RV.dp_step([a], [(x, labels, n)], 6e-4, 0.06, [50 + step])
        sb = b.step(x, labels, n, 6e-4, 0.06, 50 + step)
        assert sa == [sb]
        for u, v in ((a.net.V, b.net.V), (a.net.M, b.net.M), (a.net.V2, b.net.V2), (a.ema.w, b.ema.w),
                     (a.net.buffer_vec(), b.net.buffer_vec())):
            assert np.array_equal(u, v)


def test_dp_step_two_ranks_share_one_update():
    """Two ranks on different shards: identical parameters, moments, EMA and
    buffers after each step, and neither equals the step on its shard alone."""
    ranks = [RV.Trainer(RV.RustViT(RV.Cfg(**TINY), TINY_PARENT, 3, 8)) for _ in range(2)]
    alone = RV.Trainer(RV.RustViT(RV.Cfg(**TINY), TINY_PARENT, 3, 8))
    for step in range(2):
        shards = [_tiny_shard(r, 3, step) for r in range(2)]
        RV.dp_step(ranks, shards, 6e-4, 0.06, [50 + 7 * r + step for r in range(2)])
        alone.step(*shards[0][:2], 3, 6e-4, 0.06, 50 + step)
        r0, r1 = ranks[0].net, ranks[1].net
        assert np.array_equal(r0.V, r1.V) and np.array_equal(r0.M, r1.M)
        assert np.array_equal(r0.buffer_vec(), r1.buffer_vec())
        assert np.array_equal(ranks[0].ema.w, ranks[1].ema.w)
    assert not np.array_equal(ranks[0].net.V, alone.net.V)
