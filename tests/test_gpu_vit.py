"""The device rustvit (rustnn_b200.vit, csrc/vit.cu) against the CPU oracle's
restatement (oracle/rustvit.py): bit-identical initialisation, forward heads,
backward gradients, whole Trainer::step updates (parameters, both moments,
EMA, BatchNorm buffers, loss statistics) at bar 1e-4 relative Frobenius, and
the reference's network gradcheck (check.rs:397-455) run on the GPU."""
import numpy as np
import pytest

from oracle import oracle as O
from oracle import rustvit as RV

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-4
TINY = dict(width=4, cmid=6, dim=8, heads=2, depth3=2, dim4=12, heads4=2, depth4=1, mem_at=[1], droppath=0.2,
            img=16)
TINY_PARENT = np.array([0, 0, 1, 1, 2, 2], np.uint32)


def rel(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    den = np.linalg.norm(want)
    return float(np.linalg.norm(got - want) / (den if den > 0 else 1.0))


def dev(a, dtype=np.float32):
    return torch.from_numpy(np.ascontiguousarray(a, dtype)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def pair(cfgd, parent, nc, seed):
    from rustnn_b200 import vit

    return vit.RustViT(vit.VitCfg(**cfgd), parent, nc, seed), RV.RustViT(RV.Cfg(**cfgd), parent, nc, seed)


@pytest.mark.parametrize("which", ["tiny", "default"])
def test_init_bit_exact(which):
    cfgd, parent, nc = (TINY, TINY_PARENT, 3) if which == "tiny" else ({}, RV.cifar_parent(), 20)
    d, o = pair(cfgd, parent, nc, 1234)
    assert d.nparams == o.V.size
    assert np.array_equal(d.params(), o.V)
    assert np.array_equal(d.buffers(), o.buffer_vec())
    d.close()


def _batch(rng, n, img, nf):
    x = rng.rand_vec(n * 3 * img * img)
    labels = np.array([rng.below(nf) for _ in range(n)], np.uint32)
    return x, labels


def test_forward_backward_parity():
    d, o = pair({}, RV.cifar_parent(), 20, 99)
    rng = O.Rng(5)
    n = 4
    x, _ = _batch(rng, n, 32, 100)
    o.drop_seed = 77
    out_o = o.forward(x, n, True)
    out_d = d.forward(dev(x), n, True, 77)
    for k in ("logits", "coarse", "e1", "e2", "h1", "h2", "feat"):
        assert rel(host(out_d[k]), out_o[k]) < TOL, k
    g = {k: rng.rand_vec(out_o[k].size) for k in ("logits", "coarse", "e1", "e2", "h1", "h2")}
    g["hfinal"] = rng.rand_vec(out_o["feat"].size)
    o.backward(g)
    d.zero_grads()
    d.backward({k: dev(v) for k, v in g.items()})
    gd = d.grads()
    assert rel(gd, o.G) < TOL
    # per parameter tensor, for the tensors that carry gradient
    off = 0
    worst = 0.0
    for p in o.plist:
        k = p.v.size
        if np.linalg.norm(p.g) > 1e-6 * np.linalg.norm(o.G):
            worst = max(worst, rel(gd[off:off + k], p.g))
        off += k
    assert worst < 1e-3, worst
    assert rel(d.buffers(), o.buffer_vec()) < TOL
    d.close()


@pytest.mark.parametrize("n", [4, 128])
def test_train_steps_parity(n):
    """Two Trainer::step calls (forward, build_loss, backward, clip, Muon +
    AdamW, EMA) from the same initialisation on the same batches; n = 128 is
    BASELINE config 4's batch, the one bench.py --config rustvit times."""
    from rustnn_b200 import vit

    d, o = pair({}, RV.cifar_parent(), 20, 4321)
    tr = RV.Trainer(o)
    rng = O.Rng(17)
    for step, seed in enumerate((11, 12)):
        x, labels = _batch(rng, n, 32, 100)
        tf, tc, coarse = vit.targets(labels, d.parent, 20)
        tf_o, tc_o, coarse_o = RV.targets(labels, o.head.parent, 20, RV.LossCfg())
        assert np.array_equal(tf, tf_o) and np.array_equal(tc, tc_o) and np.array_equal(coarse, coarse_o)
        total_o, ce_o, corr_o = tr.step(x, labels, n, 6e-4, 0.06, seed)
        total_d, ce_d, corr_d = d.train_step(dev(x), dev(tf), dev(tc), dev(labels.astype(np.int32), np.int32),
                                             dev(coarse.astype(np.int32), np.int32), lr=6e-4, wd=0.06, clip=1.0,
                                             ema=0.9998, drop_seed=seed)
        assert abs(total_d - total_o) <= 1e-4 * abs(total_o), (step, total_d, total_o)
        assert abs(ce_d - ce_o) <= 1e-4 * abs(ce_o)
        assert corr_d == corr_o
        assert rel(d.params(), o.V) < TOL, step
        m, v2 = d.moments()
        assert rel(m, o.M) < TOL and rel(v2, o.V2) < TOL
        assert rel(d.ema(), tr.ema.w) < TOL
        assert rel(d.buffers(), o.buffer_vec()) < TOL
        assert not np.any(d.grads())
    d.close()


def test_host_tier_matches_device_tier():
    from rustnn_b200 import vit

    a = vit.RustViT(vit.VitCfg(**TINY), TINY_PARENT, 3, 8)
    b = vit.RustViT(vit.VitCfg(**TINY), TINY_PARENT, 3, 8)
    rng = O.Rng(2)
    n = 3
    x, labels = _batch(rng, n, 16, 6)
    tf, tc, coarse = vit.targets(labels, TINY_PARENT, 3)
    sa = a.train_step(dev(x), dev(tf), dev(tc), dev(labels.astype(np.int32), np.int32),
                      dev(coarse.astype(np.int32), np.int32), drop_seed=5)
    sb = b.train_step_host(x, tf, tc, labels, coarse, drop_seed=5)
    assert sa == sb
    assert np.array_equal(a.params(), b.params())
    a.close()
    b.close()


def test_gpu_network_gradcheck():
    """check.rs:397-455 with the GPU computing every loss and gradient, per
    component group (see tests/test_oracle_vit.py for why per group)."""
    from rustnn_b200 import vit

    rng = O.Rng(1234 ^ 0x1234)
    o = RV.RustViT(RV.Cfg(**TINY), TINY_PARENT, 3, 1234 ^ 0xBEEF)
    d = vit.RustViT(vit.VitCfg(**TINY), TINY_PARENT, 3, 1234 ^ 0xBEEF)
    base = (o.V + np.float32(0.15) * rng.rand_vec(o.V.size)).astype(np.float32)
    d.set_params(base)
    bs, nf = 3, 6
    x = dev(rng.rand_vec(bs * 3 * 16 * 16))
    g = dict(logits=rng.rand_vec(bs * nf), coarse=rng.rand_vec(bs * 3), e1=rng.rand_vec(bs * nf),
             e2=rng.rand_vec(bs * nf), h1=rng.rand_vec(bs * 12), h2=rng.rand_vec(bs * 12),
             hfinal=rng.rand_vec(bs * 12))
    gd = {k: dev(v) for k, v in g.items()}

    def lin(out):
        tot = 0.0
        for k in ("logits", "coarse", "e1", "e2", "h1", "h2"):
            tot += float(np.dot(host(out[k]).astype(np.float64), g[k].astype(np.float64)))
        return tot + float(np.dot(host(out["feat"]).astype(np.float64), g["hfinal"].astype(np.float64)))

    d.zero_grads()
    d.forward(x, bs, True, 4242)
    d.backward(gd)
    grad = d.grads()
    groups = [[o.stem.w, *o.stem_bn.params(), *o.c1.params(), *o.c2.params()],
              [o.memconv.w, *o.memln.params(), o.tokconv.w, *o.tok_bn.params()],
              [p for b in o.blocks3 for p in b.params()],
              [*o.mergeln.params(), *o.merge.params()],
              [p for b in o.blocks4 for p in b.params()],
              [p for m in (o.headln, o.pool, o.head, o.e1, o.pool2, o.e2) for p in m.params()]]
    offs, off = {}, 0
    for p in o.plist:
        offs[id(p)] = (off, p.v.size)
        off += p.v.size
    for gi, ps in enumerate(groups):
        idx = np.concatenate([np.arange(offs[id(p)][0], offs[id(p)][0] + offs[id(p)][1]) for p in ps])
        v = rng.rand_vec(idx.size)
        eps = np.float32(3e-4)
        vals = []
        for sgn in (1, -1):
            w = base.copy()
            w[idx] = (base[idx] + np.float32(sgn) * eps * v).astype(np.float32)
            d.set_params(w)
            vals.append(lin(d.forward(x, bs, True, 4242)))
        d.set_params(base)
        num = (vals[0] - vals[1]) / (2.0 * float(eps))
        ana = float(np.dot(grad[idx].astype(np.float64), v.astype(np.float64)))
        err = abs(num - ana) / (abs(num) + abs(ana) + 1e-6)
        assert err < 5e-3, (gi, err)
    d.close()
