"""Checkpoints of the device models (rnn_{resnet,rustvit}_{save,load}[_optim])
in the reference's format (ckpt.rs:8-247): the file decodes with the
restatement in oracle/ckpt.py to the oracle's tensor count, the reference's
configuration hash (model.rs:220-229, vit.rs:780-801) and the model's
parameters and buffers bit for bit; a load restores them; the optimiser-state
file makes a resumed run continue like the uninterrupted one."""
import numpy as np
import pytest

from oracle import ckpt as K
from oracle import oracle as O
from oracle import rustvit as RV

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

PIX = 3072


def batch(seed, n, nclass):
    rng = np.random.default_rng(seed)
    return rng.standard_normal(n * PIX).astype(np.float32), rng.integers(0, nclass, size=n).astype(np.uint32)


@pytest.mark.parametrize("depth_n,width,nclass", [(1, 16, 10), (2, 8, 100)])
def test_resnet_checkpoint(tmp_path, depth_n, width, nclass):
    from rustnn_b200 import model

    g = model.ResNet(depth_n, width, nclass, 3)
    o = O.ResNet(depth_n, width, nclass, 3)
    x, lab = batch(1, 8, nclass)
    g.train_step_host(x, lab)
    path = tmp_path / "resnet.ckpt"
    g.save(path)
    tensors, scalars, h, payload = K.decode(path.read_bytes())
    n_bn = 1 + 6 * depth_n + 2  # stem, two per block, the two downsampling shortcuts
    assert tensors == o.num_tensors() + 2 * n_bn
    assert h == K.resnet_hash(depth_n, width, nclass)
    assert np.array_equal(payload, np.concatenate([g.params(), g.buffers()]))
    # a fresh model from another seed takes the checkpoint over
    g2 = model.ResNet(depth_n, width, nclass, 99)
    g2.load(path)
    assert np.array_equal(g2.params(), g.params()) and np.array_equal(g2.buffers(), g.buffers())
    # the oracle's own initial state, written in the format, loads as well
    init = tmp_path / "init.ckpt"
    init.write_bytes(K.encode(tensors, h, np.concatenate([o.params(), o.buffers()])))
    g2.load(init)
    assert np.array_equal(g2.params(), o.params()) and np.array_equal(g2.buffers(), o.buffers())
    g.close()
    g2.close()


def test_resnet_refuses_other_config(tmp_path):
    from rustnn_b200 import model
    from rustnn_b200._lib import RnnError

    a, b = model.ResNet(1, 8, 10, 1), model.ResNet(1, 8, 100, 1)
    path = tmp_path / "a.ckpt"
    a.save(path)
    with pytest.raises(RnnError):
        b.load(path)
    a.close()
    b.close()


def test_resnet_resume_with_momentum(tmp_path):
    """save + save_optim after two steps; a fresh model that loads both takes
    the third step like the original."""
    from rustnn_b200 import model

    a = model.ResNet(1, 16, 10, 5)
    for s in range(2):
        a.train_step_host(*batch(10 + s, 8, 10))
    a.save(tmp_path / "p.ckpt")
    a.save_optim(tmp_path / "m.ckpt")
    b = model.ResNet(1, 16, 10, 77)
    b.load(tmp_path / "p.ckpt")
    b.load_optim(tmp_path / "m.ckpt")
    assert np.array_equal(b.moments(), a.moments())
    x, lab = batch(20, 8, 10)
    a.train_step_host(x, lab)
    b.train_step_host(x, lab)
    pa, pb = a.params(), b.params()
    assert np.linalg.norm(pa - pb) <= 1e-6 * np.linalg.norm(pa)
    a.close()
    b.close()


TINY = dict(width=4, cmid=6, dim=8, heads=2, depth3=2, dim4=12, heads4=2, depth4=1, mem_at=[1], droppath=0.2,
            img=16)
TINY_PARENT = np.array([0, 0, 1, 1, 2, 2], np.uint32)


def test_rustvit_checkpoint_and_resume(tmp_path):
    from rustnn_b200 import vit

    d = vit.RustViT(vit.VitCfg(**TINY), TINY_PARENT, 3, 4)
    o = RV.RustViT(RV.Cfg(**TINY), TINY_PARENT, 3, 4)
    n = 4

    def step(net, seed):
        r = np.random.default_rng(seed)
        x = r.standard_normal(n * 3 * 16 * 16).astype(np.float32)
        hard = r.integers(0, 6, size=n).astype(np.uint32)
        tf, tc, hardc = vit.targets(hard, TINY_PARENT, 3)
        return net.train_step_host(x, tf, tc, hard, hardc.astype(np.uint32), ema=0.9, drop_seed=seed)

    for s in range(2):
        step(d, s)
    d.save(tmp_path / "v.ckpt")
    d.save_optim(tmp_path / "vo.ckpt")
    tensors, scalars, h, payload = K.decode((tmp_path / "v.ckpt").read_bytes())
    assert tensors == len(o.plist) + len(list(o.buffers()))
    assert h == K.rustvit_hash(TINY, 6, 3, True, TINY_PARENT)
    assert np.array_equal(payload, np.concatenate([d.params(), d.buffers()]))
    e = vit.RustViT(vit.VitCfg(**TINY), TINY_PARENT, 3, 11)
    e.load(tmp_path / "v.ckpt")
    e.load_optim(tmp_path / "vo.ckpt")
    assert np.array_equal(e.params(), d.params()) and np.array_equal(e.buffers(), d.buffers())
    assert np.array_equal(e.ema(), d.ema())
    for a, b in zip(e.moments(), d.moments()):
        assert np.array_equal(a, b)
    sa, sb = step(d, 7), step(e, 7)
    assert abs(sa[0] - sb[0]) <= 1e-6 * abs(sa[0])
    pd, pe = d.params(), e.params()
    assert np.linalg.norm(pd - pe) <= 1e-6 * np.linalg.norm(pd)
    assert np.linalg.norm(d.ema() - e.ema()) <= 1e-6 * np.linalg.norm(d.ema())
    d.close()
    e.close()
