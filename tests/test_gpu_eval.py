"""The device evaluation path (csrc/eval.cu and the eval entries of resnet.cu
and vit.cu) against the CPU oracle: the eval batch bit-exact
(data.rs:494-512), forward with train false at 1e-4, and eval::resnet /
eval::vit (eval.rs:15-66, test-time augmentation and EMA weights included)."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from oracle import rustvit as RV

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-4
PIX = 3 * 32 * 32


def rel(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    den = np.linalg.norm(want)
    return float(np.linalg.norm(got - want) / (den if den > 0 else 1.0))


def dataset(seed, n, nclass):
    rng = np.random.default_rng(seed)
    return (rng.integers(0, 256, size=n * PIX, dtype=np.uint8), rng.integers(0, nclass, size=n, dtype=np.uint8))


def make_batch_dev(images_d, labels_d, start, bs, flip, out_offset=0):
    from rustnn_b200 import _lib
    from rustnn_b200.ops import default_context

    ctx = default_context()
    ctx.bind()
    out = torch.zeros(bs * PIX + out_offset, device="cuda")
    lab = torch.zeros(bs, dtype=torch.int32, device="cuda")
    _lib.call("rnn_make_batch_eval_dev", ctx.h, C.c_void_p(images_d.data_ptr()), C.c_void_p(labels_d.data_ptr()),
              labels_d.numel(), start, bs, int(flip), C.c_void_p(out.data_ptr() + 4 * out_offset),
              C.c_void_p(lab.data_ptr()))
    torch.cuda.synchronize()
    return out[out_offset:].cpu().numpy(), lab.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("start,bs,flip,off", [(0, 1, False, 0), (3, 9, True, 0), (2, 5, False, 1), (1, 6, True, 3)])
def test_make_batch_eval_bit_exact(start, bs, flip, off):
    """data.rs:494-512, both the float4 and the scalar store paths."""
    images, labels = dataset(start + bs, 12, 100)
    x_d, l_d = make_batch_dev(torch.from_numpy(images).cuda(), torch.from_numpy(labels).cuda(), start, bs, flip, off)
    x_o, l_o = O.make_batch_eval(images, labels, start, bs, flip)
    assert np.array_equal(x_d, x_o)
    assert np.array_equal(l_d, l_o)


def _trained_pair(seed):
    """A ResNet-8 w16 pair after one identical training step, so that the
    BatchNorm running statistics are not the initial ones."""
    from rustnn_b200 import model

    g = model.ResNet(1, 16, 100, seed)
    o = O.ResNet(1, 16, 100, seed)
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(16 * PIX).astype(np.float32)
    lab = rng.integers(0, 100, size=16).astype(np.uint32)
    o.train_step(x, lab)
    g.train_step_host(x, lab)
    assert rel(g.buffers(), o.buffers()) < 1e-5
    return g, o


def test_resnet_forward_eval_parity():
    """ResNet::forward(train=false) (model.rs:135-146, BN nn.rs:358-369)."""
    g, o = _trained_pair(5)
    images, labels = dataset(8, 24, 100)
    x, _ = O.make_batch_eval(images, labels, 0, 24, False)
    lg = g.forward(torch.from_numpy(x).cuda(), 24, hw=32, train=False)
    torch.cuda.synchronize()
    assert rel(lg.cpu().numpy(), o.forward(x, 24, hw=32, train=False)) < TOL
    g.close()


@pytest.mark.parametrize("n,batch", [(40, 16), (33, 64)])
def test_resnet_eval(n, batch):
    """eval::resnet (eval.rs:41-43) on a device dataset and through the host
    tier: the two agree exactly; against the oracle the loss is within 1e-4
    and the accuracy within one image (a near-tie of two logits)."""
    g, o = _trained_pair(7)
    images, labels = dataset(n, n, 100)
    lo, ao = o.eval(images, labels, batch)
    ld, ad = g.eval(torch.from_numpy(images).cuda(), torch.from_numpy(labels).cuda(), batch)
    lh, ah = g.eval(images, labels, batch)
    assert (ld, ad) == (lh, ah)
    assert abs(ld - lo) <= TOL * abs(lo)
    assert abs(ad - ao) <= 1.0 / n + 1e-7
    g.close()


def test_resnet_eval_empty():
    from rustnn_b200 import model

    g = model.ResNet(1, 4, 10, 1)
    loss, acc = g.eval(np.zeros(0, np.uint8), np.zeros(0, np.uint8), 8)
    assert np.isnan(loss) and np.isnan(acc)
    g.close()


TINY32 = dict(width=4, cmid=6, dim=8, heads=2, depth3=2, dim4=12, heads4=2, depth4=1, mem_at=[1], droppath=0.2,
              img=32)
TINY_PARENT = np.array([0, 0, 1, 1, 2, 2], np.uint32)


def _vit_pair(seed):
    from rustnn_b200 import vit

    return vit.RustViT(vit.VitCfg(**TINY32), TINY_PARENT, 3, seed), RV.RustViT(RV.Cfg(**TINY32), TINY_PARENT, 3, seed)


@pytest.mark.parametrize("tta", [False, True])
def test_vit_eval(tta):
    """eval::vit (eval.rs:47-66): exits off, train false, mirrored logits
    averaged when tta; ragged last batch."""
    d, o = _vit_pair(5)
    images, labels = dataset(21 + tta, 7, 6)
    lo, ao = RV.eval_vit(o, images, labels, 3, tta)
    ld, ad = d.eval(torch.from_numpy(images).cuda(), torch.from_numpy(labels).cuda(), 3, tta=tta)
    lh, ah = d.eval(images, labels, 3, tta=tta)
    assert (ld, ad) == (lh, ah)
    assert abs(ld - lo) <= TOL * abs(lo)
    assert abs(ad - ao) <= 1.0 / 7 + 1e-7
    d.close()


def test_vit_eval_ema_swaps_back():
    """Trainer::eval_ema (train.rs:390-402): the EMA weights are evaluated and
    the raw weights are back afterwards; equal to evaluating a model whose
    weights were set to the EMA."""
    from rustnn_b200 import vit

    d, _ = _vit_pair(9)
    rng = np.random.default_rng(4)
    n = 4
    x = rng.standard_normal(n * PIX).astype(np.float32)
    hard = rng.integers(0, 6, size=n).astype(np.uint32)
    tf, tc, hardc = vit.targets(hard, TINY_PARENT, 3)
    d.train_step_host(x, tf, tc, hard, hardc.astype(np.uint32), ema=0.5)
    d.train_step_host(x, tf, tc, hard, hardc.astype(np.uint32), ema=0.5)
    raw, ema = d.params(), d.ema()
    assert not np.array_equal(raw, ema)
    images, labels = dataset(30, 5, 6)
    got = d.eval(images, labels, 2, tta=True, use_ema=True)
    assert np.array_equal(d.params(), raw)
    d.set_params(ema)
    want = d.eval(images, labels, 2, tta=True)
    assert got == want
    d.close()


def test_make_batch_eval_outside_dataset():
    """A window past the end of the dataset is refused on the host."""
    from rustnn_b200._lib import RnnError

    images, labels = dataset(1, 4, 100)
    with pytest.raises(RnnError):
        make_batch_dev(torch.from_numpy(images).cuda(), torch.from_numpy(labels).cuda(), 2, 3, False)
