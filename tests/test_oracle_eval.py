"""Pins the oracle's evaluation path (oracle/rnn_oracle.c orc_make_batch_eval,
orc_resnet_eval; oracle/rustvit.py eval_vit) to the reference's own checks of
the eval batch (data.rs:546-584: no shift is plain normalisation, the flip
mirrors the columns) and to the loop of eval.rs:15-66 written out here."""
import numpy as np
import pytest

from oracle import oracle as O
from oracle import rustvit as RV

F32 = np.float32
MEAN = [F32(0.5071), F32(0.4865), F32(0.4409)]  # data.rs:13-14
STD = [F32(0.2673), F32(0.2564), F32(0.2762)]
PIX = 3 * 32 * 32


def rampa():
    """data.rs:521-523: each pixel encodes its position."""
    return (np.arange(PIX) % 251).astype(np.uint8)


def norm(v, c):
    """data.rs:95-98 in f32."""
    return (F32(v) / F32(255.0) - MEAN[c]) / STD[c]


def dataset(rng, n, nclass):
    images = rng.integers(0, 256, size=n * PIX, dtype=np.uint8)
    labels = rng.integers(0, nclass, size=n, dtype=np.uint8)
    return images, labels


def test_no_shift_is_normalisation():
    """data.rs:553-564 (sem_deslocamento_e_so_normalizacao)."""
    src = rampa()
    x, lab = O.make_batch_eval(src, np.array([42], np.uint8), 0, 1, False)
    assert lab.tolist() == [42]
    for c in range(3):
        want = norm(src[c * 1024:(c + 1) * 1024], c)
        assert np.array_equal(x[c * 1024:(c + 1) * 1024], want)


def test_flip_mirrors_columns():
    """data.rs:566-584 (flip_espelha_as_colunas)."""
    src = rampa()
    reto, _ = O.make_batch_eval(src, np.zeros(1, np.uint8), 0, 1, False)
    esp, _ = O.make_batch_eval(src, np.zeros(1, np.uint8), 0, 1, True)
    assert np.array_equal(esp.reshape(3, 32, 32), reto.reshape(3, 32, 32)[:, :, ::-1])
    assert not np.array_equal(esp, reto)


def test_batch_offset_and_labels():
    rng = np.random.default_rng(3)
    images, labels = dataset(rng, 7, 100)
    x, lab = O.make_batch_eval(images, labels, 2, 4, False)
    assert lab.dtype == np.uint32 and lab.tolist() == labels[2:6].tolist()
    for b in range(4):
        one, _ = O.make_batch_eval(images[(2 + b) * PIX:(3 + b) * PIX], labels[2 + b:3 + b], 0, 1, False)
        assert np.array_equal(x[b * PIX:(b + 1) * PIX], one)


def eval_loop(images, labels, batch, nclass, logits_of):
    """eval.rs:15-39 written out: f32 sum of l * bs, hits, means over seen."""
    total = len(labels)
    s, acc, correct, seen = 0, F32(0.0), 0, 0
    while s < total:
        bs = min(batch, total - s)
        lg = logits_of(s, bs)
        x, lab = O.make_batch_eval(images, labels, s, bs, False)
        loss, _, c = O.softmax_ce(lg, lab, nclass, 0.0)
        acc = F32(acc + F32(F32(loss) * F32(bs)))
        correct += c
        seen += bs
        s += bs
    return float(acc / F32(seen)), float(F32(correct) / F32(seen))


@pytest.mark.parametrize("n,batch", [(20, 8), (16, 16), (5, 32)])
def test_resnet_eval_loop(n, batch):
    """orc_resnet_eval against the loop written out over the oracle's own
    forward(train=false), ragged last batch included."""
    rng = np.random.default_rng(n)
    net = O.ResNet(1, 4, 10, 1234)
    images, labels = dataset(rng, n, 10)

    def logits_of(s, bs):
        x, _ = O.make_batch_eval(images, labels, s, bs, False)
        return net.forward(x, bs, hw=32, train=False)

    want = eval_loop(images, labels, batch, 10, logits_of)
    got = net.eval(images, labels, batch)
    assert got == want


def test_resnet_eval_empty_is_nan():
    """eval.rs:38 divides by seen = 0."""
    net = O.ResNet(1, 4, 10, 1234)
    loss, acc = net.eval(np.zeros(0, np.uint8), np.zeros(0, np.uint8), 8)
    assert np.isnan(loss) and np.isnan(acc)


TINY32 = dict(width=4, cmid=6, dim=8, heads=2, depth3=2, dim4=12, heads4=2, depth4=1, mem_at=[1], droppath=0.2,
              img=32)
TINY_PARENT = np.array([0, 0, 1, 1, 2, 2], np.uint32)


@pytest.mark.parametrize("tta", [False, True])
def test_vit_eval_loop(tta):
    """eval_vit against eval.rs:47-66 written out: exits off, train false,
    mirrored logits averaged as 0.5 * (a + b)."""
    rng = np.random.default_rng(11)
    net = RV.RustViT(RV.Cfg(**TINY32), TINY_PARENT, 3, 5)
    images, labels = dataset(rng, 5, 6)

    def logits_of(s, bs):
        x, _ = O.make_batch_eval(images, labels, s, bs, False)
        lg = net.forward(x, bs, False)["logits"]
        if tta:
            xm, _ = O.make_batch_eval(images, labels, s, bs, True)
            lg = (F32(0.5) * (lg + net.forward(xm, bs, False)["logits"])).astype(F32)
        return lg

    want = eval_loop(images, labels, 3, 6, logits_of)
    assert net.use_exits
    got = RV.eval_vit(net, images, labels, 3, tta)
    assert net.use_exits  # restored (eval.rs:64)
    assert got == want


def test_vit_eval_uses_running_statistics():
    """forward with train false normalises with the running statistics
    (nn.rs:358-369): a train forward moves them, an eval forward does not."""
    rng = np.random.default_rng(2)
    net = RV.RustViT(RV.Cfg(**TINY32), TINY_PARENT, 3, 5)
    images, labels = dataset(rng, 2, 6)
    x, _ = O.make_batch_eval(images, labels, 0, 2, False)
    before = net.buffer_vec().copy()
    net.forward(x, 2, False)
    assert np.array_equal(net.buffer_vec(), before)
    net.forward(x, 2, True)
    assert not np.array_equal(net.buffer_vec(), before)
