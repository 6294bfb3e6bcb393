"""The device batch builders (csrc/data.cu) against the CPU oracle
(oracle/rnn_oracle_data.c): make_batch_train (data.rs:384-412) and mix_batch
(data.rs:467-491), bit for bit.

The oracle runs in its default mode: the C library's f32 logf / cosf / sinf,
the functions the reference calls (erase noise, RandAugment magnitudes,
rotations).  The device takes the same functions' results (Box-Muller
tables over every 24-bit uniform; the rotations' cos / sin from a host
replay of the draws), so the bytes agree with no correctly-rounded mode."""
import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

PIX = 3072
F32 = np.float32


def dataset(seed, n):
    rng = np.random.default_rng(seed)
    return (rng.integers(0, 256, size=n * PIX, dtype=np.uint8), rng.integers(0, 100, size=n, dtype=np.uint8),
            rng.integers(0, 20, size=n, dtype=np.uint8))


def both(seed, n, bs, aug):
    from rustnn_b200 import data

    images, labels, coarse = dataset(seed, n)
    idx = np.random.default_rng(seed + 1).permutation(n)[:bs].astype(np.uint32)
    s = seed * 1_000_003 + 7
    want, wl, wc = O.make_batch_train(images, labels, coarse, idx, aug.pad, aug.ra_mag, aug.ra_n, aug.erase,
                                      aug.erase_side, s)
    dv = lambda a: torch.from_numpy(a).cuda()
    got, gl, gc = data.make_batch_train(dv(images), dv(labels), dv(coarse), dv(idx.view(np.int32)), aug, s)
    torch.cuda.synchronize()
    assert np.array_equal(gl.cpu().numpy().view(np.uint32), wl)
    assert np.array_equal(gc.cpu().numpy().view(np.uint32), wc)
    return got.cpu().numpy(), want


@pytest.mark.parametrize("pad,erase,side", [(4, 1.0, 8), (4, 0.0, 8), (32, 0.5, 16), (0, 1.0, 40), (4, 1.0, 1)])
def test_batch_train_no_randaugment(pad, erase, side):
    """The ResNet loop's augmentation (train.rs:654-660) and its corners."""
    from rustnn_b200.data import Aug

    aug = Aug(pad=pad, ra_mag=0.0, ra_n=0, erase=erase, erase_side=side)
    got, want = both(pad + side, 64, 48, aug)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("ra_mag,ra_n,erase,seed", [(0.5, 2, 0.0, 3), (1.0, 3, 0.5, 4), (0.8, 8, 0.0, 5),
                                                    (0.6, 2, 0.25, 6)])
def test_batch_train_randaugment(ra_mag, ra_n, erase, seed):
    """RandAugment (data.rs:100-306) before crop/flip/normalise/erase; 96
    images x up to 8 ops draw every op many times."""
    from rustnn_b200.data import Aug

    aug = Aug(pad=4, ra_mag=ra_mag, ra_n=ra_n, erase=erase, erase_side=8)
    got, want = both(seed, 96, 96, aug)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("m,c,seed", [(0.8, 0.0, 1), (0.0, 1.0, 2), (0.8, 1.0, 3), (0.0, 0.0, 4), (0.2, 0.3, 5)])
def test_mix_batch(m, c, seed):
    """mix_batch from the same generator state: the same permutation, lambdas
    and state afterwards; the mixed batch bit for bit."""
    from rustnn_b200 import data

    bs = 32
    for rep in range(4):
        x = np.random.default_rng(seed * 10 + rep).standard_normal(bs * PIX).astype(F32)
        st_o = O.Rng(seed * 100 + rep).state()
        st_d = st_o.copy()
        want = x.copy()
        _, perm_o, lam_o, _ = O.mix_batch(want, bs, m, c, 0.5, st_o)
        xd = torch.from_numpy(x).cuda()
        perm_d, lam_d = data.mix_batch(xd, bs, m, c, 0.5, st_d)
        torch.cuda.synchronize()
        assert np.array_equal(st_d, st_o)
        assert np.array_equal(perm_d, perm_o) and np.array_equal(lam_d, lam_o)
        assert np.array_equal(xd.cpu().numpy(), want)


def test_batch_train_index_outside_dataset():
    """An index past the dataset's end is flagged by the kernel (the
    reference panics on the slice): the next synchronisation reports the
    device error, the slot is left zero, and the context stays usable."""
    from rustnn_b200 import data
    from rustnn_b200._lib import RnnError
    from rustnn_b200.ops import default_context

    images, labels, coarse = dataset(3, 8)
    dv = lambda a: torch.from_numpy(a).cuda()
    idx = np.array([1, 8, 3], np.uint32)  # 8 == len
    got, gl, _ = data.make_batch_train(dv(images), dv(labels), None, dv(idx.view(np.int32)), data.Aug(), 5)
    with pytest.raises(RnnError):
        default_context().synchronize()
    assert not np.any(got[PIX:2 * PIX].cpu().numpy())
    ok = np.array([1, 7, 3], np.uint32)
    got, gl, _ = data.make_batch_train(dv(images), dv(labels), None, dv(ok.view(np.int32)), data.Aug(), 5)
    default_context().synchronize()
    assert np.array_equal(gl.cpu().numpy().view(np.uint32), labels[ok].astype(np.uint32))


def test_batch_train_follows_the_c_library_not_correct_rounding():
    """A batch whose bytes and noise differ between the C library's f32
    logf / cosf / sinf and correctly-rounded ones (checked on the oracle):
    the device reproduces the C library's."""
    from rustnn_b200 import data
    from rustnn_b200.data import Aug

    aug = Aug(pad=4, ra_mag=1.0, ra_n=4, erase=1.0, erase_side=16)
    images, labels, coarse = dataset(11, 256)
    idx = np.arange(256, dtype=np.uint32)
    args = (images, labels, coarse, idx, aug.pad, aug.ra_mag, aug.ra_n, aug.erase, aug.erase_side, 1234)
    want = O.make_batch_train(*args)[0]
    with O.cr_math():
        cr = O.make_batch_train(*args)[0]
    assert not np.array_equal(want, cr)
    dv = lambda a: torch.from_numpy(a).cuda()
    got = data.make_batch_train(dv(images), dv(labels), dv(coarse), dv(idx.view(np.int32)), aug, 1234)[0]
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), want)
