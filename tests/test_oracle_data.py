"""Pins the oracle's training batch builder and batch mixing
(oracle/rnn_oracle_data.c) to the reference's checks of data.rs
(data.rs:525-621: crop offsets inside the frame, a full shift leaves only the
border, mixing off is the identity, mixing on gives lambdas in [0, 1]) and to
an independent numpy restatement of data.rs:100-412 driven by the same
generator: every image, every RandAugment op, bit for bit."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

F32 = np.float32
IMG, PLANE, PIX = 32, 1024, 3072
MEAN = [F32(0.5071), F32(0.4865), F32(0.4409)]  # data.rs:13-14
STD = [F32(0.2673), F32(0.2564), F32(0.2762)]
GOLDEN = 0x9E3779B97F4A7C15
_libm = C.CDLL("libm.so.6")
for _fn in ("cosf", "sinf"):
    getattr(_libm, _fn).restype = C.c_float
    getattr(_libm, _fn).argtypes = [C.c_float]


def u8(v):
    """`v.clamp(0.0, 255.0) as u8` of an f32 array."""
    return np.clip(np.asarray(v, F32), F32(0), F32(255)).astype(np.uint8)


def px(src, c, y, x):
    ok = (y >= 0) & (x >= 0) & (y < IMG) & (x < IMG)
    return np.where(ok, src[c, np.clip(y, 0, IMG - 1), np.clip(x, 0, IMG - 1)], 128).astype(F32)


def affine(im, a, b, tx, c_, d, ty):
    src = im.copy()
    cy = F32(15.5)
    yy, xx = np.meshgrid(np.arange(IMG), np.arange(IMG), indexing="ij")
    fy, fx = yy.astype(F32) - cy, xx.astype(F32) - cy
    sx = F32(a) * fx + F32(b) * fy + F32(tx) + cy
    sy = F32(c_) * fx + F32(d) * fy + F32(ty) + cy
    x0, y0 = np.floor(sx), np.floor(sy)
    wx, wy = sx - x0, sy - y0
    x0, y0 = x0.astype(np.int64), y0.astype(np.int64)
    one = F32(1)
    for ch in range(3):
        v = (px(src, ch, y0, x0) * (one - wx) * (one - wy) + px(src, ch, y0, x0 + 1) * wx * (one - wy)
             + px(src, ch, y0 + 1, x0) * (one - wx) * wy + px(src, ch, y0 + 1, x0 + 1) * wx * wy)
        im[ch] = u8(v)


def blend(im, other, f):
    im[:] = u8(other.astype(F32) + F32(f) * (im.astype(F32) - other.astype(F32)))


def gray(im):
    v = F32(0.299) * im[0].astype(F32) + F32(0.587) * im[1].astype(F32) + F32(0.114) * im[2].astype(F32)
    return np.broadcast_to(u8(v), im.shape).copy()


def blur(im):
    out = im.copy()
    for c in range(3):
        for y in range(1, IMG - 1):
            for x in range(1, IMG - 1):
                s = F32(0)
                for dy in range(3):
                    for dx in range(3):
                        w = F32(5) if dy == 1 and dx == 1 else F32(0.375)
                        s = F32(s + w * F32(im[c, y + dy - 1, x + dx - 1]))
                out[c, y, x] = u8(s / F32(8))
    return out


def apply_op(im, op, v, rng):
    """data.rs:257-278"""
    sign = F32(1) if (rng.next_u64() >> 32) & 1 else F32(-1)
    f = F32(1) + sign * F32(0.9) * v
    if op == 0:
        affine(im, 1, sign * F32(0.3) * v, 0, 0, 1, 0)
    elif op == 1:
        affine(im, 1, 0, 0, sign * F32(0.3) * v, 1, 0)
    elif op == 2:
        affine(im, 1, 0, sign * F32(10) * v, 0, 1, 0)
    elif op == 3:
        affine(im, 1, 0, 0, 0, 1, sign * F32(10) * v)
    elif op == 4:
        t = F32(F32(F32(sign * F32(30)) * v) * F32(np.pi)) / F32(180)
        cs, sn = F32(_libm.cosf(t)), F32(_libm.sinf(t))
        affine(im, cs, -sn, 0, sn, cs, 0)
    elif op == 5:
        bits = 8 - int(F32(4) * v)
        im &= np.uint8((~((1 << (8 - bits)) - 1)) & 0xFF)
    elif op == 6:
        th = int(u8(F32(255) * (F32(1) - v)))
        im[:] = np.where(im >= th, 255 - im, im)
    elif op == 7:
        for c in range(3):
            lo, hi = int(im[c].min()), int(im[c].max())
            if hi > lo:
                k = F32(255) / F32(hi - lo)
                im[c] = u8((im[c].astype(np.int64) - lo).astype(F32) * k)
    elif op == 8:
        for c in range(3):
            cdf = np.cumsum(np.bincount(im[c].ravel(), minlength=256)).astype(np.int64)
            lo = int(cdf[cdf > 0][0])
            den = max(PLANE - lo, 1)
            im[c] = (((cdf[im[c]] - lo) * 255) // den).astype(np.uint8)
    elif op == 9:
        blend(im, np.zeros_like(im), f)
    elif op == 10:
        blend(im, gray(im), f)
    elif op == 11:
        mean = int(gray(im)[0].astype(np.uint32).sum()) // PLANE
        blend(im, np.full_like(im, mean), f)
    else:
        blend(im, blur(im), f)
    return op


def batch_train_np(images, labels, idx, pad, ra_mag, ra_n, erase, side, seed, ops_seen):
    """data.rs:384-412 restated over numpy with the oracle's generator."""
    out = np.empty((len(idx), 3, IMG, IMG), F32)
    for b, i in enumerate(idx):
        rng = O.Rng((seed ^ (b * GOLDEN)) & (2**64 - 1))
        work = images[i * PIX:(i + 1) * PIX].reshape(3, IMG, IMG).copy()
        if ra_mag > 0:
            for _ in range(ra_n):
                op = rng.below(13)
                v = F32(np.clip(F32(ra_mag) * (F32(1) + F32(0.5) * F32(rng.normal())), 0, 1))
                ops_seen.add(apply_op(work, op, v, rng))
        dy = dx = 0
        if pad > 0:
            dy = rng.below(2 * pad + 1) - pad
            dx = rng.below(2 * pad + 1) - pad
        flip = (rng.next_u64() >> 32) & 1
        for c in range(3):
            border = -MEAN[c] / STD[c]
            for y in range(IMG):
                sy = y + dy
                for x in range(IMG):
                    sx = (IMG - 1 - x if flip else x) + dx
                    if 0 <= sy < IMG and 0 <= sx < IMG:
                        out[b, c, y, x] = (F32(work[c, sy, sx]) / F32(255) - MEAN[c]) / STD[c]
                    else:
                        out[b, c, y, x] = border
        if erase > 0 and not rng.uniform() >= erase:
            cy, cx, h = rng.below(IMG), rng.below(IMG), side // 2
            for c in range(3):
                for y in range(max(cy - h, 0), min(cy + h, IMG)):
                    for x in range(max(cx - h, 0), min(cx + h, IMG)):
                        out[b, c, y, x] = rng.normal()
    return out.ravel(), labels[idx].astype(np.uint32)


def dataset(seed, n):
    rng = np.random.default_rng(seed)
    return (rng.integers(0, 256, size=n * PIX, dtype=np.uint8), rng.integers(0, 100, size=n, dtype=np.uint8),
            rng.integers(0, 20, size=n, dtype=np.uint8))


@pytest.mark.parametrize("pad,ra_mag,ra_n,erase,side,seed", [
    (4, 0.0, 0, 1.0, 8, 11),      # the ResNet loop's augmentation (train.rs:654-660)
    (4, 0.7, 2, 0.5, 8, 12),      # the rustvit schedule's (train.rs:48-55)
    (32, 0.0, 0, 0.0, 8, 13),     # shifts up to a whole image: border only
    (0, 1.0, 3, 1.0, 40, 14),     # erase larger than the image, magnitude at the clamp
])
def test_batch_train_matches_numpy(pad, ra_mag, ra_n, erase, side, seed):
    images, labels, coarse = dataset(seed, 40)
    idx = np.random.default_rng(seed).permutation(40)[:24].astype(np.uint32)
    ops = set()
    want, wl = batch_train_np(images, labels, idx, pad, ra_mag, ra_n, erase, side, seed * 977, ops)
    got, gl, gc = O.make_batch_train(images, labels, coarse, idx, pad, ra_mag, ra_n, erase, side, seed * 977)
    assert np.array_equal(got, want)
    assert np.array_equal(gl, wl)
    assert np.array_equal(gc, coarse[idx].astype(np.uint32))


def test_every_randaugment_op_matches_numpy():
    """Enough images that all 13 ops of data.rs:257-278 are drawn."""
    images, labels, coarse = dataset(5, 48)
    idx = np.arange(48, dtype=np.uint32)
    ops = set()
    want, _ = batch_train_np(images, labels, idx, 0, 0.9, 3, 0.0, 8, 4242, ops)
    got, _, _ = O.make_batch_train(images, labels, None, idx, 0, 0.9, 3, 0.0, 8, 4242)
    assert ops == set(range(13))
    assert np.array_equal(got, want)


def test_full_shift_leaves_border():
    """data.rs:586-598 (deslocamento_grande_so_deixa_borda) through the
    batch: with pad 32 some images are shifted a whole image away."""
    images, labels, _ = dataset(1, 64)
    idx = np.arange(64, dtype=np.uint32)
    x, _, _ = O.make_batch_train(images, labels, None, idx, 32, 0.0, 0, 0.0, 8, 77)
    x = x.reshape(64, 3, PLANE)
    border = np.array([-MEAN[c] / STD[c] for c in range(3)], F32)[None, :, None]
    full = np.all(x == border, axis=(1, 2))
    assert full.any()
    for b in range(64):  # crop_offset_respeita_a_moldura (data.rs:535-543)
        rng = O.Rng(77 ^ (b * GOLDEN))
        dy, dx = rng.below(65) - 32, rng.below(65) - 32
        assert -32 <= dy <= 32 and -32 <= dx <= 32
        assert full[b] == (abs(dy) >= 32 or abs(dx) >= 32)


def test_mix_off_is_identity():
    """data.rs:600-613 (mix_desligado_e_identidade)."""
    bs = 4
    x = (np.arange(bs * PIX) * 0.001).astype(F32)
    orig = x.copy()
    st = O.Rng(2).state()
    kind, perm, lam, _ = O.mix_batch(x, bs, 0.0, 0.0, 0.5, st)
    assert kind == 0 and np.array_equal(x, orig)
    assert np.all(lam == 1.0) and sorted(perm.tolist()) == list(range(bs))


@pytest.mark.parametrize("m,c", [(0.8, 0.0), (0.0, 1.0), (0.8, 1.0)])
def test_mix_on_gives_valid_lambdas(m, c):
    """data.rs:615-621 (mix_ligado_produz_lambda_valido), plus the restated
    mixup / cutmix of data.rs:436-469 checked against the generator."""
    bs = 8
    st = O.Rng(17).state()
    for _ in range(6):
        x = (np.arange(bs * PIX) % 97 * 0.01).astype(F32)
        src = x.copy()
        st0 = st.copy()
        kind, perm, lam, rect = O.mix_batch(x, bs, m, c, 0.5, st)
        assert np.all((lam >= 0) & (lam <= 1)) and np.all(np.isfinite(x))
        rng = O.Rng(0)
        rng.set_state(st0)
        for i in range(bs - 1, 0, -1):
            rng.below(i + 1)
        cut = c > 0 and (m <= 0 or rng.uniform() < 0.5)
        assert kind == (2 if cut else 1)
        s3 = src.reshape(bs, 3, IMG, IMG)
        if kind == 1:
            lv = lam[0]
            want = lv * s3 + (F32(1) - lv) * s3[perm]
            assert np.array_equal(x.reshape(bs, 3, IMG, IMG), want.astype(F32))
        else:
            y0, y1, x0, x1 = rect
            want = s3.copy()
            want[:, :, y0:y1, x0:x1] = s3[perm][:, :, y0:y1, x0:x1]
            assert np.array_equal(x.reshape(bs, 3, IMG, IMG), want)
            assert lam[0] == F32(1) - F32((y1 - y0) * (x1 - x0)) / F32(PLANE)


@pytest.mark.parametrize("ra_mag,ra_n,erase,seed", [(0.5, 2, 0.0, 3), (0.0, 0, 1.0, 11), (0.6, 2, 0.25, 12),
                                                    (0.8, 8, 0.0, 5)])
def test_cr_math_gap(ra_mag, ra_n, erase, seed):
    """The device evaluates logf / cosf / sinf correctly rounded; the C
    library's single-precision results (the reference's) differ in the last
    bit for a few percent of arguments.  Over a batch that moves the erase
    noise by an ulp and, through a RandAugment magnitude or angle, a handful
    of bytes: everything else is identical."""
    images, labels, _ = dataset(seed, 96)
    idx = np.arange(96, dtype=np.uint32)
    a, _, _ = O.make_batch_train(images, labels, None, idx, 4, ra_mag, ra_n, erase, 8, seed)
    with O.cr_math():
        b, _, _ = O.make_batch_train(images, labels, None, idx, 4, ra_mag, ra_n, erase, 8, seed)
    d = a != b
    assert np.count_nonzero(d) <= 1e-3 * a.size
    if ra_mag <= 0:
        # a last-bit change of ln or cos moves sqrt(-2 ln u1) * cos(.) by a few ulp
        assert np.all(np.abs(a[d] - b[d]) <= 4 * np.spacing(np.abs(a[d])))
    assert np.linalg.norm(a - b) <= 2e-4 * np.linalg.norm(a)


@pytest.mark.parametrize("m,c,seed", [(0.8, 0.0, 1), (0.0, 1.0, 2), (0.0, 0.0, 3)])
def test_mixed_targets(m, c, seed):
    """train.rs:120-155 after mix_batch: the host mirror (rustnn_b200.vit
    .targets) and the oracle's restatement give the same rows bit for bit;
    every row sums to 1 (to f32 rounding); lambda = 1 rows are the unmixed
    targets."""
    from oracle import rustvit as RV
    from rustnn_b200 import vit

    bs = 16
    rng = np.random.default_rng(seed)
    labels = rng.integers(0, 100, size=bs).astype(np.uint32)
    x = np.zeros(bs * PIX, F32)
    _, perm, lam, _ = O.mix_batch(x, bs, m, c, 0.5, O.Rng(seed).state())
    parent = RV.cifar_parent()
    lc = RV.LossCfg()
    tf_o, tc_o, _ = RV.targets(labels, parent, 20, lc, perm, lam)
    tf_h, tc_h, _ = vit.targets(labels, parent, 20, lc.smooth, lc.sib, perm=perm, lam=lam)
    assert np.array_equal(tf_o, tf_h) and np.array_equal(tc_o, tc_h)
    assert np.allclose(tf_h.reshape(bs, 100).sum(1), 1.0, atol=1e-5)
    assert np.allclose(tc_h.reshape(bs, 20).sum(1), 1.0, atol=1e-5)
    plain, _, _ = vit.targets(labels, parent, 20, lc.smooth, lc.sib)
    one = lam == 1.0
    assert np.array_equal(tf_h.reshape(bs, 100)[one], plain.reshape(bs, 100)[one])
