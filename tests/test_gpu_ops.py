"""GPU parity of the operator-level C ABI against the CPU oracle.

Bar: relative Frobenius error <= 1e-4 per output tensor (the tolerance the
north star states); the 3xTF32 contractions land near 1e-6.
"""
import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-4


def rel(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    den = np.linalg.norm(want)
    return float(np.linalg.norm(got - want) / (den if den > 0 else 1.0))


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


@pytest.fixture(scope="module")
def ops():
    from rustnn_b200 import ops as _ops

    return _ops


# ------------------------------------------------------------------ GEMM

GEMMCHECK = [(23, 37, 19), (64, 48, 96), (7, 16, 259)]  # check.rs:131
BENCH = [  # bench.rs:17-24 with M scaled down 4x so the oracle stays fast
    (4096, 768, 256, False, True),
    (4096, 704, 256, False, True),
    (4096, 256, 768, False, False),
    (768, 256, 4096, True, False),
    (4096, 256, 352, False, True),
    (1024, 384, 1024, False, True),
]


@pytest.mark.parametrize("m,n,k", GEMMCHECK)
@pytest.mark.parametrize("at", [False, True])
@pytest.mark.parametrize("bt", [False, True])
def test_gemmcheck(ops, m, n, k, at, bt):
    rng = O.Rng(1234 + m + n + k)
    a, b = rng.rand_vec(m * k), rng.rand_vec(k * n)
    want = O.naive_matmul(m, n, k, a, at, b, bt)
    c = torch.zeros(m * n, device="cuda")
    ops.matmul(m, n, k, dev(a), at, dev(b), bt, c)
    assert rel(host(c), want) < TOL
    # acc = true: C += op(A) op(B)
    ops.matmul(m, n, k, dev(a), at, dev(b), bt, c, acc=True)
    assert rel(host(c), 2 * want) < TOL


@pytest.mark.parametrize("m,n,k,at,bt", BENCH)
def test_gemm_bench_shapes(ops, m, n, k, at, bt):
    rng = O.Rng(7)
    a, b = rng.rand_vec(m * k), rng.rand_vec(k * n)
    want = O.matmul(m, n, k, a, at, b, bt)
    c = torch.empty(m * n, device="cuda")
    ops.matmul(m, n, k, dev(a), at, dev(b), bt, c)
    assert rel(host(c), want) < TOL


@pytest.mark.parametrize("m,n,k", [(768, 256, 8192), (37, 29, 1000), (256, 352, 2048)])
def test_matmul_dw(ops, m, n, k):
    rng = O.Rng(3)
    a, b, c0 = rng.rand_vec(k * m), rng.rand_vec(k * n), rng.rand_vec(m * n)
    want = O.matmul_dw(m, n, k, a, b, c0.copy())
    c = dev(c0)
    ops.matmul_dw(m, n, k, dev(a), dev(b), c)
    assert rel(host(c), want) < TOL


def test_gemm_k_zero_and_empty(ops):
    c = torch.full((12,), 3.0, device="cuda")
    a = torch.zeros(1, device="cuda")
    ops.matmul(3, 4, 0, a, False, a, False, c, acc=False)  # gemm.rs:449-453
    assert np.all(host(c) == 0)
    c.fill_(3.0)
    ops.matmul(3, 4, 0, a, False, a, False, c, acc=True)
    assert np.all(host(c) == 3)


# ------------------------------------------------------------------ conv

CONVS = [  # (n, cin, h, cout, k, stride, pad)
    (2, 3, 6, 4, 3, 1, 1),    # check.rs:510 conv 3x3/s1
    (2, 4, 8, 6, 1, 2, 0),    # check.rs:511 conv 1x1/s2
    (2, 4, 7, 5, 3, 2, 1),    # check.rs:512 conv 3x3/s2, odd H
    (8, 32, 32, 32, 3, 1, 1), # cfg1 geometry at batch 8
    (4, 64, 16, 128, 3, 2, 1),
    (4, 64, 16, 128, 1, 2, 0),
    (2, 3, 32, 64, 3, 1, 1),  # stem
    (3, 128, 8, 256, 3, 1, 1),
    (64, 64, 32, 64, 3, 1, 1),   # 512 row tiles: several tiles per persistent CTA
    (24, 128, 16, 128, 3, 1, 1),
    (40, 64, 16, 64, 1, 1, 0),
    (9, 32, 16, 96, 3, 1, 1),
    (2, 32, 64, 32, 3, 1, 1),    # rows wider than a 32-pixel K block: window edges inside a row
    (3, 32, 12, 64, 3, 1, 1),    # 12-wide rows: K blocks straddle image rows, ragged last K block
    (2, 96, 16, 160, 3, 1, 1),   # 16-wide halo: three channel blocks, 160 outputs over two column tiles
    (3, 32, 15, 64, 3, 2, 1),    # stride-2 dgrad by parity class over an odd input (classes of 8 and 7 rows)
    (4, 32, 8, 64, 3, 1, 1),     # 8-wide rows: wgrad K blocks of four image rows
    (1, 32, 24, 32, 3, 1, 1),    # 24-pixel rows: not a halo width, per-pixel gather path
    (3, 64, 15, 64, 1, 2, 0),    # strided 1x1 dgrad over an odd input: last row/column hit
    (2, 32, 16, 64, 1, 3, 0),    # stride 3: two of every three rows/columns get no gradient
    (2, 40, 32, 128, 3, 1, 1),   # 32-wide wgrad at 128 columns; 360 rows: a ragged last row tile
    (2, 16, 32, 256, 3, 1, 1),   # 32-wide wgrad at 256 columns: the per-thread row loads
]


@pytest.mark.parametrize("n,cin,h,cout,k,stride,pad", [(4, 64, 16, 128, 1, 2, 0), (2, 32, 9, 64, 3, 2, 1),
                                                       (4, 64, 8, 64, 3, 1, 1),
                                                       (2, 32, 32, 64, 3, 1, 1),   # halo kernel, 32-wide
                                                       (3, 64, 16, 32, 3, 1, 1)])  # halo kernel, 16-wide
def test_conv_dgrad_accumulate(ops, n, cin, h, cout, k, stride, pad):
    """dgrad with acc adds into dX (the projection shortcut's gradient joins the main path's)."""
    rng = O.Rng(7 + cin + k)
    w = (rng.rand_vec(cout * cin * k * k) * np.float32(np.sqrt(2.0 / (cin * k * k)))).astype(np.float32)
    oh = (h + 2 * pad - k) // stride + 1
    dy = rng.rand_vec(n * cout * oh * oh)
    base = rng.rand_vec(n * cin * h * h)
    dx_ref = base + O.conv2d_dgrad(dy, n, cin, h, h, w, cout, k, stride, pad)
    dx = dev(base)
    ops.conv2d_dgrad(dev(dy), dev(w), n, cin, h, h, cout, k, stride, pad, dx=dx, acc=True)
    assert rel(host(dx), dx_ref) < TOL


@pytest.mark.parametrize("n,cin,h,cout,k,stride,pad", CONVS)
def test_conv_parity(ops, n, cin, h, cout, k, stride, pad):
    rng = O.Rng(100 + cin + cout)
    x = rng.rand_vec(n * cin * h * h)
    w = (rng.rand_vec(cout * cin * k * k) * np.float32(np.sqrt(2.0 / (cin * k * k)))).astype(np.float32)
    y_ref = O.conv2d_fwd(x, n, cin, h, h, w, cout, k, stride, pad)
    y = ops.conv2d_forward(dev(x), dev(w), n, cin, h, h, cout, k, stride, pad)
    assert rel(host(y), y_ref) < TOL
    dy = rng.rand_vec(y_ref.size)
    dx_ref = O.conv2d_dgrad(dy, n, cin, h, h, w, cout, k, stride, pad)
    dx = ops.conv2d_dgrad(dev(dy), dev(w), n, cin, h, h, cout, k, stride, pad)
    assert rel(host(dx), dx_ref) < TOL
    dw0 = rng.rand_vec(w.size)
    dw_ref = O.conv2d_wgrad(x, dy, n, cin, h, h, cout, k, stride, pad, dw=dw0.copy())
    dw = dev(dw0)
    ops.conv2d_wgrad(dev(x), dev(dy), n, cin, h, h, cout, k, stride, pad, dw=dw)
    assert rel(host(dw), dw_ref) < TOL


@pytest.mark.parametrize("n,cin,h,cout", [(8, 32, 32, 32), (2, 3, 32, 64), (64, 64, 32, 64), (2, 40, 32, 128),
                                          (5, 64, 32, 64), (4, 64, 16, 128), (3, 40, 16, 64), (2, 128, 16, 128),
                                          (6, 16, 16, 32)])
@pytest.mark.parametrize("halo", ["1", "0"])
def test_conv_wgrad_both_kernels(ops, monkeypatch, n, cin, h, cout, halo):
    """32- and 16-wide 3x3 wgrad through the tensor-copy kernel (halo groups
    of 8 K blocks, split-K in whole groups) and through the per-thread row
    loads, at sizes where the default picks the latter."""
    monkeypatch.setenv("RNN_WGRAD_HALO", halo)
    rng = O.Rng(300 + cin + cout + n)
    x = rng.rand_vec(n * cin * h * h)
    dy = rng.rand_vec(n * cout * h * h)
    dw0 = rng.rand_vec(cout * cin * 9)
    dw_ref = O.conv2d_wgrad(x, dy, n, cin, h, h, cout, 3, 1, 1, dw=dw0.copy())
    dw = dev(dw0)
    ops.conv2d_wgrad(dev(x), dev(dy), n, cin, h, h, cout, 3, 1, 1, dw=dw)
    assert rel(host(dw), dw_ref) < TOL


def test_conv_cfg1_full(ops):
    """N=128, 32->32, 32x32, 3x3 s1 p1, He-normal weights, seed 0."""
    n, c, h = 128, 32, 32
    rng = O.Rng(0)
    x = rng.rand_vec(n * c * h * h)
    w = (rng.rand_vec(c * c * 9) * np.float32(np.sqrt(2.0 / 288))).astype(np.float32)
    dy = rng.rand_vec(n * c * h * h)
    y = ops.conv2d_forward(dev(x), dev(w), n, c, h, h, c, 3, 1, 1)
    assert rel(host(y), O.conv2d_fwd(x, n, c, h, h, w, c, 3, 1, 1)) < TOL
    dx = ops.conv2d_dgrad(dev(dy), dev(w), n, c, h, h, c, 3, 1, 1)
    assert rel(host(dx), O.conv2d_dgrad(dy, n, c, h, h, w, c, 3, 1, 1)) < TOL
    dw = ops.conv2d_wgrad(dev(x), dev(dy), n, c, h, h, c, 3, 1, 1)
    assert rel(host(dw), O.conv2d_wgrad(x, dy, n, c, h, h, c, 3, 1, 1)) < TOL


def test_conv_dgrad_accumulates(ops):
    n, cin, h, cout = 2, 8, 8, 16
    rng = O.Rng(9)
    w = rng.rand_vec(cout * cin * 9)
    dy = rng.rand_vec(n * cout * h * h)
    base = rng.rand_vec(n * cin * h * h)
    dx = dev(base)
    ops.conv2d_dgrad(dev(dy), dev(w), n, cin, h, h, cout, 3, 1, 1, dx=dx, acc=True)
    assert rel(host(dx), base + O.conv2d_dgrad(dy, n, cin, h, h, w, cout, 3, 1, 1)) < TOL


# ------------------------------------------------------------------ BN / glue


@pytest.mark.parametrize("n,c,hw,relu", [(3, 4, 25, False), (16, 64, 256, True), (8, 32, 1024, True),
                                         (64, 256, 64, True), (37, 8, 4, False), (5, 3, 12, True)])
def test_batchnorm_parity(ops, n, c, hw, relu):
    rng = O.Rng(21)
    y = (rng.rand_vec(n * c * hw) * 2.0 + 1.0).astype(np.float32)
    g = np.array([0.5 + rng.uniform() for _ in range(c)], np.float32)
    b = rng.rand_vec(c)
    rm, rv = rng.rand_vec(c), (np.abs(rng.rand_vec(c)) + 0.5).astype(np.float32)
    rm_ref, rv_ref = rm.copy(), rv.copy()
    out_ref, xhat_ref, invstd_ref = O.bn_fwd_train(y, n, c, hw, g, b, rm_ref, rv_ref, relu)
    rm_d, rv_d = dev(rm), dev(rv)
    out, mean, invstd = ops.batchnorm_forward(dev(y), n, c, hw, dev(g), dev(b), rm_d, rv_d, relu)
    assert rel(host(out), out_ref) < TOL
    assert rel(host(invstd), invstd_ref) < 1e-6
    assert rel(host(rm_d), rm_ref) < 1e-6 and rel(host(rv_d), rv_ref) < 1e-6
    dy = rng.rand_vec(y.size)
    dy_eff = dy.copy()
    if relu:
        O.lib().orc_relu_back(dy_eff, out_ref, dy_eff.size)
    dg_ref, db_ref = np.zeros(c, np.float32), np.zeros(c, np.float32)
    dx_ref = O.bn_bwd(dy_eff, xhat_ref, n, c, hw, g, invstd_ref, dg_ref, db_ref)
    dg, db = torch.zeros(c, device="cuda"), torch.zeros(c, device="cuda")
    dx = ops.batchnorm_backward(dev(dy), dev(y), n, c, hw, dev(g), mean, invstd, dg, db,
                                relu_out=out if relu else None)
    assert rel(host(dx), dx_ref) < TOL
    assert rel(host(dg), dg_ref) < TOL and rel(host(db), db_ref) < TOL


@pytest.mark.parametrize("n,nclass,smooth", [(4, 7, 0.1), (1024, 100, 0.1), (33, 10, 0.0)])
def test_softmax_ce_parity(ops, n, nclass, smooth):
    rng = O.Rng(5)
    z = (rng.rand_vec(n * nclass) * 3).astype(np.float32)
    labels = np.array([rng.below(nclass) for _ in range(n)], np.uint32)
    loss_ref, d_ref, corr_ref = O.softmax_ce(z, labels, nclass, smooth)
    loss, d, corr = ops.softmax_ce(dev(z), torch.from_numpy(labels.astype(np.int32)).cuda(), nclass, smooth)
    assert abs(float(host(loss)[0]) - loss_ref) <= 1e-5 * abs(loss_ref) + 1e-6
    assert rel(host(d), d_ref) < TOL
    assert int(host(corr)[0]) == corr_ref


def test_elementwise(ops):
    rng = O.Rng(8)
    a, b = rng.rand_vec(1003), rng.rand_vec(1003)
    t = dev(a)
    ops.add_relu_(t, dev(b))
    want = a.copy()
    O.lib().orc_add_relu(want, b, want.size)
    assert np.array_equal(host(t), want)
    t = dev(a)
    ops.relu_back_(t, dev(b))
    want = a.copy()
    O.lib().orc_relu_back(want, b, want.size)
    assert np.array_equal(host(t), want)
    x = rng.rand_vec(6 * 64)
    y = ops.gap_forward(dev(x), 6, 64)
    want = np.empty(6, np.float32)
    O.lib().orc_gap_fwd(x, 6, 64, want)
    assert rel(host(y), want) < 1e-6


def test_bad_arguments_raise(ops):
    from rustnn_b200 import RnnError

    x = torch.zeros(16, device="cuda")
    with pytest.raises(RnnError):
        ops.conv2d_forward(x, x, 1, 1, 4, 4, 1, 5, 1, 0)  # 5x5 kernels are not a reference shape
    with pytest.raises(RnnError):
        ops.matmul(-1, 2, 2, x, False, x, False, x)
