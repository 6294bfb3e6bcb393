"""GPU parity of the rustvit glue ops against the CPU oracle at the rustvit
shapes (batch 128, 8x8 tokens of 256 channels; 4x4 of 384; 100/20 classes),
bar 1e-4 relative Frobenius; layout ops and the DropPath mask are exact."""
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


def dev(a, dtype=np.float32):
    return torch.from_numpy(np.ascontiguousarray(a, dtype)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


@pytest.fixture(scope="module")
def ops():
    from rustnn_b200 import ops as _ops

    return _ops


L = O.lib


@pytest.mark.parametrize("n,th,c", [(128, 8, 256), (128, 4, 384), (3, 3, 8)])
def test_token_layers(ops, n, th, c):
    rng = O.Rng(n + th + c)
    rows = n * th * th
    x, dy = rng.rand_vec(rows * c), rng.rand_vec(rows * c)
    # LayerScale
    lv = rng.rand_vec(c)
    want = np.empty_like(x)
    L().orc_layerscale_fwd(x, rows, c, lv, want)
    assert rel(host(ops.layerscale_forward(dev(x), rows, c, dev(lv))), want) < 1e-6
    dl_ref, dx_ref = np.zeros(c, np.float32), np.empty_like(x)
    L().orc_layerscale_bwd(dy, x, rows, c, lv, dl_ref, dx_ref)
    dl = torch.zeros(c, device="cuda")
    dx = ops.layerscale_backward(dev(dy), dev(x), rows, c, dev(lv), dl)
    assert rel(host(dx), dx_ref) < 1e-6 and rel(host(dl), dl_ref) < TOL
    # DwConv3
    w, b = (0.1 * rng.rand_vec(9 * c)).astype(np.float32), rng.rand_vec(c)
    y_ref = np.empty_like(x)
    L().orc_dwconv3_fwd(x, n, th, th, c, w, b, y_ref)
    assert rel(host(ops.dwconv3_forward(dev(x), n, th, th, c, dev(w), dev(b))), y_ref) < TOL
    dw_ref, db_ref, dx_ref = np.zeros(9 * c, np.float32), np.zeros(c, np.float32), np.empty_like(x)
    L().orc_dwconv3_bwd(dy, x, n, th, th, c, w, dw_ref, db_ref, dx_ref)
    dw, db = torch.zeros(9 * c, device="cuda"), torch.zeros(c, device="cuda")
    dx = ops.dwconv3_backward(dev(dy), dev(x), n, th, th, c, dev(w), dw, db)
    assert rel(host(dx), dx_ref) < TOL and rel(host(dw), dw_ref) < TOL and rel(host(db), db_ref) < TOL
    # SeqPool
    t = th * th
    pv = (0.02 * rng.rand_vec(c)).astype(np.float32)
    z_ref, w_ref = np.empty(n * c, np.float32), np.empty(n * t, np.float32)
    L().orc_seqpool_fwd(x, n, t, c, pv, z_ref, w_ref)
    z, wt = ops.seqpool_forward(dev(x), n, t, c, dev(pv))
    assert rel(host(z), z_ref) < TOL and rel(host(wt), w_ref) < TOL
    dz = rng.rand_vec(n * c)
    dp_ref, dxs_ref = np.zeros(c, np.float32), np.empty_like(x)
    L().orc_seqpool_bwd(dz, x, w_ref, n, t, c, pv, dp_ref, dxs_ref)
    dp = torch.zeros(c, device="cuda")
    dxs = ops.seqpool_backward(dev(dz), dev(x), wt, n, t, c, dev(pv), dp)
    assert rel(host(dxs), dxs_ref) < TOL and rel(host(dp), dp_ref) < TOL
    # token merge and layout: exact permutations
    if th % 2 == 0:
        y_ref = np.empty_like(x)
        L().orc_token_merge_fwd(x, n, th, c, y_ref)
        ym = ops.token_merge(dev(x), n, th, c)
        assert np.array_equal(host(ym), y_ref)
        assert np.array_equal(host(ops.token_merge(ym, n, th, c, backward=True)), x)
    t_ref = np.empty_like(x)
    L().orc_tok_from_nchw(x, n, c, th * th, t_ref)
    tk = ops.tok_layout(dev(x), n, c, th * th)
    assert np.array_equal(host(tk), t_ref)
    assert np.array_equal(host(ops.tok_layout(tk, n, c, th * th, to_nchw=True)), x)


@pytest.mark.parametrize("rows,h", [(8192, 352), (2048, 512), (27, 16)])
def test_swiglu(ops, rows, h):
    rng = O.Rng(rows + h)
    ab, du = rng.rand_vec(rows * 2 * h), rng.rand_vec(rows * h)
    u_ref, dab_ref = np.empty(rows * h, np.float32), np.empty(rows * 2 * h, np.float32)
    L().orc_swiglu_act_fwd(ab, rows, h, u_ref)
    L().orc_swiglu_act_bwd(du, ab, rows, h, dab_ref)
    abd = dev(ab)
    assert rel(host(ops.swiglu_forward(abd, rows, h)), u_ref) < TOL
    assert rel(host(ops.swiglu_backward(dev(du), abd, rows, h)), dab_ref) < TOL


def test_droppath_mask_matches_reference_stream(ops):
    n, per, p, seed = 128, 64 * 256, 0.1, 99
    x = torch.ones(n * per, device="cuda")
    mask = ops.droppath_forward_(x, n, per, p, seed)
    want = np.empty(n, np.float32)
    L().orc_droppath_mask(n, p, seed, want)
    assert np.array_equal(host(mask), want)
    assert np.array_equal(host(x).reshape(n, per)[:, 0], want)
    dy = torch.ones(n * per, device="cuda")
    ops.droppath_backward_(dy, n, per, mask)
    assert np.array_equal(host(dy).reshape(n, per)[:, -1], want)


def test_heads_and_losses(ops):
    rng = O.Rng(8)
    n, nf, nc = 128, 100, 20
    parent = np.array([k // 5 for k in range(nf)], np.uint32)
    zf, zc = rng.rand_vec(n * nf), rng.rand_vec(n * nc)
    zf_ref = zf.copy()
    L().orc_taxo_fwd(zf_ref, zc, n, nf, nc, parent)
    zfd = dev(zf)
    pd = dev(parent.astype(np.int32), np.int32)
    ops.taxo_forward_(zfd, dev(zc), n, nf, nc, pd)
    assert rel(host(zfd), zf_ref) < 1e-6
    dzf, dzc = rng.rand_vec(n * nf), rng.rand_vec(n * nc)
    dc_ref = np.empty(n * nc, np.float32)
    L().orc_taxo_bwd(dzf, dzc, n, nf, nc, parent, dc_ref)
    assert rel(host(ops.taxo_backward(dev(dzf), dev(dzc), n, nf, nc, pd)), dc_ref) < 1e-6
    labels = np.array([rng.below(nf) for _ in range(n)], np.uint32)
    t = np.abs(rng.rand_vec(n * nf)) + 0.01
    t = (t.reshape(n, nf) / t.reshape(n, nf).sum(1, keepdims=True)).astype(np.float32).ravel()
    d_ref = np.empty(n * nf, np.float32)
    import ctypes as C

    corr = C.c_int(0)
    loss_ref = L().orc_ce_soft(zf, t, labels, n, nf, 0.5, d_ref, C.byref(corr))
    loss, dz, cr = ops.ce_soft(dev(zf), dev(t), dev(labels.astype(np.int32), np.int32), nf, 0.5)
    assert abs(float(host(loss)[0]) - loss_ref) <= 1e-5 * abs(loss_ref)
    assert rel(host(dz), d_ref) < TOL and int(host(cr)[0]) == corr.value
    teach = rng.rand_vec(n * nf)
    d_ref = np.zeros(n * nf, np.float32)
    kl_ref = L().orc_kl_distill(zf, teach, n, nf, 2.0, 0.3, d_ref)
    dzk = torch.zeros(n * nf, device="cuda")
    kl = ops.kl_distill(dev(zf), dev(teach), n, nf, 2.0, 0.3, dzk)
    assert abs(float(host(kl)[0]) - kl_ref) <= 1e-5 * abs(kl_ref) and rel(host(dzk), d_ref) < TOL
    pred, tgt = rng.rand_vec(n * 256), rng.rand_vec(n * 256)
    d_ref = np.zeros(n * 256, np.float32)
    hm_ref = L().orc_hint_mse(pred, tgt, n, 256, 0.7, d_ref)
    dzh = torch.zeros(n * 256, device="cuda")
    hm = ops.hint_mse(dev(pred), dev(tgt), n, 256, 0.7, dzh)
    assert abs(float(host(hm)[0]) - hm_ref) <= 1e-5 * abs(hm_ref) and rel(host(dzh), d_ref) < 1e-6
