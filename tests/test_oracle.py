"""Pins the CPU oracle to the reference's own known-answer checks.

The reference ships no stored tensors, so the oracle is pinned to what its
tests hold:

* the naive-GEMM check, check.rs:124-161 (3 shapes x 4 transposes);
* the directional-derivative gradchecks, check.rs:19-40 (dircheck),
  check.rs:503-724 (layercheck) and check.rs:727-770 (full ResNet);
* the published parameter/MAC counts, README.md:116-117, and the rng
  contract of rng.rs:74-118.
"""
import numpy as np
import pytest

from oracle import oracle as O

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


def max_rel(want, got):
    """check.rs:135-141."""
    return float(np.max(np.abs(want - got)) / max(1e-6, float(np.max(np.abs(want)))))


# ------------------------------------------------------------------ rng.rs


def test_rng_contract():
    a, b = O.Rng(1234), O.Rng(1234)
    assert all(a.next_u64() == b.next_u64() for _ in range(1000))
    assert O.Rng(1).next_u64() != O.Rng(2).next_u64()
    r = O.Rng(7)
    xs = [r.uniform() for _ in range(10000)]
    assert min(xs) >= 0.0 and max(xs) < 1.0
    r = O.Rng(9)
    for n in (1, 2, 7, 100):
        assert all(r.below(n) < n for _ in range(1000))


def test_rng_xoshiro_known_answer():
    """SplitMix64 seeding + xoshiro256++, written out independently in Python."""
    M = 2**64 - 1

    def rotl(x, k):
        return ((x << k) | (x >> (64 - k))) & M

    z = (5 + 0x9E3779B97F4A7C15) & M
    s = []
    for _ in range(4):
        z = (z + 0x9E3779B97F4A7C15) & M
        x = z
        x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & M
        x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & M
        s.append(x ^ (x >> 31))
    r = O.Rng(5)
    for _ in range(64):
        res = (rotl((s[0] + s[3]) & M, 23) + s[0]) & M
        t = (s[1] << 17) & M
        s[2] ^= s[0]
        s[3] ^= s[1]
        s[1] ^= s[2]
        s[0] ^= s[3]
        s[2] ^= t
        s[3] = rotl(s[3], 45)
        assert r.next_u64() == res


def test_normal_moments():
    v = O.Rng(0).rand_vec(200000)
    assert abs(v.mean()) < 0.01 and abs(v.std() - 1.0) < 0.01


# ------------------------------------------------------------------ gemm


@pytest.mark.parametrize("m,n,k", [(23, 37, 19), (64, 48, 96), (7, 16, 259)])
@pytest.mark.parametrize("at", [False, True])
@pytest.mark.parametrize("bt", [False, True])
def test_gemmcheck(m, n, k, at, bt):
    """check.rs:124-161, with a much tighter bar than the reference's 5e-3."""
    rng = O.Rng(1234 ^ m ^ (n << 8) ^ (k << 16))
    a = rng.rand_vec(m * k)
    b = rng.rand_vec(k * n)
    want = O.naive_matmul(m, n, k, a, at, b, bt)
    got = O.matmul(m, n, k, a, at, b, bt)
    assert max_rel(want, got) < 1e-5
    # acc = true adds on top of C
    got2 = O.matmul(m, n, k, a, at, b, bt, c=got.copy(), acc=True)
    assert max_rel(2 * want, got2) < 1e-5


def test_matmul_dw_against_naive():
    rng = O.Rng(3)
    m, n, k = 37, 29, 1000
    a = rng.rand_vec(k * m)
    b = rng.rand_vec(k * n)
    c0 = rng.rand_vec(m * n)
    want = c0 + O.naive_matmul(m, n, k, a, True, b, False)
    got = O.matmul_dw(m, n, k, a, b, c0.copy())
    assert max_rel(want, got) < 1e-5


# ------------------------------------------------------------------ layers


def kaiming(rng, fan_in, n):
    s = np.float32(np.sqrt(np.float32(2.0) / np.float32(fan_in)))
    return (rng.rand_vec(n) * s).astype(np.float32)


@pytest.mark.parametrize(
    "cin,cout,k,stride,pad,hh",
    [(3, 4, 3, 1, 1, 6), (4, 6, 1, 2, 0, 8), (4, 5, 3, 2, 1, 7)],  # check.rs:509-513
)
def test_conv_gradcheck(cin, cout, k, stride, pad, hh):
    rng = O.Rng(1234)
    w = kaiming(rng, cin * k * k, cout * cin * k * k)
    x = rng.rand_vec(2 * cin * hh * hh)
    y0 = O.conv2d_fwd(x, 2, cin, hh, hh, w, cout, k, stride, pad)
    r = rng.rand_vec(y0.size)
    dw = O.conv2d_wgrad(x, r, 2, cin, hh, hh, cout, k, stride, pad)
    dx = O.conv2d_dgrad(r, 2, cin, hh, hh, w, cout, k, stride, pad)
    e = dircheck(x, dx, EPS, rng, lambda c: float(np.dot(O.conv2d_fwd(c, 2, cin, hh, hh, w, cout, k, stride, pad), r)))
    assert e < TOL, e
    e = dircheck(w, dw, EPS, rng, lambda c: float(np.dot(O.conv2d_fwd(x, 2, cin, hh, hh, c, cout, k, stride, pad), r)))
    assert e < TOL, e


def test_batchnorm_gradcheck():
    """check.rs:546-596."""
    rng = O.Rng(99)
    c, n, hw = 4, 3, 25
    g = np.array([0.5 + rng.uniform() for _ in range(c)], np.float32)
    b = rng.rand_vec(c)
    x = (rng.rand_vec(n * c * hw) * 2.0 + 1.0).astype(np.float32)

    def fwd(xx, gg, bb):
        rm, rv = np.zeros(c, np.float32), np.ones(c, np.float32)
        return O.bn_fwd_train(xx, n, c, hw, gg, bb, rm, rv, relu=False)

    y0, xhat, invstd = fwd(x, g, b)
    r = rng.rand_vec(y0.size)
    dg, db = np.zeros(c, np.float32), np.zeros(c, np.float32)
    dx = O.bn_bwd(r, xhat, n, c, hw, g, invstd, dg, db)
    assert dircheck(x, dx, EPS, rng, lambda cc: float(np.dot(fwd(cc, g, b)[0], r))) < TOL
    assert dircheck(g, dg, EPS, rng, lambda cc: float(np.dot(fwd(x, cc, b)[0], r))) < TOL
    assert dircheck(b, db, EPS, rng, lambda cc: float(np.dot(fwd(x, g, cc)[0], r))) < TOL


def test_fc_gradcheck():
    """check.rs:598-623 (nn::Linear)."""
    import ctypes as C

    L = O.lib()
    rng = O.Rng(5)
    fin, fout, n = 6, 5, 3
    w = (kaiming(rng, fin, fin * fout) * np.float32(0.5)).astype(np.float32)
    b = rng.rand_vec(fout)
    x = rng.rand_vec(n * fin)

    def fwd(xx, ww):
        y = np.empty(n * fout, np.float32)
        L.orc_fc_fwd(np.ascontiguousarray(xx, np.float32), n, fin, fout, np.ascontiguousarray(ww, np.float32), b, y)
        return y

    r = rng.rand_vec(n * fout)
    dw, db, dx = np.zeros(fin * fout, np.float32), np.zeros(fout, np.float32), np.zeros(n * fin, np.float32)
    L.orc_fc_bwd(x, r, n, fin, fout, w, dw, db, dx)
    assert dircheck(x, dx, EPS, rng, lambda c: float(np.dot(fwd(c, w), r))) < TOL
    assert dircheck(w, dw, EPS, rng, lambda c: float(np.dot(fwd(x, c), r))) < TOL
    del C


def test_softmax_ce_gradcheck():
    """check.rs:665-676."""
    rng = O.Rng(11)
    n, nc = 4, 7
    z = rng.rand_vec(n * nc)
    labels = np.array([rng.below(nc) for _ in range(n)], np.uint32)
    _, d, _ = O.softmax_ce(z, labels, nc, 0.1)
    e = dircheck(z, d, EPS, rng, lambda c: O.softmax_ce(c, labels, nc, 0.1)[0])
    assert e < TOL, e


# ------------------------------------------------------------------ model


def test_resnet_param_and_mac_counts():
    """README.md:116-117 (resnet14 w32: 708,228 params, 105.8 MMAC/img)."""
    net = O.ResNet(2, 32, 100, 1234)
    assert net.num_params() == 708228
    assert round(net.flops() / 2e6, 1) == 105.8
    # ResNet-56 W=64, the data-parallel config: 13,651,364 params
    assert O.ResNet(9, 64, 100, 0).num_params() == 13651364


def test_resnet_full_gradcheck():
    """check.rs:727-770: ResNet-8 w4, 16x16, batch 8, all parameters."""
    NC, BS, seed = 10, 8, 1234
    net = O.ResNet(1, 4, NC, seed)
    rng = O.Rng(seed ^ 0x5EED)
    sizes, _ = net.param_info()
    p = net.params()
    p = (p + np.float32(0.3) * rng.rand_vec(p.size)).astype(np.float32)
    net.set_params(p)
    x = rng.rand_vec(BS * 3 * 16 * 16)
    labels = np.array([rng.below(NC) for _ in range(BS)], np.uint32)
    logits = net.forward(x, BS, hw=16, train=True)
    _, dl, _ = O.softmax_ce(logits, labels, NC, 0.0)
    net.zero_grads()
    net.backward(dl)
    g = net.grads()

    def lossf(c):
        net.set_params(c)
        lg = net.forward(x, BS, hw=16, train=True)
        return O.softmax_ce(lg, labels, NC, 0.0)[0]

    e = dircheck(p, g, EPS, rng, lossf)
    net.set_params(p)
    assert e < TOL, e


# ------------------------------------------------------------------ attention, LN, linear, NS


def test_rel_index_geometry():
    """attn.rs:23-72: self 3x3 -> 5x5 offsets; cross 3x3 over 6x6 -> 10x10."""
    idx, nrel = O.rel_index(3, 3, 3, 3)
    assert nrel == 25 and idx.max() == 24 and idx.min() == 0
    assert idx[0] == 12  # q (0,0) vs k (0,0): zero offset = origin (2,2)
    idx, nrel = O.rel_index(3, 3, 6, 6)
    assert nrel == 100 and idx.max() < 100


def _attn_fixture(rng, n, h, dh, th, mh, self_attn):
    c = h * dh
    tq, tk = th * th, mh * mh
    relidx, nrel = O.rel_index(th, th, mh, mh)
    tau = np.full(h, np.float32(1.0 / np.sqrt(np.float32(dh))), np.float32)
    rel = rng.rand_vec(h * nrel)
    if self_attn:
        ab = rng.rand_vec(n * tq * 3 * c)
        geo = dict(q=ab, qstride=3 * c, qoff=0, kv=ab, kvstride=3 * c, koff=c, voff=2 * c)
    else:
        q = rng.rand_vec(n * tq * c)
        mem = rng.rand_vec(n * tk * 2 * c)
        geo = dict(q=q, qstride=c, qoff=0, kv=mem, kvstride=2 * c, koff=0, voff=c)
    return c, tq, tk, relidx, nrel, tau, rel, geo


@pytest.mark.parametrize("self_attn", [True, False])
def test_attention_core_gradcheck(self_attn):
    """check.rs:300-348 geometry (c=8, h=2, 3x3 grid, 6x6 memory) on Core."""
    rng = O.Rng(77 + int(self_attn))
    n, h, dh, th, mh = 3, 2, 4, 3, 3 if self_attn else 6
    c, tq, tk, relidx, nrel, tau, rel, geo = _attn_fixture(rng, n, h, dh, th, mh, self_attn)
    mask = self_attn

    def fwd(geo_, tau_, rel_):
        return O.attn_fwd(n, h, dh, tq, tk, mask, relidx, nrel, geo_["q"], geo_["qstride"], geo_["qoff"],
                          geo_["kv"], geo_["kvstride"], geo_["koff"], geo_["voff"], tau_, rel_)

    p, o = fwd(geo, tau, rel)
    r = rng.rand_vec(o.size)
    dq = np.zeros_like(geo["q"])
    dkv = np.zeros_like(geo["kv"]) if not self_attn else dq  # self: fused buffer, one gradient
    dtau, drel = np.zeros(h, np.float32), np.zeros(h * nrel, np.float32)
    O.attn_bwd(n, h, dh, tq, tk, relidx, nrel, geo["q"], geo["qstride"], geo["qoff"], geo["kv"], geo["kvstride"],
               geo["koff"], geo["voff"], tau, p, r, dq, dkv, dtau, drel)
    loss = lambda g_, t_, r_: float(np.dot(fwd(g_, t_, r_)[1], r))
    if self_attn:
        e = dircheck(geo["q"], dq, EPS, rng, lambda v: loss({**geo, "q": v, "kv": v}, tau, rel))
        assert e < TOL, e
    else:
        assert dircheck(geo["q"], dq, EPS, rng, lambda v: loss({**geo, "q": v}, tau, rel)) < TOL
        assert dircheck(geo["kv"], dkv, EPS, rng, lambda v: loss({**geo, "kv": v}, tau, rel)) < TOL
    assert dircheck(tau, dtau, EPS, rng, lambda v: loss(geo, v, rel)) < TOL
    assert dircheck(rel, drel, EPS, rng, lambda v: loss(geo, tau, v)) < TOL


def test_layernorm_gradcheck():
    """check.rs:183-213 (Tok 3x9x8)."""
    rng = O.Rng(31)
    rows, c = 27, 8
    x = rng.rand_vec(rows * c)
    g = (1.0 + 0.2 * rng.rand_vec(c)).astype(np.float32)
    b = rng.rand_vec(c)
    r = rng.rand_vec(rows * c)
    y, xhat, invstd = O.layernorm_fwd(x, rows, c, g, b)
    dg, db = np.zeros(c, np.float32), np.zeros(c, np.float32)
    dx = O.layernorm_bwd(r, xhat, invstd, rows, c, g, dg, db)
    f = lambda xx, gg, bb: float(np.dot(O.layernorm_fwd(xx, rows, c, gg, bb)[0], r))
    assert dircheck(x, dx, EPS, rng, lambda v: f(v, g, b)) < TOL
    assert dircheck(g, dg, EPS, rng, lambda v: f(x, v, b)) < TOL
    assert dircheck(b, db, EPS, rng, lambda v: f(x, g, v)) < TOL


def test_linear_gradcheck():
    rng = O.Rng(41)
    rows, fin, fout = 27, 8, 12
    x, w, b = rng.rand_vec(rows * fin), rng.rand_vec(fout * fin), rng.rand_vec(fout)
    r = rng.rand_vec(rows * fout)
    dw, db = np.zeros(fout * fin, np.float32), np.zeros(fout, np.float32)
    dx = O.linear_bwd(x, r, rows, fin, fout, w, dw, db)
    f = lambda xx, ww, bb: float(np.dot(O.linear_fwd(xx, rows, fin, fout, ww, bb), r))
    assert dircheck(x, dx, EPS, rng, lambda v: f(v, w, b)) < TOL
    assert dircheck(w, dw, EPS, rng, lambda v: f(x, v, b)) < TOL
    assert dircheck(b, db, EPS, rng, lambda v: f(x, w, v)) < TOL


def gram_error(g, m, n):
    """check.rs:462-482."""
    G = np.asarray(g, np.float64).reshape(m, n)
    M = G @ G.T if m <= n else G.T @ G
    return float(np.abs(M - np.eye(M.shape[0])).max())


@pytest.mark.parametrize("m,n", [(12, 20), (20, 12), (16, 16)])
def test_newton_schulz_band(m, n):
    """check.rs:484-497: singular values in a band around 1 (tol 0.5)."""
    g = O.Rng(m * 100 + n).rand_vec(m * n)
    out = O.newton_schulz(g, m, n, 5)
    assert gram_error(out, m, n) < 0.5


# ------------------------------------------------------------------ rustvit glue (check.rs normcheck / losses)


def _gc(x, g, f, rng):
    return dircheck(x, g, EPS, rng, f)


def test_glue_gradchecks():
    L = O.lib()
    rng = O.Rng(2024)
    n, th, c = 3, 3, 8
    rows = n * th * th
    x = rng.rand_vec(rows * c)
    r = rng.rand_vec(rows * c)
    # LayerScale (norm.rs:151-212)
    lv = rng.rand_vec(c)
    fwd = lambda xx, ll: (lambda y: (L.orc_layerscale_fwd(np.ascontiguousarray(xx, np.float32), rows, c,
                                                          np.ascontiguousarray(ll, np.float32), y), y)[1])(
        np.empty(rows * c, np.float32))
    dl, dx = np.zeros(c, np.float32), np.empty(rows * c, np.float32)
    L.orc_layerscale_bwd(r, x, rows, c, lv, dl, dx)
    assert _gc(x, dx, lambda v: float(np.dot(fwd(v, lv), r)), rng) < TOL
    assert _gc(lv, dl, lambda v: float(np.dot(fwd(x, v), r)), rng) < TOL
    # SwiGLU gate (norm.rs:250-286)
    h = 6
    ab = rng.rand_vec(rows * 2 * h)
    ru = rng.rand_vec(rows * h)
    act = lambda v: (lambda u: (L.orc_swiglu_act_fwd(np.ascontiguousarray(v, np.float32), rows, h, u), u)[1])(
        np.empty(rows * h, np.float32))
    dab = np.empty(rows * 2 * h, np.float32)
    L.orc_swiglu_act_bwd(ru, ab, rows, h, dab)
    assert _gc(ab, dab, lambda v: float(np.dot(act(v), ru)), rng) < TOL
    # DwConv3 (norm.rs:304-451)
    w, b = (0.1 * rng.rand_vec(9 * c)).astype(np.float32), rng.rand_vec(c)
    dwf = lambda xx, ww, bb: (lambda y: (L.orc_dwconv3_fwd(np.ascontiguousarray(xx, np.float32), n, th, th, c,
                                                            np.ascontiguousarray(ww, np.float32),
                                                            np.ascontiguousarray(bb, np.float32), y), y)[1])(
        np.empty(rows * c, np.float32))
    dw, db, dx = np.zeros(9 * c, np.float32), np.zeros(c, np.float32), np.empty(rows * c, np.float32)
    L.orc_dwconv3_bwd(r, x, n, th, th, c, w, dw, db, dx)
    assert _gc(x, dx, lambda v: float(np.dot(dwf(v, w, b), r)), rng) < TOL
    assert _gc(w, dw, lambda v: float(np.dot(dwf(x, v, b), r)), rng) < TOL
    assert _gc(b, db, lambda v: float(np.dot(dwf(x, w, v), r)), rng) < TOL
    # SeqPool (norm.rs:466-581)
    t = th * th
    pv = rng.rand_vec(c)
    rz = rng.rand_vec(n * c)

    def sp(xx, pp):
        z, wt = np.empty(n * c, np.float32), np.empty(n * t, np.float32)
        L.orc_seqpool_fwd(np.ascontiguousarray(xx, np.float32), n, t, c, np.ascontiguousarray(pp, np.float32), z, wt)
        return z, wt

    _, wt = sp(x, pv)
    dp, dx = np.zeros(c, np.float32), np.empty(rows * c, np.float32)
    L.orc_seqpool_bwd(rz, x, wt, n, t, c, pv, dp, dx)
    assert _gc(x, dx, lambda v: float(np.dot(sp(v, pv)[0], rz)), rng) < TOL
    assert _gc(pv, dp, lambda v: float(np.dot(sp(x, v)[0], rz)), rng) < TOL


def test_loss_gradchecks():
    """check.rs:678-722 (ce_soft, kl_distill) and hint_mse."""
    L = O.lib()
    rng = O.Rng(77)
    n, nc = 4, 7
    z = rng.rand_vec(n * nc)
    labels = np.array([rng.below(nc) for _ in range(n)], np.uint32)
    t = np.abs(rng.rand_vec(n * nc)) + 0.1
    t = (t.reshape(n, nc) / t.reshape(n, nc).sum(1, keepdims=True)).astype(np.float32).ravel()
    d = np.empty(n * nc, np.float32)
    L.orc_ce_soft(z, t, labels, n, nc, 1.0, d, None)
    tmp = np.empty(n * nc, np.float32)
    assert dircheck(z, d, EPS, rng, lambda v: L.orc_ce_soft(np.ascontiguousarray(v, np.float32), t, labels, n, nc,
                                                            1.0, tmp, None)) < TOL
    teach = rng.rand_vec(n * nc)
    d = np.zeros(n * nc, np.float32)
    L.orc_kl_distill(z, teach, n, nc, 2.0, 1.0, d)

    def kl(v):
        tmp2 = np.zeros(n * nc, np.float32)
        return L.orc_kl_distill(np.ascontiguousarray(v, np.float32), teach, n, nc, 2.0, 1.0, tmp2)

    assert dircheck(z, d, EPS, rng, kl) < TOL
    pred, tgt = rng.rand_vec(n * 5), rng.rand_vec(n * 5)
    d = np.zeros(n * 5, np.float32)
    L.orc_hint_mse(pred, tgt, n, 5, 0.7, d)

    def hm(v):
        tmp3 = np.zeros(n * 5, np.float32)
        return L.orc_hint_mse(np.ascontiguousarray(v, np.float32), tgt, n, 5, 0.7, tmp3)

    assert dircheck(pred, d, EPS, rng, hm) < TOL


def test_layout_round_trips():
    L = O.lib()
    rng = O.Rng(3)
    n, th, c = 2, 4, 3
    z = rng.rand_vec(n * th * th * c)
    y, back = np.empty_like(z), np.empty_like(z)
    L.orc_token_merge_fwd(z, n, th, c, y)
    L.orc_token_merge_bwd(y, n, th, c, back)
    assert np.array_equal(back, z)
    # merged token (0,0) holds source tokens (0,0), (0,1), (1,0), (1,1)
    zz = z.reshape(n, th, th, c)
    assert np.array_equal(y.reshape(n, 4, 4 * c)[0, 0], np.concatenate([zz[0, 0, 0], zz[0, 0, 1], zz[0, 1, 0], zz[0, 1, 1]]))
    x = rng.rand_vec(n * c * 16)
    tk, nchw = np.empty_like(x), np.empty_like(x)
    L.orc_tok_from_nchw(x, n, c, 16, tk)
    L.orc_tok_to_nchw(tk, n, c, 16, nchw)
    assert np.array_equal(nchw, x)
    assert np.array_equal(tk.reshape(n, 16, c), x.reshape(n, c, 16).transpose(0, 2, 1))
