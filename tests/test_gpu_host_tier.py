"""The host-pointer tier of the attention / normalisation / optimiser entry
points against the CPU oracle (bar 1e-4 relative Frobenius; accumulating
outputs start from nonzero values so the read-back is exercised)."""
import ctypes as C

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


def P(a):
    return C.c_void_p(a.ctypes.data)


@pytest.fixture(scope="module")
def api():
    from rustnn_b200 import _lib, ops

    ctx = ops.default_context()
    return _lib, ctx


def test_attention_host_tier(api):
    _lib, ctx = api
    rng = O.Rng(3)
    n, h, dh, th = 4, 2, 8, 4
    c, t = h * dh, th * th
    ab = (rng.rand_vec(n * t * 3 * c) * 0.5).astype(np.float32)
    tau = np.array([0.3, 0.4], np.float32)
    idx, nrel = O.rel_index(th, th, th, th)
    relb = rng.rand_vec(h * nrel)
    p_ref, o_ref = O.attn_fwd(n, h, dh, t, t, True, idx, nrel, ab, 3 * c, 0, ab, 3 * c, c, 2 * c, tau, relb)
    p, o = np.empty_like(p_ref), np.empty_like(o_ref)
    _lib.call("rnn_attn_fwd", ctx.bind(), n, h, dh, th, th, th, th, 1, P(ab), 3 * c, 0, P(ab), 3 * c, c, 2 * c,
              P(tau), P(relb), P(p), P(o))
    assert rel(p, p_ref) < TOL and rel(o, o_ref) < TOL
    dout = rng.rand_vec(o.size)
    dq0, dkv0 = rng.rand_vec(ab.size), rng.rand_vec(ab.size)
    dt0, dr0 = rng.rand_vec(h), rng.rand_vec(h * nrel)
    want = [a.copy() for a in (dq0, dkv0, dt0, dr0)]
    O.attn_bwd(n, h, dh, t, t, idx, nrel, ab, 3 * c, 0, ab, 3 * c, c, 2 * c, tau, p_ref, dout, *want)
    got = [a.copy() for a in (dq0, dkv0, dt0, dr0)]
    _lib.call("rnn_attn_bwd", ctx.bind(), n, h, dh, th, th, th, th, P(ab), 3 * c, 0, P(ab), 3 * c, c, 2 * c, P(tau),
              P(p), P(dout), *[P(a) for a in got])
    for g_, w_ in zip(got, want):
        assert rel(g_, w_) < TOL


def test_norm_and_linear_host_tier(api):
    _lib, ctx = api
    rng = O.Rng(4)
    rows, c = 37, 24
    x = (rng.rand_vec(rows * c) * 2 + 0.5).astype(np.float32)
    g, b = (1 + 0.1 * rng.rand_vec(c)).astype(np.float32), rng.rand_vec(c)
    y_ref, xh_ref, is_ref = O.layernorm_fwd(x, rows, c, g, b)
    y, xh, inv = np.empty_like(x), np.empty_like(x), np.empty(rows, np.float32)
    _lib.call("rnn_layernorm_fwd", ctx.bind(), P(x), rows, c, P(g), P(b), 1e-5, P(y), P(xh), P(inv))
    assert rel(y, y_ref) < TOL and rel(xh, xh_ref) < TOL and rel(inv, is_ref) < TOL
    dy = rng.rand_vec(x.size)
    dg0, db0 = rng.rand_vec(c), rng.rand_vec(c)
    dg_ref, db_ref = dg0.copy(), db0.copy()
    dx_ref = O.layernorm_bwd(dy, xh_ref, is_ref, rows, c, g, dg_ref, db_ref)
    dx, dg_, db_ = np.empty_like(x), dg0.copy(), db0.copy()
    _lib.call("rnn_layernorm_bwd", ctx.bind(), P(dy), P(xh), P(inv), rows, c, P(g), P(dx), P(dg_), P(db_))
    assert rel(dx, dx_ref) < TOL and rel(dg_, dg_ref) < TOL and rel(db_, db_ref) < TOL
    fin, fout = c, 40
    w = (0.1 * rng.rand_vec(fout * fin)).astype(np.float32)
    bias = rng.rand_vec(fout)
    yl_ref = O.linear_fwd(x, rows, fin, fout, w, bias)
    yl = np.empty(rows * fout, np.float32)
    _lib.call("rnn_linear_fwd", ctx.bind(), P(x), rows, fin, fout, P(w), P(bias), P(yl))
    assert rel(yl, yl_ref) < TOL
    dyl = rng.rand_vec(rows * fout)
    dw0, dbias0 = rng.rand_vec(w.size), rng.rand_vec(fout)
    dw_ref, dbias_ref = dw0.copy(), dbias0.copy()
    dxl_ref = O.linear_bwd(x, dyl, rows, fin, fout, w, dw_ref, dbias_ref)
    dw_, dbias_, dxl = dw0.copy(), dbias0.copy(), np.empty(rows * fin, np.float32)
    _lib.call("rnn_linear_bwd", ctx.bind(), P(x), P(dyl), rows, fin, fout, P(w), P(dw_), P(dbias_), P(dxl))
    assert rel(dxl, dxl_ref) < TOL and rel(dw_, dw_ref) < TOL and rel(dbias_, dbias_ref) < TOL


def test_batchnorm_host_tier(api):
    _lib, ctx = api
    rng = O.Rng(5)
    n, c, hw = 6, 8, 25
    y = (rng.rand_vec(n * c * hw) * 2 + 1).astype(np.float32)
    g, b = (1 + 0.2 * rng.rand_vec(c)).astype(np.float32), rng.rand_vec(c)
    rm, rv = rng.rand_vec(c), (np.abs(rng.rand_vec(c)) + 0.5).astype(np.float32)
    rm_ref, rv_ref = rm.copy(), rv.copy()
    out_ref, xh_ref, is_ref = O.bn_fwd_train(y, n, c, hw, g, b, rm_ref, rv_ref, True)
    out, mean, inv = np.empty_like(y), np.empty(c, np.float32), np.empty(c, np.float32)
    rm_, rv_ = rm.copy(), rv.copy()
    _lib.call("rnn_batchnorm_fwd", ctx.bind(), P(y), n, c, hw, P(g), P(b), P(rm_), P(rv_), 0.1, 1e-5, 1, P(mean),
              P(inv), P(out))
    assert rel(out, out_ref) < TOL and rel(inv, is_ref) < TOL and rel(rm_, rm_ref) < TOL and rel(rv_, rv_ref) < TOL
    dy = rng.rand_vec(y.size)
    dy_eff = dy.copy()
    O.lib().orc_relu_back(dy_eff, out_ref, dy_eff.size)
    dg0, db0 = rng.rand_vec(c), rng.rand_vec(c)
    dg_ref, db_ref = dg0.copy(), db0.copy()
    dx_ref = O.bn_bwd(dy_eff, xh_ref, n, c, hw, g, is_ref, dg_ref, db_ref)
    dx, dg_, db_ = np.empty_like(y), dg0.copy(), db0.copy()
    _lib.call("rnn_batchnorm_bwd", ctx.bind(), P(dy), P(y), n, c, hw, P(g), P(mean), P(inv), P(out), P(dx), P(dg_),
              P(db_))
    assert rel(dx, dx_ref) < TOL and rel(dg_, dg_ref) < TOL and rel(db_, db_ref) < TOL


def test_optimisers_host_tier(api):
    _lib, ctx = api
    L = O.lib()
    rng = O.Rng(6)
    shapes = [(24, 40), (40, 24), (16, 16)]
    mats = [rng.rand_vec(r * c_) for r, c_ in shapes]
    want = [O.newton_schulz(m, r, c_, 3) for m, (r, c_) in zip(mats, shapes)]
    got = [m.copy() for m in mats]
    ptrs = (C.c_void_p * len(got))(*[a.ctypes.data for a in got])
    rows = (C.c_int * 3)(*[s[0] for s in shapes])
    cols = (C.c_int * 3)(*[s[1] for s in shapes])
    _lib.call("rnn_newton_schulz_batched", ctx.bind(), 3, C.cast(ptrs, C.c_void_p), C.cast(rows, C.c_void_p),
              C.cast(cols, C.c_void_p), 3)
    for g_, w_ in zip(got, want):
        assert rel(g_, w_) < TOL
    r, c_ = 24, 40
    v, g, m = rng.rand_vec(r * c_), rng.rand_vec(r * c_), rng.rand_vec(r * c_)
    vr, gr, mr = v.copy(), g.copy(), m.copy()
    L.orc_muon_step(vr, gr, mr, r, c_, 3, 0.02, 0.95, 0.1, 1)
    vd, gd, md = v.copy(), g.copy(), m.copy()
    _lib.call("rnn_muon_step", ctx.bind(), P(vd), P(gd), P(md), r, c_, 3, 0.02, 0.95, 0.1, 1)
    assert rel(vd, vr) < TOL and rel(md, mr) < TOL and not np.any(gd)
    k = 1000
    v, g, m, v2 = rng.rand_vec(k), rng.rand_vec(k), rng.rand_vec(k), np.abs(rng.rand_vec(k))
    ref = [a.copy() for a in (v, g, m, v2)]
    L.orc_adamw_step(*ref, k, 1e-3, 0.05, 1, 0.9, 0.999, 1e-8, 4)
    got = [a.copy() for a in (v, g, m, v2)]
    _lib.call("rnn_adamw_step", ctx.bind(), *[P(a) for a in got], k, 1e-3, 0.05, 1, 0.9, 0.999, 1e-8, 4)
    for g_, w_ in zip(got, ref):
        assert rel(g_, w_) < TOL
    v, g, m = rng.rand_vec(k), rng.rand_vec(k), rng.rand_vec(k)
    ref = [a.copy() for a in (v, g, m)]
    L.orc_sgd_step(*ref, k, 0.1, 0.9, 5e-4, 1)
    got = [a.copy() for a in (v, g, m)]
    _lib.call("rnn_sgd_nesterov", ctx.bind(), *[P(a) for a in got], k, 0.1, 0.9, 5e-4, 1)
    for g_, w_ in zip(got, ref):
        assert rel(g_, w_) < TOL
    g = (rng.rand_vec(k) * 3).astype(np.float32)
    gr = g.copy()
    norm_ref = L.orc_clip(gr, k, 1.0)
    gd, norm = g.copy(), np.zeros(1, np.float32)
    _lib.call("rnn_clip", ctx.bind(), P(gd), k, 1.0, P(norm))
    assert rel(gd, gr) < TOL and abs(norm[0] - norm_ref) <= 1e-5 * norm_ref
    e, v = rng.rand_vec(k), rng.rand_vec(k)
    er = e.copy()
    L.orc_ema_update(er, v, k, 0.9998, 5)
    ed = e.copy()
    _lib.call("rnn_ema_update", ctx.bind(), P(ed), P(v), k, 0.9998, 5)
    assert rel(ed, er) < TOL
