"""GPU parity of the attention, LayerNorm, Linear and optimiser entry points
against the CPU oracle (bar: 1e-4 relative Frobenius per output tensor), and
the reference's directional-derivative gradchecks (check.rs:19-40, tol 5e-3)
run with the GPU computing every loss and gradient."""
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


# ------------------------------------------------------------------ attention

ATTN = [
    # (n, h, dh, th, mh, self)  -- BASELINE config 3 (batch 128, 4 heads, dh 32, 8x8, cross 8x8 -> 16x16)
    (128, 4, 32, 8, 8, True),
    (128, 4, 32, 8, 16, False),
    (8, 4, 64, 8, 8, True),      # rustvit stage 3 (dim 256 / 4 heads)
    (8, 4, 64, 8, 16, False),    # rustvit cross attention over the 16x16 memory
    (3, 2, 4, 3, 3, True),       # check.rs:300 fixture
    (3, 2, 4, 3, 6, False),      # check.rs:327 fixture
    (4, 6, 64, 4, 4, True),      # rustvit stage 4 (dim 384 / 6 heads, 4x4)
    (3, 2, 6, 2, 2, True),       # check.rs:397 tiny network, stage 4 (dim 12 / 2 heads)
    (2, 3, 12, 4, 8, False),
    (2, 2, 24, 4, 4, True),
    (2, 2, 48, 4, 8, False),
]


def _geometry(rng, n, h, dh, th, mh, self_attn):
    c = h * dh
    tq, tk = th * th, mh * mh
    if self_attn:
        ab = (rng.rand_vec(n * tq * 3 * c) * np.float32(1 / np.sqrt(32))).astype(np.float32)
        return c, tq, tk, dict(q=ab, qstride=3 * c, qoff=0, kv=ab, kvstride=3 * c, koff=c, voff=2 * c)
    q = (rng.rand_vec(n * tq * c) * np.float32(1 / np.sqrt(32))).astype(np.float32)
    mem = (rng.rand_vec(n * tk * 2 * c) * np.float32(1 / np.sqrt(32))).astype(np.float32)
    return c, tq, tk, dict(q=q, qstride=c, qoff=0, kv=mem, kvstride=2 * c, koff=0, voff=c)


@pytest.mark.parametrize("n,h,dh,th,mh,self_attn", ATTN)
def test_attention_parity(ops, n, h, dh, th, mh, self_attn):
    rng = O.Rng(n * 1000 + dh + mh)
    c, tq, tk, g = _geometry(rng, n, h, dh, th, mh, self_attn)
    relidx, nrel = O.rel_index(th, th, mh, mh)
    gidx, gnrel = ops.rel_index(th, th, mh, mh)
    assert gnrel == nrel and np.array_equal(gidx, relidx)
    tau = np.full(h, np.float32(1.0 / np.sqrt(np.float32(dh))), np.float32)
    relv = rng.rand_vec(h * nrel)
    p_ref, o_ref = O.attn_fwd(n, h, dh, tq, tk, self_attn, relidx, nrel, g["q"], g["qstride"], g["qoff"], g["kv"],
                              g["kvstride"], g["koff"], g["voff"], tau, relv)
    qd = dev(g["q"])
    kvd = qd if self_attn else dev(g["kv"])
    p, o = ops.attn_forward(n, h, dh, th, th, mh, mh, self_attn, qd, g["qstride"], g["qoff"], kvd, g["kvstride"],
                            g["koff"], g["voff"], dev(tau), dev(relv))
    assert rel(host(p), p_ref) < TOL
    assert rel(host(o), o_ref) < TOL
    dout = rng.rand_vec(o_ref.size)
    dq_ref = np.zeros_like(g["q"])
    dkv_ref = dq_ref if self_attn else np.zeros_like(g["kv"])
    dtau_ref, drel_ref = np.zeros(h, np.float32), np.zeros(h * nrel, np.float32)
    O.attn_bwd(n, h, dh, tq, tk, relidx, nrel, g["q"], g["qstride"], g["qoff"], g["kv"], g["kvstride"], g["koff"],
               g["voff"], tau, p_ref, dout, dq_ref, dkv_ref, dtau_ref, drel_ref)
    dq = torch.zeros_like(qd)
    dkv = dq if self_attn else torch.zeros_like(kvd)
    dtau, drel = torch.zeros(h, device="cuda"), torch.zeros(h * nrel, device="cuda")
    ops.attn_backward(n, h, dh, th, th, mh, mh, qd, g["qstride"], g["qoff"], kvd, g["kvstride"], g["koff"], g["voff"],
                      dev(tau), p, dev(dout), dq, dkv, dtau, drel)
    assert rel(host(dq), dq_ref) < TOL
    if not self_attn:
        assert rel(host(dkv), dkv_ref) < TOL
    assert rel(host(dtau), dtau_ref) < TOL
    assert rel(host(drel), drel_ref) < TOL


def test_attention_backward_is_deterministic(ops):
    rng = O.Rng(5)
    n, h, dh, th, mh = 16, 4, 32, 8, 16
    c, tq, tk, g = _geometry(rng, n, h, dh, th, mh, False)
    _, nrel = ops.rel_index(th, th, mh, mh)
    tau, relv = dev(np.full(h, 0.17, np.float32)), dev(rng.rand_vec(h * nrel))
    qd, kvd = dev(g["q"]), dev(g["kv"])
    p, o = ops.attn_forward(n, h, dh, th, th, mh, mh, False, qd, c, 0, kvd, 2 * c, 0, c, tau, relv)
    dout = dev(rng.rand_vec(n * tq * c))
    outs = []
    for _ in range(2):
        dq, dkv = torch.zeros_like(qd), torch.zeros_like(kvd)
        dt, dr = torch.zeros(h, device="cuda"), torch.zeros(h * nrel, device="cuda")
        ops.attn_backward(n, h, dh, th, th, mh, mh, qd, c, 0, kvd, 2 * c, 0, c, tau, p, dout, dq, dkv, dt, dr)
        outs.append([host(t) for t in (dq, dkv, dt, dr)])
    for a, b in zip(*outs):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("n,h,dh,th,mh,self_attn", [(128, 4, 32, 8, 8, True), (128, 4, 32, 8, 16, False),
                                                    (16, 4, 64, 8, 8, True), (16, 4, 64, 8, 16, False)])
def test_attention_tensor_core_path_matches_simt(ops, monkeypatch, n, h, dh, th, mh, self_attn):
    """At 64 query tokens with head dim 32/64 the calls run on the tcgen05
    engine (3 forward launches: bias table, scores+softmax, P V; 6 backward:
    dS, dQ, dK/dV, the dtau reduction, the image sum of dS, the drel gather)
    and agree with the SIMT kernels (RNN_ATTN_SIMT=1)."""
    from rustnn_b200 import _lib

    L = _lib.lib()
    rng = O.Rng(700 + dh + mh)
    c, tq, tk, g = _geometry(rng, n, h, dh, th, mh, self_attn)
    _, nrel = ops.rel_index(th, th, mh, mh)
    tau = dev(np.full(h, np.float32(1.0 / np.sqrt(np.float32(dh))), np.float32))
    relv = dev(rng.rand_vec(h * nrel))
    qd = dev(g["q"])
    kvd = qd if self_attn else dev(g["kv"])
    dout = dev(rng.rand_vec(n * tq * c))
    res = {}
    for simt in (False, True):
        monkeypatch.setenv("RNN_ATTN_SIMT", "1" if simt else "0")
        l0 = L.rnn_launch_count()
        p, o = ops.attn_forward(n, h, dh, th, th, mh, mh, self_attn, qd, g["qstride"], g["qoff"], kvd,
                                g["kvstride"], g["koff"], g["voff"], tau, relv)
        l1 = L.rnn_launch_count()
        dq = torch.zeros_like(qd)
        dkv = dq if self_attn else torch.zeros_like(kvd)
        dt, dr = torch.zeros(h, device="cuda"), torch.zeros(h * nrel, device="cuda")
        ops.attn_backward(n, h, dh, th, th, mh, mh, qd, g["qstride"], g["qoff"], kvd, g["kvstride"], g["koff"],
                          g["voff"], tau, p, dout, dq, dkv, dt, dr)
        l2 = L.rnn_launch_count()
        if not simt:
            assert (l1 - l0, l2 - l1) == (3, 6), (l1 - l0, l2 - l1)
        res[simt] = [host(t) for t in (p, o, dq, dkv, dt, dr)]
    for name, a, b in zip(("p", "o", "dq", "dkv", "dtau", "drel"), res[False], res[True]):
        assert rel(a, b) < TOL, (name, rel(a, b))


def _dircheck(base, grad, eps, rng, lossf):
    base = np.asarray(base, np.float32)
    v = rng.rand_vec(base.size)
    lp = lossf((base + np.float32(eps) * v).astype(np.float32))
    lm = lossf((base - np.float32(eps) * v).astype(np.float32))
    num = (lp - lm) / (2.0 * eps)
    ana = float(np.dot(np.asarray(grad, np.float64), v.astype(np.float64)))
    return abs(num - ana) / (abs(num) + abs(ana) + 1e-6)


@pytest.mark.parametrize("self_attn", [True, False])
def test_attention_gradcheck_on_gpu(ops, self_attn):
    """check.rs:300-348 fixture, every loss and gradient on the GPU."""
    rng = O.Rng(90 + int(self_attn))
    n, h, dh, th = 3, 2, 4, 3
    mh = 3 if self_attn else 6
    c, tq, tk, g = _geometry(rng, n, h, dh, th, mh, self_attn)
    g = {k: (v * np.float32(np.sqrt(32)) if isinstance(v, np.ndarray) else v) for k, v in g.items()}
    _, nrel = ops.rel_index(th, th, mh, mh)
    tau = np.full(h, np.float32(0.5), np.float32)
    relv = rng.rand_vec(h * nrel)
    r = rng.rand_vec(n * tq * c)

    def loss(q, kv):
        qd = dev(q)
        kvd = qd if self_attn else dev(kv)
        _, o = ops.attn_forward(n, h, dh, th, th, mh, mh, self_attn, qd, g["qstride"], 0, kvd, g["kvstride"],
                                g["koff"], g["voff"], dev(tau), dev(relv))
        return float(np.dot(host(o).astype(np.float64), r))

    qd = dev(g["q"])
    kvd = qd if self_attn else dev(g["kv"])
    p, _ = ops.attn_forward(n, h, dh, th, th, mh, mh, self_attn, qd, g["qstride"], 0, kvd, g["kvstride"], g["koff"],
                            g["voff"], dev(tau), dev(relv))
    dq = torch.zeros_like(qd)
    dkv = dq if self_attn else torch.zeros_like(kvd)
    dt, dr = torch.zeros(h, device="cuda"), torch.zeros(h * nrel, device="cuda")
    ops.attn_backward(n, h, dh, th, th, mh, mh, qd, g["qstride"], 0, kvd, g["kvstride"], g["koff"], g["voff"],
                      dev(tau), p, dev(r), dq, dkv, dt, dr)
    if self_attn:
        assert _dircheck(g["q"], host(dq), 3e-4, rng, lambda v: loss(v, v)) < 5e-3
    else:
        assert _dircheck(g["q"], host(dq), 3e-4, rng, lambda v: loss(v, g["kv"])) < 5e-3
        assert _dircheck(g["kv"], host(dkv), 3e-4, rng, lambda v: loss(g["q"], v)) < 5e-3


# ------------------------------------------------------------------ LayerNorm / Linear


@pytest.mark.parametrize("rows,c", [(8192, 256), (2048, 384), (27, 8), (4096, 512), (100, 128), (1000, 384)])
def test_layernorm_parity(ops, rows, c):
    rng = O.Rng(rows + c)
    x = (rng.rand_vec(rows * c) * 3 + 1).astype(np.float32)
    gm = (1 + 0.2 * rng.rand_vec(c)).astype(np.float32)
    bt = rng.rand_vec(c)
    y_ref, xh_ref, is_ref = O.layernorm_fwd(x, rows, c, gm, bt)
    y, xh, isd = ops.layernorm_forward(dev(x), rows, c, dev(gm), dev(bt))
    assert rel(host(y), y_ref) < TOL and rel(host(xh), xh_ref) < TOL and rel(host(isd), is_ref) < 1e-6
    dy = rng.rand_vec(rows * c)
    # the gradients accumulate (+=) into what the buffers hold
    dg_ref, db_ref = rng.rand_vec(c), rng.rand_vec(c)
    dg, db = dev(dg_ref.copy()), dev(db_ref.copy())
    dx_ref = O.layernorm_bwd(dy, xh_ref, is_ref, rows, c, gm, dg_ref, db_ref)
    dx = ops.layernorm_backward(dev(dy), xh, isd, rows, c, dev(gm), dg, db)
    assert rel(host(dx), dx_ref) < TOL and rel(host(dg), dg_ref) < TOL and rel(host(db), db_ref) < TOL


@pytest.mark.parametrize("rows,fin,fout,bias", [(8192, 256, 768, True), (2048, 384, 1152, True), (27, 8, 12, False),
                                               (8192, 704 // 2, 256, True)])
def test_linear_parity(ops, rows, fin, fout, bias):
    rng = O.Rng(rows + fin + fout)
    x = rng.rand_vec(rows * fin)
    w = (rng.rand_vec(fout * fin) * np.float32(0.05)).astype(np.float32)
    b = rng.rand_vec(fout) if bias else None
    y_ref = O.linear_fwd(x, rows, fin, fout, w, b)
    y = ops.linear_forward(dev(x), rows, fin, fout, dev(w), dev(b) if bias else None)
    assert rel(host(y), y_ref) < TOL
    dy = rng.rand_vec(rows * fout)
    dw0 = rng.rand_vec(fout * fin)
    dw_ref = dw0.copy()
    db_ref = np.zeros(fout, np.float32) if bias else None
    dx_ref = O.linear_bwd(x, dy, rows, fin, fout, w, dw_ref, db_ref)
    dw = dev(dw0)
    db = torch.zeros(fout, device="cuda") if bias else None
    dx = ops.linear_backward(dev(x), dev(dy), rows, fin, fout, dev(w), dw, db)
    assert rel(host(dx), dx_ref) < TOL and rel(host(dw), dw_ref) < TOL
    if bias:
        assert rel(host(db), db_ref) < TOL


# ------------------------------------------------------------------ optim.rs


@pytest.mark.parametrize("rows,cols", [(1152, 384), (384, 1152), (256, 256), (12, 20), (20, 12), (100, 256)])
def test_newton_schulz_parity(ops, rows, cols):
    g = O.Rng(rows * 7 + cols).rand_vec(rows * cols)
    want = O.newton_schulz(g, rows, cols, 3)
    gd = dev(g)
    ops.newton_schulz_(gd, rows, cols, 3)
    assert rel(host(gd), want) < TOL


def test_muon_adamw_clip_ema_parity(ops):
    rng = O.Rng(12)
    rows, cols = 256, 768
    v, gr, m = rng.rand_vec(rows * cols), rng.rand_vec(rows * cols), rng.rand_vec(rows * cols)
    vr, gref, mr = v.copy(), gr.copy(), m.copy()
    O.lib().orc_muon_step(vr, gref, mr, rows, cols, 3, 6e-4, 0.95, 0.06, 1)
    vd, gd, md = dev(v), dev(gr), dev(m)
    ops.muon_step_(vd, gd, md, rows, cols, 3, 6e-4, 0.95, 0.06, True)
    assert rel(host(vd), vr) < TOL and rel(host(md), mr) < TOL and np.all(host(gd) == 0)
    n = 100003
    v, gr, m, v2 = rng.rand_vec(n), rng.rand_vec(n), rng.rand_vec(n), np.abs(rng.rand_vec(n))
    vr, gref, mr, v2r = v.copy(), gr.copy(), m.copy(), v2.copy()
    O.lib().orc_adamw_step(vr, gref, mr, v2r, n, 6e-4, 0.06, 1, 0.9, 0.999, 1e-8, 7)
    vd, gd, md, v2d = dev(v), dev(gr), dev(m), dev(v2)
    ops.adamw_step_(vd, gd, md, v2d, 6e-4, 0.06, True, 7)
    assert rel(host(vd), vr) < 1e-6 and rel(host(md), mr) < 1e-6 and rel(host(v2d), v2r) < 1e-6
    gq = rng.rand_vec(n)
    gref = gq.copy()
    nref = O.lib().orc_clip(gref, n, 1.0)
    gd = dev(gq)
    nd = ops.clip_(gd, 1.0)
    assert abs(float(host(nd)[0]) - nref) <= 1e-6 * nref and rel(host(gd), gref) < 1e-6
    e, w = rng.rand_vec(n), rng.rand_vec(n)
    er = e.copy()
    O.lib().orc_ema_update(er, w, n, 0.9998, 5)
    ed = dev(e)
    ops.ema_update_(ed, dev(w), 0.9998, 5)
    assert rel(host(ed), er) < 1e-6


def test_newton_schulz_grouped_rustvit_matrices(ops):
    """Newton-Schulz over all 39 Muon matrices of the default rustvit at once
    (rnn_newton_schulz_batched_dev: same-shape matrices batched into shared
    GEMM launches, tall ones transposed in and out) against one matrix at a
    time, and the small shapes against the oracle (optim.rs:124-145)."""
    import ctypes as C

    from rustnn_b200 import _lib
    from rustnn_b200.kernel_bench import RUSTVIT_2D

    rng = np.random.default_rng(8)
    mats = [rng.standard_normal(r * c).astype(np.float32) for r, c in RUSTVIT_2D]
    one = [dev(m) for m in mats]
    for t, (r, c) in zip(one, RUSTVIT_2D):
        ops.newton_schulz_(t, r, c, 3)
    grp = [dev(m) for m in mats]
    ptrs = (C.c_void_p * len(grp))(*[t.data_ptr() for t in grp])
    rows = (C.c_int * len(grp))(*[r for r, _ in RUSTVIT_2D])
    cols = (C.c_int * len(grp))(*[c for _, c in RUSTVIT_2D])
    ctx = ops.default_context()
    _lib.call("rnn_newton_schulz_batched_dev", ctx.bind(), len(grp), C.cast(ptrs, C.c_void_p),
              C.cast(rows, C.c_void_p), C.cast(cols, C.c_void_p), 3)
    torch.cuda.synchronize()
    for a, b, (r, c), m in zip(grp, one, RUSTVIT_2D, mats):
        assert rel(host(a), host(b)) < TOL, (r, c)
        if r * c <= 40000:
            assert rel(host(a), O.newton_schulz(m, r, c, 3)) < TOL, (r, c)
