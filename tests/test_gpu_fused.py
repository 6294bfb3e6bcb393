"""The rustvit fusions of csrc/fused.cu (README.md:549-552 of the reference
lists them as identified and not built): the residual add joined into
LayerNorm, LayerNorm writing the packed A operand of the next GEMM, and the
SiLU gate in the SwiGLU first GEMM's epilogue.  Each is checked against the
CPU oracle (bar 1e-4) and against the unfused device sequence, which it
reproduces bit for bit where both run the same summation order."""
import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-4


def rel(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.fixture(scope="module")
def ops():
    from rustnn_b200 import ops as _ops

    return _ops


# rows x c: rustvit stage 3 (8192 x 256 at batch 128), stage 4 (2048 x 384),
# a ragged last row tile, and the 512-wide memory LayerNorm
@pytest.mark.parametrize("rows,c,nres", [(8192, 256, 2), (2048, 384, 1), (300, 256, 0), (640, 512, 2)])
def test_layernorm_residual_and_packed_linear(ops, rows, c, nres):
    rng = O.Rng(rows + c + nres)
    x = rng.rand_vec(rows * c)
    res = [rng.rand_vec(rows * c) for _ in range(nres)]
    g = (np.float32(1) + np.float32(0.1) * rng.rand_vec(c)).astype(np.float32)
    b = (np.float32(0.1) * rng.rand_vec(c)).astype(np.float32)
    s_ref = x.copy()
    for r in res:
        s_ref = (s_ref + r).astype(np.float32)  # vit.rs:160-176, one rounding per add
    y_ref, xh_ref, is_ref = O.layernorm_fwd(s_ref, rows, c, g, b)
    rd = [dev(r) for r in res] + [None, None]
    s, y, xh, inv, img = ops.layernorm_res_forward(dev(x), rows, c, dev(g), dev(b), r1=rd[0], r2=rd[1], pack=True)
    if nres:
        assert np.array_equal(host(s), s_ref)
    assert rel(host(y), y_ref) < TOL and rel(host(xh), xh_ref) < TOL and rel(host(inv), is_ref) < TOL
    # the unfused device path gives the same bits
    y2, xh2, inv2 = ops.layernorm_forward(dev(s_ref), rows, c, dev(g), dev(b))
    assert np.array_equal(host(y), host(y2)) and np.array_equal(host(inv), host(inv2))
    fout = 384
    w = (np.float32(0.05) * rng.rand_vec(fout * c)).astype(np.float32)
    bias = rng.rand_vec(fout)
    out = ops.linear_forward_packed(img, rows, c, fout, dev(w), dev(bias))
    ref = O.linear_fwd(y_ref, rows, c, fout, w, bias)
    assert rel(host(out), ref) < TOL
    # the unfused GEMM may split K for small row counts (another summation order)
    assert rel(host(out), host(ops.linear_forward(y, rows, c, fout, dev(w), dev(bias)))) < 1e-5


@pytest.mark.parametrize("rows,c,h", [(8192, 256, 352), (2048, 384, 512), (200, 64, 48)])
def test_swiglu_gate_in_the_gemm_epilogue(ops, rows, c, h):
    rng = O.Rng(rows + h)
    x = rng.rand_vec(rows * c)
    wg = (np.float32(0.05) * rng.rand_vec(2 * h * c)).astype(np.float32)
    bg = (np.float32(0.1) * rng.rand_vec(2 * h)).astype(np.float32)
    ab_ref = O.linear_fwd(x, rows, c, 2 * h, wg, bg)
    u_ref = np.empty(rows * h, np.float32)
    O.lib().orc_swiglu_act_fwd(ab_ref, rows, h, u_ref)
    xd, wd, bd = dev(x), dev(wg), dev(bg)
    ab, u = ops.swiglu_fused_forward(xd, rows, c, h, wd, bd)
    assert rel(host(ab), ab_ref) < TOL and rel(host(u), u_ref) < TOL
    ab2 = ops.linear_forward(xd, rows, c, 2 * h, wd, bd)
    u2 = ops.swiglu_forward(ab2, rows, h)
    assert np.array_equal(host(ab), host(ab2)) and np.array_equal(host(u), host(u2))
    if c % 128 == 0:  # from the LayerNorm's packed image of x (identity affine)
        one, zero = dev(np.ones(c, np.float32)), dev(np.zeros(c, np.float32))
        _, y, _, _, img = ops.layernorm_res_forward(xd, rows, c, one, zero, pack=True)
        ab3, u3 = ops.swiglu_fused_forward(None, rows, c, h, wd, bd, a_image=img)
        ab4, u4 = ops.swiglu_fused_forward(y, rows, c, h, wd, bd)
        assert np.array_equal(host(ab3), host(ab4)) and np.array_equal(host(u3), host(u4))
