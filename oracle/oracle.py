"""ctypes bindings for the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle is a plain-C restatement of the reference's CPU arithmetic
(``rnn_oracle.c``).  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline legs of ``bench.py`` may import this module; the product package
``rustnn_b200`` never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librnn_oracle.so")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(dtype=np.uint64, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def build(force: bool = False) -> str:
    """Compile the oracle with the recipe in ``oracle/Makefile``."""
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < max(
        os.path.getmtime(os.path.join(HERE, f)) for f in ("rnn_oracle.c", "rnn_oracle_data.c", "rnn_oracle.h",
                                                          "Makefile")
    ):
        subprocess.check_call(["make", "-s", "-C", HERE])
    return LIB_PATH


class _Rng(C.Structure):
    _fields_ = [("s", C.c_uint64 * 4)]


_lib = None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    build()
    L = C.CDLL(LIB_PATH)
    V, I, F, Z, U64 = None, C.c_int, C.c_float, C.c_size_t, C.c_uint64
    P = C.c_void_p
    sig = {
        "orc_rng_new": (V, [C.POINTER(_Rng), U64]),
        "orc_rng_next_u64": (U64, [C.POINTER(_Rng)]),
        "orc_rng_uniform": (F, [C.POINTER(_Rng)]),
        "orc_rng_normal": (F, [C.POINTER(_Rng)]),
        "orc_rng_below": (U64, [C.POINTER(_Rng), U64]),
        "orc_rand_vec": (V, [_f32p, Z, C.POINTER(_Rng)]),
        "orc_matmul": (V, [I, I, I, _f32p, I, _f32p, I, _f32p, I]),
        "orc_matmul_dw": (V, [I, I, I, _f32p, _f32p, _f32p]),
        "orc_naive_matmul": (V, [I, I, I, _f32p, I, _f32p, I, _f32p]),
        "orc_conv2d_fwd": (V, [_f32p, I, I, I, I, _f32p, I, I, I, I, _f32p]),
        "orc_conv2d_dgrad": (V, [_f32p, I, I, I, I, _f32p, I, I, I, I, _f32p]),
        "orc_conv2d_wgrad": (V, [_f32p, _f32p, I, I, I, I, I, I, I, I, _f32p]),
        "orc_bn_fwd_train": (V, [_f32p, I, I, I, _f32p, _f32p, _f32p, _f32p, F, F, I, _f32p, _f32p]),
        "orc_bn_fwd_eval": (V, [_f32p, I, I, I, _f32p, _f32p, _f32p, _f32p, F, I]),
        "orc_bn_bwd": (V, [_f32p, _f32p, I, I, I, _f32p, _f32p, _f32p, _f32p, _f32p]),
        "orc_relu_back": (V, [_f32p, _f32p, Z]),
        "orc_add": (V, [_f32p, _f32p, Z]),
        "orc_add_relu": (V, [_f32p, _f32p, Z]),
        "orc_gap_fwd": (V, [_f32p, I, I, _f32p]),
        "orc_gap_bwd": (V, [_f32p, I, I, _f32p]),
        "orc_fc_fwd": (V, [_f32p, I, I, I, _f32p, _f32p, _f32p]),
        "orc_fc_bwd": (V, [_f32p, _f32p, I, I, I, _f32p, _f32p, _f32p, _f32p]),
        "orc_softmax_ce": (F, [_f32p, _u32p, I, I, F, _f32p, C.POINTER(C.c_int)]),
        "orc_sgd_step": (V, [_f32p, _f32p, _f32p, Z, F, F, F, I]),
        "orc_resnet_new": (P, [I, I, I, U64]),
        "orc_resnet_free": (V, [P]),
        "orc_resnet_num_params": (Z, [P]),
        "orc_resnet_num_tensors": (I, [P]),
        "orc_resnet_get_params": (V, [P, _f32p]),
        "orc_resnet_set_params": (V, [P, _f32p]),
        "orc_resnet_get_grads": (V, [P, _f32p]),
        "orc_resnet_get_moments": (V, [P, _f32p]),
        "orc_resnet_zero_grads": (V, [P]),
        "orc_resnet_num_buffers": (Z, [P]),
        "orc_resnet_get_buffers": (V, [P, _f32p]),
        "orc_resnet_param_info": (V, [P, _i64p, _i32p]),
        "orc_resnet_forward": (V, [P, _f32p, I, I, I, I, _f32p]),
        "orc_resnet_backward": (V, [P, _f32p]),
        "orc_resnet_step": (V, [P, F, F, F]),
        "orc_resnet_train_step": (F, [P, _f32p, _u32p, I, F, F, F, F, C.POINTER(C.c_int)]),
        "orc_resnet_flops": (U64, [P, I, I]),
        "orc_make_batch_eval": (V, [_u8p, _u8p, Z, I, I, _f32p, _u32p]),
        "orc_resnet_eval": (V, [P, _u8p, _u8p, I, I, _f32p]),
        "orc_make_batch_train": (V, [_u8p, _u8p, C.c_void_p, _u32p, I, I, F, I, F, I, U64, _f32p, _u32p,
                                     C.c_void_p]),
        "orc_mix_batch": (I, [_f32p, I, F, F, F, _u64p, _u32p, _f32p, _i32p]),
        "orc_data_set_cr_math": (V, [I]),
        "orc_rel_index": (I, [I, I, I, I, C.c_void_p]),
        "orc_attn_fwd": (V, [I, I, I, I, I, I, _u32p, I, _f32p, I, I, _f32p, I, I, I, _f32p, _f32p, _f32p, _f32p]),
        "orc_attn_bwd": (V, [I, I, I, I, I, _u32p, I, _f32p, I, I, _f32p, I, I, I, _f32p, _f32p, _f32p,
                             _f32p, _f32p, _f32p, _f32p]),
        "orc_layernorm_fwd": (V, [_f32p, I, I, _f32p, _f32p, F, _f32p, _f32p, _f32p]),
        "orc_layernorm_bwd": (V, [_f32p, _f32p, _f32p, I, I, _f32p, _f32p, _f32p, _f32p]),
        "orc_linear_fwd": (V, [_f32p, I, I, I, _f32p, C.c_void_p, _f32p]),
        "orc_linear_bwd": (V, [_f32p, _f32p, I, I, I, _f32p, _f32p, C.c_void_p, _f32p]),
        "orc_newton_schulz": (V, [_f32p, I, I, I]),
        "orc_muon_step": (V, [_f32p, _f32p, _f32p, I, I, I, F, F, F, I]),
        "orc_adamw_step": (V, [_f32p, _f32p, _f32p, _f32p, Z, F, F, I, F, F, F, I]),
        "orc_clip": (F, [_f32p, Z, F]),
        "orc_ema_update": (V, [_f32p, _f32p, Z, F, I]),
        "orc_layerscale_fwd": (V, [_f32p, I, I, _f32p, _f32p]),
        "orc_layerscale_bwd": (V, [_f32p, _f32p, I, I, _f32p, _f32p, _f32p]),
        "orc_swiglu_act_fwd": (V, [_f32p, I, I, _f32p]),
        "orc_swiglu_act_bwd": (V, [_f32p, _f32p, I, I, _f32p]),
        "orc_dwconv3_fwd": (V, [_f32p, I, I, I, I, _f32p, _f32p, _f32p]),
        "orc_dwconv3_bwd": (V, [_f32p, _f32p, I, I, I, I, _f32p, _f32p, _f32p, _f32p]),
        "orc_seqpool_fwd": (V, [_f32p, I, I, I, _f32p, _f32p, _f32p]),
        "orc_seqpool_bwd": (V, [_f32p, _f32p, _f32p, I, I, I, _f32p, _f32p, _f32p]),
        "orc_droppath_mask": (V, [I, F, U64, _f32p]),
        "orc_token_merge_fwd": (V, [_f32p, I, I, I, _f32p]),
        "orc_token_merge_bwd": (V, [_f32p, I, I, I, _f32p]),
        "orc_tok_from_nchw": (V, [_f32p, I, I, I, _f32p]),
        "orc_tok_to_nchw": (V, [_f32p, I, I, I, _f32p]),
        "orc_taxo_fwd": (V, [_f32p, _f32p, I, I, I, _u32p]),
        "orc_taxo_bwd": (V, [_f32p, _f32p, I, I, I, _u32p, _f32p]),
        "orc_ce_soft": (F, [_f32p, _f32p, _u32p, I, I, F, _f32p, C.POINTER(C.c_int)]),
        "orc_kl_distill": (F, [_f32p, _f32p, I, I, F, F, _f32p]),
        "orc_hint_mse": (F, [_f32p, _f32p, I, I, F, _f32p]),
        "orc_trunc_normal": (V, [C.POINTER(_Rng), _f32p, Z, F]),
        "orc_kaiming": (V, [C.POINTER(_Rng), _f32p, Z, I]),
        "orc_set_threads": (V, [I]),
        "orc_get_threads": (I, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------- rng.rs


class Rng:
    """rng.rs Rng: SplitMix64-seeded xoshiro256++ (bit exact)."""

    def __init__(self, seed: int):
        self._s = _Rng()
        lib().orc_rng_new(C.byref(self._s), C.c_uint64(seed & (2**64 - 1)))

    def next_u64(self) -> int:
        return lib().orc_rng_next_u64(C.byref(self._s))

    def uniform(self) -> float:
        return lib().orc_rng_uniform(C.byref(self._s))

    def normal(self) -> float:
        return lib().orc_rng_normal(C.byref(self._s))

    def below(self, n: int) -> int:
        return lib().orc_rng_below(C.byref(self._s), n)

    def rand_vec(self, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        lib().orc_rand_vec(out, n, C.byref(self._s))
        return out

    def state(self) -> np.ndarray:
        """The xoshiro256++ state words (rng.rs:3-5)."""
        return np.array(list(self._s.s), np.uint64)

    def set_state(self, st) -> None:
        for i in range(4):
            self._s.s[i] = int(st[i])


# ---------------------------------------------------------------- gemm.rs


def matmul(m, n, k, a, at, b, bt, c=None, acc=False):
    if c is None:
        c = np.zeros(m * n, np.float32)
    lib().orc_matmul(m, n, k, _f32(a).ravel(), int(at), _f32(b).ravel(), int(bt), c, int(acc))
    return c


def matmul_dw(m, n, k, a, b, c):
    lib().orc_matmul_dw(m, n, k, _f32(a).ravel(), _f32(b).ravel(), c)
    return c


def naive_matmul(m, n, k, a, at, b, bt):
    c = np.zeros(m * n, np.float32)
    lib().orc_naive_matmul(m, n, k, _f32(a).ravel(), int(at), _f32(b).ravel(), int(bt), c)
    return c


# ---------------------------------------------------------------- conv


def out_dim(h, k, stride, pad):
    return (h + 2 * pad - k) // stride + 1


def conv2d_fwd(x, n, cin, h, w, wt, cout, k, stride, pad):
    oh, ow = out_dim(h, k, stride, pad), out_dim(w, k, stride, pad)
    y = np.empty(n * cout * oh * ow, np.float32)
    lib().orc_conv2d_fwd(_f32(x).ravel(), n, cin, h, w, _f32(wt).ravel(), cout, k, stride, pad, y)
    return y


def conv2d_dgrad(dy, n, cin, h, w, wt, cout, k, stride, pad):
    dx = np.empty(n * cin * h * w, np.float32)
    lib().orc_conv2d_dgrad(_f32(dy).ravel(), n, cin, h, w, _f32(wt).ravel(), cout, k, stride, pad, dx)
    return dx


def conv2d_wgrad(x, dy, n, cin, h, w, cout, k, stride, pad, dw=None):
    if dw is None:
        dw = np.zeros(cout * cin * k * k, np.float32)
    lib().orc_conv2d_wgrad(_f32(x).ravel(), _f32(dy).ravel(), n, cin, h, w, cout, k, stride, pad, dw)
    return dw


# ---------------------------------------------------------------- BN / glue


def bn_fwd_train(y, n, c, hw, gamma, beta, rmean, rvar, relu, mom=0.1, eps=1e-5):
    """In place on a copy of y; returns (out, xhat, invstd); rmean/rvar updated."""
    out = _f32(y).ravel().copy()
    xhat = np.empty_like(out)
    invstd = np.empty(c, np.float32)
    lib().orc_bn_fwd_train(out, n, c, hw, _f32(gamma), _f32(beta), rmean, rvar, mom, eps, int(relu), xhat, invstd)
    return out, xhat, invstd


def bn_fwd_eval(y, n, c, hw, gamma, beta, rmean, rvar, relu, eps=1e-5):
    """BatchNorm2d with running statistics (nn.rs:358-369); returns a new array."""
    out = _f32(y).ravel().copy()
    lib().orc_bn_fwd_eval(out, n, c, hw, _f32(gamma), _f32(beta), _f32(rmean), _f32(rvar), eps, int(relu))
    return out


def make_batch_train(images, labels, coarse, idx, pad=4, ra_mag=0.0, ra_n=2, erase=0.0, erase_side=8, seed=0):
    """data::make_batch_train (data.rs:384-412): (x [bs*3072] f32, labels u32,
    coarse u32 or None)."""
    images = np.ascontiguousarray(images, dtype=np.uint8).ravel()
    labels = np.ascontiguousarray(labels, dtype=np.uint8).ravel()
    idx = np.ascontiguousarray(idx, dtype=np.uint32).ravel()
    bs = len(idx)
    x = np.empty(bs * 3 * 32 * 32, np.float32)
    lab = np.empty(bs, np.uint32)
    cz = None if coarse is None else np.ascontiguousarray(coarse, dtype=np.uint8).ravel()
    cout = None if coarse is None else np.empty(bs, np.uint32)
    lib().orc_make_batch_train(images, labels, None if cz is None else cz.ctypes.data, idx, bs, pad, ra_mag, ra_n,
                               erase, erase_side, seed & (2**64 - 1), x, lab,
                               None if cout is None else cout.ctypes.data)
    return x, lab, cout


class cr_math:
    """Within this context the data pipeline's logf / cosf / sinf are
    correctly rounded (the device's convention) instead of the C library's."""

    def __enter__(self):
        lib().orc_data_set_cr_math(1)

    def __exit__(self, *a):
        lib().orc_data_set_cr_math(0)


def mix_batch(x, bs, alpha_mix, alpha_cut, sw, state):
    """data::mix_batch (data.rs:467-491) in place on x; state (uint64[4]) is the
    caller's generator, advanced.  Returns (kind, perm, lam, rect)."""
    perm = np.empty(bs, np.uint32)
    lam = np.empty(bs, np.float32)
    rect = np.zeros(4, np.int32)
    kind = lib().orc_mix_batch(x, bs, alpha_mix, alpha_cut, sw, state, perm, lam, rect)
    return kind, perm, lam, rect


def make_batch_eval(images, labels, start, bs, flip):
    """data::make_batch_eval (data.rs:494-512): (x [bs*3072] f32, labels u32)."""
    images = np.ascontiguousarray(images, dtype=np.uint8).ravel()
    labels = np.ascontiguousarray(labels, dtype=np.uint8).ravel()
    x = np.empty(bs * 3 * 32 * 32, np.float32)
    lab = np.empty(bs, np.uint32)
    lib().orc_make_batch_eval(images, labels, start, bs, int(flip), x, lab)
    return x, lab


def bn_bwd(dy, xhat, n, c, hw, gamma, invstd, dgamma, dbeta):
    dx = np.empty(n * c * hw, np.float32)
    lib().orc_bn_bwd(_f32(dy).ravel(), _f32(xhat).ravel(), n, c, hw, _f32(gamma), _f32(invstd), dx, dgamma, dbeta)
    return dx


def softmax_ce(logits, labels, nclass, smooth):
    logits = _f32(logits).ravel()
    labels = np.ascontiguousarray(labels, dtype=np.uint32)
    d = np.empty_like(logits)
    corr = C.c_int(0)
    loss = lib().orc_softmax_ce(logits, labels, len(labels), nclass, smooth, d, C.byref(corr))
    return loss, d, corr.value


# ---------------------------------------------------------------- model.rs


class ResNet:
    """model.rs ResNet restated in C."""

    def __init__(self, depth_n, width, nclass, seed):
        self.h = lib().orc_resnet_new(depth_n, width, nclass, seed)
        self.nclass = nclass
        self.width = width
        self.depth_n = depth_n

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.orc_resnet_free(self.h)
            self.h = None

    def num_params(self):
        return lib().orc_resnet_num_params(self.h)

    def num_tensors(self):
        return lib().orc_resnet_num_tensors(self.h)

    def param_info(self):
        k = self.num_tensors()
        sizes = np.zeros(k, np.int64)
        decay = np.zeros(k, np.int32)
        lib().orc_resnet_param_info(self.h, sizes, decay)
        return sizes, decay

    def params(self):
        out = np.empty(self.num_params(), np.float32)
        lib().orc_resnet_get_params(self.h, out)
        return out

    def set_params(self, v):
        lib().orc_resnet_set_params(self.h, _f32(v).ravel())

    def grads(self):
        out = np.empty(self.num_params(), np.float32)
        lib().orc_resnet_get_grads(self.h, out)
        return out

    def moments(self):
        out = np.empty(self.num_params(), np.float32)
        lib().orc_resnet_get_moments(self.h, out)
        return out

    def buffers(self):
        out = np.empty(lib().orc_resnet_num_buffers(self.h), np.float32)
        lib().orc_resnet_get_buffers(self.h, out)
        return out

    def zero_grads(self):
        lib().orc_resnet_zero_grads(self.h)

    def forward(self, x, n, hw=32, train=True):
        logits = np.empty(n * self.nclass, np.float32)
        lib().orc_resnet_forward(self.h, _f32(x).ravel(), n, hw, hw, int(train), logits)
        return logits

    def backward(self, dlogits):
        lib().orc_resnet_backward(self.h, _f32(dlogits).ravel())

    def step(self, lr, mom, wd):
        lib().orc_resnet_step(self.h, lr, mom, wd)

    def train_step(self, x, labels, smooth=0.1, lr=0.2, mom=0.9, wd=5e-4):
        labels = np.ascontiguousarray(labels, dtype=np.uint32)
        corr = C.c_int(0)
        loss = lib().orc_resnet_train_step(self.h, _f32(x).ravel(), labels, len(labels), smooth, lr, mom, wd, C.byref(corr))
        return loss, corr.value

    def flops(self, h=32, w=32):
        return lib().orc_resnet_flops(self.h, h, w)

    def eval(self, images, labels, batch):
        """eval::resnet (eval.rs:41-43) over a u8 CHW dataset: (loss, accuracy)."""
        assert batch > 0
        images = np.ascontiguousarray(images, dtype=np.uint8).ravel()
        labels = np.ascontiguousarray(labels, dtype=np.uint8).ravel()
        out = np.empty(2, np.float32)
        lib().orc_resnet_eval(self.h, images, labels, len(labels), batch, out)
        return float(out[0]), float(out[1])


# ---------------------------------------------------------------- attn.rs


def rel_index(th, tw, mh, mw):
    """(relidx [th*tw*mh*mw] u32, nrel), attn.rs:53-72."""
    idx = np.empty(th * tw * mh * mw, np.uint32)
    nrel = lib().orc_rel_index(th, tw, mh, mw, C.c_void_p(idx.ctypes.data))
    return idx, nrel


def attn_fwd(n, h, dh, tq, tk, mask_diag, relidx, nrel, q, qstride, qoff, kv, kvstride, koff, voff, tau, rel):
    p = np.empty(n * h * tq * tk, np.float32)
    o = np.empty(n * tq * h * dh, np.float32)
    lib().orc_attn_fwd(n, h, dh, tq, tk, int(mask_diag), np.ascontiguousarray(relidx, np.uint32), nrel,
                       _f32(q).ravel(), qstride, qoff, _f32(kv).ravel(), kvstride, koff, voff, _f32(tau), _f32(rel),
                       p, o)
    return p, o


def attn_bwd(n, h, dh, tq, tk, relidx, nrel, q, qstride, qoff, kv, kvstride, koff, voff, tau, p, dout,
             dq, dkv, dtau, drel):
    """dq, dkv, dtau, drel are float32 arrays that accumulate."""
    lib().orc_attn_bwd(n, h, dh, tq, tk, np.ascontiguousarray(relidx, np.uint32), nrel, _f32(q).ravel(), qstride,
                       qoff, _f32(kv).ravel(), kvstride, koff, voff, _f32(tau), _f32(p).ravel(), _f32(dout).ravel(),
                       dq, dkv, dtau, drel)


def layernorm_fwd(x, rows, c, g, b, eps=1e-5):
    y = np.empty(rows * c, np.float32)
    xhat = np.empty(rows * c, np.float32)
    invstd = np.empty(rows, np.float32)
    lib().orc_layernorm_fwd(_f32(x).ravel(), rows, c, _f32(g), _f32(b), eps, y, xhat, invstd)
    return y, xhat, invstd


def layernorm_bwd(dy, xhat, invstd, rows, c, g, dg, db):
    dx = np.empty(rows * c, np.float32)
    lib().orc_layernorm_bwd(_f32(dy).ravel(), _f32(xhat).ravel(), _f32(invstd), rows, c, _f32(g), dx, dg, db)
    return dx


def _opt(b):
    return None if b is None else C.c_void_p(b.ctypes.data)


def linear_fwd(x, rows, fin, fout, w, b=None):
    y = np.empty(rows * fout, np.float32)
    bb = None if b is None else _f32(b)
    lib().orc_linear_fwd(_f32(x).ravel(), rows, fin, fout, _f32(w).ravel(), _opt(bb), y)
    return y


def linear_bwd(x, dy, rows, fin, fout, w, dw, db=None):
    dx = np.empty(rows * fin, np.float32)
    lib().orc_linear_bwd(_f32(x).ravel(), _f32(dy).ravel(), rows, fin, fout, _f32(w).ravel(), dw, _opt(db), dx)
    return dx


def newton_schulz(g, rows, cols, steps):
    out = _f32(g).ravel().copy()
    lib().orc_newton_schulz(out, rows, cols, steps)
    return out


def set_threads(n: int):
    lib().orc_set_threads(n)


def get_threads() -> int:
    return lib().orc_get_threads()
