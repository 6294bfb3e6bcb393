"""Operator-level API over the C ABI, mirroring the reference's Rust calls.

Tensors are torch CUDA float32 tensors (torch is used only for device memory
and streams).  Every op runs on the current torch stream, through a context
bound to it, and raises ``RnnError`` on any failure; there is no CPU path.

Reference interfaces mirrored here:
  matmul      gemm.rs:434-444 (C (+)= op(A) op(B))
  gemm_small  gemm.rs:500-512 (same contract; no packing scratch needed)
  matmul_dw   gemm.rs:555     (C += A^T B)
  conv2d_*    nn.rs:166/193/230 (Conv2d forward / backward_w / backward)
  batchnorm_* nn.rs:290-427
  softmax_ce  nn.rs:615-637
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import CTX, RnnError, call, check, lib

__all__ = [
    "Context", "default_context", "matmul", "gemm_small", "matmul_dw", "conv2d_forward", "conv2d_dgrad",
    "conv2d_wgrad", "batchnorm_forward", "batchnorm_eval", "batchnorm_backward", "relu_back_", "add_",
    "add_relu_", "gap_forward", "gap_backward", "softmax_ce", "sgd_nesterov_", "out_dim", "RnnError",
    "rel_index", "attn_forward", "attn_backward", "layernorm_forward", "layernorm_backward", "linear_forward",
    "linear_backward", "layernorm_res_forward", "linear_forward_packed", "swiglu_fused_forward", "newton_schulz_", "muon_step_", "adamw_step_", "clip_", "ema_update_",
    "layerscale_forward", "layerscale_backward", "swiglu_forward", "swiglu_backward", "dwconv3_forward",
    "dwconv3_backward", "seqpool_forward", "seqpool_backward", "droppath_forward_", "droppath_backward_",
    "token_merge", "tok_layout", "taxo_forward_", "taxo_backward", "ce_soft", "kl_distill", "hint_mse",
]


class Context:
    """An rnn_ctx on one device (its stream follows torch's current stream)."""

    def __init__(self, device: int = 0):
        if not torch.cuda.is_available():
            raise RnnError("rustnn_b200 needs a CUDA device (sm_100a); there is no CPU fallback")
        self.device = device
        h = CTX()
        with torch.cuda.device(device):
            check(lib().rnn_ctx_create(C.byref(h), device), "rnn_ctx_create")
        self.h = h
        self._stream = None

    def bind(self):
        s = torch.cuda.current_stream(self.device).cuda_stream
        if s != self._stream:
            call("rnn_ctx_set_stream", self.h, C.c_void_p(s))
            self._stream = s
        return self.h

    def synchronize(self):
        call("rnn_ctx_synchronize", self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().rnn_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_ctx = {}


def default_context(device=None) -> Context:
    if device is None:
        device = torch.cuda.current_device()
    if device not in _ctx:
        _ctx[device] = Context(device)
    return _ctx[device]


def _ptr(t: torch.Tensor, name: str):
    if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.float32 and t.dtype != torch.int32:
        raise RnnError(f"{name}: expected a CUDA float32 tensor")
    if not t.is_contiguous():
        raise RnnError(f"{name}: tensor must be contiguous")
    return C.c_void_p(t.data_ptr())


def _ctx_of(t: torch.Tensor, ctx):
    c = ctx or default_context(t.device.index)
    return c.bind()


def out_dim(h: int, k: int, stride: int, pad: int) -> int:
    """nn.rs:148-150."""
    return (h + 2 * pad - k) // stride + 1


# ---------------------------------------------------------------- gemm.rs


def matmul(m, n, k, a, at, b, bt, c, acc=False, ctx=None):
    """C[m x n] (+)= op(A) op(B) (gemm.rs:434)."""
    call("rnn_gemm_dev", _ctx_of(c, ctx), m, n, k, _ptr(a, "a"), int(bool(at)), _ptr(b, "b"), int(bool(bt)),
         _ptr(c, "c"), int(bool(acc)))
    return c


gemm_small = matmul  # gemm.rs:500: same contract; batching happens inside the engine


def matmul_dw(m, n, k, a, b, c, ctx=None):
    """C[m x n] += A^T B, A [k x m], B [k x n] (gemm.rs:555)."""
    call("rnn_gemm_dw_dev", _ctx_of(c, ctx), m, n, k, _ptr(a, "a"), _ptr(b, "b"), _ptr(c, "c"))
    return c


# ---------------------------------------------------------------- conv


def conv2d_forward(x, w, n, cin, h, wd, cout, k, stride, pad, y=None, acc=False, ctx=None):
    oh, ow = out_dim(h, k, stride, pad), out_dim(wd, k, stride, pad)
    if y is None:
        y = torch.empty(n * cout * oh * ow, device=x.device, dtype=torch.float32)
    call("rnn_conv2d_fwd_dev", _ctx_of(x, ctx), _ptr(x, "x"), n, cin, h, wd, _ptr(w, "w"), cout, k, stride, pad,
         _ptr(y, "y"), int(bool(acc)))
    return y


def conv2d_dgrad(dy, w, n, cin, h, wd, cout, k, stride, pad, dx=None, acc=False, ctx=None):
    if dx is None:
        dx = torch.empty(n * cin * h * wd, device=dy.device, dtype=torch.float32)
    call("rnn_conv2d_dgrad_dev", _ctx_of(dy, ctx), _ptr(dy, "dy"), n, cin, h, wd, _ptr(w, "w"), cout, k, stride,
         pad, _ptr(dx, "dx"), int(bool(acc)))
    return dx


def conv2d_wgrad(x, dy, n, cin, h, wd, cout, k, stride, pad, dw=None, ctx=None):
    """dw += dy im2col(x)^T (accumulates, like nn.rs:226)."""
    if dw is None:
        dw = torch.zeros(cout * cin * k * k, device=x.device, dtype=torch.float32)
    call("rnn_conv2d_wgrad_dev", _ctx_of(x, ctx), _ptr(x, "x"), _ptr(dy, "dy"), n, cin, h, wd, cout, k, stride,
         pad, _ptr(dw, "dw"))
    return dw


# ---------------------------------------------------------------- BatchNorm


def batchnorm_forward(y, n, c, hw, gamma, beta, rmean, rvar, relu, mom=0.1, eps=1e-5, out=None, ctx=None):
    """Returns (out, mean, invstd); rmean/rvar updated in place."""
    if out is None:
        out = torch.empty_like(y)
    mean = torch.empty(c, device=y.device, dtype=torch.float32)
    invstd = torch.empty(c, device=y.device, dtype=torch.float32)
    call("rnn_batchnorm_fwd_dev", _ctx_of(y, ctx), _ptr(y, "y"), n, c, hw, _ptr(gamma, "gamma"),
         _ptr(beta, "beta"), _ptr(rmean, "rmean"), _ptr(rvar, "rvar"), mom, eps, int(bool(relu)), _ptr(mean, "mean"),
         _ptr(invstd, "invstd"), _ptr(out, "out"))
    return out, mean, invstd


def batchnorm_eval(y, n, c, hw, gamma, beta, rmean, rvar, relu, eps=1e-5, out=None, ctx=None):
    if out is None:
        out = torch.empty_like(y)
    call("rnn_batchnorm_eval_dev", _ctx_of(y, ctx), _ptr(y, "y"), n, c, hw, _ptr(gamma, "gamma"), _ptr(beta, "beta"),
         _ptr(rmean, "rmean"), _ptr(rvar, "rvar"), eps, int(bool(relu)), _ptr(out, "out"))
    return out


def batchnorm_backward(dy, y, n, c, hw, gamma, mean, invstd, dgamma, dbeta, relu_out=None, dx=None, ctx=None):
    if dx is None:
        dx = torch.empty_like(dy)
    ro = _ptr(relu_out, "relu_out") if relu_out is not None else None
    call("rnn_batchnorm_bwd_dev", _ctx_of(dy, ctx), _ptr(dy, "dy"), _ptr(y, "y"), n, c, hw, _ptr(gamma, "gamma"),
         _ptr(mean, "mean"), _ptr(invstd, "invstd"), ro, _ptr(dx, "dx"), _ptr(dgamma, "dgamma"), _ptr(dbeta, "dbeta"))
    return dx


# ---------------------------------------------------------------- glue


def relu_back_(d, y, ctx=None):
    call("rnn_relu_back_dev", _ctx_of(d, ctx), _ptr(d, "d"), _ptr(y, "y"), d.numel())
    return d


def add_(a, b, ctx=None):
    call("rnn_add_dev", _ctx_of(a, ctx), _ptr(a, "a"), _ptr(b, "b"), a.numel())
    return a


def add_relu_(a, b, ctx=None):
    call("rnn_add_relu_dev", _ctx_of(a, ctx), _ptr(a, "a"), _ptr(b, "b"), a.numel())
    return a


def gap_forward(x, nc, hw, ctx=None):
    y = torch.empty(nc, device=x.device, dtype=torch.float32)
    call("rnn_gap_fwd_dev", _ctx_of(x, ctx), _ptr(x, "x"), nc, hw, _ptr(y, "y"))
    return y


def gap_backward(dy, nc, hw, ctx=None):
    dx = torch.empty(nc * hw, device=dy.device, dtype=torch.float32)
    call("rnn_gap_bwd_dev", _ctx_of(dy, ctx), _ptr(dy, "dy"), nc, hw, _ptr(dx, "dx"))
    return dx


def softmax_ce(logits, labels, nclass, smooth, ctx=None):
    """Returns (loss tensor[1], dlogits, correct tensor[1]) (nn.rs:615-637)."""
    n = labels.numel()
    lab = labels.to(torch.int32).contiguous()
    d = torch.empty_like(logits)
    loss = torch.empty(1, device=logits.device, dtype=torch.float32)
    corr = torch.empty(1, device=logits.device, dtype=torch.int32)
    call("rnn_softmax_ce_dev", _ctx_of(logits, ctx), _ptr(logits, "logits"), _ptr(lab, "labels"), n, nclass, smooth,
         _ptr(d, "dlogits"), _ptr(loss, "loss"), _ptr(corr, "correct"))
    return loss, d, corr


def sgd_nesterov_(v, g, m, lr, mom, wd, decay, ctx=None):
    """Param::step (nn.rs:102-110); g is zeroed."""
    call("rnn_sgd_nesterov_dev", _ctx_of(v, ctx), _ptr(v, "v"), _ptr(g, "g"), _ptr(m, "m"), v.numel(), lr, mom, wd,
         int(bool(decay)))
    return v


# ---------------------------------------------------------------- attn.rs


def _opt_ptr(t, name):
    return None if t is None else _ptr(t, name)


def rel_index(th, tw, mh, mw):
    """(relidx numpy u32 [th*tw*mh*mw], nrel) -- attn.rs:53-72."""
    import numpy as np

    idx = np.empty(th * tw * mh * mw, np.uint32)
    nrel = C.c_int()
    call("rnn_rel_index", th, tw, mh, mw, C.c_void_p(idx.ctypes.data), C.byref(nrel))
    return idx, nrel.value


def attn_forward(n, h, dh, th, tw, mh, mw, mask_diag, q, qstride, qoff, kv, kvstride, koff, voff, tau, rel,
                 ctx=None):
    """Core::forward (attn.rs:148): returns (p [n,h,tq,tk], o [n,tq,h*dh])."""
    tq, tk = th * tw, mh * mw
    p = torch.empty(n * h * tq * tk, device=q.device, dtype=torch.float32)
    o = torch.empty(n * tq * h * dh, device=q.device, dtype=torch.float32)
    call("rnn_attn_fwd_dev", _ctx_of(q, ctx), n, h, dh, th, tw, mh, mw, int(bool(mask_diag)), _ptr(q, "q"), qstride,
         qoff, _ptr(kv, "kv"), kvstride, koff, voff, _ptr(tau, "tau"), _ptr(rel, "rel"), _ptr(p, "p"), _ptr(o, "o"))
    return p, o


def attn_backward(n, h, dh, th, tw, mh, mw, q, qstride, qoff, kv, kvstride, koff, voff, tau, p, dout, dq, dkv,
                  dtau, drel, ctx=None):
    """Core::backward (attn.rs:226): dq, dkv, dtau, drel accumulate."""
    call("rnn_attn_bwd_dev", _ctx_of(q, ctx), n, h, dh, th, tw, mh, mw, _ptr(q, "q"), qstride, qoff, _ptr(kv, "kv"),
         kvstride, koff, voff, _ptr(tau, "tau"), _ptr(p, "p"), _ptr(dout, "dout"), _ptr(dq, "dq"), _ptr(dkv, "dkv"),
         _ptr(dtau, "dtau"), _ptr(drel, "drel"))


# ---------------------------------------------------------------- norm.rs / linear.rs


def layernorm_forward(x, rows, c, gamma, beta, eps=1e-5, ctx=None):
    """LayerNorm::forward (norm.rs:38): returns (y, xhat, invstd)."""
    y = torch.empty_like(x)
    xhat = torch.empty_like(x)
    invstd = torch.empty(rows, device=x.device, dtype=torch.float32)
    call("rnn_layernorm_fwd_dev", _ctx_of(x, ctx), _ptr(x, "x"), rows, c, _ptr(gamma, "gamma"), _ptr(beta, "beta"),
         eps, _ptr(y, "y"), _ptr(xhat, "xhat"), _ptr(invstd, "invstd"))
    return y, xhat, invstd


def layernorm_backward(dy, xhat, invstd, rows, c, gamma, dgamma, dbeta, ctx=None):
    dx = torch.empty_like(dy)
    call("rnn_layernorm_bwd_dev", _ctx_of(dy, ctx), _ptr(dy, "dy"), _ptr(xhat, "xhat"), _ptr(invstd, "invstd"), rows,
         c, _ptr(gamma, "gamma"), _ptr(dx, "dx"), _ptr(dgamma, "dgamma"), _ptr(dbeta, "dbeta"))
    return dx


def linear_forward(x, rows, fin, fout, w, b=None, ctx=None):
    """Linear::forward (linear.rs:44): y = x W^T + b."""
    y = torch.empty(rows * fout, device=x.device, dtype=torch.float32)
    call("rnn_linear_fwd_dev", _ctx_of(x, ctx), _ptr(x, "x"), rows, fin, fout, _ptr(w, "w"), _opt_ptr(b, "b"),
         _ptr(y, "y"))
    return y


def layernorm_res_forward(x, rows, c, gamma, beta, r1=None, r2=None, eps=1e-5, pack=False, ctx=None):
    """s = x (+ r1) (+ r2) and LayerNorm::forward of s in one pass
    (vit.rs:160-176 + norm.rs:38); returns (s, y, xhat, invstd, a_image),
    a_image (the packed A operand of the next GEMM) only when pack."""
    s = torch.empty_like(x) if r1 is not None else None
    y, xhat = torch.empty_like(x), torch.empty_like(x)
    invstd = torch.empty(rows, device=x.device, dtype=torch.float32)
    img = torch.empty(((rows + 127) // 128) * 128 * c * 2, device=x.device, dtype=torch.float32) if pack else None
    call("rnn_layernorm_res_fwd_dev", _ctx_of(x, ctx), _ptr(x, "x"), _opt_ptr(r1, "r1"), _opt_ptr(r2, "r2"), rows, c,
         _ptr(gamma, "gamma"), _ptr(beta, "beta"), eps, _opt_ptr(s, "sum"), _ptr(y, "y"), _ptr(xhat, "xhat"),
         _ptr(invstd, "invstd"), _opt_ptr(img, "a_image"))
    return s, y, xhat, invstd, img


def linear_forward_packed(a_image, rows, fin, fout, w, b=None, ctx=None):
    """Linear::forward from the packed A image of x (bias in the epilogue)."""
    y = torch.empty(rows * fout, device=a_image.device, dtype=torch.float32)
    call("rnn_linear_fwd_packed_dev", _ctx_of(a_image, ctx), _ptr(a_image, "a_image"), rows, fin, fout,
         _ptr(w, "w"), _opt_ptr(b, "b"), _ptr(y, "y"))
    return y


def swiglu_fused_forward(x, rows, c, h, wg, bg, a_image=None, ctx=None):
    """SwiGlu::forward's first GEMM with the gate in its epilogue: (ab, u)."""
    src = a_image if a_image is not None else x
    ab = torch.empty(rows * 2 * h, device=src.device, dtype=torch.float32)
    u = torch.empty(rows * h, device=src.device, dtype=torch.float32)
    call("rnn_swiglu_fwd_dev", _ctx_of(src, ctx), _opt_ptr(x, "x"), _opt_ptr(a_image, "a_image"), rows, c, h,
         _ptr(wg, "wg"), _ptr(bg, "bg"), _ptr(ab, "ab"), _ptr(u, "u"))
    return ab, u


def linear_backward(x, dy, rows, fin, fout, w, dw, db=None, ctx=None):
    """Linear::backward (linear.rs:66): dW, db accumulate; returns dx."""
    dx = torch.empty(rows * fin, device=x.device, dtype=torch.float32)
    call("rnn_linear_bwd_dev", _ctx_of(x, ctx), _ptr(x, "x"), _ptr(dy, "dy"), rows, fin, fout, _ptr(w, "w"),
         _ptr(dw, "dw"), _opt_ptr(db, "db"), _ptr(dx, "dx"))
    return dx


# ---------------------------------------------------------------- optim.rs


def newton_schulz_(g, rows, cols, steps, ctx=None):
    call("rnn_newton_schulz_dev", _ctx_of(g, ctx), _ptr(g, "g"), rows, cols, steps)
    return g


def muon_step_(v, g, m, rows, cols, steps, lr, mom=0.95, wd=0.0, decay=True, ctx=None):
    call("rnn_muon_step_dev", _ctx_of(v, ctx), _ptr(v, "v"), _ptr(g, "g"), _ptr(m, "m"), rows, cols, steps, lr, mom,
         wd, int(bool(decay)))
    return v


def adamw_step_(v, g, m, v2, lr, wd, decay, t, b1=0.9, b2=0.999, eps=1e-8, ctx=None):
    call("rnn_adamw_step_dev", _ctx_of(v, ctx), _ptr(v, "v"), _ptr(g, "g"), _ptr(m, "m"), _ptr(v2, "v2"), v.numel(),
         lr, wd, int(bool(decay)), b1, b2, eps, t)
    return v


def clip_(g, max_norm, ctx=None):
    """Returns the pre-clip norm as a 1-element device tensor."""
    norm = torch.empty(1, device=g.device, dtype=torch.float32)
    call("rnn_clip_dev", _ctx_of(g, ctx), _ptr(g, "g"), g.numel(), max_norm, _ptr(norm, "norm"))
    return norm


def ema_update_(e, v, decay, t, ctx=None):
    call("rnn_ema_update_dev", _ctx_of(e, ctx), _ptr(e, "e"), _ptr(v, "v"), e.numel(), decay, t)
    return e


# ---------------------------------------------------------------- rustvit glue


def _new(shape_numel, like):
    return torch.empty(shape_numel, device=like.device, dtype=torch.float32)


def layerscale_forward(x, rows, c, l, out=None, ctx=None):
    y = out if out is not None else torch.empty_like(x)
    call("rnn_layerscale_fwd_dev", _ctx_of(x, ctx), _ptr(x, "x"), rows, c, _ptr(l, "l"), _ptr(y, "y"))
    return y


def layerscale_backward(dy, x, rows, c, l, dl, ctx=None):
    dx = torch.empty_like(dy)
    call("rnn_layerscale_bwd_dev", _ctx_of(dy, ctx), _ptr(dy, "dy"), _ptr(x, "x"), rows, c, _ptr(l, "l"),
         _ptr(dl, "dl"), _ptr(dx, "dx"))
    return dx


def swiglu_forward(ab, rows, h, ctx=None):
    u = _new(rows * h, ab)
    call("rnn_swiglu_act_fwd_dev", _ctx_of(ab, ctx), _ptr(ab, "ab"), rows, h, _ptr(u, "u"))
    return u


def swiglu_backward(du, ab, rows, h, ctx=None):
    dab = torch.empty_like(ab)
    call("rnn_swiglu_act_bwd_dev", _ctx_of(du, ctx), _ptr(du, "du"), _ptr(ab, "ab"), rows, h, _ptr(dab, "dab"))
    return dab


def dwconv3_forward(x, n, th, tw, c, w, b, ctx=None):
    y = torch.empty_like(x)
    call("rnn_dwconv3_fwd_dev", _ctx_of(x, ctx), _ptr(x, "x"), n, th, tw, c, _ptr(w, "w"), _ptr(b, "b"), _ptr(y, "y"))
    return y


def dwconv3_backward(dy, x, n, th, tw, c, w, dw, db, ctx=None):
    dx = torch.empty_like(dy)
    call("rnn_dwconv3_bwd_dev", _ctx_of(dy, ctx), _ptr(dy, "dy"), _ptr(x, "x"), n, th, tw, c, _ptr(w, "w"),
         _ptr(dw, "dw"), _ptr(db, "db"), _ptr(dx, "dx"))
    return dx


def seqpool_forward(x, n, t, c, p, ctx=None):
    z, w = _new(n * c, x), _new(n * t, x)
    call("rnn_seqpool_fwd_dev", _ctx_of(x, ctx), _ptr(x, "x"), n, t, c, _ptr(p, "p"), _ptr(z, "z"), _ptr(w, "w"))
    return z, w


def seqpool_backward(dz, x, w, n, t, c, p, dp, ctx=None):
    dx = torch.empty_like(x)
    call("rnn_seqpool_bwd_dev", _ctx_of(dz, ctx), _ptr(dz, "dz"), _ptr(x, "x"), _ptr(w, "w"), n, t, c, _ptr(p, "p"),
         _ptr(dp, "dp"), _ptr(dx, "dx"))
    return dx


def droppath_forward_(x, n, per_image, p, seed, ctx=None):
    mask = _new(n, x)
    call("rnn_droppath_fwd_dev", _ctx_of(x, ctx), _ptr(x, "x"), n, per_image, p, seed & (2**64 - 1), _ptr(mask, "mask"))
    return mask


def droppath_backward_(dy, n, per_image, mask, ctx=None):
    call("rnn_droppath_bwd_dev", _ctx_of(dy, ctx), _ptr(dy, "dy"), n, per_image, _ptr(mask, "mask"))
    return dy


def token_merge(src, n, th, c, backward=False, ctx=None):
    dst = torch.empty_like(src)
    call("rnn_token_merge_dev", _ctx_of(src, ctx), _ptr(src, "src"), n, th, c, _ptr(dst, "dst"), int(bool(backward)))
    return dst


def tok_layout(x, n, c, hw, to_nchw=False, ctx=None):
    y = torch.empty_like(x)
    call("rnn_tok_layout_dev", _ctx_of(x, ctx), _ptr(x, "x"), n, c, hw, _ptr(y, "y"), int(bool(to_nchw)))
    return y


def taxo_forward_(zf, zc, n, nf, nc, parent, ctx=None):
    call("rnn_taxo_combine_fwd_dev", _ctx_of(zf, ctx), _ptr(zf, "zf"), _ptr(zc, "zc"), n, nf, nc, _ptr(parent, "parent"))
    return zf


def taxo_backward(dzf, dzc, n, nf, nc, parent, ctx=None):
    dc = torch.empty_like(dzc)
    call("rnn_taxo_combine_bwd_dev", _ctx_of(dzf, ctx), _ptr(dzf, "dzf"), _ptr(dzc, "dzc"), n, nf, nc,
         _ptr(parent, "parent"), _ptr(dc, "dc"))
    return dc


def ce_soft(logits, target, hard, nclass, scale=1.0, ctx=None):
    n = hard.numel()
    dz = torch.empty_like(logits)
    loss = _new(1, logits)
    corr = torch.empty(1, device=logits.device, dtype=torch.int32)
    call("rnn_ce_soft_dev", _ctx_of(logits, ctx), _ptr(logits, "logits"), _ptr(target, "target"), _ptr(hard, "hard"), n,
         nclass, scale, _ptr(dz, "dz"), _ptr(loss, "loss"), _ptr(corr, "correct"))
    return loss, dz, corr


def kl_distill(student, teacher, n, nclass, temp, scale, dz, ctx=None):
    loss = _new(1, student)
    call("rnn_kl_distill_dev", _ctx_of(student, ctx), _ptr(student, "student"), _ptr(teacher, "teacher"), n, nclass,
         temp, scale, _ptr(dz, "dz"), _ptr(loss, "loss"))
    return loss


def hint_mse(pred, target, n, c, scale, dz, ctx=None):
    loss = _new(1, pred)
    call("rnn_hint_mse_dev", _ctx_of(pred, ctx), _ptr(pred, "pred"), _ptr(target, "target"), n, c, scale,
         _ptr(dz, "dz"), _ptr(loss, "loss"))
    return loss
