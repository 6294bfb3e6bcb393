"""rustvit (vit.rs) restated over the C oracle kernels.  TEST INFRASTRUCTURE ONLY.

The composition — layer wiring, initialisation order, parameter order, the
multi-exit loss and the optimiser — follows the reference file by file; the
arithmetic of every layer is the C restatement in ``rnn_oracle.c`` reached
through ``oracle.oracle``.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU legs of ``bench.py`` may import this module.

Parameters live in four flat float32 buffers (value, gradient, first moment,
second moment) in the reference's ``for_each_param`` order (vit.rs:687-719),
each ``Param`` holding views into them, so whole-model vectors compare
elementwise with the device implementation.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from oracle import oracle as O

F32 = np.float32


def _L():
    return O.lib()


# ---------------------------------------------------------------- Param (nn.rs:44-111)


class Param:
    def __init__(self, v, decay, rows=0, cols=0):
        self.v = np.ascontiguousarray(v, F32)
        self.g = np.zeros_like(self.v)
        self.m = np.zeros_like(self.v)
        self.v2 = np.zeros_like(self.v)
        self.decay = bool(decay)
        self.rows, self.cols = rows, cols


def p_new(n, decay):
    return Param(np.zeros(n, F32), decay)


def p_filled(n, val, decay):
    return Param(np.full(n, F32(val), F32), decay)


def p_trunc(n, std, decay, rng):
    """Param::trunc_normal, nn.rs:77-89."""
    out = np.empty(n, F32)
    _L().orc_trunc_normal(C.byref(rng._s), out, n, F32(std))
    return Param(out, decay)


def p_kaiming(fan_in, n, rng):
    """Param::kaiming, nn.rs:95-100."""
    out = np.empty(n, F32)
    _L().orc_kaiming(C.byref(rng._s), out, n, fan_in)
    return Param(out, True)


# ---------------------------------------------------------------- tok.rs


def tok_from_nchw(x, n, c, hw):
    y = np.empty(n * hw * c, F32)
    _L().orc_tok_from_nchw(O._f32(x).ravel(), n, c, hw, y)
    return y


def tok_to_nchw(t, n, c, hw):
    y = np.empty(n * hw * c, F32)
    _L().orc_tok_to_nchw(O._f32(t).ravel(), n, c, hw, y)
    return y


# ---------------------------------------------------------------- nn.rs layers


class Conv2d:
    """nn.rs:115-250; backward accumulates dW (backward_w) and returns dX."""

    def __init__(self, cin, cout, k, stride, pad, rng):
        self.w = p_kaiming(cin * k * k, cout * cin * k * k, rng)
        self.cin, self.cout, self.k, self.stride, self.pad = cin, cout, k, stride, pad

    def forward(self, x, n, h, w):
        self.x, self.n, self.h, self.wd = x, n, h, w
        return O.conv2d_fwd(x, n, self.cin, h, w, self.w.v, self.cout, self.k, self.stride, self.pad)

    def out_hw(self, h):
        return O.out_dim(h, self.k, self.stride, self.pad)

    def backward_w(self, dy):
        O.conv2d_wgrad(self.x, dy, self.n, self.cin, self.h, self.wd, self.cout, self.k, self.stride, self.pad,
                       self.w.g)

    def backward(self, dy):
        self.backward_w(dy)
        return O.conv2d_dgrad(dy, self.n, self.cin, self.h, self.wd, self.w.v, self.cout, self.k, self.stride,
                              self.pad)

    def params(self):
        yield self.w


class BatchNorm2d:
    """nn.rs:255-428 (train statistics in f64, momentum 0.1, eps 1e-5)."""

    def __init__(self, c):
        self.g = p_filled(c, 1.0, False)
        self.b = p_new(c, False)
        self.rm = np.zeros(c, F32)
        self.rv = np.ones(c, F32)
        self.c = c

    def forward(self, y, n, hw, relu, train=True):
        if not train:  # running statistics (nn.rs:358-369)
            return O.bn_fwd_eval(y, n, self.c, hw, self.g.v, self.b.v, self.rm, self.rv, relu)
        out, self.xhat, self.invstd = O.bn_fwd_train(y, n, self.c, hw, self.g.v, self.b.v, self.rm, self.rv, relu)
        self.n, self.hw = n, hw
        return out

    def backward(self, dy):
        return O.bn_bwd(dy, self.xhat, self.n, self.c, self.hw, self.g.v, self.invstd, self.g.g, self.b.g)

    def params(self):
        yield self.g
        yield self.b

    def buffers(self):
        yield self.rm
        yield self.rv


def relu_back(d, y):
    d = O._f32(d).copy()
    _L().orc_relu_back(d, O._f32(y), d.size)
    return d


class BasicBlock:
    """model.rs:10-98: conv-BN-ReLU-conv-BN (+ 1x1 down) + ReLU, b2 gamma zeroed."""

    def __init__(self, cin, cout, stride, rng):
        self.b2 = BatchNorm2d(cout)
        self.b2.g.v[:] = 0.0  # zero_gamma
        self.c1 = Conv2d(cin, cout, 3, stride, 1, rng)
        self.b1 = BatchNorm2d(cout)
        self.c2 = Conv2d(cout, cout, 3, 1, 1, rng)
        self.down = (Conv2d(cin, cout, 1, stride, 0, rng), BatchNorm2d(cout)) if (stride != 1 or cin != cout) else None
        self.cout = cout

    def forward(self, x, n, h, w, train=True):
        y1 = self.c1.forward(x, n, h, w)
        oh = self.c1.out_hw(h)
        hh = self.b1.forward(y1, n, oh * oh, True, train)
        y = self.b2.forward(self.c2.forward(hh, n, oh, oh), n, oh * oh, False, train)
        if self.down is not None:
            c, b = self.down
            s = b.forward(c.forward(x, n, h, w), n, oh * oh, False, train)
        else:
            s = x
        _L().orc_add_relu(y, O._f32(s), y.size)
        self.h1, self.out, self.oh = hh, y, oh
        return y

    def backward(self, d):
        d = relu_back(d, self.out)
        dmain = self.c2.backward(self.b2.backward(d))
        dmain = relu_back(dmain, self.h1)
        dx = self.c1.backward(self.b1.backward(dmain))
        if self.down is not None:
            c, b = self.down
            dx = dx + c.backward(b.backward(d))
        else:
            dx = dx + d
        return dx.astype(F32)

    def params(self):
        yield from self.c1.params()
        yield from self.b1.params()
        yield from self.c2.params()
        yield from self.b2.params()
        if self.down is not None:
            yield from self.down[0].params()
            yield from self.down[1].params()

    def buffers(self):
        yield from self.b1.buffers()
        yield from self.b2.buffers()
        if self.down is not None:
            yield from self.down[1].buffers()


# ---------------------------------------------------------------- linear.rs, norm.rs


class Linear:
    """linear.rs:14-104."""

    def __init__(self, fin, fout, bias, std, rng):
        self.w = p_trunc(fin * fout, std, True, rng)
        self.w.rows, self.w.cols = fout, fin
        self.b = p_new(fout, False) if bias else None
        self.fin, self.fout = fin, fout

    @staticmethod
    def scaled(fin, fout, bias, depth, rng):
        return Linear(fin, fout, bias, F32(0.02) / np.sqrt(F32(2.0 * depth), dtype=F32), rng)

    def forward(self, x, rows):
        self.x, self.rows = O._f32(x).ravel(), rows
        return O.linear_fwd(self.x, rows, self.fin, self.fout, self.w.v, None if self.b is None else self.b.v)

    def backward(self, dy):
        return O.linear_bwd(self.x, dy, self.rows, self.fin, self.fout, self.w.v, self.w.g,
                            None if self.b is None else self.b.g)

    def params(self):
        yield self.w
        if self.b is not None:
            yield self.b


class LayerNorm:
    """norm.rs:18-137 (f64 row statistics, eps 1e-5)."""

    def __init__(self, c):
        self.g = p_filled(c, 1.0, False)
        self.b = p_new(c, False)
        self.c = c

    def forward(self, x, rows):
        y, self.xhat, self.invstd = O.layernorm_fwd(x, rows, self.c, self.g.v, self.b.v)
        self.rows = rows
        return y

    def backward(self, dy):
        return O.layernorm_bwd(dy, self.xhat, self.invstd, self.rows, self.c, self.g.v, self.g.g, self.b.g)

    def params(self):
        yield self.g
        yield self.b


class LayerScale:
    """norm.rs:151-212."""

    def __init__(self, c, init):
        self.l = p_filled(c, init, False)
        self.c = c

    def forward(self, x, rows):
        self.x, self.rows = O._f32(x).ravel().copy(), rows
        y = np.empty_like(self.x)
        _L().orc_layerscale_fwd(self.x, rows, self.c, self.l.v, y)
        return y

    def backward(self, dy):
        dx = np.empty(self.rows * self.c, F32)
        _L().orc_layerscale_bwd(O._f32(dy).ravel(), self.x, self.rows, self.c, self.l.v, self.l.g, dx)
        return dx

    def params(self):
        yield self.l


class SwiGlu:
    """norm.rs:225-288: y = (silu(x W1) * (x W2)) W3 with W1|W2 fused."""

    def __init__(self, c, h, depth, rng):
        self.wg = Linear(c, 2 * h, True, 0.02, rng)
        self.wd = Linear.scaled(h, c, True, depth, rng)
        self.h = h

    def forward(self, x, rows):
        self.ab = self.wg.forward(x, rows)
        self.rows = rows
        u = np.empty(rows * self.h, F32)
        _L().orc_swiglu_act_fwd(self.ab, rows, self.h, u)
        return self.wd.forward(u, rows)

    def backward(self, dy):
        du = self.wd.backward(dy)
        dab = np.empty(self.rows * 2 * self.h, F32)
        _L().orc_swiglu_act_bwd(du, self.ab, self.rows, self.h, dab)
        return self.wg.backward(dab)

    def params(self):
        yield from self.wg.params()
        yield from self.wd.params()


class DwConv3:
    """norm.rs:304-451: depthwise 3x3 over the token grid, channel-last."""

    def __init__(self, c, th, tw, rng):
        self.w = p_trunc(9 * c, 0.1, False, rng)
        self.b = p_new(c, False)
        self.c, self.th, self.tw = c, th, tw

    def forward(self, x, n):
        self.x, self.n = O._f32(x).ravel(), n
        y = np.empty_like(self.x)
        _L().orc_dwconv3_fwd(self.x, n, self.th, self.tw, self.c, self.w.v, self.b.v, y)
        return y

    def backward(self, dy):
        dx = np.empty_like(self.x)
        _L().orc_dwconv3_bwd(O._f32(dy).ravel(), self.x, self.n, self.th, self.tw, self.c, self.w.v, self.w.g,
                             self.b.g, dx)
        return dx

    def params(self):
        yield self.w
        yield self.b


class SeqPool:
    """norm.rs:460-581: w = softmax(x . p), z = sum_t w_t x_t."""

    def __init__(self, c, rng):
        self.p = p_trunc(c, 0.02, True, rng)
        self.c = c

    def forward(self, x, n, t):
        self.x, self.n, self.t = O._f32(x).ravel(), n, t
        z = np.empty(n * self.c, F32)
        self.w = np.empty(n * t, F32)
        _L().orc_seqpool_fwd(self.x, n, t, self.c, self.p.v, z, self.w)
        return z

    def backward(self, dz):
        dx = np.empty_like(self.x)
        _L().orc_seqpool_bwd(O._f32(dz).ravel(), self.x, self.w, self.n, self.t, self.c, self.p.v, self.p.g, dx)
        return dx

    def params(self):
        yield self.p


# ---------------------------------------------------------------- attn.rs wrappers


class SelfAttn:
    """attn.rs:347-442: fused qkv projection, LSA temperature, relative bias."""

    def __init__(self, c, h, th, tw, depth, rng):
        dh = c // h
        self.relidx, self.nrel = O.rel_index(th, tw, th, tw)
        self.qkv = Linear(c, 3 * c, True, 0.02, rng)
        self.proj = Linear.scaled(c, c, True, depth, rng)
        self.tau = p_filled(h, F32(1.0) / np.sqrt(F32(dh), dtype=F32), False)
        self.rel = p_new(h * self.nrel, False)
        self.c, self.h, self.dh, self.t = c, h, dh, th * tw

    def forward(self, x, n):
        c, t = self.c, self.t
        self.ab = self.qkv.forward(x, n * t)
        self.p, o = O.attn_fwd(n, self.h, self.dh, t, t, True, self.relidx, self.nrel, self.ab, 3 * c, 0, self.ab,
                               3 * c, c, 2 * c, self.tau.v, self.rel.v)
        self.n = n
        return self.proj.forward(o, n * t)

    def backward(self, dy):
        c, t, n = self.c, self.t, self.n
        dobuf = self.proj.backward(dy)
        dab = np.zeros(n * t * 3 * c, F32)
        dkv = np.zeros(n * t * 3 * c, F32)
        O.attn_bwd(n, self.h, self.dh, t, t, self.relidx, self.nrel, self.ab, 3 * c, 0, self.ab, 3 * c, c, 2 * c,
                   self.tau.v, self.p, dobuf, dab, dkv, self.tau.g, self.rel.g)
        dab += dkv
        return self.qkv.backward(dab)

    def params(self):
        yield from self.qkv.params()
        yield from self.proj.params()
        yield self.tau
        yield self.rel


class CrossAttn:
    """attn.rs:444-560: queries from the tokens, K|V from the memory [n, tk, 2c]."""

    def __init__(self, c, h, th, tw, mh, mw, depth, rng):
        dh = c // h
        self.relidx, self.nrel = O.rel_index(th, tw, mh, mw)
        self.wq = Linear(c, c, True, 0.02, rng)
        self.proj = Linear.scaled(c, c, True, depth, rng)
        self.tau = p_filled(h, F32(1.0) / np.sqrt(F32(dh), dtype=F32), False)
        self.rel = p_new(h * self.nrel, False)
        self.c, self.h, self.dh, self.t, self.tk = c, h, dh, th * tw, mh * mw

    def forward(self, x, mem, n):
        c, t = self.c, self.t
        self.q = self.wq.forward(x, n * t)
        self.p, o = O.attn_fwd(n, self.h, self.dh, t, self.tk, False, self.relidx, self.nrel, self.q, c, 0, mem,
                               2 * c, 0, c, self.tau.v, self.rel.v)
        self.n = n
        return self.proj.forward(o, n * t)

    def backward(self, dy, mem, dmem):
        c, t, n = self.c, self.t, self.n
        dobuf = self.proj.backward(dy)
        dq = np.zeros(n * t * c, F32)
        O.attn_bwd(n, self.h, self.dh, t, self.tk, self.relidx, self.nrel, self.q, c, 0, mem, 2 * c, 0, c,
                   self.tau.v, self.p, dobuf, dq, dmem, self.tau.g, self.rel.g)
        return self.wq.backward(dq)

    def params(self):
        yield from self.wq.params()
        yield from self.proj.params()
        yield self.tau
        yield self.rel


# ---------------------------------------------------------------- vit.rs


class DropPath:
    """vit.rs:26-73: whole-branch drop per image from an explicit seed."""

    def __init__(self, p):
        self.p = F32(p)
        self.mask = None

    def forward(self, x, n, per, train, seed):
        if not train or self.p <= 0.0:
            self.mask = None
            return x
        self.mask = np.empty(n, F32)
        _L().orc_droppath_mask(n, self.p, C.c_uint64(seed & (2**64 - 1)), self.mask)
        return (x.reshape(n, per) * self.mask[:, None]).astype(F32).ravel()

    def backward(self, dy, n, per):
        if self.mask is None:
            return dy
        return (dy.reshape(n, per) * self.mask[:, None]).astype(F32).ravel()


class Block:
    """vit.rs:75-232: pre-LN block with self-attention + gamma * depthwise branch,
    optional cross-attention into the memory, and a SwiGLU MLP."""

    def __init__(self, c, h, th, tw, mem, depth, drop, idx, ls_init, rng):
        hidden = -(-(4 * c // 3) // 16) * 16
        self.n1 = LayerNorm(c)
        self.attn = SelfAttn(c, h, th, tw, depth, rng)
        self.dw = DwConv3(c, th, tw, rng)
        self.gamma = p_filled(c, 0.5, False)
        self.ls1 = LayerScale(c, ls_init)
        self.cross = CrossAttn(c, h, th, tw, mem[0], mem[1], depth, rng) if mem is not None else None
        self.lsm = LayerScale(c, ls_init) if mem is not None else None
        self.n2 = LayerNorm(c)
        self.mlp = SwiGlu(c, hidden, depth, rng)
        self.ls2 = LayerScale(c, ls_init)
        self.dp1, self.dp2, self.dp3 = DropPath(drop), DropPath(drop), DropPath(drop)
        self.c, self.t, self.idx = c, th * tw, idx

    def forward(self, x, mem, n, train, seed):
        c, t = self.c, self.t
        rows = n * t
        hh = self.n1.forward(x, rows)
        a = self.attn.forward(hh, n)
        d = self.dw.forward(hh, n)
        a = (a.reshape(rows, c) + self.gamma.v[None, :] * d.reshape(rows, c)).astype(F32).ravel()
        self.dwo = d
        a = self.dp1.forward(self.ls1.forward(a, rows), n, t * c, train, seed ^ self.idx)
        y = (O._f32(x).ravel() + a).astype(F32)
        self.n, self.hbuf = n, hh
        if self.cross is not None:
            cm = self.cross.forward(hh, mem, n)
            cm = self.dp2.forward(self.lsm.forward(cm, rows), n, t * c, train, seed ^ self.idx ^ 0x5151)
            y = (y + cm).astype(F32)
        h2 = self.n2.forward(y, rows)
        m = self.mlp.forward(h2, rows)
        m = self.dp3.forward(self.ls2.forward(m, rows), n, t * c, train, seed ^ self.idx ^ 0xA2A2)
        return (y + m).astype(F32)

    def backward(self, dz, mem, dmem):
        c, t, n = self.c, self.t, self.n
        rows = n * t
        dm = self.ls2.backward(self.dp3.backward(dz, n, t * c))
        dh2 = self.mlp.backward(dm)
        dy = (dz + self.n2.backward(dh2)).astype(F32)
        dh = np.zeros(rows * c, F32)
        if self.cross is not None:
            dc = self.lsm.backward(self.dp2.backward(dy, n, t * c))
            dh += self.cross.backward(dc, mem, dmem)
        da = self.ls1.backward(self.dp1.backward(dy, n, t * c))
        # gamma gradient and the depthwise branch's upstream gradient in one
        # LayerScale-shaped pass: dgamma += sum(da * dwo), ddw = gamma * da
        ddw = np.empty(rows * c, F32)
        _L().orc_layerscale_bwd(da, self.dwo, rows, c, self.gamma.v, self.gamma.g, ddw)
        dh += self.attn.backward(da)
        dh += self.dw.backward(ddw)
        return (dy + self.n1.backward(dh)).astype(F32)

    def params(self):
        yield from self.n1.params()
        yield from self.attn.params()
        yield from self.dw.params()
        yield self.gamma
        yield from self.ls1.params()
        if self.cross is not None:
            yield from self.cross.params()
        if self.lsm is not None:
            yield from self.lsm.params()
        yield from self.n2.params()
        yield from self.mlp.params()
        yield from self.ls2.params()


class TaxoHead:
    """vit.rs:236-315: z_f[c] = z_coarse[parent(c)] + r[c]."""

    def __init__(self, c, parent, nc, rng):
        self.parent = np.ascontiguousarray(parent, np.uint32)
        self.nf, self.nc = len(parent), nc
        self.coarse = Linear(c, nc, True, 0.02, rng)
        self.resid = Linear(c, self.nf, True, 0.02, rng)

    def forward(self, f, n):
        zc = self.coarse.forward(f, n)
        zf = self.resid.forward(f, n)
        _L().orc_taxo_fwd(zf, zc, n, self.nf, self.nc, self.parent)
        self.n = n
        return zf, zc

    def backward(self, dzf, dzc):
        dc = np.empty(self.n * self.nc, F32)
        _L().orc_taxo_bwd(O._f32(dzf), O._f32(dzc), self.n, self.nf, self.nc, self.parent, dc)
        df = self.resid.backward(dzf)
        return (df + self.coarse.backward(dc)).astype(F32)

    def params(self):
        yield from self.coarse.params()
        yield from self.resid.params()


class Exit:
    """vit.rs:317-347: auxiliary classifier + hint projection."""

    def __init__(self, cin, nclass, chint, rng):
        self.fc = Linear(cin, nclass, True, 0.02, rng)
        self.hint = Linear(cin, chint, False, 0.02, rng)

    def forward(self, f, n):
        return self.fc.forward(f, n), self.hint.forward(f, n)

    def backward(self, dz, dh):
        return (self.fc.backward(dz) + self.hint.backward(dh)).astype(F32)

    def params(self):
        yield from self.fc.params()
        yield from self.hint.params()


@dataclass
class Cfg:
    """vit.rs:349-387 (defaults = Cfg::default)."""
    width: int = 32
    cmid: int = 96
    dim: int = 256
    heads: int = 4
    depth3: int = 5
    dim4: int = 384
    heads4: int = 6
    depth4: int = 2
    mem_at: list = field(default_factory=lambda: [1, 3])
    droppath: float = 0.1
    img: int = 32


def cifar_parent():
    """Synthetic 20 x 5 taxonomy: parent[i] = i / 5."""
    return np.array([i // 5 for i in range(100)], np.uint32)


class RustViT:
    """vit.rs:389-802."""

    def __init__(self, cfg: Cfg, parent, ncoarse, seed):
        rng = O.Rng(seed)
        w, cm, d, d4 = cfg.width, cfg.cmid, cfg.dim, cfg.dim4
        self.mh = cfg.img // 2
        self.th = cfg.img // 4
        th4 = self.th // 2
        depth = cfg.depth3 + cfg.depth4
        nf = len(parent)
        den = F32(max(depth, 2) - 1)
        self.blocks3 = []
        for i in range(cfg.depth3):
            dp = F32(cfg.droppath) * F32(i) / den
            self.blocks3.append(Block(d, cfg.heads, self.th, self.th, (self.mh, self.mh) if i in cfg.mem_at else None,
                                      depth, dp, i + 1, 1e-4, rng))
        self.blocks4 = []
        for i in range(cfg.depth4):
            dp = F32(cfg.droppath) * F32(cfg.depth3 + i) / den
            self.blocks4.append(Block(d4, cfg.heads4, th4, th4, None, depth, dp, cfg.depth3 + i + 1, 1e-4, rng))
        # struct-literal order (vit.rs:478-509)
        self.stem = Conv2d(3, w, 3, 1, 1, rng)
        self.stem_bn = BatchNorm2d(w)
        self.c1 = BasicBlock(w, w, 1, rng)
        self.c2 = BasicBlock(w, cm, 2, rng)
        self.memconv = Conv2d(cm, 2 * d, 1, 1, 0, rng)
        self.memln = LayerNorm(2 * d)
        self.tokconv = Conv2d(cm, d, 3, 2, 1, rng)
        self.tok_bn = BatchNorm2d(d)
        self.mergeln = LayerNorm(4 * d)
        self.merge = Linear(4 * d, d4, True, 0.02, rng)
        self.headln = LayerNorm(d4)
        self.pool = SeqPool(d4, rng)
        self.head = TaxoHead(d4, parent, ncoarse, rng)
        self.e1 = Exit(cm, nf, d4, rng)
        self.pool2 = SeqPool(d, rng)
        self.e2 = Exit(d, nf, d4, rng)
        self.cfg, self.nf, self.nc = cfg, nf, ncoarse
        self.drop_seed = 0
        self.use_exits = True
        self._flatten()

    # -- parameter storage
    def params(self):
        yield self.stem.w
        yield from self.stem_bn.params()
        yield from self.c1.params()
        yield from self.c2.params()
        yield self.memconv.w
        yield from self.memln.params()
        yield self.tokconv.w
        yield from self.tok_bn.params()
        for b in self.blocks3:
            yield from b.params()
        yield from self.mergeln.params()
        yield from self.merge.params()
        for b in self.blocks4:
            yield from b.params()
        yield from self.headln.params()
        yield from self.pool.params()
        yield from self.head.params()
        if self.use_exits:
            yield from self.e1.params()
            yield from self.pool2.params()
            yield from self.e2.params()

    def buffers(self):
        yield from self.stem_bn.buffers()
        yield from self.c1.buffers()
        yield from self.c2.buffers()
        yield from self.tok_bn.buffers()

    def _flatten(self):
        ps = list(self.params())
        total = sum(p.v.size for p in ps)
        self.V, self.G = np.zeros(total, F32), np.zeros(total, F32)
        self.M, self.V2 = np.zeros(total, F32), np.zeros(total, F32)
        off = 0
        self.plist = ps
        for p in ps:
            n = p.v.size
            self.V[off:off + n] = p.v
            p.v, p.g, p.m, p.v2 = self.V[off:off + n], self.G[off:off + n], self.M[off:off + n], self.V2[off:off + n]
            off += n

    def num_params(self):
        return self.V.size

    def buffer_vec(self):
        return np.concatenate([b for b in self.buffers()])

    # -- forward (vit.rs:511-582)
    def forward(self, x, n, train=True):
        cfg, d = self.cfg, self.cfg.dim
        img, th, mh = cfg.img, self.th, self.mh
        h = self.stem_bn.forward(self.stem.forward(x, n, img, img), n, img * img, True, train)
        self.stem_out = h
        h = self.c1.forward(h, n, img, img, train)
        h = self.c2.forward(h, n, img, img, train)
        self.c2_out = h
        cm = cfg.cmid
        memt = tok_from_nchw(self.memconv.forward(h, n, mh, mh), n, 2 * d, mh * mh)
        mem = self.memln.forward(memt, n * mh * mh)
        t = self.tok_bn.forward(self.tokconv.forward(h, n, mh, mh), n, th * th, False, train)
        z = tok_from_nchw(t, n, d, th * th)
        seed = self.drop_seed
        for b in self.blocks3:
            z = b.forward(z, mem, n, train, seed)
        self.mem = mem
        e2l = h2v = None
        if self.use_exits and train:
            f = self.pool2.forward(z, n, th * th)
            e2l, h2v = self.e2.forward(f, n)
        zm = np.empty(z.size, F32)
        _L().orc_token_merge_fwd(z, n, th, d, zm)
        th4 = th // 2
        zn = self.mergeln.forward(zm, n * th4 * th4)
        z4 = self.merge.forward(zn, n * th4 * th4)
        for b in self.blocks4:
            z4 = b.forward(z4, None, n, train, seed)
        zf = self.headln.forward(z4, n * th4 * th4)
        feat = self.pool.forward(zf, n, th4 * th4)
        logits, coarse = self.head.forward(feat, n)
        e1l = h1v = None
        if self.use_exits and train:
            g = np.empty(n * cm, F32)
            _L().orc_gap_fwd(self.c2_out, n * cm, mh * mh, g)
            e1l, h1v = self.e1.forward(g, n)
        self.n = n
        return dict(logits=logits, coarse=coarse, e1=e1l, e2=e2l, h1=h1v, h2=h2v, feat=feat)

    # -- backward (vit.rs:627-685)
    def backward(self, g):
        cfg, d3, n = self.cfg, self.cfg.dim, self.n
        th, mh = self.th, self.mh
        dfeat = self.head.backward(g["logits"], g["coarse"])
        if g.get("hfinal") is not None:
            dfeat = (dfeat + g["hfinal"]).astype(F32)
        dzf = self.pool.backward(dfeat)
        dz4 = self.headln.backward(dzf)
        for b in reversed(self.blocks4):
            dz4 = b.backward(dz4, None, None)
        dmg = self.merge.backward(dz4)
        dzn = self.mergeln.backward(dmg)
        dz = np.empty(dzn.size, F32)
        _L().orc_token_merge_bwd(dzn, n, th, d3, dz)
        if self.use_exits and g.get("e2") is not None:
            df2 = self.e2.backward(g["e2"], g["h2"])
            dz = (dz + self.pool2.backward(df2)).astype(F32)
        dmem = np.zeros(self.mem.size, F32)
        for b in reversed(self.blocks3):
            dz = b.backward(dz, self.mem, dmem)
        dt = tok_to_nchw(dz, n, d3, th * th)
        dtc = self.tokconv.backward(self.tok_bn.backward(dt))
        dmemn = self.memln.backward(dmem)
        dmc = self.memconv.backward(tok_to_nchw(dmemn, n, 2 * d3, mh * mh))
        dc2 = (dtc + dmc).astype(F32)
        if self.use_exits and g.get("e1") is not None:
            dg = self.e1.backward(g["e1"], g["h1"])
            dgap = np.empty(n * cfg.cmid * mh * mh, F32)
            _L().orc_gap_bwd(dg, n * cfg.cmid, mh * mh, dgap)
            dc2 = (dc2 + dgap).astype(F32)
        dh = self.c2.backward(dc2)
        dh = self.c1.backward(dh)
        dh = relu_back(dh, self.stem_out)
        dh = self.stem_bn.backward(dh)
        self.stem.backward_w(dh)

    def macs(self):
        """vit.rs:745-771, per image."""
        c = self.cfg
        w, cm, d, d4, img = c.width, c.cmid, c.dim, c.dim4, c.img
        r1, r2, t, t4 = img * img, img * img // 4, self.th * self.th, self.th * self.th // 4
        m = 3 * 9 * w * r1 + 2 * (w * 9 * w * r1) + (w * 9 * cm * r2 + cm * 9 * cm * r2 + w * cm * r2)
        m += cm * 2 * d * r2 + cm * 9 * d * t
        hid3 = -(-(4 * d // 3) // 16) * 16
        m += (t * d * 3 * d + 2 * t * t * d + t * d * d + 3 * t * d * hid3 + 9 * d * t) * c.depth3
        m += 2 * t * r2 * d * len(c.mem_at)
        m += t4 * 4 * d * d4
        hid4 = -(-(4 * d4 // 3) // 16) * 16
        m += (t4 * d4 * 3 * d4 + 2 * t4 * t4 * d4 + t4 * d4 * d4 + 3 * t4 * d4 * hid4 + 9 * d4 * t4) * c.depth4
        m += d4 * (self.nf + self.nc)
        return m


# ---------------------------------------------------------------- loss.rs / train.rs


@dataclass
class LossCfg:
    """The build_loss weights of cli.rs:98-112 (defaults)."""
    smooth: float = 0.1
    sib: float = 0.7
    coarse_w: float = 0.4
    exit_w: tuple = (0.3, 0.6)
    alpha: float = 1.0
    temp: float = 3.0
    beta: float = 0.03


def taxo_target(y, parent, nf, eps, sib):
    """loss.rs:11-28 with groups[g] = the classes whose parent is g."""
    g = np.nonzero(parent == parent[y])[0]
    k = len(g)
    out = np.full(nf, F32(eps) * (F32(1.0) - F32(sib)) / F32(nf - k) if nf > k else F32(0.0), F32)
    if k > 1:
        out[g] = F32(eps) * F32(sib) / F32(k - 1)
    out[y] = F32(1.0) - F32(eps)
    return out


def uniform_target(y, k, eps):
    """loss.rs:30-34."""
    out = np.full(k, F32(eps) / F32(k), F32)
    out[y] += F32(1.0) - F32(eps)
    return out


def targets(labels, parent, nc, lc: LossCfg, perm=None, lam=None):
    """train.rs:120-155: (tf [n, nf], tc [n, nc], coarse labels).  With perm /
    lam (data::mix_batch's) row i is lam[i] * target(i) + (1 - lam[i]) *
    target(perm[i]) in f32, unfused; without them lambda = 1."""
    nf = len(parent)
    coarse = parent[labels].astype(np.uint32)
    fa = [taxo_target(int(y), parent, nf, lc.smooth, lc.sib).astype(F32) for y in labels]
    ca = [uniform_target(int(c), nc, lc.smooth).astype(F32) for c in coarse]
    if perm is None:
        return np.concatenate(fa), np.concatenate(ca), coarse
    tf, tc = [], []
    for i in range(len(labels)):
        lv = F32(lam[i])
        tf.append(lv * fa[i] + (F32(1.0) - lv) * fa[perm[i]])
        tc.append(lv * ca[i] + (F32(1.0) - lv) * ca[perm[i]])
    return np.concatenate(tf).astype(F32), np.concatenate(tc).astype(F32), coarse


def ce_soft(logits, target, hard, nclass, scale):
    d = np.empty(logits.size, F32)
    corr = C.c_int(0)
    loss = _L().orc_ce_soft(O._f32(logits), O._f32(target), np.ascontiguousarray(hard, np.uint32), len(hard), nclass,
                            F32(scale), d, C.byref(corr))
    return loss, d, corr.value


def build_loss(out, tf, tc, hard, hardc, lc: LossCfg, nf, nc, n):
    """train.rs:70-118: returns (grads dict, total, ce, correct)."""
    L = _L()
    ce, dlog, correct = ce_soft(out["logits"], tf, hard, nf, 1.0)
    g = dict(logits=dlog, coarse=np.zeros(n * nc, F32))
    total = F32(ce)
    if lc.coarse_w > 0.0:
        lcoarse, g["coarse"], _ = ce_soft(out["coarse"], tc, hardc, nc, lc.coarse_w)
        total += F32(lc.coarse_w) * F32(lcoarse)
    if out["e1"] is not None:
        d4 = out["feat"].size // n
        l1, g["e1"], _ = ce_soft(out["e1"], tf, hard, nf, lc.exit_w[0])
        l2, g["e2"], _ = ce_soft(out["e2"], tf, hard, nf, lc.exit_w[1])
        g["h1"], g["h2"] = np.zeros(n * d4, F32), np.zeros(n * d4, F32)
        total += F32(lc.exit_w[0]) * F32(l1) + F32(lc.exit_w[1]) * F32(l2)
        if lc.alpha > 0.0:
            k1 = L.orc_kl_distill(O._f32(out["e1"]), O._f32(out["logits"]), n, nf, F32(lc.temp), F32(lc.alpha), g["e1"])
            k2 = L.orc_kl_distill(O._f32(out["e2"]), O._f32(out["logits"]), n, nf, F32(lc.temp), F32(lc.alpha), g["e2"])
            total += F32(lc.alpha) * (F32(k1) + F32(k2))
        if lc.beta > 0.0:
            total += F32(L.orc_hint_mse(O._f32(out["h1"]), O._f32(out["feat"]), n, d4, F32(lc.beta), g["h1"])) + F32(
                L.orc_hint_mse(O._f32(out["h2"]), O._f32(out["feat"]), n, d4, F32(lc.beta), g["h2"]))
    return g, float(total), float(ce), correct


class Optim:
    """optim.rs:149-234: Muon (momentum 0.95, 3 NS steps) for the 2-D Linear
    weights, AdamW (0.9, 0.999, 1e-8) for everything else."""

    def __init__(self, muon=True, ns_steps=3):
        self.muon, self.ns, self.mom = muon, ns_steps, F32(0.95)
        self.b1, self.b2, self.eps = F32(0.9), F32(0.999), F32(1e-8)
        self.t = 0

    def step_all(self, params, lr, wd):
        L = _L()
        for p in params:
            if self.muon and p.rows > 0 and min(p.rows, p.cols) > 1:
                L.orc_muon_step(p.v, p.g, p.m, p.rows, p.cols, self.ns, F32(lr), self.mom, F32(wd), int(p.decay))
        for p in params:
            if not (self.muon and p.rows > 0 and min(p.rows, p.cols) > 1):
                L.orc_adamw_step(p.v, p.g, p.m, p.v2, p.v.size, F32(lr), F32(wd), int(p.decay), self.b1, self.b2,
                                 self.eps, self.t)
        self.t += 1


class Ema:
    """optim.rs:253-317 (update only)."""

    def __init__(self, d):
        self.d, self.w, self.t = F32(d), None, 0

    def update(self, flat_v):
        self.t += 1
        if self.w is None:
            self.w = flat_v.copy()
            return
        _L().orc_ema_update(self.w, flat_v, flat_v.size, self.d, self.t)


class Trainer:
    """train.rs:346-387 with a fixed learning rate and no augmentation."""

    def __init__(self, net: RustViT, lc: LossCfg = LossCfg(), clip=1.0, ema=0.9998, muon=True, ns=3):
        self.net, self.lc, self.clip = net, lc, F32(clip)
        self.opt = Optim(muon, ns)
        self.ema = Ema(ema) if ema > 0 else None

    def step(self, x, labels, n, lr, wd, drop_seed):
        net = self.net
        tf, tc, coarse = targets(labels, net.head.parent, net.nc, self.lc)
        net.drop_seed = drop_seed
        out = net.forward(x, n, True)
        g, total, ce, correct = build_loss(out, tf, tc, labels, coarse, self.lc, net.nf, net.nc, n)
        net.backward(g)
        if self.clip > 0.0:
            _L().orc_clip(net.G, net.G.size, self.clip)
        self.opt.step_all(net.plist, lr, wd)
        if self.ema is not None:
            self.ema.update(net.V)
        return total, ce, correct


def dp_step(trainers, shards, lr, wd, seeds):
    """One batch-sharded Trainer::step over len(trainers) ranks, the
    semantics of rnn_rustvit_dp_attach (no counterpart in the reference,
    whose step, train.rs:346-387, runs in one process).  Every trainer holds
    a network built from the same seed; rank r runs forward, build_loss and
    backward on shards[r] = (x, labels, n) with drop seed seeds[r] (its
    BatchNorm layers on its own batch statistics); then the ranks' BatchNorm
    running statistics and gradients are replaced by their mean (f32 sum in
    rank order, then the division by the rank count), and every rank runs
    clip_, Optim::step_all and Ema::update as Trainer.step does.  Returns
    each rank's (total, ce, correct)."""
    world = len(trainers)
    stats = []
    for tr, (x, labels, n), seed in zip(trainers, shards, seeds):
        net = tr.net
        tf, tc, coarse = targets(labels, net.head.parent, net.nc, tr.lc)
        net.drop_seed = seed
        out = net.forward(x, n, True)
        g, total, ce, correct = build_loss(out, tf, tc, labels, coarse, tr.lc, net.nf, net.nc, n)
        net.backward(g)
        stats.append((total, ce, correct))

    def mean(arrays):
        acc = arrays[0].astype(F32).copy()
        for a in arrays[1:]:
            acc = (acc + a).astype(F32)
        return (acc / F32(world)).astype(F32)

    gmean = mean([tr.net.G for tr in trainers])
    bufs = [list(tr.net.buffers()) for tr in trainers]
    bmean = [mean([b[i] for b in bufs]) for i in range(len(bufs[0]))]
    for tr, b in zip(trainers, bufs):
        net = tr.net
        net.G[:] = gmean
        for dst, src in zip(b, bmean):
            dst[:] = src
        if tr.clip > 0.0:
            _L().orc_clip(net.G, net.G.size, tr.clip)
        tr.opt.step_all(net.plist, lr, wd)
        if tr.ema is not None:
            tr.ema.update(net.V)
    return stats


def eval_vit(net: RustViT, images, labels, batch, tta):
    """eval::vit (eval.rs:47-66) over a u8 CHW dataset: the exits are off, each
    batch runs forward with train false, and with tta its logits are averaged
    with those of the mirrored batch, 0.5 * (a + b); softmax_ce without
    smoothing, loss summed as l * bs in f32 (eval.rs:15-39).  Returns
    (loss, accuracy)."""
    assert batch > 0
    exits = net.use_exits
    net.use_exits = False
    total = len(labels)
    acc_sum, correct, seen, s = F32(0.0), 0, 0, 0
    while s < total:
        bs = min(batch, total - s)
        x, lab = O.make_batch_eval(images, labels, s, bs, False)
        lg = net.forward(x, bs, False)["logits"]
        if tta:
            xm, lab = O.make_batch_eval(images, labels, s, bs, True)
            mirrored = net.forward(xm, bs, False)["logits"]
            lg = (F32(0.5) * (lg + mirrored)).astype(F32)
        loss, _, c = O.softmax_ce(lg, lab, net.nf, 0.0)
        acc_sum = F32(acc_sum + F32(F32(loss) * F32(bs)))
        correct += c
        seen += bs
        s += bs
    net.use_exits = exits
    if seen == 0:
        return float("nan"), float("nan")
    return float(acc_sum / F32(seen)), float(F32(correct) / F32(seen))
