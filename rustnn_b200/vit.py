"""The rustvit training step (vit.rs RustViT, train.rs Trainer::step) on the GPU.

``RustViT(cfg, parent, ncoarse, seed)`` mirrors ``RustViT::new`` and draws
the same initial parameters; ``train_step`` runs forward, the multi-exit loss
(build_loss, train.rs:70-118), backward, clip_, Optim::step_all (Muon for
the 2-D Linear weights, AdamW for the rest) and the EMA update as one
device-resident sequence of this library's kernels.  ``targets`` builds the
soft targets of train.rs:120-155 on the host (mixup off), as the reference's
data pipeline does.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np
import torch

from ._lib import VIT, RnnError, call, check, lib
from .ops import default_context


@dataclass
class VitCfg:
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


def cifar_parent() -> np.ndarray:
    """The CIFAR-100 shape of the taxonomy: 20 coarse groups of 5, parent[i] = i / 5."""
    return np.array([i // 5 for i in range(100)], np.uint32)


def targets(labels, parent, ncoarse, smooth=0.1, sib=0.7, perm=None, lam=None):
    """Soft targets of train.rs:120-155: taxo_target for the fine labels
    (loss.rs:11-28), uniform_target for the coarse ones (loss.rs:30-34).
    With perm / lam from mix_batch (data.rs:467-491) row i becomes
    lam[i] * target(i) + (1 - lam[i]) * target(perm[i]).  Returns
    (tf [n * nf], tc [n * nc], coarse labels)."""
    parent = np.asarray(parent, np.uint32)
    labels = np.asarray(labels, np.uint32)
    nf = len(parent)
    f32 = np.float32
    tf = np.empty((len(labels), nf), f32)
    for i, y in enumerate(labels):
        g = np.nonzero(parent == parent[y])[0]
        k = len(g)
        tf[i] = f32(smooth) * (f32(1.0) - f32(sib)) / f32(nf - k) if nf > k else f32(0.0)
        if k > 1:
            tf[i, g] = f32(smooth) * f32(sib) / f32(k - 1)
        tf[i, y] = f32(1.0) - f32(smooth)
    coarse = parent[labels].astype(np.uint32)
    tc = np.full((len(labels), ncoarse), f32(smooth) / f32(ncoarse), f32)
    tc[np.arange(len(labels)), coarse] += f32(1.0) - f32(smooth)
    if perm is not None:  # train.rs:148-153, each product rounded before the add
        perm = np.asarray(perm, np.int64)
        lv = np.asarray(lam, f32)[:, None]
        tf = (lv * tf + (f32(1.0) - lv) * tf[perm]).astype(f32)
        tc = (lv * tc + (f32(1.0) - lv) * tc[perm]).astype(f32)
    return tf.ravel(), tc.ravel(), coarse


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return C.c_void_p(t.ctypes.data)
    return C.c_void_p(t.data_ptr())


class RustViT:
    def __init__(self, cfg: VitCfg = None, parent=None, ncoarse: int = 20, seed: int = 1234,
                 device: int | None = None):
        cfg = cfg or VitCfg()
        parent = cifar_parent() if parent is None else np.ascontiguousarray(parent, np.uint32)
        self.cfg, self.parent, self.nf, self.nc = cfg, parent, len(parent), ncoarse
        self.ctx = default_context(device)
        self.device = self.ctx.device
        cfg9 = np.array([cfg.width, cfg.cmid, cfg.dim, cfg.heads, cfg.depth3, cfg.dim4, cfg.heads4, cfg.depth4,
                         cfg.img], np.int32)
        mem = np.array(cfg.mem_at, np.int32) if cfg.mem_at else np.zeros(1, np.int32)
        h = VIT()
        check(lib().rnn_rustvit_create(self.ctx.bind(), _ptr(cfg9), _ptr(mem), len(cfg.mem_at), cfg.droppath,
                                       _ptr(parent), self.nf, ncoarse, seed & (2**64 - 1), C.byref(h)),
              "rnn_rustvit_create")
        self.h = h
        n = C.c_size_t()
        call("rnn_rustvit_num_params", self.h, C.byref(n))
        self.nparams = n.value
        call("rnn_rustvit_num_buffers", self.h, C.byref(n))
        self.nbuffers = n.value

    def close(self):
        if getattr(self, "h", None):
            lib().rnn_rustvit_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -------------------------------------------------------------- state
    def _get(self, name, n):
        self.ctx.bind()
        out = np.empty(n, np.float32)
        call(name, self.h, _ptr(out))
        return out

    def params(self):
        return self._get("rnn_rustvit_get_params", self.nparams)

    def grads(self):
        return self._get("rnn_rustvit_get_grads", self.nparams)

    def ema(self):
        return self._get("rnn_rustvit_get_ema", self.nparams)

    def buffers(self):
        return self._get("rnn_rustvit_get_buffers", self.nbuffers)

    def moments(self):
        self.ctx.bind()
        m, v2 = np.empty(self.nparams, np.float32), np.empty(self.nparams, np.float32)
        call("rnn_rustvit_get_moments", self.h, _ptr(m), _ptr(v2))
        return m, v2

    def set_params(self, v):
        v = np.ascontiguousarray(v, np.float32)
        if v.size != self.nparams:
            raise RnnError(f"set_params: expected {self.nparams} values, got {v.size}")
        self.ctx.bind()
        call("rnn_rustvit_set_params", self.h, _ptr(v))

    def zero_grads(self):
        self.ctx.bind()
        call("rnn_rustvit_zero_grads", self.h)

    # -------------------------------------------------------------- passes
    def forward(self, x: torch.Tensor, n: int, train: bool = True, drop_seed: int = 0) -> dict:
        """RustViT::forward; returns the heads as device tensors (exits only when train)."""
        dev = x.device
        d4 = self.cfg.dim4
        out = {"logits": torch.empty(n * self.nf, device=dev), "coarse": torch.empty(n * self.nc, device=dev),
               "feat": torch.empty(n * d4, device=dev)}
        if train:
            out.update(e1=torch.empty(n * self.nf, device=dev), e2=torch.empty(n * self.nf, device=dev),
                       h1=torch.empty(n * d4, device=dev), h2=torch.empty(n * d4, device=dev))
        self.ctx.bind()
        call("rnn_rustvit_forward_dev", self.h, _ptr(x), n, int(train), drop_seed & (2**64 - 1),
             _ptr(out["logits"]), _ptr(out["coarse"]), _ptr(out.get("e1")), _ptr(out.get("e2")),
             _ptr(out.get("h1")), _ptr(out.get("h2")), _ptr(out["feat"]))
        return out

    def backward(self, g: dict):
        """RustViT::backward with vit::Grads (device tensors; exits and hfinal optional)."""
        self.ctx.bind()
        call("rnn_rustvit_backward_dev", self.h, _ptr(g["logits"]), _ptr(g["coarse"]), _ptr(g.get("e1")),
             _ptr(g.get("e2")), _ptr(g.get("h1")), _ptr(g.get("h2")), _ptr(g.get("hfinal")))

    def dp_attach(self, comm):
        """Makes later train steps one rank of a batch-sharded step over
        comm (a ``dp.Comm`` on this network's device; None detaches): the
        gradient and the BatchNorm running statistics are averaged over the
        ranks inside the step.  The network keeps a borrowed reference."""
        self._comm = comm
        call("rnn_rustvit_dp_attach", self.h, comm.h if comm is not None else None)

    def train_step(self, x, tf, tc, hard, hardc, lr=6e-4, wd=0.06, clip=1.0, ema=0.9998, drop_seed=0,
                   stats=True):
        """Trainer::step on device inputs; returns (total loss, ce, correct),
        or None without waiting for the device when stats is False."""
        self.ctx.bind()
        st = np.zeros(3, np.float32)
        call("rnn_rustvit_train_step_dev", self.h, _ptr(x), _ptr(tf), _ptr(tc), _ptr(hard), _ptr(hardc),
             hard.numel(), lr, wd, clip, ema, drop_seed & (2**64 - 1), _ptr(st) if stats else None)
        return (float(st[0]), float(st[1]), int(st[2])) if stats else None

    def eval(self, images, labels, batch: int, tta: bool = False, use_ema: bool = False):
        """eval::vit (eval.rs:47-66) over a u8 CHW dataset [len, 3, 32, 32]
        with u8 labels: (mean loss, accuracy); use_ema evaluates the EMA
        weights (Trainer::eval_ema, train.rs:390-402).  Device tensors are
        read in place; host arrays go through the host tier."""
        self.ctx.bind()
        out = np.zeros(2, np.float32)
        dev = isinstance(labels, torch.Tensor) and labels.is_cuda
        n = int(labels.size) if isinstance(labels, np.ndarray) else int(labels.numel())
        call("rnn_rustvit_eval_dev" if dev else "rnn_rustvit_eval", self.h, _ptr(images), _ptr(labels), n, batch,
             int(bool(tta)), int(bool(use_ema)), _ptr(out[0:1]), _ptr(out[1:2]))
        return float(out[0]), float(out[1])

    def save(self, path: str):
        """Checkpointed::save (ckpt.rs:62-68) in the reference's format."""
        self.ctx.bind()
        call("rnn_rustvit_save", self.h, str(path).encode())

    def load(self, path: str):
        self.ctx.bind()
        call("rnn_rustvit_load", self.h, str(path).encode())

    def save_optim(self, path: str):
        """Both moments, the EMA weights and the step counters, which the
        reference's checkpoint omits."""
        self.ctx.bind()
        call("rnn_rustvit_save_optim", self.h, str(path).encode())

    def load_optim(self, path: str):
        self.ctx.bind()
        call("rnn_rustvit_load_optim", self.h, str(path).encode())

    def train_step_host(self, x, tf, tc, hard, hardc, lr=6e-4, wd=0.06, clip=1.0, ema=0.9998, drop_seed=0):
        """The same step through the host tier of the C ABI (host batch arrays)."""
        self.ctx.bind()
        stats = np.zeros(3, np.float32)
        call("rnn_rustvit_train_step", self.h, _ptr(x), _ptr(tf), _ptr(tc), _ptr(hard), _ptr(hardc), len(hard),
             lr, wd, clip, ema, drop_seed & (2**64 - 1), _ptr(stats))
        return float(stats[0]), float(stats[1]), int(stats[2])
