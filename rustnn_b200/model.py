"""The ResNet training step (model.rs ResNet, train.rs:684-699) on the GPU.

``ResNet(depth_n, width, nclass, seed)`` mirrors ``ResNet::new`` and draws
the same initial parameters.  ``train_step`` runs forward, softmax_ce,
backward, the optional data-parallel gradient allreduce and the
SGD-Nesterov update (Param::step) as one device-resident sequence.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import NET, RnnError, call, check, lib
from .ops import default_context

UID_BYTES = 128


def dp_unique_id() -> bytes:
    buf = (C.c_ubyte * UID_BYTES)()
    call("rnn_dp_unique_id", C.cast(buf, C.c_void_p))
    return bytes(buf)


def _addr(t):
    if isinstance(t, np.ndarray):
        return C.c_void_p(t.ctypes.data)
    return C.c_void_p(t.data_ptr())


def _numel(t):
    return int(t.size) if isinstance(t, np.ndarray) else int(t.numel())


class ResNet:
    def __init__(self, depth_n: int, width: int, nclass: int, seed: int, device: int | None = None):
        self.ctx = default_context(device)
        self.device = self.ctx.device
        self.depth_n, self.width, self.nclass = depth_n, width, nclass
        h = NET()
        check(lib().rnn_resnet_create(self.ctx.bind(), depth_n, width, nclass, seed & (2**64 - 1), C.byref(h)),
              "rnn_resnet_create")
        self.h = h
        n = C.c_size_t()
        call("rnn_resnet_num_params", self.h, C.byref(n))
        self.nparams = n.value
        call("rnn_resnet_num_buffers", self.h, C.byref(n))
        self.nbuffers = n.value
        self._loss = torch.zeros(1, device=f"cuda:{self.device}", dtype=torch.float32)
        self._corr = torch.zeros(1, device=f"cuda:{self.device}", dtype=torch.int32)

    def close(self):
        if getattr(self, "h", None):
            lib().rnn_resnet_destroy(self.h)
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
        call(name, self.h, C.c_void_p(out.ctypes.data))
        return out

    def params(self):
        return self._get("rnn_resnet_get_params", self.nparams)

    def grads(self):
        return self._get("rnn_resnet_get_grads", self.nparams)

    def moments(self):
        return self._get("rnn_resnet_get_moments", self.nparams)

    def buffers(self):
        return self._get("rnn_resnet_get_buffers", self.nbuffers)

    def set_params(self, v):
        v = np.ascontiguousarray(v, np.float32)
        if v.size != self.nparams:
            raise RnnError(f"set_params: expected {self.nparams} values, got {v.size}")
        self.ctx.bind()
        call("rnn_resnet_set_params", self.h, C.c_void_p(v.ctypes.data))

    def grad_buffer(self) -> tuple[int, int]:
        p, n = C.c_void_p(), C.c_size_t()
        call("rnn_resnet_grad_buffer", self.h, C.byref(p), C.byref(n))
        return p.value, n.value

    # -------------------------------------------------------------- step
    def forward(self, x: torch.Tensor, n: int, hw: int = 32, train: bool = True) -> torch.Tensor:
        logits = torch.empty(n * self.nclass, device=x.device, dtype=torch.float32)
        self.ctx.bind()
        call("rnn_resnet_forward_dev", self.h, C.c_void_p(x.data_ptr()), n, hw, hw, int(train),
             C.c_void_p(logits.data_ptr()))
        return logits

    def backward(self, dlogits: torch.Tensor):
        self.ctx.bind()
        call("rnn_resnet_backward_dev", self.h, C.c_void_p(dlogits.data_ptr()))

    def use_graph(self, enable: bool = True):
        """Replay the training step from a CUDA graph (see rnn_resnet_set_graph)."""
        call("rnn_resnet_set_graph", self.h, int(bool(enable)))

    def step(self, lr: float, mom: float, wd: float):
        self.ctx.bind()
        call("rnn_resnet_step", self.h, lr, mom, wd)

    def train_step(self, x: torch.Tensor, labels: torch.Tensor, smooth=0.1, lr=0.2, mom=0.9, wd=5e-4):
        """Device inputs; returns (loss, correct) as 1-element device tensors."""
        self.ctx.bind()
        n = labels.numel()
        call("rnn_resnet_train_step_dev", self.h, C.c_void_p(x.data_ptr()), C.c_void_p(labels.data_ptr()), n,
             smooth, lr, mom, wd, C.c_void_p(self._loss.data_ptr()), C.c_void_p(self._corr.data_ptr()))
        return self._loss, self._corr

    def train_step_host(self, x: np.ndarray, labels: np.ndarray, smooth=0.1, lr=0.2, mom=0.9, wd=5e-4):
        """Host (pinned or pageable) inputs through the host tier of the C ABI."""
        self.ctx.bind()
        loss, corr = C.c_float(), C.c_int()
        call("rnn_resnet_train_step", self.h, C.c_void_p(x.ctypes.data if isinstance(x, np.ndarray) else x.data_ptr()),
             C.c_void_p(labels.ctypes.data if isinstance(labels, np.ndarray) else labels.data_ptr()), len(labels),
             smooth, lr, mom, wd, C.c_void_p(C.addressof(loss)), C.c_void_p(C.addressof(corr)))
        return loss.value, corr.value

    def eval(self, images, labels, batch: int):
        """eval::resnet (eval.rs:41-43) over a u8 CHW dataset [len, 3, 32, 32]
        with u8 labels: (mean loss, accuracy).  Device tensors are read in
        place; host arrays go through the host tier (one copy in)."""
        self.ctx.bind()
        loss, acc = C.c_float(), C.c_float()
        name = "rnn_resnet_eval_dev" if isinstance(labels, torch.Tensor) and labels.is_cuda else "rnn_resnet_eval"
        call(name, self.h, _addr(images), _addr(labels), _numel(labels), batch,
             C.c_void_p(C.addressof(loss)), C.c_void_p(C.addressof(acc)))
        return loss.value, acc.value

    def save(self, path: str):
        """Checkpointed::save (ckpt.rs:62-68) in the reference's format."""
        self.ctx.bind()
        call("rnn_resnet_save", self.h, str(path).encode())

    def load(self, path: str):
        """Checkpointed::load (ckpt.rs:70-76)."""
        self.ctx.bind()
        call("rnn_resnet_load", self.h, str(path).encode())

    def save_optim(self, path: str):
        """The SGD momentum, which the reference's checkpoint omits."""
        self.ctx.bind()
        call("rnn_resnet_save_optim", self.h, str(path).encode())

    def load_optim(self, path: str):
        self.ctx.bind()
        call("rnn_resnet_load_optim", self.h, str(path).encode())

    def dp_init(self, rank: int, world: int, uid: bytes, sync_bn: bool = True):
        buf = (C.c_ubyte * UID_BYTES).from_buffer_copy(uid)
        call("rnn_resnet_dp_init", self.h, rank, world, C.cast(buf, C.c_void_p), int(sync_bn))
