"""Batch construction on the device: data::make_batch_train (data.rs:384-412),
data::make_batch_eval (data.rs:494-512) and data::mix_batch (data.rs:467-491).

The dataset lives on the device as data::Dataset's bytes (data.rs:16-24):
``images`` u8 [len, 3, 32, 32] (CHW), ``labels`` / ``coarse`` u8 [len]."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import call
from .ops import default_context

PIX = 3 * 32 * 32


@dataclass
class Aug:
    """data::Aug (data.rs:281-304); the defaults are Aug::default."""
    pad: int = 4
    ra_mag: float = 0.0
    ra_n: int = 2
    erase: float = 0.0
    erase_side: int = 8


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def make_batch_train(images: torch.Tensor, labels: torch.Tensor, coarse: torch.Tensor | None, idx: torch.Tensor,
                     aug: Aug, seed: int, out: torch.Tensor | None = None, labels_out: torch.Tensor | None = None):
    """Returns (x [bs*3072] f32, labels u32 as int32, coarse or None), all on
    the device; idx holds the dataset indices (int32 / uint32)."""
    ctx = default_context()
    ctx.bind()
    bs = idx.numel()
    dev = images.device
    out = torch.empty(bs * PIX, dtype=torch.float32, device=dev) if out is None else out
    lab = torch.empty(bs, dtype=torch.int32, device=dev) if labels_out is None else labels_out
    co = None if coarse is None else torch.empty(bs, dtype=torch.int32, device=dev)
    call("rnn_make_batch_train_dev", ctx.h, _p(images), _p(labels), _p(coarse), labels.numel(), _p(idx), bs,
         aug.pad, aug.ra_mag,
         aug.ra_n, aug.erase, aug.erase_side, seed & (2**64 - 1), _p(out), _p(lab), _p(co))
    return out, lab, co


def make_batch_eval(images: torch.Tensor, labels: torch.Tensor, start: int, bs: int, flip: bool,
                    out: torch.Tensor | None = None):
    ctx = default_context()
    ctx.bind()
    out = torch.empty(bs * PIX, dtype=torch.float32, device=images.device) if out is None else out
    lab = torch.empty(bs, dtype=torch.int32, device=images.device)
    call("rnn_make_batch_eval_dev", ctx.h, _p(images), _p(labels), labels.numel(), start, bs, int(flip), _p(out),
         _p(lab))
    return out, lab


def mix_batch(x: torch.Tensor, bs: int, alpha_mix: float, alpha_cut: float, sw: float, state: np.ndarray):
    """In place on the device batch x; state = the caller's xoshiro256++ words
    (numpy uint64[4]), advanced.  Returns (perm, lam) as numpy arrays."""
    ctx = default_context()
    ctx.bind()
    assert state.dtype == np.uint64 and state.flags["C_CONTIGUOUS"] and state.size == 4
    perm = np.empty(bs, np.uint32)
    lam = np.empty(bs, np.float32)
    call("rnn_mix_batch_dev", ctx.h, _p(x), bs, alpha_mix, alpha_cut, sw, C.c_void_p(state.ctypes.data),
         C.c_void_p(perm.ctypes.data), C.c_void_p(lam.ctypes.data))
    return perm, lam
