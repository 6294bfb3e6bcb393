"""Loads librnn_b200.so and declares its C ABI (include/rnn_b200.h).

The product path has no fallback: if the library is missing or the device is
not an sm_100a part, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "librnn_b200.so")

RNN_OK = 0
ERRORS = {-1: "RNN_ERR_ARG", -2: "RNN_ERR_CUDA", -3: "RNN_ERR_NCCL", -4: "RNN_ERR_DEVICE", -5: "RNN_ERR_UNSUPPORTED",
          -6: "RNN_ERR_IO"}

_lock = threading.Lock()
_lib = None

I, F, Z, U64, P = C.c_int, C.c_float, C.c_size_t, C.c_uint64, C.c_void_p
FP = C.c_void_p  # device or host float pointer, passed as an integer address


class _CtxS(C.Structure):
    """opaque rnn_ctx"""


class _NetS(C.Structure):
    """opaque rnn_resnet"""


class _VitS(C.Structure):
    """opaque rnn_rustvit"""


# distinct handle types: ctypes rejects a context where a network is expected
CTX = C.POINTER(_CtxS)
NET = C.POINTER(_NetS)
VIT = C.POINTER(_VitS)

# name -> argtypes; every function returns int unless listed in _RESTYPE
SIGS = {
    "rnn_device_ok": [I],
    "rnn_launch_count": [],
    "rnn_ctx_create": [C.POINTER(CTX), I],
    "rnn_ctx_destroy": [CTX],
    "rnn_ctx_set_stream": [CTX, P],
    "rnn_ctx_use_own_stream": [CTX],
    "rnn_ctx_stream": [CTX],
    "rnn_ctx_synchronize": [CTX],
    "rnn_gemm_dev": [CTX, I, I, I, FP, I, FP, I, FP, I],
    "rnn_gemm": [CTX, I, I, I, FP, I, FP, I, FP, I],
    "rnn_gemm_dw_dev": [CTX, I, I, I, FP, FP, FP],
    "rnn_gemm_dw": [CTX, I, I, I, FP, FP, FP],
    "rnn_gemm_dw_noalloc_dev": [I, I, I, FP, FP, FP, P],
    "rnn_gemm_dw_noalloc_status": [P],
    "rnn_layernorm_res_fwd_dev": [CTX, FP, FP, FP, I, I, FP, FP, F, FP, FP, FP, FP, FP],
    "rnn_linear_fwd_packed_dev": [CTX, FP, I, I, I, FP, FP, FP],
    "rnn_swiglu_fwd_dev": [CTX, FP, FP, I, I, I, FP, FP, FP, FP],
    "rnn_batchnorm_stats_peer_dev": [CTX, FP, I, I, I, I, I, P, P, I, I, P],
    "rnn_peer_mailbox_bytes": [I],
    "rnn_alloc": [CTX, Z, P],
    "rnn_free": [CTX, P],
    "rnn_memcpy_h2d": [CTX, P, P, Z],
    "rnn_memcpy_d2h": [CTX, P, P, Z],
    "rnn_comm_init": [P, I, I, I, P],
    "rnn_comm_destroy": [P],
    "rnn_allreduce_grads": [CTX, P, P, Z, I],
    "rnn_comm_check": [P],
    "rnn_comm_abort": [P],
    "rnn_comm_wait": [CTX, P, I],
    "rnn_resnet_comm": [NET, P],
    "rnn_conv2d_fwd_dev": [CTX, FP, I, I, I, I, FP, I, I, I, I, FP, I],
    "rnn_conv2d_fwd": [CTX, FP, I, I, I, I, FP, I, I, I, I, FP],
    "rnn_conv2d_dgrad_dev": [CTX, FP, I, I, I, I, FP, I, I, I, I, FP, I],
    "rnn_conv2d_dgrad": [CTX, FP, I, I, I, I, FP, I, I, I, I, FP],
    "rnn_conv2d_wgrad_dev": [CTX, FP, FP, I, I, I, I, I, I, I, I, FP],
    "rnn_conv2d_wgrad": [CTX, FP, FP, I, I, I, I, I, I, I, I, FP],
    "rnn_batchnorm_fwd_dev": [CTX, FP, I, I, I, FP, FP, FP, FP, F, F, I, FP, FP, FP],
    "rnn_batchnorm_eval_dev": [CTX, FP, I, I, I, FP, FP, FP, FP, F, I, FP],
    "rnn_batchnorm_bwd_dev": [CTX, FP, FP, I, I, I, FP, FP, FP, FP, FP, FP, FP],
    "rnn_relu_back_dev": [CTX, FP, FP, Z],
    "rnn_add_dev": [CTX, FP, FP, Z],
    "rnn_add_relu_dev": [CTX, FP, FP, Z],
    "rnn_gap_fwd_dev": [CTX, FP, I, I, FP],
    "rnn_gap_bwd_dev": [CTX, FP, I, I, FP],
    "rnn_softmax_ce_dev": [CTX, FP, FP, I, I, F, FP, FP, FP],
    "rnn_sgd_nesterov_dev": [CTX, FP, FP, FP, Z, F, F, F, I],
    "rnn_rel_index": [I, I, I, I, P, C.POINTER(I)],
    "rnn_attn_fwd_dev": [CTX, I, I, I, I, I, I, I, I, FP, I, I, FP, I, I, I, FP, FP, FP, FP],
    "rnn_attn_bwd_dev": [CTX, I, I, I, I, I, I, I, FP, I, I, FP, I, I, I, FP, FP, FP, FP, FP, FP, FP],
    "rnn_layernorm_fwd_dev": [CTX, FP, I, I, FP, FP, F, FP, FP, FP],
    "rnn_layernorm_bwd_dev": [CTX, FP, FP, FP, I, I, FP, FP, FP, FP],
    "rnn_linear_fwd_dev": [CTX, FP, I, I, I, FP, FP, FP],
    "rnn_linear_bwd_dev": [CTX, FP, FP, I, I, I, FP, FP, FP, FP],
    "rnn_newton_schulz_dev": [CTX, FP, I, I, I],
    "rnn_muon_step_dev": [CTX, FP, FP, FP, I, I, I, F, F, F, I],
    "rnn_adamw_step_dev": [CTX, FP, FP, FP, FP, Z, F, F, I, F, F, F, I],
    "rnn_clip_dev": [CTX, FP, Z, F, FP],
    "rnn_ema_update_dev": [CTX, FP, FP, Z, F, I],
    "rnn_layerscale_fwd_dev": [CTX, FP, I, I, FP, FP],
    "rnn_layerscale_bwd_dev": [CTX, FP, FP, I, I, FP, FP, FP],
    "rnn_swiglu_act_fwd_dev": [CTX, FP, I, I, FP],
    "rnn_swiglu_act_bwd_dev": [CTX, FP, FP, I, I, FP],
    "rnn_dwconv3_fwd_dev": [CTX, FP, I, I, I, I, FP, FP, FP],
    "rnn_dwconv3_bwd_dev": [CTX, FP, FP, I, I, I, I, FP, FP, FP, FP],
    "rnn_seqpool_fwd_dev": [CTX, FP, I, I, I, FP, FP, FP],
    "rnn_seqpool_bwd_dev": [CTX, FP, FP, FP, I, I, I, FP, FP, FP],
    "rnn_droppath_fwd_dev": [CTX, FP, I, Z, F, U64, FP],
    "rnn_droppath_bwd_dev": [CTX, FP, I, Z, FP],
    "rnn_token_merge_dev": [CTX, FP, I, I, I, FP, I],
    "rnn_tok_layout_dev": [CTX, FP, I, I, I, FP, I],
    "rnn_taxo_combine_fwd_dev": [CTX, FP, FP, I, I, I, FP],
    "rnn_taxo_combine_bwd_dev": [CTX, FP, FP, I, I, I, FP, FP],
    "rnn_ce_soft_dev": [CTX, FP, FP, FP, I, I, F, FP, FP, FP],
    "rnn_kl_distill_dev": [CTX, FP, FP, I, I, F, F, FP, FP],
    "rnn_hint_mse_dev": [CTX, FP, FP, I, I, F, FP, FP],
    "rnn_attn_fwd": [CTX, I, I, I, I, I, I, I, I, FP, I, I, FP, I, I, I, FP, FP, FP, FP],
    "rnn_attn_bwd": [CTX, I, I, I, I, I, I, I, FP, I, I, FP, I, I, I, FP, FP, FP, FP, FP, FP, FP],
    "rnn_layernorm_fwd": [CTX, FP, I, I, FP, FP, F, FP, FP, FP],
    "rnn_layernorm_bwd": [CTX, FP, FP, FP, I, I, FP, FP, FP, FP],
    "rnn_linear_fwd": [CTX, FP, I, I, I, FP, FP, FP],
    "rnn_linear_bwd": [CTX, FP, FP, I, I, I, FP, FP, FP, FP],
    "rnn_batchnorm_fwd": [CTX, FP, I, I, I, FP, FP, FP, FP, F, F, I, FP, FP, FP],
    "rnn_batchnorm_bwd": [CTX, FP, FP, I, I, I, FP, FP, FP, FP, FP, FP, FP],
    "rnn_newton_schulz_batched_dev": [CTX, I, P, P, P, I],
    "rnn_newton_schulz_batched": [CTX, I, P, P, P, I],
    "rnn_muon_step": [CTX, FP, FP, FP, I, I, I, F, F, F, I],
    "rnn_adamw_step": [CTX, FP, FP, FP, FP, Z, F, F, I, F, F, F, I],
    "rnn_sgd_nesterov": [CTX, FP, FP, FP, Z, F, F, F, I],
    "rnn_clip": [CTX, FP, Z, F, FP],
    "rnn_ema_update": [CTX, FP, FP, Z, F, I],
    "rnn_resnet_create": [CTX, I, I, I, U64, C.POINTER(NET)],
    "rnn_resnet_destroy": [NET],
    "rnn_resnet_num_params": [NET, C.POINTER(Z)],
    "rnn_resnet_num_buffers": [NET, C.POINTER(Z)],
    "rnn_resnet_get_params": [NET, FP],
    "rnn_resnet_set_params": [NET, FP],
    "rnn_resnet_get_grads": [NET, FP],
    "rnn_resnet_get_moments": [NET, FP],
    "rnn_resnet_get_buffers": [NET, FP],
    "rnn_resnet_grad_buffer": [NET, C.POINTER(P), C.POINTER(Z)],
    "rnn_resnet_forward_dev": [NET, FP, I, I, I, I, FP],
    "rnn_resnet_backward_dev": [NET, FP],
    "rnn_resnet_step": [NET, F, F, F],
    "rnn_resnet_set_graph": [NET, I],
    "rnn_resnet_train_step_dev": [NET, FP, FP, I, F, F, F, F, FP, FP],
    "rnn_resnet_train_step": [NET, FP, FP, I, F, F, F, F, FP, FP],
    "rnn_dp_unique_id": [FP],
    "rnn_resnet_dp_init": [NET, I, I, FP, I],
    "rnn_rustvit_create": [CTX, FP, FP, I, F, FP, I, I, U64, C.POINTER(VIT)],
    "rnn_rustvit_destroy": [VIT],
    "rnn_rustvit_num_params": [VIT, C.POINTER(Z)],
    "rnn_rustvit_num_buffers": [VIT, C.POINTER(Z)],
    "rnn_rustvit_get_params": [VIT, FP],
    "rnn_rustvit_set_params": [VIT, FP],
    "rnn_rustvit_get_grads": [VIT, FP],
    "rnn_rustvit_get_moments": [VIT, FP, FP],
    "rnn_rustvit_get_ema": [VIT, FP],
    "rnn_rustvit_get_buffers": [VIT, FP],
    "rnn_rustvit_zero_grads": [VIT],
    "rnn_rustvit_forward_dev": [VIT, FP, I, I, U64, FP, FP, FP, FP, FP, FP, FP],
    "rnn_rustvit_backward_dev": [VIT, FP, FP, FP, FP, FP, FP, FP],
    "rnn_rustvit_train_step_dev": [VIT, FP, FP, FP, FP, FP, I, F, F, F, F, U64, FP],
    "rnn_rustvit_train_step": [VIT, FP, FP, FP, FP, FP, I, F, F, F, F, U64, FP],
    "rnn_rustvit_dp_attach": [VIT, P],
    "rnn_make_batch_eval_dev": [CTX, FP, FP, Z, Z, I, I, FP, FP],
    "rnn_make_batch_train_dev": [CTX, FP, FP, FP, Z, FP, I, I, F, I, F, I, U64, FP, FP, FP],
    "rnn_mix_batch_dev": [CTX, FP, I, F, F, F, FP, FP, FP],
    "rnn_ckpt_config_hash": [C.c_char_p, Z, FP, Z],
    "rnn_ckpt_write": [C.c_char_p, C.c_uint32, U64, FP, Z],
    "rnn_ckpt_read": [C.c_char_p, C.c_uint32, U64, FP, Z],
    "rnn_resnet_save": [NET, C.c_char_p],
    "rnn_resnet_load": [NET, C.c_char_p],
    "rnn_resnet_save_optim": [NET, C.c_char_p],
    "rnn_resnet_load_optim": [NET, C.c_char_p],
    "rnn_rustvit_save": [VIT, C.c_char_p],
    "rnn_rustvit_load": [VIT, C.c_char_p],
    "rnn_rustvit_save_optim": [VIT, C.c_char_p],
    "rnn_rustvit_load_optim": [VIT, C.c_char_p],
    "rnn_resnet_eval_dev": [NET, FP, FP, I, I, FP, FP],
    "rnn_resnet_eval": [NET, FP, FP, I, I, FP, FP],
    "rnn_rustvit_eval_dev": [VIT, FP, FP, I, I, I, I, FP, FP],
    "rnn_rustvit_eval": [VIT, FP, FP, I, I, I, I, FP, FP],
}
_RESTYPE = {
    "rnn_ctx_stream": P,
    "rnn_launch_count": C.c_ulonglong,
    "rnn_ckpt_config_hash": C.c_uint64,
    "rnn_peer_mailbox_bytes": C.c_size_t,
}


class RnnError(RuntimeError):
    pass


def lib():
    """The loaded library; raises if it was not built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RnnError(
                f"{LIB_PATH} is missing: build it with `python -m rustnn_b200.build` (there is no CPU fallback)"
            )
        L = C.CDLL(LIB_PATH)
        L.rnn_last_error.restype = C.c_char_p
        L.rnn_last_error.argtypes = []
        for name, args in SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _RESTYPE.get(name, C.c_int)
        _lib = L
        return L


def check(code: int, what: str = "") -> None:
    if code != RNN_OK:
        msg = lib().rnn_last_error().decode(errors="replace")
        raise RnnError(f"{what}: {ERRORS.get(code, code)}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
