//! Raw bindings to `librnn_b200.so`, the B200 (sm_100a) backend of rustnn's
//! dense-contraction path.  Every item mirrors a declaration of
//! `include/rnn_b200.h` (C ABI): device pointers on the `_dev` entries, host
//! pointers on the others, an `int` status (0 or a negative `RNN_ERR_*`) from
//! every call.  `check` turns a status into a `Result` carrying
//! `rnn_last_error()`.
//!
//! The reference crate swaps the bodies of its operators for these calls and
//! keeps its signatures: `gemm::matmul` (gemm.rs:434) -> `rnn_gemm`,
//! `gemm::matmul_dw` (gemm.rs:555) -> `rnn_gemm_dw`, `Conv2d::forward /
//! backward_w / backward` (nn.rs:166, 193, 230) -> `rnn_conv2d_*`,
//! `Core::forward / backward` (attn.rs:148, 226) -> `rnn_attn_*`, the
//! training steps (train.rs:346-387, 684-699) -> `rnn_rustvit_train_step` /
//! `rnn_resnet_train_step`.
#![allow(non_camel_case_types)]

use std::ffi::CStr;
use std::os::raw::{c_char, c_int, c_void};

pub const RNN_OK: c_int = 0;
pub const RNN_ERR_ARG: c_int = -1;
pub const RNN_ERR_CUDA: c_int = -2;
pub const RNN_ERR_NCCL: c_int = -3;
pub const RNN_ERR_DEVICE: c_int = -4;
pub const RNN_ERR_UNSUPPORTED: c_int = -5;
pub const RNN_ERR_IO: c_int = -6;
pub const RNN_UID_BYTES: usize = 128;

#[repr(C)]
pub struct RnnCtx {
    _p: [u8; 0],
}
#[repr(C)]
pub struct RnnResnet {
    _p: [u8; 0],
}
#[repr(C)]
pub struct RnnRustvit {
    _p: [u8; 0],
}
#[repr(C)]
pub struct RnnComm {
    _p: [u8; 0],
}

extern "C" {
    pub fn rnn_last_error() -> *const c_char;
    pub fn rnn_launch_count() -> u64;
    pub fn rnn_device_ok(device: c_int) -> c_int;
    pub fn rnn_ctx_create(out: *mut *mut RnnCtx, device: c_int) -> c_int;
    pub fn rnn_ctx_destroy(ctx: *mut RnnCtx) -> c_int;
    pub fn rnn_ctx_set_stream(ctx: *mut RnnCtx, cuda_stream: *mut c_void) -> c_int;
    pub fn rnn_ctx_use_own_stream(ctx: *mut RnnCtx) -> c_int;
    pub fn rnn_ctx_stream(ctx: *mut RnnCtx) -> *mut c_void;
    pub fn rnn_ctx_synchronize(ctx: *mut RnnCtx) -> c_int;
    pub fn rnn_gemm_dev(ctx: *mut RnnCtx, m: c_int, n: c_int, k: c_int, a: *const f32, at: c_int, b: *const f32, bt: c_int, c: *mut f32, acc: c_int) -> c_int;
    pub fn rnn_gemm(ctx: *mut RnnCtx, m: c_int, n: c_int, k: c_int, a: *const f32, at: c_int, b: *const f32, bt: c_int, c: *mut f32, acc: c_int) -> c_int;
    pub fn rnn_gemm_dw_dev(ctx: *mut RnnCtx, m: c_int, n: c_int, k: c_int, a: *const f32, b: *const f32, c: *mut f32) -> c_int;
    pub fn rnn_gemm_dw(ctx: *mut RnnCtx, m: c_int, n: c_int, k: c_int, a: *const f32, b: *const f32, c: *mut f32) -> c_int;
    pub fn rnn_gemm_dw_noalloc_dev(m: c_int, n: c_int, k: c_int, a: *const f32, b: *const f32, c: *mut f32, cuda_stream: *mut c_void) -> c_int;
    pub fn rnn_gemm_dw_noalloc_status(cuda_stream: *mut c_void) -> c_int;
    pub fn rnn_conv2d_fwd_dev(ctx: *mut RnnCtx, x: *const f32, n: c_int, cin: c_int, h: c_int, w: c_int, wt: *const f32, cout: c_int, k: c_int, stride: c_int, pad: c_int, y: *mut f32, acc: c_int) -> c_int;
    pub fn rnn_conv2d_fwd(ctx: *mut RnnCtx, x: *const f32, n: c_int, cin: c_int, h: c_int, w: c_int, wt: *const f32, cout: c_int, k: c_int, stride: c_int, pad: c_int, y: *mut f32) -> c_int;
    pub fn rnn_conv2d_dgrad_dev(ctx: *mut RnnCtx, dy: *const f32, n: c_int, cin: c_int, h: c_int, w: c_int, wt: *const f32, cout: c_int, k: c_int, stride: c_int, pad: c_int, dx: *mut f32, acc: c_int) -> c_int;
    pub fn rnn_conv2d_dgrad(ctx: *mut RnnCtx, dy: *const f32, n: c_int, cin: c_int, h: c_int, w: c_int, wt: *const f32, cout: c_int, k: c_int, stride: c_int, pad: c_int, dx: *mut f32) -> c_int;
    pub fn rnn_conv2d_wgrad_dev(ctx: *mut RnnCtx, x: *const f32, dy: *const f32, n: c_int, cin: c_int, h: c_int, w: c_int, cout: c_int, k: c_int, stride: c_int, pad: c_int, dw: *mut f32) -> c_int;
    pub fn rnn_conv2d_wgrad(ctx: *mut RnnCtx, x: *const f32, dy: *const f32, n: c_int, cin: c_int, h: c_int, w: c_int, cout: c_int, k: c_int, stride: c_int, pad: c_int, dw: *mut f32) -> c_int;
    pub fn rnn_batchnorm_fwd_dev(ctx: *mut RnnCtx, y: *const f32, n: c_int, c: c_int, hw: c_int, gamma: *const f32, beta: *const f32, rmean: *mut f32, rvar: *mut f32, mom: f32, eps: f32, relu: c_int, mean: *mut f32, invstd: *mut f32, out: *mut f32) -> c_int;
    pub fn rnn_batchnorm_eval_dev(ctx: *mut RnnCtx, y: *const f32, n: c_int, c: c_int, hw: c_int, gamma: *const f32, beta: *const f32, rmean: *const f32, rvar: *const f32, eps: f32, relu: c_int, out: *mut f32) -> c_int;
    pub fn rnn_batchnorm_bwd_dev(ctx: *mut RnnCtx, dy: *const f32, y: *const f32, n: c_int, c: c_int, hw: c_int, gamma: *const f32, mean: *const f32, invstd: *const f32, relu_out: *const f32, dx: *mut f32, dgamma: *mut f32, dbeta: *mut f32) -> c_int;
    pub fn rnn_batchnorm_stats_peer_dev(ctx: *mut RnnCtx, y: *const f32, n: c_int, c: c_int, hw: c_int, rank: c_int, world: c_int, mailboxes: *const *mut c_void, seq: *mut u64, cmax: c_int, wait_ms: c_int, sums: *mut f64) -> c_int;
    pub fn rnn_peer_mailbox_bytes(cmax: c_int) -> usize;
    pub fn rnn_relu_back_dev(ctx: *mut RnnCtx, d: *mut f32, y: *const f32, len: usize) -> c_int;
    pub fn rnn_add_dev(ctx: *mut RnnCtx, a: *mut f32, b: *const f32, len: usize) -> c_int;
    pub fn rnn_add_relu_dev(ctx: *mut RnnCtx, a: *mut f32, b: *const f32, len: usize) -> c_int;
    pub fn rnn_gap_fwd_dev(ctx: *mut RnnCtx, x: *const f32, nc: c_int, hw: c_int, y: *mut f32) -> c_int;
    pub fn rnn_gap_bwd_dev(ctx: *mut RnnCtx, dy: *const f32, nc: c_int, hw: c_int, dx: *mut f32) -> c_int;
    pub fn rnn_softmax_ce_dev(ctx: *mut RnnCtx, logits: *const f32, labels: *const u32, n: c_int, nclass: c_int, smooth: f32, dlogits: *mut f32, loss_out: *mut f32, correct_out: *mut c_int) -> c_int;
    pub fn rnn_sgd_nesterov_dev(ctx: *mut RnnCtx, v: *mut f32, g: *mut f32, m: *mut f32, len: usize, lr: f32, mom: f32, wd: f32, decay: c_int) -> c_int;
    pub fn rnn_rel_index(th: c_int, tw: c_int, mh: c_int, mw: c_int, idx: *mut u32, nrel: *mut c_int) -> c_int;
    pub fn rnn_attn_fwd_dev(ctx: *mut RnnCtx, n: c_int, h: c_int, dh: c_int, th: c_int, tw: c_int, mh: c_int, mw: c_int, mask_diag: c_int, q: *const f32, qstride: c_int, qoff: c_int, kv: *const f32, kvstride: c_int, koff: c_int, voff: c_int, tau: *const f32, rel: *const f32, p: *mut f32, o: *mut f32) -> c_int;
    pub fn rnn_attn_bwd_dev(ctx: *mut RnnCtx, n: c_int, h: c_int, dh: c_int, th: c_int, tw: c_int, mh: c_int, mw: c_int, q: *const f32, qstride: c_int, qoff: c_int, kv: *const f32, kvstride: c_int, koff: c_int, voff: c_int, tau: *const f32, p: *const f32, dout: *const f32, dq: *mut f32, dkv: *mut f32, dtau: *mut f32, drel: *mut f32) -> c_int;
    pub fn rnn_layernorm_fwd_dev(ctx: *mut RnnCtx, x: *const f32, rows: c_int, c: c_int, gamma: *const f32, beta: *const f32, eps: f32, y: *mut f32, xhat: *mut f32, invstd: *mut f32) -> c_int;
    pub fn rnn_layernorm_bwd_dev(ctx: *mut RnnCtx, dy: *const f32, xhat: *const f32, invstd: *const f32, rows: c_int, c: c_int, gamma: *const f32, dx: *mut f32, dgamma: *mut f32, dbeta: *mut f32) -> c_int;
    pub fn rnn_linear_fwd_dev(ctx: *mut RnnCtx, x: *const f32, rows: c_int, fin: c_int, fout: c_int, w: *const f32, b: *const f32, y: *mut f32) -> c_int;
    pub fn rnn_linear_bwd_dev(ctx: *mut RnnCtx, x: *const f32, dy: *const f32, rows: c_int, fin: c_int, fout: c_int, w: *const f32, dw: *mut f32, db: *mut f32, dx: *mut f32) -> c_int;
    pub fn rnn_newton_schulz_dev(ctx: *mut RnnCtx, g: *mut f32, rows: c_int, cols: c_int, steps: c_int) -> c_int;
    pub fn rnn_muon_step_dev(ctx: *mut RnnCtx, v: *mut f32, g: *mut f32, m: *mut f32, rows: c_int, cols: c_int, steps: c_int, lr: f32, mom: f32, wd: f32, decay: c_int) -> c_int;
    pub fn rnn_adamw_step_dev(ctx: *mut RnnCtx, v: *mut f32, g: *mut f32, m: *mut f32, v2: *mut f32, n: usize, lr: f32, wd: f32, decay: c_int, b1: f32, b2: f32, eps: f32, t: c_int) -> c_int;
    pub fn rnn_clip_dev(ctx: *mut RnnCtx, g: *mut f32, n: usize, max: f32, norm_out: *mut f32) -> c_int;
    pub fn rnn_ema_update_dev(ctx: *mut RnnCtx, e: *mut f32, v: *const f32, n: usize, decay: f32, t: c_int) -> c_int;
    pub fn rnn_layerscale_fwd_dev(ctx: *mut RnnCtx, x: *const f32, rows: c_int, c: c_int, l: *const f32, y: *mut f32) -> c_int;
    pub fn rnn_layerscale_bwd_dev(ctx: *mut RnnCtx, dy: *const f32, x: *const f32, rows: c_int, c: c_int, l: *const f32, dl: *mut f32, dx: *mut f32) -> c_int;
    pub fn rnn_swiglu_act_fwd_dev(ctx: *mut RnnCtx, ab: *const f32, rows: c_int, h: c_int, u: *mut f32) -> c_int;
    pub fn rnn_swiglu_act_bwd_dev(ctx: *mut RnnCtx, du: *const f32, ab: *const f32, rows: c_int, h: c_int, dab: *mut f32) -> c_int;
    pub fn rnn_dwconv3_fwd_dev(ctx: *mut RnnCtx, x: *const f32, n: c_int, th: c_int, tw: c_int, c: c_int, w: *const f32, b: *const f32, y: *mut f32) -> c_int;
    pub fn rnn_dwconv3_bwd_dev(ctx: *mut RnnCtx, dy: *const f32, x: *const f32, n: c_int, th: c_int, tw: c_int, c: c_int, w: *const f32, dw: *mut f32, db: *mut f32, dx: *mut f32) -> c_int;
    pub fn rnn_seqpool_fwd_dev(ctx: *mut RnnCtx, x: *const f32, n: c_int, t: c_int, c: c_int, p: *const f32, z: *mut f32, w: *mut f32) -> c_int;
    pub fn rnn_seqpool_bwd_dev(ctx: *mut RnnCtx, dz: *const f32, x: *const f32, w: *const f32, n: c_int, t: c_int, c: c_int, p: *const f32, dp: *mut f32, dx: *mut f32) -> c_int;
    pub fn rnn_droppath_fwd_dev(ctx: *mut RnnCtx, x: *mut f32, n: c_int, per_image: usize, p: f32, seed: u64, mask: *mut f32) -> c_int;
    pub fn rnn_droppath_bwd_dev(ctx: *mut RnnCtx, dy: *mut f32, n: c_int, per_image: usize, mask: *const f32) -> c_int;
    pub fn rnn_token_merge_dev(ctx: *mut RnnCtx, src: *const f32, n: c_int, th: c_int, c: c_int, dst: *mut f32, backward: c_int) -> c_int;
    pub fn rnn_tok_layout_dev(ctx: *mut RnnCtx, r#in: *const f32, n: c_int, c: c_int, hw: c_int, out: *mut f32, to_nchw: c_int) -> c_int;
    pub fn rnn_taxo_combine_fwd_dev(ctx: *mut RnnCtx, zf: *mut f32, zc: *const f32, n: c_int, nf: c_int, nc: c_int, parent: *const u32) -> c_int;
    pub fn rnn_taxo_combine_bwd_dev(ctx: *mut RnnCtx, dzf: *const f32, dzc: *const f32, n: c_int, nf: c_int, nc: c_int, parent: *const u32, dc: *mut f32) -> c_int;
    pub fn rnn_ce_soft_dev(ctx: *mut RnnCtx, logits: *const f32, target: *const f32, hard: *const u32, n: c_int, nclass: c_int, scale: f32, dz: *mut f32, loss_out: *mut f32, correct_out: *mut c_int) -> c_int;
    pub fn rnn_kl_distill_dev(ctx: *mut RnnCtx, student: *const f32, teacher: *const f32, n: c_int, nclass: c_int, temp: f32, scale: f32, dz: *mut f32, loss_out: *mut f32) -> c_int;
    pub fn rnn_hint_mse_dev(ctx: *mut RnnCtx, pred: *const f32, target: *const f32, n: c_int, c: c_int, scale: f32, dz: *mut f32, loss_out: *mut f32) -> c_int;
    pub fn rnn_attn_fwd(ctx: *mut RnnCtx, n: c_int, h: c_int, dh: c_int, th: c_int, tw: c_int, mh: c_int, mw: c_int, mask_diag: c_int, q: *const f32, qstride: c_int, qoff: c_int, kv: *const f32, kvstride: c_int, koff: c_int, voff: c_int, tau: *const f32, rel: *const f32, p: *mut f32, o: *mut f32) -> c_int;
    pub fn rnn_attn_bwd(ctx: *mut RnnCtx, n: c_int, h: c_int, dh: c_int, th: c_int, tw: c_int, mh: c_int, mw: c_int, q: *const f32, qstride: c_int, qoff: c_int, kv: *const f32, kvstride: c_int, koff: c_int, voff: c_int, tau: *const f32, p: *const f32, dout: *const f32, dq: *mut f32, dkv: *mut f32, dtau: *mut f32, drel: *mut f32) -> c_int;
    pub fn rnn_layernorm_fwd(ctx: *mut RnnCtx, x: *const f32, rows: c_int, c: c_int, gamma: *const f32, beta: *const f32, eps: f32, y: *mut f32, xhat: *mut f32, invstd: *mut f32) -> c_int;
    pub fn rnn_layernorm_bwd(ctx: *mut RnnCtx, dy: *const f32, xhat: *const f32, invstd: *const f32, rows: c_int, c: c_int, gamma: *const f32, dx: *mut f32, dgamma: *mut f32, dbeta: *mut f32) -> c_int;
    pub fn rnn_linear_fwd(ctx: *mut RnnCtx, x: *const f32, rows: c_int, fin: c_int, fout: c_int, w: *const f32, b: *const f32, y: *mut f32) -> c_int;
    pub fn rnn_linear_bwd(ctx: *mut RnnCtx, x: *const f32, dy: *const f32, rows: c_int, fin: c_int, fout: c_int, w: *const f32, dw: *mut f32, db: *mut f32, dx: *mut f32) -> c_int;
    pub fn rnn_batchnorm_fwd(ctx: *mut RnnCtx, y: *const f32, n: c_int, c: c_int, hw: c_int, gamma: *const f32, beta: *const f32, rmean: *mut f32, rvar: *mut f32, mom: f32, eps: f32, relu: c_int, mean: *mut f32, invstd: *mut f32, out: *mut f32) -> c_int;
    pub fn rnn_batchnorm_bwd(ctx: *mut RnnCtx, dy: *const f32, y: *const f32, n: c_int, c: c_int, hw: c_int, gamma: *const f32, mean: *const f32, invstd: *const f32, relu_out: *const f32, dx: *mut f32, dgamma: *mut f32, dbeta: *mut f32) -> c_int;
    pub fn rnn_newton_schulz_batched_dev(ctx: *mut RnnCtx, count: c_int, g: *const *mut f32, rows: *const c_int, cols: *const c_int, steps: c_int) -> c_int;
    pub fn rnn_newton_schulz_batched(ctx: *mut RnnCtx, count: c_int, g: *const *mut f32, rows: *const c_int, cols: *const c_int, steps: c_int) -> c_int;
    pub fn rnn_muon_step(ctx: *mut RnnCtx, v: *mut f32, g: *mut f32, m: *mut f32, rows: c_int, cols: c_int, steps: c_int, lr: f32, mom: f32, wd: f32, decay: c_int) -> c_int;
    pub fn rnn_adamw_step(ctx: *mut RnnCtx, v: *mut f32, g: *mut f32, m: *mut f32, v2: *mut f32, n: usize, lr: f32, wd: f32, decay: c_int, b1: f32, b2: f32, eps: f32, t: c_int) -> c_int;
    pub fn rnn_sgd_nesterov(ctx: *mut RnnCtx, v: *mut f32, g: *mut f32, m: *mut f32, len: usize, lr: f32, mom: f32, wd: f32, decay: c_int) -> c_int;
    pub fn rnn_clip(ctx: *mut RnnCtx, g: *mut f32, n: usize, max: f32, norm_out: *mut f32) -> c_int;
    pub fn rnn_ema_update(ctx: *mut RnnCtx, e: *mut f32, v: *const f32, n: usize, decay: f32, t: c_int) -> c_int;
    pub fn rnn_resnet_create(ctx: *mut RnnCtx, depth_n: c_int, width: c_int, nclass: c_int, seed: u64, out: *mut *mut RnnResnet) -> c_int;
    pub fn rnn_resnet_destroy(net: *mut RnnResnet) -> c_int;
    pub fn rnn_resnet_num_params(net: *mut RnnResnet, out: *mut usize) -> c_int;
    pub fn rnn_resnet_num_buffers(net: *mut RnnResnet, out: *mut usize) -> c_int;
    pub fn rnn_resnet_get_params(net: *mut RnnResnet, out: *mut f32) -> c_int;
    pub fn rnn_resnet_set_params(net: *mut RnnResnet, r#in: *const f32) -> c_int;
    pub fn rnn_resnet_get_grads(net: *mut RnnResnet, out: *mut f32) -> c_int;
    pub fn rnn_resnet_get_moments(net: *mut RnnResnet, out: *mut f32) -> c_int;
    pub fn rnn_resnet_get_buffers(net: *mut RnnResnet, out: *mut f32) -> c_int;
    pub fn rnn_resnet_grad_buffer(net: *mut RnnResnet, out: *mut *mut f32, len: *mut usize) -> c_int;
    pub fn rnn_resnet_forward_dev(net: *mut RnnResnet, x: *const f32, n: c_int, h: c_int, w: c_int, train: c_int, logits: *mut f32) -> c_int;
    pub fn rnn_resnet_backward_dev(net: *mut RnnResnet, dlogits: *const f32) -> c_int;
    pub fn rnn_resnet_step(net: *mut RnnResnet, lr: f32, mom: f32, wd: f32) -> c_int;
    pub fn rnn_resnet_set_graph(net: *mut RnnResnet, enable: c_int) -> c_int;
    pub fn rnn_resnet_train_step_dev(net: *mut RnnResnet, x: *const f32, labels: *const u32, n: c_int, smooth: f32, lr: f32, mom: f32, wd: f32, loss: *mut f32, correct: *mut c_int) -> c_int;
    pub fn rnn_resnet_train_step(net: *mut RnnResnet, x: *const f32, labels: *const u32, n: c_int, smooth: f32, lr: f32, mom: f32, wd: f32, loss: *mut f32, correct: *mut c_int) -> c_int;
    pub fn rnn_dp_unique_id(uid_out: *mut u8) -> c_int;
    pub fn rnn_resnet_dp_init(net: *mut RnnResnet, rank: c_int, world: c_int, uid: *const u8, sync_bn: c_int) -> c_int;
    pub fn rnn_resnet_comm(net: *mut RnnResnet, out: *mut *mut RnnComm) -> c_int;
    pub fn rnn_alloc(ctx: *mut RnnCtx, bytes: usize, out: *mut *mut c_void) -> c_int;
    pub fn rnn_free(ctx: *mut RnnCtx, p: *mut c_void) -> c_int;
    pub fn rnn_memcpy_h2d(ctx: *mut RnnCtx, dst: *mut c_void, src: *const c_void, bytes: usize) -> c_int;
    pub fn rnn_memcpy_d2h(ctx: *mut RnnCtx, dst: *mut c_void, src: *const c_void, bytes: usize) -> c_int;
    pub fn rnn_comm_init(out: *mut *mut RnnComm, device: c_int, rank: c_int, world: c_int, uid: *const u8) -> c_int;
    pub fn rnn_comm_destroy(comm: *mut RnnComm) -> c_int;
    pub fn rnn_allreduce_grads(ctx: *mut RnnCtx, comm: *mut RnnComm, grads: *mut f32, n: usize, average: c_int) -> c_int;
    pub fn rnn_comm_check(comm: *mut RnnComm) -> c_int;
    pub fn rnn_comm_abort(comm: *mut RnnComm) -> c_int;
    pub fn rnn_comm_wait(ctx: *mut RnnCtx, comm: *mut RnnComm, timeout_ms: c_int) -> c_int;
    pub fn rnn_layernorm_res_fwd_dev(ctx: *mut RnnCtx, x: *const f32, r1: *const f32, r2: *const f32, rows: c_int, c: c_int, g: *const f32, b: *const f32, eps: f32, sum_out: *mut f32, y: *mut f32, xhat: *mut f32, invstd: *mut f32, a_image: *mut f32) -> c_int;
    pub fn rnn_linear_fwd_packed_dev(ctx: *mut RnnCtx, a_image: *const f32, rows: c_int, fin: c_int, fout: c_int, w: *const f32, b: *const f32, y: *mut f32) -> c_int;
    pub fn rnn_swiglu_fwd_dev(ctx: *mut RnnCtx, x: *const f32, a_image: *const f32, rows: c_int, c: c_int, h: c_int, wg: *const f32, bg: *const f32, ab: *mut f32, u: *mut f32) -> c_int;
    pub fn rnn_rustvit_create(ctx: *mut RnnCtx, cfg9: *const c_int, mem_at: *const c_int, n_mem: c_int, droppath: f32, parent: *const u32, nf: c_int, ncoarse: c_int, seed: u64, out: *mut *mut RnnRustvit) -> c_int;
    pub fn rnn_rustvit_destroy(net: *mut RnnRustvit) -> c_int;
    pub fn rnn_rustvit_num_params(net: *mut RnnRustvit, out: *mut usize) -> c_int;
    pub fn rnn_rustvit_num_buffers(net: *mut RnnRustvit, out: *mut usize) -> c_int;
    pub fn rnn_rustvit_get_params(net: *mut RnnRustvit, out: *mut f32) -> c_int;
    pub fn rnn_rustvit_set_params(net: *mut RnnRustvit, r#in: *const f32) -> c_int;
    pub fn rnn_rustvit_get_grads(net: *mut RnnRustvit, out: *mut f32) -> c_int;
    pub fn rnn_rustvit_get_moments(net: *mut RnnRustvit, m: *mut f32, v2: *mut f32) -> c_int;
    pub fn rnn_rustvit_get_ema(net: *mut RnnRustvit, out: *mut f32) -> c_int;
    pub fn rnn_rustvit_get_buffers(net: *mut RnnRustvit, out: *mut f32) -> c_int;
    pub fn rnn_rustvit_zero_grads(net: *mut RnnRustvit) -> c_int;
    pub fn rnn_rustvit_forward_dev(net: *mut RnnRustvit, x: *const f32, n: c_int, train: c_int, drop_seed: u64, logits: *mut f32, coarse: *mut f32, e1: *mut f32, e2: *mut f32, h1: *mut f32, h2: *mut f32, feat: *mut f32) -> c_int;
    pub fn rnn_rustvit_backward_dev(net: *mut RnnRustvit, dlogits: *const f32, dcoarse: *const f32, de1: *const f32, de2: *const f32, dh1: *const f32, dh2: *const f32, dhfinal: *const f32) -> c_int;
    pub fn rnn_rustvit_train_step_dev(net: *mut RnnRustvit, x: *const f32, tf: *const f32, tc: *const f32, hard: *const u32, hardc: *const u32, n: c_int, lr: f32, wd: f32, clip: f32, ema: f32, drop_seed: u64, stats: *mut f32) -> c_int;
    pub fn rnn_rustvit_dp_attach(net: *mut RnnRustvit, comm: *mut RnnComm) -> c_int;
    pub fn rnn_rustvit_train_step(net: *mut RnnRustvit, x: *const f32, tf: *const f32, tc: *const f32, hard: *const u32, hardc: *const u32, n: c_int, lr: f32, wd: f32, clip: f32, ema: f32, drop_seed: u64, stats: *mut f32) -> c_int;
    pub fn rnn_make_batch_eval_dev(ctx: *mut RnnCtx, images: *const u8, labels: *const u8, len: usize, start: usize, bs: c_int, flip: c_int, out: *mut f32, labels_out: *mut u32) -> c_int;
    pub fn rnn_make_batch_train_dev(ctx: *mut RnnCtx, images: *const u8, labels: *const u8, coarse: *const u8, len: usize, idx: *const u32, bs: c_int, pad: c_int, ra_mag: f32, ra_n: c_int, erase: f32, erase_side: c_int, seed: u64, out: *mut f32, labels_out: *mut u32, coarse_out: *mut u32) -> c_int;
    pub fn rnn_mix_batch_dev(ctx: *mut RnnCtx, x: *mut f32, bs: c_int, alpha_mix: f32, alpha_cut: f32, sw: f32, rng_state: *mut u64, perm: *mut u32, lam: *mut f32) -> c_int;
    pub fn rnn_resnet_eval_dev(net: *mut RnnResnet, images: *const u8, labels: *const u8, len: c_int, batch: c_int, loss: *mut f32, acc: *mut f32) -> c_int;
    pub fn rnn_resnet_eval(net: *mut RnnResnet, images: *const u8, labels: *const u8, len: c_int, batch: c_int, loss: *mut f32, acc: *mut f32) -> c_int;
    pub fn rnn_rustvit_eval_dev(net: *mut RnnRustvit, images: *const u8, labels: *const u8, len: c_int, batch: c_int, tta: c_int, use_ema: c_int, loss: *mut f32, acc: *mut f32) -> c_int;
    pub fn rnn_rustvit_eval(net: *mut RnnRustvit, images: *const u8, labels: *const u8, len: c_int, batch: c_int, tta: c_int, use_ema: c_int, loss: *mut f32, acc: *mut f32) -> c_int;
    pub fn rnn_ckpt_config_hash(kind: *const c_char, kind_len: usize, values: *const u64, n: usize) -> u64;
    pub fn rnn_ckpt_write(path: *const c_char, tensors: u32, config_hash: u64, payload: *const f32, scalars: usize) -> c_int;
    pub fn rnn_ckpt_read(path: *const c_char, tensors: u32, config_hash: u64, payload: *mut f32, scalars: usize) -> c_int;
    pub fn rnn_resnet_save(net: *mut RnnResnet, path: *const c_char) -> c_int;
    pub fn rnn_resnet_load(net: *mut RnnResnet, path: *const c_char) -> c_int;
    pub fn rnn_rustvit_save(net: *mut RnnRustvit, path: *const c_char) -> c_int;
    pub fn rnn_rustvit_load(net: *mut RnnRustvit, path: *const c_char) -> c_int;
    pub fn rnn_resnet_save_optim(net: *mut RnnResnet, path: *const c_char) -> c_int;
    pub fn rnn_resnet_load_optim(net: *mut RnnResnet, path: *const c_char) -> c_int;
    pub fn rnn_rustvit_save_optim(net: *mut RnnRustvit, path: *const c_char) -> c_int;
    pub fn rnn_rustvit_load_optim(net: *mut RnnRustvit, path: *const c_char) -> c_int;
}

/// A failed call: its status code and the library's message.
#[derive(Debug, Clone)]
pub struct Error {
    pub code: c_int,
    pub message: String,
}

impl std::fmt::Display for Error {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        write!(f, "librnn_b200 error {}: {}", self.code, self.message)
    }
}

impl std::error::Error for Error {}

/// `Ok(())` for `RNN_OK`, else the code with `rnn_last_error()` of this thread.
pub fn check(code: c_int) -> Result<(), Error> {
    if code == RNN_OK {
        return Ok(());
    }
    let message = unsafe {
        let p = rnn_last_error();
        if p.is_null() {
            String::new()
        } else {
            CStr::from_ptr(p).to_string_lossy().into_owned()
        }
    };
    Err(Error { code, message })
}
