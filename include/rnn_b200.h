/*
 * librnn_b200 -- C ABI of the B200 (sm_100a) backend for rustnn's
 * dense-contraction path.
 *
 * Every entry point returns RNN_OK (0) or a negative RNN_ERR_* code; nothing
 * unwinds across the boundary.  rnn_last_error() gives the message of the
 * last failure on the calling thread.
 *
 * Two tiers:
 *   - "_dev" entry points take DEVICE pointers and enqueue on the context's
 *     stream (asynchronous; call rnn_ctx_synchronize to wait and to collect
 *     device-side error flags);
 *   - the plain-named entry points take HOST pointers, mirror the reference's
 *     Rust signatures, copy in, run, copy out and synchronise.
 * All tensors are f32, row-major / NCHW exactly as in the reference.
 * Gradients accumulate (+=) wherever the reference accumulates.
 *
 * A context owns one CUDA stream and a growable device workspace.  Calls on
 * one context must come from one host thread at a time.
 */
#ifndef RNN_B200_H
#define RNN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RNN_OK 0
#define RNN_ERR_ARG -1     /* bad shape, stride, alignment or pointer */
#define RNN_ERR_CUDA -2    /* CUDA runtime error */
#define RNN_ERR_NCCL -3    /* NCCL error */
#define RNN_ERR_DEVICE -4  /* a kernel raised its device error word (timeout) */
#define RNN_ERR_UNSUPPORTED -5
#define RNN_ERR_IO -6       /* a checkpoint file could not be read or written */

typedef struct rnn_ctx rnn_ctx;
typedef struct rnn_resnet rnn_resnet;
typedef struct rnn_rustvit rnn_rustvit;
typedef struct rnn_comm rnn_comm;

const char *rnn_last_error(void);
/* Number of kernels this library has launched in this process. */
unsigned long long rnn_launch_count(void);
/* 1 when the library was built for sm_100a and a B200-class device is present */
int rnn_device_ok(int device);

/* ---- context ------------------------------------------------------------ */
int rnn_ctx_create(rnn_ctx **out, int device);
int rnn_ctx_destroy(rnn_ctx *ctx);
/* Enqueue on `cuda_stream` (e.g. the caller's framework stream; NULL is the
 * legacy default stream) instead of the context's own stream.  Work already
 * queued on the previous stream is waited for first. */
int rnn_ctx_set_stream(rnn_ctx *ctx, void *cuda_stream);
/* Go back to the context's own (non-blocking) stream. */
int rnn_ctx_use_own_stream(rnn_ctx *ctx);
void *rnn_ctx_stream(rnn_ctx *ctx);
/* Waits for the stream and reports kernel timeouts as RNN_ERR_DEVICE. */
int rnn_ctx_synchronize(rnn_ctx *ctx);

/* ---- GEMM (gemm.rs) ----------------------------------------------------- */
/* C[m x n] (+)= op(A) op(B).  at: A is [k x m]; bt: B is [n x k]; acc: add to
 * C instead of overwriting.  Replaces gemm::matmul (gemm.rs:434-444) and
 * gemm::gemm_small (gemm.rs:500-512; the PackedA/PackedB scratch arguments
 * have no counterpart: packing happens in shared memory). */
int rnn_gemm_dev(rnn_ctx *ctx, int m, int n, int k, const float *a, int at,
                 const float *b, int bt, float *c, int acc);
int rnn_gemm(rnn_ctx *ctx, int m, int n, int k, const float *a, int at,
             const float *b, int bt, float *c, int acc);
/* C[m x n] += A^T B, A [k x m], B [k x n]: gemm::matmul_dw (gemm.rs:555).
 * Split over K with a deterministic fixed-order reduction. */
int rnn_gemm_dw_dev(rnn_ctx *ctx, int m, int n, int k, const float *a,
                    const float *b, float *c);
int rnn_gemm_dw(rnn_ctx *ctx, int m, int n, int k, const float *a,
                const float *b, float *c);
/* No counterpart in the reference.  The same C += A^T B for callers that may
 * not allocate device memory (a framework that keeps all device memory in its
 * own pool, a loop that cannot pay cudaMalloc's implicit synchronisation): no
 * context, device pointers, enqueued on `cuda_stream` (NULL = legacy default
 * stream).  Split-K partials live in a fixed 16-MiB device array inside the
 * library, held by every GPU that loads it until exit; m*n may not exceed
 * 2,097,152 (RNN_ERR_ARG otherwise).  The first call on a device looks up the
 * array's device address, and the first call of each tile width on a device
 * sets that kernel's shared-memory opt-in, so make those first calls before
 * any stream capture.  All calls share the array: calls that overlap on a GPU
 * race.  A kernel that gives up waiting on its pipeline (a 2 s bound) does not
 * fail the call, which has already returned: it sets a device word that
 * rnn_gemm_dw_noalloc_status reports. */
int rnn_gemm_dw_noalloc_dev(int m, int n, int k, const float *a,
                            const float *b, float *c, void *cuda_stream);
/* No counterpart in the reference.  Companion of rnn_gemm_dw_noalloc_dev:
 * waits for `cuda_stream`, then returns RNN_ERR_DEVICE (and clears the word)
 * if a kernel of that entry on the current device gave up waiting since the
 * last query, else RNN_OK.  Allocates nothing. */
int rnn_gemm_dw_noalloc_status(void *cuda_stream);

/* ---- Conv2d (nn.rs:115-251, conv.rs) ------------------------------------ */
/* x [n,cin,h,w], w [cout, cin*k*k] in (ci,kh,kw) order, y [n,cout,oh,ow]
 * with oh = (h + 2 pad - k)/stride + 1.  acc: y += conv(x) instead of =.
 * Replaces Conv2d::forward (nn.rs:166) / conv::forward_image (conv.rs:169). */
int rnn_conv2d_fwd_dev(rnn_ctx *ctx, const float *x, int n, int cin, int h,
                       int w, const float *wt, int cout, int k, int stride,
                       int pad, float *y, int acc);
int rnn_conv2d_fwd(rnn_ctx *ctx, const float *x, int n, int cin, int h, int w,
                   const float *wt, int cout, int k, int stride, int pad,
                   float *y);
/* dx (+)= col2im(W^T dy).  Replaces the dX half of Conv2d::backward
 * (nn.rs:230-250) / conv::dx_image (conv.rs:207).  acc=0 overwrites dx like
 * the reference (conv.rs:218); acc=1 adds (fuses the residual add_). */
int rnn_conv2d_dgrad_dev(rnn_ctx *ctx, const float *dy, int n, int cin, int h,
                         int w, const float *wt, int cout, int k, int stride,
                         int pad, float *dx, int acc);
int rnn_conv2d_dgrad(rnn_ctx *ctx, const float *dy, int n, int cin, int h,
                     int w, const float *wt, int cout, int k, int stride,
                     int pad, float *dx);
/* dw += dy im2col(x)^T.  Replaces Conv2d::backward_w (nn.rs:193-227) /
 * conv::dw_image (conv.rs:283).  Deterministic split-K reduction. */
int rnn_conv2d_wgrad_dev(rnn_ctx *ctx, const float *x, const float *dy, int n,
                         int cin, int h, int w, int cout, int k, int stride,
                         int pad, float *dw);
int rnn_conv2d_wgrad(rnn_ctx *ctx, const float *x, const float *dy, int n,
                     int cin, int h, int w, int cout, int k, int stride,
                     int pad, float *dw);

/* ---- BatchNorm2d (nn.rs:255-428) ---------------------------------------- */
/* Train-mode forward over y [n,c,hw]: per-channel batch statistics in f64
 * (nn.rs:301-322), running mean/var update with momentum `mom` and unbiased
 * variance (nn.rs:330-336), out = gamma*xhat + beta, optionally ReLU
 * (nn.rs:326-354).  Writes mean[c] and invstd[c]; xhat is not stored (the
 * backward recomputes it from y).  out may alias y. */
int rnn_batchnorm_fwd_dev(rnn_ctx *ctx, const float *y, int n, int c, int hw,
                          const float *gamma, const float *beta, float *rmean,
                          float *rvar, float mom, float eps, int relu,
                          float *mean, float *invstd, float *out);
/* Eval-mode forward (nn.rs:358-369). */
int rnn_batchnorm_eval_dev(rnn_ctx *ctx, const float *y, int n, int c, int hw,
                           const float *gamma, const float *beta,
                           const float *rmean, const float *rvar, float eps,
                           int relu, float *out);
/* Backward (nn.rs:384-427) with xhat = (y - mean) * invstd.  When
 * relu_out != NULL the incoming gradient is first masked by relu_out > 0
 * (relu_back_, nn.rs:433).  dgamma/dbeta accumulate; dx is written. */
int rnn_batchnorm_bwd_dev(rnn_ctx *ctx, const float *dy, const float *y, int n,
                          int c, int hw, const float *gamma, const float *mean,
                          const float *invstd, const float *relu_out,
                          float *dx, float *dgamma, float *dbeta);

/* ---- elementwise / loss / optimiser (nn.rs) ----------------------------- */
int rnn_relu_back_dev(rnn_ctx *ctx, float *d, const float *y, size_t len);   /* nn.rs:433 */
int rnn_add_dev(rnn_ctx *ctx, float *a, const float *b, size_t len);         /* nn.rs:441 */
int rnn_add_relu_dev(rnn_ctx *ctx, float *a, const float *b, size_t len);    /* nn.rs:446 */
int rnn_gap_fwd_dev(rnn_ctx *ctx, const float *x, int nc, int hw, float *y); /* nn.rs:455 */
int rnn_gap_bwd_dev(rnn_ctx *ctx, const float *dy, int nc, int hw, float *dx); /* nn.rs:465 */
/* softmax + cross-entropy with label smoothing (nn.rs:615-637): writes
 * dlogits (already divided by n), loss_out[0] = mean loss, correct_out[0] =
 * number of argmax hits.  Deterministic. */
int rnn_softmax_ce_dev(rnn_ctx *ctx, const float *logits, const uint32_t *labels,
                       int n, int nclass, float smooth, float *dlogits,
                       float *loss_out, int *correct_out);
/* Param::step (nn.rs:102-110) over `len` elements; g is zeroed. */
int rnn_sgd_nesterov_dev(rnn_ctx *ctx, float *v, float *g, float *m, size_t len,
                         float lr, float mom, float wd, int decay);

/* ---- attention (attn.rs) ------------------------------------------------ */
/* rel_index (attn.rs:53-72) for a th x tw query grid over an mh x mw key grid
 * (equal grids: self attention; otherwise the memory is at twice the
 * resolution and offsets are in half-token units).  Writes th*tw*mh*mw
 * indices when idx != NULL; *nrel = number of bias entries per head. */
int rnn_rel_index(int th, int tw, int mh, int mw, uint32_t *idx, int *nrel);
/* Core::forward (attn.rs:148-223) for all n images and h heads in one launch:
 * S = tau_h Q K^T + rel_h[rel_index], diagonal masked when mask_diag (LSA),
 * P = softmax(S) written to p [n,h,tq,tk] (the backward reads it), O = P V
 * written to o [n,tq,h*dh].  Q rows are qstride floats apart with head hd at
 * column qoff + hd*dh; K/V rows kvstride apart at koff/voff + hd*dh (the fused
 * qkv [n*t,3c] buffer: qstride=kvstride=3c, qoff=0, koff=c, voff=2c; the
 * cross-attention memory [n*tk,2c]: koff=0, voff=c).  dh in {4,8,16,32,64}. */
int rnn_attn_fwd_dev(rnn_ctx *ctx, int n, int h, int dh, int th, int tw, int mh,
                     int mw, int mask_diag, const float *q, int qstride,
                     int qoff, const float *kv, int kvstride, int koff,
                     int voff, const float *tau, const float *rel, float *p,
                     float *o);
/* Core::backward (attn.rs:226-343): dq, dkv, dtau, drel accumulate (+=); dq
 * and dkv may be the same buffer (the fused qkv gradient).  Deterministic. */
int rnn_attn_bwd_dev(rnn_ctx *ctx, int n, int h, int dh, int th, int tw, int mh,
                     int mw, const float *q, int qstride, int qoff,
                     const float *kv, int kvstride, int koff, int voff,
                     const float *tau, const float *p, const float *dout,
                     float *dq, float *dkv, float *dtau, float *drel);

/* ---- LayerNorm (norm.rs:17-143) and Linear (linear.rs:44-96) ------------ */
/* y = gamma * xhat + beta over rows of c, f64 row statistics; xhat [rows*c]
 * and invstd [rows] are written when non-NULL (the backward needs them). */
int rnn_layernorm_fwd_dev(rnn_ctx *ctx, const float *x, int rows, int c,
                          const float *gamma, const float *beta, float eps,
                          float *y, float *xhat, float *invstd);
/* dx written; dgamma, dbeta accumulate (norm.rs:92-137). */
int rnn_layernorm_bwd_dev(rnn_ctx *ctx, const float *dy, const float *xhat,
                          const float *invstd, int rows, int c,
                          const float *gamma, float *dx, float *dgamma,
                          float *dbeta);
/* Linear::forward: y[rows,fout] = x W^T (+ b; b may be NULL), W [fout,fin]. */
int rnn_linear_fwd_dev(rnn_ctx *ctx, const float *x, int rows, int fin, int fout,
                       const float *w, const float *b, float *y);
/* Linear::backward: dW += dY^T X, db += colsum(dY) (b may be NULL), dx = dY W. */
int rnn_linear_bwd_dev(rnn_ctx *ctx, const float *x, const float *dy, int rows,
                       int fin, int fout, const float *w, float *dw, float *db,
                       float *dx);

/* ---- optimisers (optim.rs) ---------------------------------------------- */
/* newton_schulz in place on g [rows x cols] (optim.rs:124-145). */
int rnn_newton_schulz_dev(rnn_ctx *ctx, float *g, int rows, int cols, int steps);
/* One Muon update of one matrix (optim.rs:184-197); g is zeroed. */
int rnn_muon_step_dev(rnn_ctx *ctx, float *v, float *g, float *m, int rows,
                      int cols, int steps, float lr, float mom, float wd,
                      int decay);
/* step_adam (optim.rs:205-233); t = updates already taken; g is zeroed. */
int rnn_adamw_step_dev(rnn_ctx *ctx, float *v, float *g, float *m, float *v2,
                       size_t n, float lr, float wd, int decay, float b1,
                       float b2, float eps, int t);
/* clip_ (optim.rs:237-250) over one flat gradient buffer; the pre-clip norm
 * goes to norm_out[0] (device) when non-NULL. */
int rnn_clip_dev(rnn_ctx *ctx, float *g, size_t n, float max, float *norm_out);
/* Ema::update (optim.rs:270-287) for its t-th call (t >= 2; the first call
 * copies the weights): e = d e + (1-d) v, d = min(decay, (1+t)/(10+t)). */
int rnn_ema_update_dev(rnn_ctx *ctx, float *e, const float *v, size_t n,
                       float decay, int t);

/* ---- rustvit glue (norm.rs, vit.rs, tok.rs, loss.rs); [n,t,c] tokens ---- */
/* LayerScale (norm.rs:151-212): y = l * x per channel (y may alias x);
 * backward: dl += sum dy*x, dx = l * dy. */
int rnn_layerscale_fwd_dev(rnn_ctx *ctx, const float *x, int rows, int c,
                           const float *l, float *y);
int rnn_layerscale_bwd_dev(rnn_ctx *ctx, const float *dy, const float *x,
                           int rows, int c, const float *l, float *dl, float *dx);
/* SwiGLU gate (norm.rs:250-286): u = silu(a) * b from ab [rows, 2h]. */
int rnn_swiglu_act_fwd_dev(rnn_ctx *ctx, const float *ab, int rows, int h,
                           float *u);
int rnn_swiglu_act_bwd_dev(rnn_ctx *ctx, const float *du, const float *ab,
                           int rows, int h, float *dab);
/* DwConv3 (norm.rs:304-451): depthwise 3x3 over the th x tw token grid,
 * channels-last, w [9, c], b [c]; dw, db accumulate; dx written. */
int rnn_dwconv3_fwd_dev(rnn_ctx *ctx, const float *x, int n, int th, int tw,
                        int c, const float *w, const float *b, float *y);
int rnn_dwconv3_bwd_dev(rnn_ctx *ctx, const float *dy, const float *x, int n,
                        int th, int tw, int c, const float *w, float *dw,
                        float *db, float *dx);
/* SeqPool (norm.rs:466-581): w = softmax_t(x.p) [n,t], z = sum_t w x [n,c];
 * dp accumulates, dx written. */
int rnn_seqpool_fwd_dev(rnn_ctx *ctx, const float *x, int n, int t, int c,
                        const float *p, float *z, float *w);
int rnn_seqpool_bwd_dev(rnn_ctx *ctx, const float *dz, const float *x,
                        const float *w, int n, int t, int c, const float *p,
                        float *dp, float *dx);
/* DropPath (vit.rs:30-74): per-image keep mask drawn from Rng::new(seed)
 * exactly like the reference (mask [n] device, 1/keep or 0); x scaled in
 * place.  The backward scales dy by the same mask. */
int rnn_droppath_fwd_dev(rnn_ctx *ctx, float *x, int n, size_t per_image,
                         float p, uint64_t seed, float *mask);
int rnn_droppath_bwd_dev(rnn_ctx *ctx, float *dy, int n, size_t per_image,
                         const float *mask);
/* token_merge (vit.rs:586-624): [n, th*th, c] -> [n, (th/2)^2, 4c] (2x2
 * neighbours concatenated); backward=1 copies the gradient back. */
int rnn_token_merge_dev(rnn_ctx *ctx, const float *src, int n, int th, int c,
                        float *dst, int backward);
/* Tok::from_tensor / to_tensor (tok.rs:54-87): [n,c,hw] <-> [n,hw,c]. */
int rnn_tok_layout_dev(rnn_ctx *ctx, const float *in, int n, int c, int hw,
                       float *out, int to_nchw);
/* TaxoHead (vit.rs:283-310): zf[i,k] += zc[i,parent[k]]; backward writes
 * dc = dzc + scatter(dzf). */
int rnn_taxo_combine_fwd_dev(rnn_ctx *ctx, float *zf, const float *zc, int n,
                             int nf, int nc, const uint32_t *parent);
int rnn_taxo_combine_bwd_dev(rnn_ctx *ctx, const float *dzf, const float *dzc,
                             int n, int nf, int nc, const uint32_t *parent,
                             float *dc);
/* ce_soft (loss.rs:39-81): dz = scale * d(mean CE)/dz written; loss_out[0],
 * correct_out[0] (device) when non-NULL. */
int rnn_ce_soft_dev(rnn_ctx *ctx, const float *logits, const float *target,
                    const uint32_t *hard, int n, int nclass, float scale,
                    float *dz, float *loss_out, int *correct_out);
/* kl_distill (loss.rs:87-130): T^2 KL(teacher || student); dz accumulates. */
int rnn_kl_distill_dev(rnn_ctx *ctx, const float *student, const float *teacher,
                       int n, int nclass, float temp, float scale, float *dz,
                       float *loss_out);
/* hint_mse (loss.rs:133-151): dz accumulates. */
int rnn_hint_mse_dev(rnn_ctx *ctx, const float *pred, const float *target,
                     int n, int c, float scale, float *dz, float *loss_out);

/* ---- host-pointer tier of the attention / norm / optimiser entries -------
 * Same arguments as the _dev entries above, on host memory: the call stages
 * the operands, runs the device entry, copies results back and
 * synchronises.  Accumulating outputs are read and written back. */
int rnn_attn_fwd(rnn_ctx *ctx, int n, int h, int dh, int th, int tw, int mh,
                 int mw, int mask_diag, const float *q, int qstride, int qoff,
                 const float *kv, int kvstride, int koff, int voff,
                 const float *tau, const float *rel, float *p, float *o);   /* attn.rs:148 */
int rnn_attn_bwd(rnn_ctx *ctx, int n, int h, int dh, int th, int tw, int mh,
                 int mw, const float *q, int qstride, int qoff,
                 const float *kv, int kvstride, int koff, int voff,
                 const float *tau, const float *p, const float *dout,
                 float *dq, float *dkv, float *dtau, float *drel);          /* attn.rs:226 */
int rnn_layernorm_fwd(rnn_ctx *ctx, const float *x, int rows, int c,
                      const float *gamma, const float *beta, float eps,
                      float *y, float *xhat, float *invstd);                 /* norm.rs:59 */
int rnn_layernorm_bwd(rnn_ctx *ctx, const float *dy, const float *xhat,
                      const float *invstd, int rows, int c, const float *gamma,
                      float *dx, float *dgamma, float *dbeta);               /* norm.rs:101 */
int rnn_linear_fwd(rnn_ctx *ctx, const float *x, int rows, int fin, int fout,
                   const float *w, const float *b, float *y);                /* linear.rs:44 */
int rnn_linear_bwd(rnn_ctx *ctx, const float *x, const float *dy, int rows,
                   int fin, int fout, const float *w, float *dw, float *db,
                   float *dx);                                               /* linear.rs:66 */
int rnn_batchnorm_fwd(rnn_ctx *ctx, const float *y, int n, int c, int hw,
                      const float *gamma, const float *beta, float *rmean,
                      float *rvar, float mom, float eps, int relu,
                      float *mean, float *invstd, float *out);               /* nn.rs:290-354 */
int rnn_batchnorm_bwd(rnn_ctx *ctx, const float *dy, const float *y, int n,
                      int c, int hw, const float *gamma, const float *mean,
                      const float *invstd, const float *relu_out, float *dx,
                      float *dgamma, float *dbeta);                          /* nn.rs:384-427 */
/* newton_schulz (optim.rs:124-145) over `count` matrices in one call, each
 * in place; the device form takes an array of device pointers (the 39
 * matrices of Optim::step_all, optim.rs:182-190, in one call). */
int rnn_newton_schulz_batched_dev(rnn_ctx *ctx, int count, float *const *g,
                                  const int *rows, const int *cols, int steps);
int rnn_newton_schulz_batched(rnn_ctx *ctx, int count, float *const *g,
                              const int *rows, const int *cols, int steps);
int rnn_muon_step(rnn_ctx *ctx, float *v, float *g, float *m, int rows,
                  int cols, int steps, float lr, float mom, float wd,
                  int decay);                                                /* optim.rs:183-199 */
int rnn_adamw_step(rnn_ctx *ctx, float *v, float *g, float *m, float *v2,
                   size_t n, float lr, float wd, int decay, float b1, float b2,
                   float eps, int t);                                        /* optim.rs:205-233 */
int rnn_sgd_nesterov(rnn_ctx *ctx, float *v, float *g, float *m, size_t len,
                     float lr, float mom, float wd, int decay);              /* nn.rs:102-110 */
int rnn_clip(rnn_ctx *ctx, float *g, size_t n, float max, float *norm_out);  /* optim.rs:237-250 */
int rnn_ema_update(rnn_ctx *ctx, float *e, const float *v, size_t n,
                   float decay, int t);                                      /* optim.rs:270-287 */

/* No reference counterpart (the reference is one process): the SyncBN
 * exchange of the data-parallel step on its own.  Per-channel forward sums
 * (sum y, sum y^2; f64, [c][2]) of this rank's y [n,c,hw] (nn.rs:301-322),
 * published in this rank's mailbox and summed with every peer's in rank order:
 * mailboxes is a device array of `world` device pointers (peers' mapped
 * through CUDA IPC by the caller), each mailbox rnn_peer_mailbox_bytes(cmax)
 * bytes, zeroed before first use: a u64 flag at offset 0, then two slots of
 * [cmax][2] doubles from offset 128.  seq is this rank's device u64 exchange
 * counter (starts at 0).  A peer that does not publish within wait_ms sets the
 * device error word (rnn_ctx_synchronize -> RNN_ERR_DEVICE) and the call
 * returns with that peer's stale slot in the sums instead of hanging.
 * hw % 4 == 0; y 16-byte aligned. */
int rnn_batchnorm_stats_peer_dev(rnn_ctx *ctx, const float *y, int n, int c,
                                 int hw, int rank, int world,
                                 void *const *mailboxes,
                                 unsigned long long *seq, int cmax, int wait_ms,
                                 double *sums);
size_t rnn_peer_mailbox_bytes(int cmax);

/* ---- ResNet training step (model.rs, train.rs:684-699) ------------------ */
/* ResNet::new(depth_n, width, nclass, seed) (model.rs:112-133), with the
 * reference's initialisation drawn from the same xoshiro256++ stream, so
 * parameters are bit-identical to the reference's at creation. */
int rnn_resnet_create(rnn_ctx *ctx, int depth_n, int width, int nclass,
                      uint64_t seed, rnn_resnet **out);
int rnn_resnet_destroy(rnn_resnet *net);
int rnn_resnet_num_params(rnn_resnet *net, size_t *out);
int rnn_resnet_num_buffers(rnn_resnet *net, size_t *out);
/* flat host copies in for_each_param order (model.rs:159-168) */
int rnn_resnet_get_params(rnn_resnet *net, float *out);
int rnn_resnet_set_params(rnn_resnet *net, const float *in);
int rnn_resnet_get_grads(rnn_resnet *net, float *out);
int rnn_resnet_get_moments(rnn_resnet *net, float *out);
/* running mean/var, for_each_buffer order (model.rs:170-176) */
int rnn_resnet_get_buffers(rnn_resnet *net, float *out);
/* device pointer to the flat gradient buffer (for external collectives) */
int rnn_resnet_grad_buffer(rnn_resnet *net, float **out, size_t *len);
/* ResNet::forward (model.rs:135): x [n,3,h,w] device, logits [n,nclass] */
int rnn_resnet_forward_dev(rnn_resnet *net, const float *x, int n, int h, int w,
                           int train, float *logits);
/* ResNet::backward (model.rs:148): gradients accumulate */
int rnn_resnet_backward_dev(rnn_resnet *net, const float *dlogits);
/* ResNet::step (model.rs:206) */
int rnn_resnet_step(rnn_resnet *net, float lr, float mom, float wd);
/* No reference counterpart (a device-side execution option): when enabled,
 * rnn_resnet_train_step[_dev] records the whole step (kernels and NCCL
 * calls) into a CUDA graph on its second call with the same arguments and
 * replays it afterwards; any change of pointers, sizes or hyperparameters
 * runs the step eagerly and recaptures.  Results are identical. */
int rnn_resnet_set_graph(rnn_resnet *net, int enable);
/* forward + softmax_ce + backward (+ gradient allreduce when data-parallel)
 * + step, on device inputs.  loss/correct are device pointers (1 element). */
int rnn_resnet_train_step_dev(rnn_resnet *net, const float *x,
                              const uint32_t *labels, int n, float smooth,
                              float lr, float mom, float wd, float *loss,
                              int *correct);
/* Same from host inputs: copies x/labels in and loss/correct out. */
int rnn_resnet_train_step(rnn_resnet *net, const float *x,
                          const uint32_t *labels, int n, float smooth, float lr,
                          float mom, float wd, float *loss, int *correct);

/* ---- data parallel (no reference counterpart: the reference is one process) */
#define RNN_UID_BYTES 128
int rnn_dp_unique_id(unsigned char *uid_out);
/* Joins an NCCL communicator (one rank per GPU).  The train step then sums
 * gradients across ranks and divides by world (each rank's softmax_ce divides
 * by its local batch), and, when sync_bn != 0, BatchNorm statistics are
 * reduced across ranks so every rank normalises with whole-batch statistics
 * like the single-process reference. */
int rnn_resnet_dp_init(rnn_resnet *net, int rank, int world,
                       const unsigned char *uid, int sync_bn);
/* The network's communicator as a handle for rnn_comm_wait / rnn_comm_check
 * (failure detection of its collectives); it belongs to the network. */
int rnn_resnet_comm(rnn_resnet *net, rnn_comm **out);

/* ---- Tier-2 runtime (no reference counterpart: the reference is one process
 * with host memory only; pool.rs is its allocator and it has no collective).
 * Device memory on the context's device; copies enqueued on its stream. */
int rnn_alloc(rnn_ctx *ctx, size_t bytes, void **out);
/* waits for the context's stream first (queued work may still read p) */
int rnn_free(rnn_ctx *ctx, void *p);
int rnn_memcpy_h2d(rnn_ctx *ctx, void *dst, const void *src, size_t bytes);
int rnn_memcpy_d2h(rnn_ctx *ctx, void *dst, const void *src, size_t bytes);
/* An NCCL communicator for the batch-sharded step (one rank per GPU; uid from
 * rnn_dp_unique_id, the same bytes on every rank). */
int rnn_comm_init(rnn_comm **out, int device, int rank, int world,
                  const unsigned char *uid);
int rnn_comm_destroy(rnn_comm *comm);
/* Sum (average != 0: mean) of a flat f32 gradient buffer over all ranks, in
 * place, on the context's stream (train.rs:684-699 with the batch sharded). */
int rnn_allreduce_grads(rnn_ctx *ctx, rnn_comm *comm, float *grads, size_t n,
                        int average);
/* RNN_ERR_NCCL when the communicator has an asynchronous error. */
int rnn_comm_check(rnn_comm *comm);
/* Makes every pending collective of the communicator return; it is unusable
 * afterwards. */
int rnn_comm_abort(rnn_comm *comm);
/* Host watchdog: waits for the context's stream, polling the communicator's
 * asynchronous error every millisecond.  On an error, or when the stream has
 * not finished within timeout_ms (a peer never joined a collective), aborts
 * the communicator and returns RNN_ERR_NCCL. */
int rnn_comm_wait(rnn_ctx *ctx, rnn_comm *comm, int timeout_ms);

/* ---- rustvit fusions the reference identified and did not build
 * (README.md:549-552) ------------------------------------------------------ */
/* s = x (+ r1) (+ r2) (vit.rs:160-176: the block's residual adds, each rounded
 * like the reference's add_), written to sum_out when non-null, then
 * LayerNorm::forward of s (norm.rs:38-100) into y / xhat / invstd.  With
 * a_image, y is also written as the packed A operand of the GEMM that reads
 * it: per 128-row tile and 32-column block, a [hi | lo] pair of 16 KB TF32
 * tiles in the engine's shared-memory layout (rnn_linear_fwd_packed_dev,
 * rnn_swiglu_fwd_dev bulk-copy it); it holds ceil(rows/128)*128*c*2 floats.
 * c a multiple of 128 up to 512; 16-byte aligned tensors. */
int rnn_layernorm_res_fwd_dev(rnn_ctx *ctx, const float *x, const float *r1,
                              const float *r2, int rows, int c, const float *g,
                              const float *b, float eps, float *sum_out,
                              float *y, float *xhat, float *invstd,
                              float *a_image);
/* Linear::forward (linear.rs:44-63) from a packed A image of x: y = x W^T + b,
 * the bias added in the GEMM's epilogue.  fin a multiple of 32. */
int rnn_linear_fwd_packed_dev(rnn_ctx *ctx, const float *a_image, int rows,
                              int fin, int fout, const float *w, const float *b,
                              float *y);
/* SwiGlu::forward's first half (norm.rs:250-260) as one GEMM: ab = x Wg^T + bg
 * ([rows, 2h], value columns then gate columns, kept for the backward) and
 * u = silu(a) * g ([rows, h]) from its epilogue.  x row-major, or a_image
 * (then x may be null).  c a multiple of 32, h a multiple of 16. */
int rnn_swiglu_fwd_dev(rnn_ctx *ctx, const float *x, const float *a_image,
                       int rows, int c, int h, const float *wg, const float *bg,
                       float *ab, float *u);

/* ---- rustvit training step (vit.rs, train.rs:70-118 and 346-387) -------- */
/* RustViT::new (vit.rs:441-509) on the device.  cfg9 = {width, cmid, dim,
 * heads, depth3, dim4, heads4, depth4, img} (vit.rs:349-365); mem_at lists the
 * reader blocks of stage 3; parent[nf] maps each fine class to its coarse
 * group (TaxoHead, vit.rs:236-262).  Initial parameters are drawn from the
 * reference's rng stream in its construction order (bit-identical).
 * Parameters, gradients and moments are flat in for_each_param order
 * (vit.rs:687-719); buffers (BatchNorm running statistics) in
 * for_each_buffer order (vit.rs:721-728). */
int rnn_rustvit_create(rnn_ctx *ctx, const int *cfg9, const int *mem_at,
                       int n_mem, float droppath, const uint32_t *parent,
                       int nf, int ncoarse, uint64_t seed, rnn_rustvit **out);
int rnn_rustvit_destroy(rnn_rustvit *net);
int rnn_rustvit_num_params(rnn_rustvit *net, size_t *out);
int rnn_rustvit_num_buffers(rnn_rustvit *net, size_t *out);
int rnn_rustvit_get_params(rnn_rustvit *net, float *out);   /* host or device dst */
int rnn_rustvit_set_params(rnn_rustvit *net, const float *in);
int rnn_rustvit_get_grads(rnn_rustvit *net, float *out);
int rnn_rustvit_get_moments(rnn_rustvit *net, float *m, float *v2);
int rnn_rustvit_get_ema(rnn_rustvit *net, float *out);
int rnn_rustvit_get_buffers(rnn_rustvit *net, float *out);
int rnn_rustvit_zero_grads(rnn_rustvit *net);
/* RustViT::forward (vit.rs:511-582) with drop_seed = RustViT::drop_seed.
 * Outputs (device, nullable) are copied out: logits/e1/e2 [n, nf], coarse
 * [n, ncoarse], h1/h2/feat [n, dim4]; the exits exist only when train. */
int rnn_rustvit_forward_dev(rnn_rustvit *net, const float *x, int n, int train,
                            uint64_t drop_seed, float *logits, float *coarse,
                            float *e1, float *e2, float *h1, float *h2,
                            float *feat);
/* RustViT::backward (vit.rs:627-685) with vit::Grads; gradients accumulate
 * into the flat gradient buffer.  The exit gradients come as a set or not
 * at all; dhfinal is nullable (an empty Grads::hfinal). */
int rnn_rustvit_backward_dev(rnn_rustvit *net, const float *dlogits,
                             const float *dcoarse, const float *de1,
                             const float *de2, const float *dh1,
                             const float *dh2, const float *dhfinal);
/* Trainer::step (train.rs:346-387) at a given learning rate: forward,
 * build_loss with the cli.rs defaults (tf/tc the soft targets of
 * train.rs:120-155, hard/hardc the fine and coarse labels), backward, clip_
 * at `clip` (0 = off), Optim::step_all (Muon + AdamW), Ema::update at
 * `ema` (0 = off).  stats (host, nullable) = {total loss, ce, correct}. */
int rnn_rustvit_train_step_dev(rnn_rustvit *net, const float *x,
                               const float *tf, const float *tc,
                               const uint32_t *hard, const uint32_t *hardc,
                               int n, float lr, float wd, float clip, float ema,
                               uint64_t drop_seed, float *stats);
/* Data-parallel Trainer::step.  No counterpart in the reference, whose
 * step (train.rs:346-387) runs in one process.  comm (borrowed, from
 * rnn_comm_init on the network's device; NULL detaches) makes every later
 * train step of this network one rank of a batch-sharded step: each rank
 * passes its own equal shard (and its own drop_seed); after the forward the
 * BatchNorm running statistics are averaged over the ranks, after the
 * backward the flat gradient is (before clip_), so clip_, the optimiser and
 * the EMA run identically on every rank.  BatchNorm batch statistics stay
 * per rank; the loss and accuracy in stats are the rank's own shard's. */
int rnn_rustvit_dp_attach(rnn_rustvit *net, rnn_comm *comm);
/* Host tier of the step: the batch comes from host memory. */
int rnn_rustvit_train_step(rnn_rustvit *net, const float *x, const float *tf,
                           const float *tc, const uint32_t *hard,
                           const uint32_t *hardc, int n, float lr, float wd,
                           float clip, float ema, uint64_t drop_seed,
                           float *stats);

/* ---- evaluation (data.rs:494-512, eval.rs:15-66) ------------------------ */
/* A dataset is data::Dataset's images and fine labels (data.rs:16-24): len
 * images of 3 x 32 x 32 bytes in CHW order, then len label bytes. */
/* data::make_batch_eval (data.rs:494-512): images/labels (len images) and
 * out/labels_out on the device; [start, start + bs) must lie inside the
 * dataset (RNN_ERR_ARG otherwise); writes bs images from `start`, normalised per channel
 * ((v / 255 - mean) / std, data.rs:95-98), mirrored left-right when flip, and
 * their labels widened to u32. */
int rnn_make_batch_eval_dev(rnn_ctx *ctx, const uint8_t *images,
                            const uint8_t *labels, size_t len, size_t start,
                            int bs, int flip, float *out,
                            uint32_t *labels_out);
/* data::make_batch_train (data.rs:384-412): images/labels (and coarse
 * labels, nullable) of a dataset of len images, idx [bs] (u32) its images to
 * use, all on the device.  An index >= len raises the device error
 * (RNN_ERR_DEVICE at the next rnn_ctx_synchronize) and leaves that image's
 * slot zero, where the reference panics.  Augmentation = data::Aug (data.rs:281-293): RandAugment of
 * ra_n ops (at most 8) at magnitude ra_mag (off at 0), crop offset within
 * pad, flip, normalise, random erasing with probability `erase` of an
 * erase_side square of normal noise.  Image b draws from
 * Rng::new(seed ^ b * 0x9E3779B97F4A7C15) in the reference's order.
 * out [bs, 3, 32, 32], labels_out / coarse_out (nullable) [bs] u32.
 * The f32 logf / cosf / sinf results are the host C library's, as the
 * reference's: the first call with erasing or RandAugment on a device builds
 * two 64-MB Box-Muller tables there from the C library (kept until exit;
 * make that call before any stream capture), and with RandAugment each call
 * replays the images' RandAugment draws on the host for the rotations'
 * cos / sin. */
int rnn_make_batch_train_dev(rnn_ctx *ctx, const uint8_t *images,
                             const uint8_t *labels, const uint8_t *coarse,
                             size_t len, const uint32_t *idx, int bs, int pad,
                             float ra_mag, int ra_n, float erase,
                             int erase_side, uint64_t seed, float *out,
                             uint32_t *labels_out, uint32_t *coarse_out);
/* data::mix_batch (data.rs:467-491) in place on the device batch x
 * [bs, 3, 32, 32] (16-byte aligned): mixup or cutmix with a permutation of
 * the batch, drawn from the caller's generator, rng_state = the four
 * xoshiro256++ words of rng.rs's Rng (host, advanced in place).  perm and
 * lam (host, [bs], nullable) receive the permutation and the per-image
 * lambdas (1 = not mixed). */
int rnn_mix_batch_dev(rnn_ctx *ctx, float *x, int bs, float alpha_mix,
                      float alpha_cut, float sw, uint64_t *rng_state,
                      uint32_t *perm, float *lam);
/* eval::resnet (eval.rs:41-43): batches of `batch` images, forward with
 * train false (BatchNorm on running statistics), softmax_ce without
 * smoothing; loss = sum(batch loss * bs) / len, acc = correct / len (host
 * floats, NaN both when len == 0).  _dev takes the dataset on the device;
 * the plain form copies a host dataset in first. */
int rnn_resnet_eval_dev(rnn_resnet *net, const uint8_t *images,
                        const uint8_t *labels, int len, int batch, float *loss,
                        float *acc);
int rnn_resnet_eval(rnn_resnet *net, const uint8_t *images,
                    const uint8_t *labels, int len, int batch, float *loss,
                    float *acc);
/* eval::vit (eval.rs:47-66): exits off, forward with train false; with tta
 * the logits of each batch and of its mirror are averaged (0.5 * (a + b)).
 * use_ema evaluates the EMA weights, swapped in for the pass and out again
 * (Trainer::eval_ema, train.rs:390-402).  The model's img must be 32. */
int rnn_rustvit_eval_dev(rnn_rustvit *net, const uint8_t *images,
                         const uint8_t *labels, int len, int batch, int tta,
                         int use_ema, float *loss, float *acc);
int rnn_rustvit_eval(rnn_rustvit *net, const uint8_t *images,
                     const uint8_t *labels, int len, int batch, int tta,
                     int use_ema, float *loss, float *acc);

/* ---- checkpoints (ckpt.rs:8-247) ---------------------------------------- */
/* The reference's file format: "RUSTNN\0", tensor count (u32), scalar count
 * (u64), configuration hash (u64), little endian, then the f32 payload
 * (every parameter in for_each_param order, then every buffer in
 * for_each_buffer order).  Saves go to path.tmp, renamed over path; loads
 * check count, size and hash (or accept a bare legacy payload of the right
 * size) before any value is replaced. */
/* ckpt::config_hash (ckpt.rs:83-96): FNV-1a of kind, then of each value's 8
 * little-endian bytes. */
uint64_t rnn_ckpt_config_hash(const char *kind, size_t kind_len,
                              const uint64_t *values, size_t n);
/* write_checkpoint / read_checkpoint (ckpt.rs:99-189) of a host payload. */
int rnn_ckpt_write(const char *path, uint32_t tensors, uint64_t config_hash,
                   const float *payload, size_t scalars);
int rnn_ckpt_read(const char *path, uint32_t tensors, uint64_t config_hash,
                  float *payload, size_t scalars);
/* Checkpointed::save / load (ckpt.rs:51-77) of the device models, with
 * ResNet's hash of ("resnet", [depth_n, width, nclass]) (model.rs:220-229)
 * and rustvit's of ("rustvit", cfg, nclass, ncoarse, use_exits, mem_at,
 * parent) (vit.rs:780-801). */
int rnn_resnet_save(rnn_resnet *net, const char *path);
int rnn_resnet_load(rnn_resnet *net, const char *path);
int rnn_rustvit_save(rnn_rustvit *net, const char *path);
int rnn_rustvit_load(rnn_rustvit *net, const char *path);
/* No reference counterpart: the optimiser state the reference's checkpoint
 * omits, in the same format under the hash of "<kind>-optim" — ResNet: the
 * SGD momentum; rustvit: the first and second moments, the EMA weights and
 * the step counters (Adam t, EMA t, EMA ready: three u32 words at the end of
 * the payload). */
int rnn_resnet_save_optim(rnn_resnet *net, const char *path);
int rnn_resnet_load_optim(rnn_resnet *net, const char *path);
int rnn_rustvit_save_optim(rnn_rustvit *net, const char *path);
int rnn_rustvit_load_optim(rnn_rustvit *net, const char *path);

#ifdef __cplusplus
}
#endif
#endif
