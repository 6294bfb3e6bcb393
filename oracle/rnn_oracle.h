/*
 * CPU oracle for the rustnn dense-contraction path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is a plain-C restatement of the
 * reference's own CPU arithmetic (lsiddd/rustnn, Rust).  It exists to check
 * the CUDA library and to time a CPU baseline.  Only tests/, the smoke check
 * in __graft_entry__.py and the cpu_baseline / --impl reference legs of
 * bench.py may load it.  The product library (rustnn_b200) never calls it.
 *
 * Every function names the reference file:line it restates.  All arithmetic
 * is f32 except where the reference itself accumulates in f64 (BatchNorm and
 * LayerNorm statistics, the global-norm clip).
 *
 * Pinning: the reference is Rust and no Rust toolchain exists on this
 * machine, so it cannot be run to produce golden tensors.  The reference ships
 * no stored tensors either.  The oracle is pinned to what the reference's own
 * tests hold: the naive-GEMM check (check.rs:105-161), the directional
 * derivative gradchecks (check.rs:19-40, 503-770) and the published parameter
 * and MAC counts (README.md:116-117).  tests/test_oracle.py runs all of them.
 */
#ifndef RNN_ORACLE_H
#define RNN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- rng.rs ------------------------------------------------------------ */
typedef struct { uint64_t s[4]; } orc_rng;
void     orc_rng_new(orc_rng *r, uint64_t seed);          /* rng.rs:8-20  */
uint64_t orc_rng_next_u64(orc_rng *r);                     /* rng.rs:23-36 */
float    orc_rng_uniform(orc_rng *r);                      /* rng.rs:50-52 */
float    orc_rng_normal(orc_rng *r);                       /* rng.rs:55-59 */
uint64_t orc_rng_below(orc_rng *r, uint64_t n);            /* rng.rs:45-47 */
void     orc_rand_vec(float *out, size_t n, orc_rng *r);   /* rng.rs:70-72 */

/* ---- gemm.rs ----------------------------------------------------------- */
/* C[m x n] (+)= op(A) op(B); at: A is [k x m]; bt: B is [n x k]. gemm.rs:434 */
void orc_matmul(int m, int n, int k, const float *a, int at, const float *b,
                int bt, float *c, int acc);
/* C[m x n] += A^T B, A [k x m], B [k x n].  gemm.rs:555-598 */
void orc_matmul_dw(int m, int n, int k, const float *a, const float *b, float *c);
/* naive triple loop, check.rs:105-122 */
void orc_naive_matmul(int m, int n, int k, const float *a, int at,
                      const float *b, int bt, float *c);

/* ---- conv.rs / nn.rs Conv2d -------------------------------------------- */
/* NCHW x [n,cin,h,w]; W [cout, cin*k*k]; y [n,cout,oh,ow].  nn.rs:166-185 */
void orc_conv2d_fwd(const float *x, int n, int cin, int h, int w,
                    const float *wt, int cout, int k, int stride, int pad,
                    float *y);
/* dX = col2im(W^T dY), overwrites dx.  nn.rs:230-250, conv.rs:207-246 */
void orc_conv2d_dgrad(const float *dy, int n, int cin, int h, int w,
                      const float *wt, int cout, int k, int stride, int pad,
                      float *dx);
/* dW += dY im2col(X)^T.  nn.rs:193-227, conv.rs:283-322 */
void orc_conv2d_wgrad(const float *x, const float *dy, int n, int cin, int h,
                      int w, int cout, int k, int stride, int pad, float *dw);

/* ---- nn.rs BatchNorm2d -------------------------------------------------- */
/* Train-mode forward in place on y [n,c,hw] (nn.rs:326-354).  Writes xhat,
 * invstd; updates running mean/var (mom, unbiased var). */
void orc_bn_fwd_train(float *y, int n, int c, int hw, const float *gamma,
                      const float *beta, float *rmean, float *rvar, float mom,
                      float eps, int relu, float *xhat, float *invstd);
/* Eval-mode forward in place (nn.rs:358-369). */
void orc_bn_fwd_eval(float *y, int n, int c, int hw, const float *gamma,
                     const float *beta, const float *rmean, const float *rvar,
                     float eps, int relu);
/* Backward (nn.rs:384-427): dx written, dgamma/dbeta accumulated. */
void orc_bn_bwd(const float *dy, const float *xhat, int n, int c, int hw,
                const float *gamma, const float *invstd, float *dx,
                float *dgamma, float *dbeta);

/* ---- nn.rs glue --------------------------------------------------------- */
void orc_relu_back(float *d, const float *y, size_t len);         /* nn.rs:433 */
void orc_add(float *a, const float *b, size_t len);               /* nn.rs:441 */
void orc_add_relu(float *a, const float *b, size_t len);          /* nn.rs:446 */
void orc_gap_fwd(const float *x, int nc, int hw, float *y);       /* nn.rs:455 */
void orc_gap_bwd(const float *dy, int nc, int hw, float *dx);     /* nn.rs:465 */
/* scalar classifier nn::Linear (nn.rs:501-563) */
void orc_fc_fwd(const float *x, int n, int fin, int fout, const float *w,
                const float *b, float *y);
void orc_fc_bwd(const float *x, const float *dy, int n, int fin, int fout,
                const float *w, float *dw, float *db, float *dx);
/* softmax + CE with smoothing; returns mean loss, writes dlogits (/n).
 * nn.rs:573-637 */
float orc_softmax_ce(const float *logits, const uint32_t *labels, int n,
                     int nclass, float smooth, float *dlogits, int *correct);
/* Param::step, SGD-Nesterov with decoupled wd.  nn.rs:102-110 */
void orc_sgd_step(float *v, float *g, float *m, size_t len, float lr,
                  float mom, float wd, int decay);

/* ---- model.rs ResNet ---------------------------------------------------- */
typedef struct orc_resnet orc_resnet;
orc_resnet *orc_resnet_new(int depth_n, int width, int nclass, uint64_t seed);
void   orc_resnet_free(orc_resnet *net);
size_t orc_resnet_num_params(const orc_resnet *net);
int    orc_resnet_num_tensors(const orc_resnet *net);
/* flat copies in for_each_param order (model.rs:159-168) */
void   orc_resnet_get_params(const orc_resnet *net, float *out);
void   orc_resnet_set_params(orc_resnet *net, const float *in);
void   orc_resnet_get_grads(const orc_resnet *net, float *out);
void   orc_resnet_get_moments(const orc_resnet *net, float *out);
void   orc_resnet_zero_grads(orc_resnet *net);
/* running mean/var of every BN, for_each_buffer order (model.rs:170-176) */
size_t orc_resnet_num_buffers(const orc_resnet *net);
void   orc_resnet_get_buffers(const orc_resnet *net, float *out);
/* per-tensor sizes and decay flags, for_each_param order */
void   orc_resnet_param_info(const orc_resnet *net, int64_t *sizes, int *decay);
/* model.rs:135-146; logits [n, nclass] */
void   orc_resnet_forward(orc_resnet *net, const float *x, int n, int h,
                          int w, int train, float *logits);
/* model.rs:148-157 */
void   orc_resnet_backward(orc_resnet *net, const float *dlogits);
/* model.rs:206-208 */
void   orc_resnet_step(orc_resnet *net, float lr, float mom, float wd);
/* forward + softmax_ce + backward + step (train.rs:684-699) */
float  orc_resnet_train_step(orc_resnet *net, const float *x,
                             const uint32_t *labels, int n, float smooth,
                             float lr, float mom, float wd, int *correct);
/* model.rs:179-198 */
uint64_t orc_resnet_flops(const orc_resnet *net, int h, int w);

/* ---- data.rs / eval.rs: evaluation batches and the eval loop ------------ */
/* make_batch_train (data.rs:384-412) with the augmentation of data.rs:
 * RandAugment on the bytes (ra_n ops of magnitude ra_mag, off at 0,
 * data.rs:100-306), crop offset within `pad` (data.rs:309-318), flip,
 * normalise (data.rs:331-360) and random erasing with probability `erase`
 * of an erase_side square of normal noise (data.rs:364-377).  Image b draws
 * from Rng::new(seed ^ b * 0x9E3779B97F4A7C15).  coarse / coarse_out may be
 * NULL.  (rnn_oracle_data.c) */
void   orc_make_batch_train(const uint8_t *images, const uint8_t *labels,
                            const uint8_t *coarse, const uint32_t *idx, int bs,
                            int pad, float ra_mag, int ra_n, float erase,
                            int erase_side, uint64_t seed, float *out,
                            uint32_t *labels_out, uint32_t *coarse_out);
/* 1: the data pipeline's logf / cosf / sinf return correctly rounded
 * values instead of the C library's (see rnn_oracle_data.c); 0 (default):
 * the C library's, as the reference. */
void   orc_data_set_cr_math(int on);
/* mix_batch (data.rs:467-491): state = the caller's xoshiro256++ state,
 * advanced in place; perm/lam [bs] out; rect (nullable) = {y0, y1, x0, x1}
 * of a cutmix.  Returns 0 (no mixing), 1 (mixup) or 2 (cutmix). */
int    orc_mix_batch(float *x, int bs, float alpha_mix, float alpha_cut,
                     float sw, uint64_t *state, uint32_t *perm, float *lam,
                     int *rect);
/* make_batch_eval (data.rs:494-512): bs images from `start` of a CHW u8
 * dataset of 3 x 32 x 32 images, normalised per channel (data.rs:95-98),
 * mirrored left-right when flip (crop_flip_normalize with no shift,
 * data.rs:331-360); labels widened to u32. */
void   orc_make_batch_eval(const uint8_t *images, const uint8_t *labels,
                           size_t start, int bs, int flip, float *out,
                           uint32_t *labels_out);
/* eval::resnet (eval.rs:15-43): batches of `batch`, forward with train
 * false, softmax_ce without smoothing; out2 = {mean loss, accuracy}. */
void   orc_resnet_eval(orc_resnet *net, const uint8_t *images,
                       const uint8_t *labels, int len, int batch, float *out2);

/* ---- attn.rs ------------------------------------------------------------ */
/* rel_index (attn.rs:53-72): writes th*tw*mh*mw indices when idx != NULL,
 * returns nrel = span_y * span_x (attn.rs:23-46). */
int  orc_rel_index(int th, int tw, int mh, int mw, uint32_t *idx);
/* Core::forward (attn.rs:148-223) over n images: q rows strided by qstride
 * (head hd at column qoff + hd*dh), kv rows by kvstride (K at koff, V at
 * voff), tau[h], rel[h*nrel]; writes p [n,h,tq,tk] and o [n,tq,h*dh]. */
void orc_attn_fwd(int n, int h, int dh, int tq, int tk, int mask_diag,
                  const uint32_t *relidx, int nrel, const float *q, int qstride,
                  int qoff, const float *kv, int kvstride, int koff, int voff,
                  const float *tau, const float *rel, float *p, float *o);
/* Core::backward (attn.rs:226-343): dq, dkv, dtau, drel accumulate. */
void orc_attn_bwd(int n, int h, int dh, int tq, int tk, const uint32_t *relidx,
                  int nrel, const float *q, int qstride, int qoff,
                  const float *kv, int kvstride, int koff, int voff,
                  const float *tau, const float *p, const float *dout,
                  float *dq, float *dkv, float *dtau, float *drel);

/* ---- norm.rs LayerNorm (f64 row statistics) ----------------------------- */
void orc_layernorm_fwd(const float *x, int rows, int c, const float *g,
                       const float *b, float eps, float *y, float *xhat,
                       float *invstd);                         /* norm.rs:38-90 */
void orc_layernorm_bwd(const float *dy, const float *xhat, const float *invstd,
                       int rows, int c, const float *g, float *dx, float *dg,
                       float *db);                             /* norm.rs:92-137 */

/* ---- linear.rs ----------------------------------------------------------- */
/* y[rows, fout] = x W^T + b (b may be NULL), linear.rs:44-63 */
void orc_linear_fwd(const float *x, int rows, int fin, int fout, const float *w,
                    const float *b, float *y);
/* dW += dY^T X; db += colsum(dY) (b may be NULL); dx = dY W; linear.rs:66-96 */
void orc_linear_bwd(const float *x, const float *dy, int rows, int fin, int fout,
                    const float *w, float *dw, float *db, float *dx);

/* ---- optim.rs ------------------------------------------------------------ */
/* newton_schulz in place on g [rows x cols] (optim.rs:70-145) */
void orc_newton_schulz(float *g, int rows, int cols, int steps);
/* one Muon update of one matrix parameter (optim.rs:182-197) */
void orc_muon_step(float *v, float *g, float *m, int rows, int cols, int steps,
                   float lr, float mom, float wd, int decay);
/* step_adam (optim.rs:205-233); t = steps taken before this one */
void orc_adamw_step(float *v, float *g, float *m, float *v2, size_t n, float lr,
                    float wd, int decay, float b1, float b2, float eps, int t);
/* clip_ (optim.rs:237-250) over one flat gradient buffer; returns the norm */
float orc_clip(float *g, size_t n, float max);
/* Ema::update for t >= 2 (optim.rs:270-287): e = d e + (1-d) v */
void orc_ema_update(float *e, const float *v, size_t n, float decay, int t);

/* ---- rustvit glue (norm.rs, vit.rs, tok.rs, loss.rs) -------------------- */
void orc_layerscale_fwd(const float *x, int rows, int c, const float *l, float *y);      /* norm.rs:170-181 */
void orc_layerscale_bwd(const float *dy, const float *x, int rows, int c, const float *l,
                        float *dl, float *dx);                                           /* norm.rs:183-212 */
void orc_swiglu_act_fwd(const float *ab, int rows, int h, float *u);                     /* norm.rs:250-266 */
void orc_swiglu_act_bwd(const float *du, const float *ab, int rows, int h, float *dab);  /* norm.rs:272-286 */
void orc_dwconv3_fwd(const float *x, int n, int th, int tw, int c, const float *w,
                     const float *b, float *y);                                          /* norm.rs:328-368 */
void orc_dwconv3_bwd(const float *dy, const float *x, int n, int th, int tw, int c,
                     const float *w, float *dw, float *db, float *dx);                   /* norm.rs:370-451 */
void orc_seqpool_fwd(const float *x, int n, int t, int c, const float *p, float *z,
                     float *w);                                                          /* norm.rs:488-528 */
void orc_seqpool_bwd(const float *dz, const float *x, const float *w, int n, int t, int c,
                     const float *p, float *dp, float *dx);                              /* norm.rs:530-581 */
void orc_droppath_mask(int n, float p, uint64_t seed, float *mask);                      /* vit.rs:40-60 */
void orc_token_merge_fwd(const float *z, int n, int th, int c, float *y);                /* vit.rs:586-604 */
void orc_token_merge_bwd(const float *dy, int n, int th, int c, float *dz);              /* vit.rs:606-624 */
void orc_tok_from_nchw(const float *x, int n, int c, int hw, float *y);                  /* tok.rs:54-68 */
void orc_tok_to_nchw(const float *x, int n, int c, int hw, float *y);                    /* tok.rs:71-87 */
void orc_taxo_fwd(float *zf, const float *zc, int n, int nf, int nc, const uint32_t *parent); /* vit.rs:283-295 */
void orc_taxo_bwd(const float *dzf, const float *dzc, int n, int nf, int nc,
                  const uint32_t *parent, float *dc);                                    /* vit.rs:297-310 */
float orc_ce_soft(const float *logits, const float *target, const uint32_t *hard, int n,
                  int nclass, float scale, float *dz, int *correct);                     /* loss.rs:39-81 */
float orc_kl_distill(const float *s, const float *t, int n, int nclass, float temp,
                     float scale, float *dz);                                            /* loss.rs:87-130 */
float orc_hint_mse(const float *pred, const float *target, int n, int c, float scale,
                   float *dz);                                                           /* loss.rs:133-151 */

/* rustvit parameter initialisers */
void orc_trunc_normal(orc_rng *r, float *out, size_t n, float std); /* nn.rs:77-89 */
void orc_kaiming(orc_rng *r, float *out, size_t n, int fan_in);      /* nn.rs:95-100 */

/* ---- threads ------------------------------------------------------------ */
void orc_set_threads(int n);
int  orc_get_threads(void);

#ifdef __cplusplus
}
#endif

#endif
