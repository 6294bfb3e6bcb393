// Glue kernels of the ResNet step (nn.rs), callable from the model code.
#pragma once

#include "common.cuh"

namespace rnn {

int relu_back(rnn_ctx* ctx, float* d, const float* y, size_t n);
int add(rnn_ctx* ctx, float* a, const float* b, size_t n, bool relu);
// a += (y <= 0 ? 0 : b)
// (with `mask`, the ReLU outcome as bits instead of y: bit e of word e/32)
int add_masked(rnn_ctx* ctx, float* a, const float* b, const float* y, size_t n, const uint32_t* mask = nullptr);
int gap_fwd(rnn_ctx* ctx, const float* x, int nc, int hw, float* y);
int gap_bwd(rnn_ctx* ctx, const float* dy, int nc, int hw, float* dx);
int fc_fwd(rnn_ctx* ctx, const float* x, int n, int fin, int fout, const float* w, const float* b, float* y);
int fc_bwd(rnn_ctx* ctx, const float* x, const float* dy, int n, int fin, int fout, const float* w, float* dw,
           float* db, float* dx);
int softmax_ce(rnn_ctx* ctx, const float* logits, const uint32_t* labels, int n, int nclass, float smooth,
               float* dlogits, float* row_loss, int* hit, float* loss_out, int* correct_out);
int sgd_nesterov(rnn_ctx* ctx, float* v, float* g, float* m, const uint8_t* decay_mask, int decay_all, size_t n,
                 float lr, float mom, float wd, float gscale);

struct PeerSums;
namespace tc {
// BatchNorm statistics requested from a forward convolution's epilogue:
// with `sums` set, conv_fwd may fill it with per-channel (sum y, sum y^2)
// of its output (over every rank when `ps` has peers) and sets `fused`;
// `reduced` says the sums already cover all ranks.
struct ConvStats {
  double* sums = nullptr;
  const PeerSums* ps = nullptr;
  bool fused = false;
  bool reduced = false;
};
int gemm_dev(rnn_ctx* ctx, int m, int n, int k, const float* a, bool at, const float* b, bool bt, float* c,
             bool acc, bool force_split);
// batch same-shape GEMMs in one launch: C_i (+)= op(A_i) op(B_i), item i at
// a + i*sa, b + i*sb, c + i*sc (strides in floats)
int gemm_batched_dev(rnn_ctx* ctx, int batch, int m, int n, int k, const float* a, size_t sa, bool at,
                     const float* b, size_t sb, bool bt, float* c, size_t sc, bool acc);
int conv_fwd(rnn_ctx* ctx, const float* x, int n, int cin, int h, int w, const float* wt, int cout, int k,
             int stride, int pad, float* y, bool acc, ConvStats* stats = nullptr);
int conv_dgrad(rnn_ctx* ctx, const float* dy, int n, int cin, int h, int w, const float* wt, int cout, int k,
               int stride, int pad, float* dx, bool acc);
int conv_wgrad(rnn_ctx* ctx, const float* x, const float* dy, int n, int cin, int h, int w, int cout, int k,
               int stride, int pad, float* dw, int force_splits, const float* dy_packed = nullptr);
// Tile width of the packed dY image conv_wgrad would build for these shapes
// when a producer of dY may write it instead (one column tile, cout == the
// tile width, 32-pixel K blocks); 0 when it would not use one.
int wgrad_dy_pack_bn(int n, int cout, int k, int oh, int ow, const void* dy);
}  // namespace tc
// Backward of LayerNorm (norm.rs:96-135), Linear (linear.rs:66-96) and the
// depthwise 3x3 (vit.rs DwConv3) as the C entries compute them, except that
// with acc_dx the input gradient is added into dx (dx += ...) instead of
// stored: the residual joins of the rustvit backward take it that way.
int layernorm_bwd(rnn_ctx* ctx, const float* dy, const float* xhat, const float* invstd, int rows, int c,
                  const float* g, float* dx, float* dg, float* db, bool acc_dx);
int linear_bwd(rnn_ctx* ctx, const float* x, const float* dy, int rows, int fin, int fout, const float* w, float* dw,
               float* db, float* dx, bool acc_dx);
int dwconv3_bwd(rnn_ctx* ctx, const float* dy, const float* x, int n, int th, int tw, int c, const float* w,
                float* dw, float* db, float* dx, bool acc_dx);
// One launch of an optimiser update over many parameter segments of the flat
// value / gradient / moment buffers (a table in device memory): segment s
// covers elements [off, off + n); scale is Muon's update scale and decay the
// parameter's weight-decay flag.  Per element the arithmetic is that of the
// single-tensor kernels, so a segmented launch equals one launch per segment.
struct OptSeg {
  size_t off, n;
  float scale;
  int decay;
};
int muon_momentum_segs(rnn_ctx* ctx, float* g, float* m, const OptSeg* segs, int nseg, size_t max_n, float mom);
int muon_update_segs(rnn_ctx* ctx, float* v, float* g, const OptSeg* segs, int nseg, size_t max_n, float lr,
                     float wd);
int adamw_segs(rnn_ctx* ctx, float* v, float* g, float* m, float* v2, const OptSeg* segs, int nseg, size_t max_n,
               float lr, float wd, float b1, float b2, float eps, int t);
float muon_scale(int rows, int cols);
// Newton-Schulz (optim.rs:124-145) in place on `count` matrices, the
// matrices of one working shape batched into shared launches (optim.cu)
int newton_schulz_grouped(rnn_ctx* ctx, int count, float* const* g, const int* rows, const int* cols, int steps);
// Muon's momentum (optim.rs:186-190) and update (optim.rs:192-196) of one
// matrix; rnn_muon_step_dev is momentum, newton_schulz, update
int muon_momentum(rnn_ctx* ctx, float* g, float* m, size_t n, float mom);
int muon_update(rnn_ctx* ctx, float* v, float* g, int rows, int cols, float lr, float wd, int decay);

}  // namespace rnn
