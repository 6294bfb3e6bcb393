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

}  // namespace rnn
