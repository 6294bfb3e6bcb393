// BatchNorm building blocks shared by the C ABI and the ResNet step.  The
// forward/backward are split at the per-channel [C][2] f64 sums so that the
// data-parallel step can all-reduce them (SyncBN) between the two halves.
#pragma once

#include "common.cuh"

namespace rnn {

size_t bn_scratch_bytes(int n, int C, int num_sms);
// Number of per-channel partial sums the BN kernels write ([C][P][2] f64);
// every caller that lays out its own partial buffer must use this count.
int bn_parts(int n, int C, int num_sms);

// sums[c] = (sum y, sum y^2)
int bn_fwd_sums(rnn_ctx* ctx, const float* y, int n, int C, int hw, double* part, double* sums);
int bn_fwd_finish(rnn_ctx* ctx, const float* y, int n, int C, int hw, double count, const double* sums,
                  const float* gamma, const float* beta, float* rmean, float* rvar, float mom, float eps,
                  int relu, float* mean, float* invstd, float* out);
// sums[c] = (sum dy*xhat, sum dy)
int bn_bwd_sums(rnn_ctx* ctx, const float* dy, const float* y, const float* relu_out, int n, int C, int hw,
                const float* mean, const float* invstd, double* part, double* sums);
int bn_bwd_finish(rnn_ctx* ctx, const float* dy, const float* y, const float* relu_out, int n, int C, int hw,
                  double count, const double* sums, const float* gamma, const float* mean,
                  const float* invstd, float* dgb, float* dx, float* dgamma, float* dbeta, float pscale);

}  // namespace rnn
