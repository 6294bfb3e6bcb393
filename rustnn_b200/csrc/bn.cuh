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

// SyncBN over peer memory: each rank owns a mailbox in its own HBM (flag +
// two slots of [cmax][2] f64), every rank maps every peer's mailbox (CUDA
// IPC over NVLink).  When passed to the *_sums calls below, the last CTA of
// the partial-sum kernel publishes this rank's per-channel sums, waits
// (bounded) for every peer's, and sums all ranks in rank order, so the
// statistics kernel and the cross-GPU reduction are one launch and every
// rank ends with identical sums.
struct PeerSums {
  int rank = 0, world = 1, cmax = 0;
  char* const* mail = nullptr;        // device array [world]: mailbox base of every rank (own included)
  unsigned long long* seq = nullptr;  // this rank's exchange counter (device)
  int* dev_error = nullptr;
};
constexpr size_t PEER_MAIL_HEADER = 128;
inline size_t peer_mail_bytes(int cmax) { return PEER_MAIL_HEADER + 2 * (size_t)cmax * 2 * sizeof(double); }

// sums[c] = (sum y, sum y^2); with `ps` the sums cover every rank and
// *reduced is set when the kernel did that reduction (else the caller must)
int bn_fwd_sums(rnn_ctx* ctx, const float* y, int n, int C, int hw, double* part, double* sums,
                const PeerSums* ps = nullptr, bool* reduced = nullptr);
// out = [relu](bn(y) [+ res]); res may alias out (the residual join of a block)
int bn_fwd_finish(rnn_ctx* ctx, const float* y, int n, int C, int hw, double count, const double* sums,
                  const float* gamma, const float* beta, float* rmean, float* rvar, float mom, float eps,
                  int relu, float* mean, float* invstd, float* out, const float* res = nullptr);
// sums[c] = (sum dy*xhat, sum dy)
int bn_bwd_sums(rnn_ctx* ctx, const float* dy, const float* y, const float* relu_out, int n, int C, int hw,
                const float* mean, const float* invstd, double* part, double* sums, const PeerSums* ps = nullptr,
                bool* reduced = nullptr);
int bn_bwd_finish(rnn_ctx* ctx, const float* dy, const float* y, const float* relu_out, int n, int C, int hw,
                  double count, const double* sums, const float* gamma, const float* mean,
                  const float* invstd, float* dgb, float* dx, float* dgamma, float* dbeta, float pscale);

}  // namespace rnn
