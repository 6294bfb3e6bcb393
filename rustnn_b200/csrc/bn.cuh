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
  unsigned long long wait_ns = 5000000000ull;  // bound of the wait for a peer's flag
};
constexpr size_t PEER_MAIL_HEADER = 128;
inline size_t peer_mail_bytes(int cmax) { return PEER_MAIL_HEADER + 2 * (size_t)cmax * 2 * sizeof(double); }

#ifdef __CUDACC__
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Cross-rank step of the last CTA (all its threads; `sums` holds this
// rank's totals): publish them in slot seq&1 of the own mailbox, raise the
// flag to seq, wait for every peer's flag (bounded: wait_ns, 5 s in the
// training step, then an error bit and garbage instead of a hang), and sum
// every rank's slot in rank order.
// Two slots suffice: a rank can only publish seq+2 after passing the wait
// for seq+1, which needs this rank's flag, raised after it read seq.
__device__ inline void peer_exchange(const PeerSums& ps, double* sums, int C) {
  __shared__ unsigned long long seq;
  if (threadIdx.x == 0) seq = ++(*ps.seq);
  __syncthreads();
  const size_t slot_off = PEER_MAIL_HEADER + (size_t)(seq & 1) * ps.cmax * 2 * sizeof(double);
  double* mine = reinterpret_cast<double*>(ps.mail[ps.rank] + slot_off);
  for (int c = threadIdx.x; c < 2 * C; c += blockDim.x) mine[c] = sums[c];
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<unsigned long long*>(ps.mail[ps.rank]), seq);
  }
  if ((int)threadIdx.x < ps.world && (int)threadIdx.x != ps.rank) {
    const unsigned long long* flag = reinterpret_cast<const unsigned long long*>(ps.mail[threadIdx.x]);
    const unsigned long long t0 = gtimer();
    while (ld_acquire_sys(flag) < seq) {
      if (gtimer() - t0 > ps.wait_ns) {
        if (ps.dev_error) atomicOr(ps.dev_error, DEV_ERR_PEER);
        break;
      }
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * C; c += blockDim.x) {
    double t = 0.0;
    for (int r = 0; r < ps.world; r++) {
      const double* d = reinterpret_cast<const double*>(ps.mail[r] + slot_off);
      t += r == ps.rank ? mine[c] : __ldcv(d + c);
    }
    sums[c] = t;
  }
}

#endif

// sums[c] = (sum y, sum y^2); with `ps` the sums cover every rank and
// *reduced is set when the kernel did that reduction (else the caller must)
int bn_fwd_sums(rnn_ctx* ctx, const float* y, int n, int C, int hw, double* part, double* sums,
                const PeerSums* ps = nullptr, bool* reduced = nullptr);
// out = [relu](bn(y) [+ res]); res may alias out (the residual join of a block)
int bn_fwd_finish(rnn_ctx* ctx, const float* y, int n, int C, int hw, double count, const double* sums,
                  const float* gamma, const float* beta, float* rmean, float* rvar, float mom, float eps,
                  int relu, float* mean, float* invstd, float* out, const float* res = nullptr,
                  uint32_t* mask = nullptr, bool* masked = nullptr);
// With `mask` (relu), the ReLU outcome is also stored as bits (bit e of word
// e/32 set where out[e] > 0) when the shape allows; *masked says it was.
// The backward calls below accept those bits (relu_mask) instead of
// re-reading the float relu_out (which they still use as the fallback).
// sums[c] = (sum dy*xhat, sum dy)
int bn_bwd_sums(rnn_ctx* ctx, const float* dy, const float* y, const float* relu_out, int n, int C, int hw,
                const float* mean, const float* invstd, double* part, double* sums, const PeerSums* ps = nullptr,
                bool* reduced = nullptr, const uint32_t* relu_mask = nullptr);
int bn_bwd_finish(rnn_ctx* ctx, const float* dy, const float* y, const float* relu_out, int n, int C, int hw,
                  double count, const double* sums, const float* gamma, const float* mean,
                  const float* invstd, float* dgb, float* dx, float* dgamma, float* dbeta, float pscale,
                  float* pack = nullptr, int pack_bn = 0, bool* packed = nullptr,
                  const uint32_t* relu_mask = nullptr);
// With `pack` (pack_bn == C), dx is also written as the hi/lo B image a
// 3x3 wgrad consumes (see tc::wgrad_dy_pack_bn); *packed says it was.

}  // namespace rnn
