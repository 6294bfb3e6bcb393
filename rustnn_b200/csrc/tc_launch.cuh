// Host-side launch plumbing for the tcgen05 engine: tile-width choice,
// split-K choice, the persistent grid, and the deterministic split-K
// reduction.
#pragma once

#include <algorithm>
#include <atomic>
#include <type_traits>

#include "common.cuh"
#include "tc_gemm.cuh"

namespace rnn {
namespace tc {

// Writes 32 consecutive values of one output row (row-major destination).
// `nvalid` columns are in range; `vec` means dst is 16-byte aligned and the
// row holds all 32 (vector stores).
__device__ __forceinline__ void store_row32(float* dst, int nvalid, const float (&v)[32], bool acc,
                                            bool vec) {
  if (vec && nvalid >= 32) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      float4* p = reinterpret_cast<float4*>(dst + j);
      float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      if (acc) {
        float4 c = *p;
        o.x += c.x; o.y += c.y; o.z += c.z; o.w += c.w;
      }
      *p = o;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; j++)
      if (j < nvalid) dst[j] = acc ? dst[j] + v[j] : v[j];
  }
}

// out[r, c] (+)= sum_s ws[s, r, c] over a row-major [rows x cols] result;
// when `transpose`, out is indexed [c, r] instead.  The summation order over
// s is fixed, so the result is deterministic.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, float* __restrict__ out, int rows,
                                     int cols, int splits, int acc, int transpose);

int launch_splitk_reduce(rnn_ctx* ctx, const float* ws, float* out, int rows, int cols, int splits,
                         bool acc, bool transpose);

inline int pick_bn(int N, int m_tiles, int num_sms) {
  int best = 32;
  long best_cost = -1;
  for (int bn : {32, 64, 128, 256}) {
    long nt = (N + bn - 1) / bn;
    long tiles = (long)m_tiles * nt;
    long waves = (tiles + num_sms - 1) / num_sms;
    long cost = waves * (128 + bn);
    if (best_cost < 0 || cost <= best_cost) {
      best_cost = cost;
      best = bn;
    }
    if (bn >= N) break;  // wider tiles only add padding
  }
  return best;
}

inline Sched make_sched(int M, int N, int K, int bn, int splits) {
  Sched s;
  s.m_tiles = (M + BM - 1) / BM;
  s.n_tiles = (N + bn - 1) / bn;
  s.kblocks = (K + BK - 1) / BK;
  if (splits < 1) splits = 1;
  if (splits > s.kblocks) splits = s.kblocks;
  s.kb_per_split = (s.kblocks + splits - 1) / splits;
  s.splits = (s.kblocks + s.kb_per_split - 1) / s.kb_per_split;
  s.num_tiles = s.m_tiles * s.n_tiles * s.splits;
  return s;
}

// Split count that fills the SMs when the output tiles alone cannot.
inline int pick_splits(int M, int N, int K, int bn, int num_sms) {
  long tiles = (long)((M + BM - 1) / BM) * ((N + bn - 1) / bn);
  int kblocks = (K + BK - 1) / BK;
  if (tiles * 2 > num_sms || kblocks < 8) return 1;
  long s = num_sms / tiles;
  s = std::min<long>(s, kblocks / 4);
  return (int)std::max<long>(s, 1);
}

// True for problem types written against the engine's native interface
// (they define a per-thread tile state TS); others go through ChunkProb.
template <class P, class = void>
struct has_ts : std::false_type {};
template <class P>
struct has_ts<P, std::void_t<typename P::TS>> : std::true_type {};

// cudaFuncSetAttribute acts on the current device only, so the dynamic
// shared-memory opt-in of a kernel is recorded per device: one bit per device
// ordinal below 64 in an atomic mask (two threads that race both set the same
// attribute, which is harmless); devices beyond 63 set it on every launch.
template <class Kernel>
int ensure_smem_optin(Kernel kernel, std::atomic<unsigned long long>& done, int device, int bytes) {
  const unsigned long long bit = device >= 0 && device < 64 ? 1ull << device : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return RNN_OK;
  RNN_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  if (bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return RNN_OK;
}

template <int BN, class Prob>
int launch_native(rnn_ctx* ctx, const Prob& prob, const Sched& sched) {
  using C = CfgOf<Prob, BN>;
  static std::atomic<unsigned long long> optin_done{0};  // per instantiation, one bit per device
  RNN_TRY(ensure_smem_optin(tc3_gemm_kernel<BN, Prob>, optin_done, ctx->device, C::SMEM_BYTES));
  if (sched.num_tiles <= 0) return RNN_OK;
  int grid = std::min(sched.num_tiles, ctx->num_sms);
  tc3_gemm_kernel<BN, Prob><<<grid, C::THREADS, C::SMEM_BYTES, ctx->stream>>>(prob, sched, ctx->dev_error);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

template <int BN, class Prob>
int launch(rnn_ctx* ctx, const Prob& prob, const Sched& sched) {
  if constexpr (has_ts<Prob>::value) {
    return launch_native<BN>(ctx, prob, sched);
  } else {
    ChunkProb<Prob, BN> w;
    static_cast<Prob&>(w) = prob;
    return launch_native<BN>(ctx, w, sched);
  }
}

// Packs the B operand image for every (n tile, K block) into `out`
// (ensure_pack must have sized it: n_tiles * kblocks * 2 * BN * BK floats).
template <int BN, class Src>
int launch_pack(rnn_ctx* ctx, const Src& src, int n_tiles, int kblocks, float* out) {
  const long chunks = (long)n_tiles * kblocks * BN * 8;
  const unsigned grid = (unsigned)std::min<long>((chunks + 255) / 256, (long)ctx->num_sms * 8);
  pack_b_kernel<BN, Src><<<grid, 256, 0, ctx->stream>>>(src, n_tiles, kblocks, out);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

// Dispatches on the runtime tile width.
template <template <int> class Launcher, class... Args>
int dispatch_bn(int bn, Args&&... args) {
  switch (bn) {
    case 32: return Launcher<32>::run(args...);
    case 64: return Launcher<64>::run(args...);
    case 128: return Launcher<128>::run(args...);
    default: return Launcher<256>::run(args...);
  }
}

}  // namespace tc
}  // namespace rnn
