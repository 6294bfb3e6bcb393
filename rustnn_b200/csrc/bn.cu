// BatchNorm2d on device (nn.rs:255-428), NCHW.
//
// Forward (train): per-channel sums of y and y^2 in f64 (nn.rs:301-322) as
// fixed-partition partials -> per-channel combine (the SyncBN allreduce hooks
// in between) -> finalize (mean, var, invstd, running stats, nn.rs:330-336)
// -> apply out = gamma*xhat + beta (+ReLU) (nn.rs:338-353).  xhat is not
// stored: the backward recomputes (y - mean) * invstd bit-identically.
//
// Backward (nn.rs:384-427): per-channel sums of dy and dy*xhat, then
// dx = gamma*invstd/m * (m*dy - sum(dy) - xhat*sum(dy*xhat)).  An optional
// relu_out mask applies relu_back_ (nn.rs:433) to dy on the fly.
#include <algorithm>
#include <cstdint>
#include <initializer_list>

#include "bn.cuh"
#include "tc_gemm.cuh"

namespace rnn {

static __device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Two double sums per block -> part[blk*2 + {0,1}]
template <int NT>
static __device__ __forceinline__ void block_sum2(double a, double b, double* out) {
  __shared__ double sa[NT / 32], sb[NT / 32];
  a = warp_sum_d(a);
  b = warp_sum_d(b);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { sa[w] = a; sb[w] = b; }
  __syncthreads();
  if (w == 0) {
    a = l < NT / 32 ? sa[l] : 0.0;
    b = l < NT / 32 ? sb[l] : 0.0;
    a = warp_sum_d(a);
    b = warp_sum_d(b);
    if (l == 0) { out[0] = a; out[1] = b; }
  }
}

// The last CTA of a partial-sum launch to finish sums the [C][P][2]
// partials in a fixed order (so the result is deterministic) and writes
// sums[C][2]; with peers it then runs the cross-rank exchange; it finally
// returns the counter to zero for the next launch.
static __device__ __forceinline__ void last_block_combine(const double* part, int C, int P,
                                                          unsigned* counter, double* sums, PeerSums ps) {
  __shared__ bool last;
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(counter, 1u);
    last = prev == gridDim.x * gridDim.y - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    double a = 0.0, b = 0.0;
    for (int p = 0; p < P; p++) {
      a += __ldcg(part + ((size_t)c * P + p) * 2);
      b += __ldcg(part + ((size_t)c * P + p) * 2 + 1);
    }
    sums[c * 2] = a;
    sums[c * 2 + 1] = b;
  }
  if (ps.world > 1) {
    __syncthreads();
    peer_exchange(ps, sums, C);
  }
  if (threadIdx.x == 0) *counter = 0u;
}

constexpr int BN_NT = 256;
constexpr int BN_U = 4;  // float4 loads in flight per thread and stream
constexpr int BN_FUSE_MAX_C = 4096;  // fused finalize keeps 2*C floats (<= 32 KB) per CTA in shared memory

// grid (C, P): block (c, p) sums the planes of images [n*p/P, n*(p+1)/P) of
// channel c.  Scalar form, for hw % 4 != 0 or unaligned tensors.
__global__ void __launch_bounds__(BN_NT) bn_fwd_partial_kernel(const float* __restrict__ y, int n, int C,
                                                             int hw, int P, double* __restrict__ part) {
  const int c = blockIdx.x, p = blockIdx.y;
  const int i0 = (int)((long)n * p / P), i1 = (int)((long)n * (p + 1) / P);
  double s = 0.0, s2 = 0.0;
  for (int img = i0; img < i1; img++) {
    const float* plane = y + ((size_t)img * C + c) * hw;
    for (int q = threadIdx.x; q < hw; q += BN_NT) {
      double v = __ldg(plane + q);
      s += v;
      s2 += v * v;
    }
  }
  block_sum2<BN_NT>(s, s2, part + ((size_t)c * P + p) * 2);
}

// Vector form: the block's planes are flattened into one float4 index space
// (so small planes still occupy every thread) and each thread keeps BN_U
// independent loads in flight.
__global__ void __launch_bounds__(BN_NT) bn_fwd_partial4_kernel(const float4* __restrict__ y, int n, int C,
                                                              int hw4, int P, double* __restrict__ part,
                                                              unsigned* counter, double* __restrict__ sums,
                                                              PeerSums ps) {
  const int c = blockIdx.x, p = blockIdx.y;
  const int i0 = (int)((long)n * p / P), i1 = (int)((long)n * (p + 1) / P);
  const unsigned tot = (unsigned)(i1 - i0) * (unsigned)hw4;
  double s = 0.0, s2 = 0.0;
  for (unsigned j = threadIdx.x; j < tot; j += BN_NT * BN_U) {
    float4 v[BN_U];
#pragma unroll
    for (int u = 0; u < BN_U; u++) {
      const unsigned jj = j + u * BN_NT;
      if (jj < tot) {
        const unsigned img = jj / (unsigned)hw4, q = jj - img * (unsigned)hw4;
        v[u] = __ldg(y + ((size_t)(i0 + img) * C + c) * hw4 + q);
      } else {
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int u = 0; u < BN_U; u++) {
      s += (double)v[u].x + (double)v[u].y + (double)v[u].z + (double)v[u].w;
      s2 += (double)v[u].x * v[u].x + (double)v[u].y * v[u].y + (double)v[u].z * v[u].z +
            (double)v[u].w * v[u].w;
    }
  }
  block_sum2<BN_NT>(s, s2, part + ((size_t)c * P + p) * 2);
  last_block_combine(part, C, P, counter, sums, ps);
}

// Backward partials: sum dy_eff * xhat and dy_eff (scalar form).
__global__ void __launch_bounds__(BN_NT) bn_bwd_partial_kernel(const float* __restrict__ dy,
                                                             const float* __restrict__ y,
                                                             const float* __restrict__ relu_out, int n,
                                                             int C, int hw, int P,
                                                             const float* __restrict__ mean,
                                                             const float* __restrict__ invstd,
                                                             double* __restrict__ part) {
  const int c = blockIdx.x, p = blockIdx.y;
  const int i0 = (int)((long)n * p / P), i1 = (int)((long)n * (p + 1) / P);
  const float mu = mean[c], is = invstd[c];
  double a = 0.0, b = 0.0;
  for (int img = i0; img < i1; img++) {
    const size_t base = ((size_t)img * C + c) * hw;
    for (int q = threadIdx.x; q < hw; q += BN_NT) {
      float d = __ldg(dy + base + q);
      if (relu_out && __ldg(relu_out + base + q) <= 0.0f) d = 0.0f;
      const float xh = (__ldg(y + base + q) - mu) * is;
      a += (double)d * (double)xh;
      b += (double)d;
    }
  }
  block_sum2<BN_NT>(a, b, part + ((size_t)c * P + p) * 2);
}

// ReLU masks kept as bits (RELU mode 2): bit e of word e/32 is set where the
// forward's ReLU output was > 0.  float4 index o covers bits 4*(o%8)..+3 of
// word o/8.
static __device__ __forceinline__ float4 mask4(const uint32_t* __restrict__ m, size_t o) {
  const uint32_t w = __ldg(m + (o >> 3)) >> (4 * (unsigned)(o & 7));
  return make_float4((w & 1u) ? 1.f : 0.f, (w & 2u) ? 1.f : 0.f, (w & 4u) ? 1.f : 0.f, (w & 8u) ? 1.f : 0.f);
}

// Writes the mask bits of float4 jj's four values (> 0) from a full warp
// whose lanes hold consecutive jj: eight lanes share one word.
static __device__ __forceinline__ void store_mask4(uint32_t* __restrict__ m, unsigned jj, const float (&o)[4]) {
  uint32_t v = (o[0] > 0.f ? 1u : 0u) | (o[1] > 0.f ? 2u : 0u) | (o[2] > 0.f ? 4u : 0u) | (o[3] > 0.f ? 8u : 0u);
  v <<= 4 * (jj & 7);
  v |= __shfl_xor_sync(0xffffffffu, v, 1);
  v |= __shfl_xor_sync(0xffffffffu, v, 2);
  v |= __shfl_xor_sync(0xffffffffu, v, 4);
  if ((jj & 7) == 0) m[jj >> 3] = v;
}

static __device__ __forceinline__ void bwd_acc(float d, float yv, float r, bool has_r, float mu, float is,
                                               double& a, double& b) {
  if (has_r && r <= 0.0f) d = 0.0f;
  const float xh = (yv - mu) * is;
  a += (double)d * (double)xh;
  b += (double)d;
}

// RELU: 0 no mask, 1 relu_out (float), 2 relu_mask (bits)
template <int RELU>
__global__ void __launch_bounds__(BN_NT) bn_bwd_partial4_kernel(const float4* __restrict__ dy,
                                                              const float4* __restrict__ y,
                                                              const float4* __restrict__ relu_out,
                                                              const uint32_t* __restrict__ relu_mask, int n,
                                                              int C, int hw4, int P,
                                                              const float* __restrict__ mean,
                                                              const float* __restrict__ invstd,
                                                              double* __restrict__ part, unsigned* counter,
                                                              double* __restrict__ sums, PeerSums ps) {
  const int c = blockIdx.x, p = blockIdx.y;
  const int i0 = (int)((long)n * p / P), i1 = (int)((long)n * (p + 1) / P);
  const unsigned tot = (unsigned)(i1 - i0) * (unsigned)hw4;
  const float mu = mean[c], is = invstd[c];
  double a = 0.0, b = 0.0;
  for (unsigned j = threadIdx.x; j < tot; j += BN_NT * BN_U) {
    float4 d[BN_U], v[BN_U], r[BN_U];
#pragma unroll
    for (int u = 0; u < BN_U; u++) {
      const unsigned jj = j + u * BN_NT;
      if (jj < tot) {
        const unsigned img = jj / (unsigned)hw4, q = jj - img * (unsigned)hw4;
        const size_t o = ((size_t)(i0 + img) * C + c) * hw4 + q;
        d[u] = __ldg(dy + o);
        v[u] = __ldg(y + o);
        if (RELU == 1) r[u] = __ldg(relu_out + o);
        if (RELU == 2) r[u] = mask4(relu_mask, o);
      } else {
        d[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        v[u] = make_float4(mu, mu, mu, mu);
        if (RELU) r[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int u = 0; u < BN_U; u++) {
      bwd_acc(d[u].x, v[u].x, RELU ? r[u].x : 1.f, RELU, mu, is, a, b);
      bwd_acc(d[u].y, v[u].y, RELU ? r[u].y : 1.f, RELU, mu, is, a, b);
      bwd_acc(d[u].z, v[u].z, RELU ? r[u].z : 1.f, RELU, mu, is, a, b);
      bwd_acc(d[u].w, v[u].w, RELU ? r[u].w : 1.f, RELU, mu, is, a, b);
    }
  }
  block_sum2<BN_NT>(a, b, part + ((size_t)c * P + p) * 2);
  last_block_combine(part, C, P, counter, sums, ps);
}

// part [C][P][2] -> sums [C][2] in fixed order
__global__ void bn_combine_kernel(const double* __restrict__ part, int C, int P, double* __restrict__ sums) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  double a = 0.0, b = 0.0;
  for (int p = 0; p < P; p++) {
    a += part[((size_t)c * P + p) * 2];
    b += part[((size_t)c * P + p) * 2 + 1];
  }
  sums[c * 2] = a;
  sums[c * 2 + 1] = b;
}

// nn.rs:317-319 and 330-336
__global__ void bn_finalize_kernel(const double* __restrict__ sums, int C, double m, float mom, float eps,
                                   float* __restrict__ mean, float* __restrict__ invstd,
                                   float* __restrict__ rmean, float* __restrict__ rvar) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const double mu = sums[c * 2] / m;
  double va = sums[c * 2 + 1] / m - mu * mu;
  const float muf = (float)mu;
  const float var = (float)(va > 0.0 ? va : 0.0);
  mean[c] = muf;
  invstd[c] = 1.0f / sqrtf(var + eps);
  const float mf = (float)m;
  if (rmean) rmean[c] = (1.0f - mom) * rmean[c] + mom * muf;
  if (rvar) {
    const float den = (mf - 1.0f) > 1.0f ? (mf - 1.0f) : 1.0f;
    const float unb = var * mf / den;
    rvar[c] = (1.0f - mom) * rvar[c] + mom * unb;
  }
}

// sums [C][2] = (sum dy*xhat, sum dy) -> dgamma += , dbeta +=, and the f32
// copies used by the dx kernel
__global__ void bn_bwd_finalize_kernel(const double* __restrict__ sums, int C, float* __restrict__ dg_out,
                                       float* __restrict__ db_out, float* __restrict__ dgamma,
                                       float* __restrict__ dbeta, float pscale) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const float dg = (float)sums[c * 2], db = (float)sums[c * 2 + 1];
  dg_out[c] = dg;
  db_out[c] = db;
  if (dgamma) dgamma[c] += dg * pscale;
  if (dbeta) dbeta[c] += db * pscale;
}

__global__ void bn_apply_kernel(const float* __restrict__ y, int C, int hw, size_t total,
                                const float* __restrict__ gamma, const float* __restrict__ beta,
                                const float* __restrict__ mean, const float* __restrict__ invstd, int relu,
                                const float* res, float* out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)((i / hw) % C);
    const float xh = (y[i] - mean[c]) * invstd[c];
    float v = gamma[c] * xh + beta[c];
    if (res) v += res[i];
    out[i] = relu ? fmaxf(v, 0.0f) : v;
  }
}

// Vector forms of apply and dx: float4 index j lies in plane j / hw4, whose
// channel is plane % C; BN_U independent float4s per thread per iteration.
__global__ void __launch_bounds__(256) bn_apply4_kernel(const float4* __restrict__ y, int C, unsigned hw4,
                                                        unsigned total4, const float* __restrict__ gamma,
                                                        const float* __restrict__ beta,
                                                        const float* __restrict__ mean,
                                                        const float* __restrict__ invstd, int relu,
                                                        const float4* res, float4* out, uint32_t* mask_out) {
  const unsigned stride = gridDim.x * blockDim.x;
  for (unsigned j = blockIdx.x * blockDim.x + threadIdx.x; j < total4; j += stride * BN_U) {
    float4 v[BN_U];
#pragma unroll
    for (int u = 0; u < BN_U; u++) {
      const unsigned jj = j + u * stride;
      if (jj < total4) v[u] = __ldg(y + jj);
    }
#pragma unroll
    for (int u = 0; u < BN_U; u++) {
      const unsigned jj = j + u * stride;
      if (jj >= total4) break;
      const int c = (int)((jj / hw4) % (unsigned)C);
      const float mu = __ldg(mean + c), is = __ldg(invstd + c), g = __ldg(gamma + c), bt = __ldg(beta + c);
      float4 o;
      o.x = g * ((v[u].x - mu) * is) + bt;
      o.y = g * ((v[u].y - mu) * is) + bt;
      o.z = g * ((v[u].z - mu) * is) + bt;
      o.w = g * ((v[u].w - mu) * is) + bt;
      if (res) {
        const float4 r = res[jj];
        o.x += r.x; o.y += r.y; o.z += r.z; o.w += r.w;
      }
      if (relu) {
        o.x = fmaxf(o.x, 0.0f);
        o.y = fmaxf(o.y, 0.0f);
        o.z = fmaxf(o.z, 0.0f);
        o.w = fmaxf(o.w, 0.0f);
      }
      out[jj] = o;
      if (mask_out) {
        const float m[4] = {o.x, o.y, o.z, o.w};
        store_mask4(mask_out, jj, m);
      }
    }
  }
}

template <int RELU>
__global__ void __launch_bounds__(256) bn_dx4_kernel(const float4* __restrict__ dy, const float4* __restrict__ y,
                                                     const float4* __restrict__ relu_out,
                                                     const uint32_t* __restrict__ relu_mask, int C, unsigned hw4,
                                                     unsigned total4, float m, const float* __restrict__ gamma,
                                                     const float* __restrict__ mean,
                                                     const float* __restrict__ invstd,
                                                     const float* __restrict__ dg, const float* __restrict__ db,
                                                     float4* __restrict__ dx) {
  const unsigned stride = gridDim.x * blockDim.x;
  for (unsigned j = blockIdx.x * blockDim.x + threadIdx.x; j < total4; j += stride * BN_U) {
    float4 d[BN_U], v[BN_U], r[BN_U];
#pragma unroll
    for (int u = 0; u < BN_U; u++) {
      const unsigned jj = j + u * stride;
      if (jj < total4) {
        d[u] = __ldg(dy + jj);
        v[u] = __ldg(y + jj);
        if (RELU == 1) r[u] = __ldg(relu_out + jj);
        if (RELU == 2) r[u] = mask4(relu_mask, jj);
      }
    }
#pragma unroll
    for (int u = 0; u < BN_U; u++) {
      const unsigned jj = j + u * stride;
      if (jj >= total4) break;
      const int c = (int)((jj / hw4) % (unsigned)C);
      const float mu = __ldg(mean + c), is = __ldg(invstd + c);
      const float s = __ldg(gamma + c) * is / m, dbc = __ldg(db + c), dgc = __ldg(dg + c);
      float dd[4] = {d[u].x, d[u].y, d[u].z, d[u].w};
      const float vv[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      if (RELU) {
        const float rr[4] = {r[u].x, r[u].y, r[u].z, r[u].w};
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (rr[e] <= 0.0f) dd[e] = 0.0f;
      }
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float xh = (vv[e] - mu) * is;
        o[e] = s * (m * dd[e] - dbc - xh * dgc);
      }
      dx[jj] = make_float4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Fused finalize + apply (nn.rs:317-353): every CTA derives mean and invstd
// of all channels from the f64 sums into shared memory (identical
// arithmetic to bn_finalize_kernel); CTA 0 also stores them for the backward
// and updates the running statistics.
__global__ void __launch_bounds__(256) bn_apply4_fin_kernel(const float4* __restrict__ y, int C, unsigned hw4,
                                                            unsigned total4, const float* __restrict__ gamma,
                                                            const float* __restrict__ beta,
                                                            const double* __restrict__ sums, double m, float mom,
                                                            float eps, float* __restrict__ rmean,
                                                            float* __restrict__ rvar, int relu,
                                                            float* __restrict__ mean_out,
                                                            float* __restrict__ invstd_out,
                                                            const float4* res, float4* out, uint32_t* mask_out) {
  extern __shared__ float sh[];
  float* smu = sh;
  float* sis = sh + C;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const double mu = sums[c * 2] / m;
    const double va = sums[c * 2 + 1] / m - mu * mu;
    const float muf = (float)mu;
    const float var = (float)(va > 0.0 ? va : 0.0);
    const float is = 1.0f / sqrtf(var + eps);
    smu[c] = muf;
    sis[c] = is;
    if (blockIdx.x == 0) {
      mean_out[c] = muf;
      invstd_out[c] = is;
      const float mf = (float)m;
      if (rmean) rmean[c] = (1.0f - mom) * rmean[c] + mom * muf;
      if (rvar) {
        const float den = (mf - 1.0f) > 1.0f ? (mf - 1.0f) : 1.0f;
        rvar[c] = (1.0f - mom) * rvar[c] + mom * (var * mf / den);
      }
    }
  }
  __syncthreads();
  const unsigned stride = gridDim.x * blockDim.x;
  for (unsigned j = blockIdx.x * blockDim.x + threadIdx.x; j < total4; j += stride * BN_U) {
    float4 v[BN_U];
#pragma unroll
    for (int u = 0; u < BN_U; u++) {
      const unsigned jj = j + u * stride;
      if (jj < total4) v[u] = __ldg(y + jj);
    }
#pragma unroll
    for (int u = 0; u < BN_U; u++) {
      const unsigned jj = j + u * stride;
      if (jj >= total4) break;
      const int c = (int)((jj / hw4) % (unsigned)C);
      const float mu = smu[c], is = sis[c], g = __ldg(gamma + c), bt = __ldg(beta + c);
      float4 o;
      o.x = g * ((v[u].x - mu) * is) + bt;
      o.y = g * ((v[u].y - mu) * is) + bt;
      o.z = g * ((v[u].z - mu) * is) + bt;
      o.w = g * ((v[u].w - mu) * is) + bt;
      if (res) {
        const float4 r = res[jj];
        o.x += r.x; o.y += r.y; o.z += r.z; o.w += r.w;
      }
      if (relu) {
        o.x = fmaxf(o.x, 0.0f);
        o.y = fmaxf(o.y, 0.0f);
        o.z = fmaxf(o.z, 0.0f);
        o.w = fmaxf(o.w, 0.0f);
      }
      out[jj] = o;
      if (mask_out) {
        const float m[4] = {o.x, o.y, o.z, o.w};
        store_mask4(mask_out, jj, m);
      }
    }
  }
}

// Fused backward finalize + dx (nn.rs:400-427): dgamma/dbeta sums from the
// f64 sums in every CTA; CTA 0 adds them (scaled) into the gradients.
template <int RELU>
__global__ void __launch_bounds__(256) bn_dx4_fin_kernel(const float4* __restrict__ dy,
                                                         const float4* __restrict__ y,
                                                         const float4* __restrict__ relu_out,
                                                         const uint32_t* __restrict__ relu_mask, int C, unsigned hw4,
                                                         unsigned total4, float m, const float* __restrict__ gamma,
                                                         const float* __restrict__ mean,
                                                         const float* __restrict__ invstd,
                                                         const double* __restrict__ sums,
                                                         float* __restrict__ dgamma, float* __restrict__ dbeta,
                                                         float pscale, float4* __restrict__ dx,
                                                         char* __restrict__ pack, int pack_bn) {
  extern __shared__ float sh[];
  float* sdg = sh;
  float* sdb = sh + C;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const float dg = (float)sums[c * 2], db = (float)sums[c * 2 + 1];
    sdg[c] = dg;
    sdb[c] = db;
    if (blockIdx.x == 0) {
      if (dgamma) dgamma[c] += dg * pscale;
      if (dbeta) dbeta[c] += db * pscale;
    }
  }
  __syncthreads();
  const unsigned stride = gridDim.x * blockDim.x;
  for (unsigned j = blockIdx.x * blockDim.x + threadIdx.x; j < total4; j += stride * BN_U) {
    float4 d[BN_U], v[BN_U], r[BN_U];
#pragma unroll
    for (int u = 0; u < BN_U; u++) {
      const unsigned jj = j + u * stride;
      if (jj < total4) {
        d[u] = __ldg(dy + jj);
        v[u] = __ldg(y + jj);
        if (RELU == 1) r[u] = __ldg(relu_out + jj);
        if (RELU == 2) r[u] = mask4(relu_mask, jj);
      }
    }
#pragma unroll
    for (int u = 0; u < BN_U; u++) {
      const unsigned jj = j + u * stride;
      if (jj >= total4) break;
      const int c = (int)((jj / hw4) % (unsigned)C);
      const float mu = __ldg(mean + c), is = __ldg(invstd + c);
      const float s = __ldg(gamma + c) * is / m, dbc = sdb[c], dgc = sdg[c];
      float dd[4] = {d[u].x, d[u].y, d[u].z, d[u].w};
      const float vv[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      if (RELU) {
        const float rr[4] = {r[u].x, r[u].y, r[u].z, r[u].w};
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (rr[e] <= 0.0f) dd[e] = 0.0f;
      }
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float xh = (vv[e] - mu) * is;
        o[e] = s * (m * dd[e] - dbc - xh * dgc);
      }
      dx[jj] = make_float4(o[0], o[1], o[2], o[3]);
      if (pack) {
        // the 4 pixels are one 16-byte chunk of row c of the wgrad's B
        // image for K block p / 32 (hi tile, then lo tile; SWIZZLE_128B)
        const unsigned chw4 = (unsigned)C * hw4;
        const unsigned img = jj / chw4, pix = (jj % hw4) * 4;
        const size_t p = (size_t)img * hw4 * 4 + pix;
        const size_t kb = p >> 5;
        const int ch = (int)((p & 31) >> 2);
        char* tile = pack + kb * (size_t)(2 * pack_bn * 128);
        const size_t off = (size_t)(c >> 3) * 1024 + (c & 7) * 128 + ((ch ^ (c & 7)) << 4);
        float hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
          hi[e] = tc::tf32_round(o[e]);
          lo[e] = o[e] - hi[e];
        }
        *reinterpret_cast<float4*>(tile + off) = make_float4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<float4*>(tile + (size_t)pack_bn * 128 + off) = make_float4(lo[0], lo[1], lo[2], lo[3]);
      }
    }
  }
}

__global__ void bn_eval_kernel(const float* __restrict__ y, int C, int hw, size_t total,
                               const float* __restrict__ gamma, const float* __restrict__ beta,
                               const float* __restrict__ rmean, const float* __restrict__ rvar, float eps,
                               int relu, float* __restrict__ out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)((i / hw) % C);
    const float is = 1.0f / sqrtf(rvar[c] + eps);
    const float sc = gamma[c] * is, sh = beta[c] - gamma[c] * is * rmean[c];
    const float v = sc * y[i] + sh;
    out[i] = relu ? fmaxf(v, 0.0f) : v;
  }
}

__global__ void bn_dx_kernel(const float* __restrict__ dy, const float* __restrict__ y,
                             const float* __restrict__ relu_out, int C, int hw, size_t total, float m,
                             const float* __restrict__ gamma, const float* __restrict__ mean,
                             const float* __restrict__ invstd, const float* __restrict__ dg,
                             const float* __restrict__ db, float* __restrict__ dx) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)((i / hw) % C);
    float d = dy[i];
    if (relu_out && relu_out[i] <= 0.0f) d = 0.0f;
    const float xh = (y[i] - mean[c]) * invstd[c];
    const float s = gamma[c] * invstd[c] / m;
    dx[i] = s * (m * d - db[c] - xh * dg[c]);
  }
}

int bn_parts(int n, int C, int num_sms) {
  int P = (8 * num_sms + C - 1) / C;
  if (P > n) P = n;
  if (P < 1) P = 1;
  return P;
}

static bool vec4_ok(int hw, size_t total, std::initializer_list<const void*> ptrs) {
  if (hw % 4 != 0 || total / 4 >= (size_t)INT32_MAX) return false;
  for (const void* p : ptrs)
    if (p && (reinterpret_cast<uintptr_t>(p) & 15)) return false;
  return true;
}

static unsigned ew4_grid(size_t total4, int num_sms) {
  size_t g = (total4 + 256 * BN_U - 1) / (256 * BN_U);
  size_t cap = (size_t)num_sms * 8;
  return (unsigned)std::max<size_t>(1, std::min(g, cap));
}

static unsigned ew_grid(size_t total, int num_sms) {
  size_t g = (total + 255) / 256;
  size_t cap = (size_t)num_sms * 16;
  return (unsigned)std::max<size_t>(1, std::min(g, cap));
}

int bn_fwd_sums(rnn_ctx* ctx, const float* y, int n, int C, int hw, double* part, double* sums,
                const PeerSums* ps, bool* reduced) {
  const int P = bn_parts(n, C, ctx->num_sms);
  if (reduced) *reduced = false;
  // the partials and the per-channel sums must not overlap (the combine
  // kernel reads one while it writes the other)
  RNN_REQUIRE(part + (size_t)C * P * 2 <= sums || sums + (size_t)C * 2 <= part,
              "batchnorm: partial-sum buffer (%d x %d) overlaps the sums", C, P);
  RNN_RANGE(y, sizeof(float) * (size_t)n * C * hw);
  RNN_RANGE(part, sizeof(double) * (size_t)C * P * 2);
  RNN_RANGE(sums, sizeof(double) * (size_t)C * 2);
  if (vec4_ok(hw, (size_t)n * C * hw, {y})) {  // partials + last-CTA combine in one launch
    const PeerSums pv = (ps && ps->world > 1 && C <= ps->cmax) ? *ps : PeerSums{};
    bn_fwd_partial4_kernel<<<dim3(C, P), BN_NT, 0, ctx->stream>>>(reinterpret_cast<const float4*>(y), n, C,
                                                                 hw / 4, P, part, ctx->counters + COUNTER_BN, sums, pv);
    RNN_CHECK_LAUNCH();
    if (reduced) *reduced = pv.world > 1;
    return RNN_OK;
  }
  bn_fwd_partial_kernel<<<dim3(C, P), BN_NT, 0, ctx->stream>>>(y, n, C, hw, P, part);
  RNN_CHECK_LAUNCH();
  bn_combine_kernel<<<(C + 127) / 128, 128, 0, ctx->stream>>>(part, C, P, sums);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int bn_fwd_finish(rnn_ctx* ctx, const float* y, int n, int C, int hw, double count, const double* sums,
                  const float* gamma, const float* beta, float* rmean, float* rvar, float mom, float eps,
                  int relu, float* mean, float* invstd, float* out, const float* res, uint32_t* mask,
                  bool* masked) {
  if (masked) *masked = false;
  RNN_RANGE(sums, sizeof(double) * (size_t)C * 2);
  RNN_RANGE(mean, sizeof(float) * C);
  RNN_RANGE(invstd, sizeof(float) * C);
  if (rmean) RNN_RANGE(rmean, sizeof(float) * C);
  if (rvar) RNN_RANGE(rvar, sizeof(float) * C);
  RNN_RANGE(gamma, sizeof(float) * C);
  RNN_RANGE(beta, sizeof(float) * C);
  RNN_RANGE(y, sizeof(float) * (size_t)n * C * hw);
  RNN_RANGE(out, sizeof(float) * (size_t)n * C * hw);
  if (res) RNN_RANGE(res, sizeof(float) * (size_t)n * C * hw);
  const size_t total = (size_t)n * C * hw;
  const float4* res4 = reinterpret_cast<const float4*>(res);
  // ReLU mask bits: every warp of the vector kernels covers 32 whole float4s
  uint32_t* mk = (mask && relu && total % 128 == 0 && vec4_ok(hw, total, {y, out, res})) ? mask : nullptr;
  if (mk) RNN_RANGE(mk, total / 8);
  if (masked) *masked = mk != nullptr;
  if (vec4_ok(hw, total, {y, out, res}) && C <= BN_FUSE_MAX_C) {  // finalize fused into the apply
    bn_apply4_fin_kernel<<<ew4_grid(total / 4, ctx->num_sms), 256, 2 * C * sizeof(float), ctx->stream>>>(
        reinterpret_cast<const float4*>(y), C, (unsigned)(hw / 4), (unsigned)(total / 4), gamma, beta, sums, count,
        mom, eps, rmean, rvar, relu, mean, invstd, res4, reinterpret_cast<float4*>(out), mk);
    RNN_CHECK_LAUNCH();
    return RNN_OK;
  }
  bn_finalize_kernel<<<(C + 127) / 128, 128, 0, ctx->stream>>>(sums, C, count, mom, eps, mean, invstd,
                                                                rmean, rvar);
  RNN_CHECK_LAUNCH();
  if (vec4_ok(hw, total, {y, out, res}))
    bn_apply4_kernel<<<ew4_grid(total / 4, ctx->num_sms), 256, 0, ctx->stream>>>(
        reinterpret_cast<const float4*>(y), C, (unsigned)(hw / 4), (unsigned)(total / 4), gamma, beta, mean,
        invstd, relu, res4, reinterpret_cast<float4*>(out), mk);
  else
    bn_apply_kernel<<<ew_grid(total, ctx->num_sms), 256, 0, ctx->stream>>>(y, C, hw, total, gamma, beta,
                                                                            mean, invstd, relu, res, out);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int bn_bwd_sums(rnn_ctx* ctx, const float* dy, const float* y, const float* relu_out, int n, int C, int hw,
                const float* mean, const float* invstd, double* part, double* sums, const PeerSums* ps,
                bool* reduced, const uint32_t* relu_mask) {
  const int P = bn_parts(n, C, ctx->num_sms);
  if (reduced) *reduced = false;
  // the partials and the per-channel sums must not overlap (the combine
  // kernel reads one while it writes the other)
  RNN_REQUIRE(part + (size_t)C * P * 2 <= sums || sums + (size_t)C * 2 <= part,
              "batchnorm: partial-sum buffer (%d x %d) overlaps the sums", C, P);
  RNN_RANGE(dy, sizeof(float) * (size_t)n * C * hw);
  RNN_RANGE(y, sizeof(float) * (size_t)n * C * hw);
  if (relu_out) RNN_RANGE(relu_out, sizeof(float) * (size_t)n * C * hw);
  RNN_RANGE(mean, sizeof(float) * C);
  RNN_RANGE(invstd, sizeof(float) * C);
  RNN_RANGE(part, sizeof(double) * (size_t)C * P * 2);
  RNN_RANGE(sums, sizeof(double) * (size_t)C * 2);
  if (vec4_ok(hw, (size_t)n * C * hw, {dy, y, relu_out})) {
    const float4 *d4 = reinterpret_cast<const float4*>(dy), *y4 = reinterpret_cast<const float4*>(y),
                 *r4 = reinterpret_cast<const float4*>(relu_out);
    const PeerSums pv = (ps && ps->world > 1 && C <= ps->cmax) ? *ps : PeerSums{};
    unsigned* cnt = ctx->counters + COUNTER_BN;
    if (relu_mask) {
      RNN_RANGE(relu_mask, (size_t)n * C * hw / 8);
      bn_bwd_partial4_kernel<2><<<dim3(C, P), BN_NT, 0, ctx->stream>>>(d4, y4, r4, relu_mask, n, C, hw / 4, P,
                                                                      mean, invstd, part, cnt, sums, pv);
    } else if (relu_out) {
      bn_bwd_partial4_kernel<1><<<dim3(C, P), BN_NT, 0, ctx->stream>>>(d4, y4, r4, nullptr, n, C, hw / 4, P,
                                                                      mean, invstd, part, cnt, sums, pv);
    } else {
      bn_bwd_partial4_kernel<0><<<dim3(C, P), BN_NT, 0, ctx->stream>>>(d4, y4, r4, nullptr, n, C, hw / 4, P,
                                                                      mean, invstd, part, cnt, sums, pv);
    }
    RNN_CHECK_LAUNCH();
    if (reduced) *reduced = pv.world > 1;
    return RNN_OK;  // partials + last-CTA combine (+ cross-rank sum) in one launch
  } else {
    bn_bwd_partial_kernel<<<dim3(C, P), BN_NT, 0, ctx->stream>>>(dy, y, relu_out, n, C, hw, P, mean, invstd,
                                                                 part);
  }
  RNN_CHECK_LAUNCH();
  bn_combine_kernel<<<(C + 127) / 128, 128, 0, ctx->stream>>>(part, C, P, sums);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int bn_bwd_finish(rnn_ctx* ctx, const float* dy, const float* y, const float* relu_out, int n, int C, int hw,
                  double count, const double* sums, const float* gamma, const float* mean,
                  const float* invstd, float* dgb /* [2C] scratch */, float* dx, float* dgamma,
                  float* dbeta, float pscale, float* pack, int pack_bn, bool* packed,
                  const uint32_t* relu_mask) {
  if (packed) *packed = false;
  RNN_RANGE(sums, sizeof(double) * (size_t)C * 2);
  RNN_RANGE(dgb, sizeof(float) * (size_t)C * 2);
  if (dgamma) RNN_RANGE(dgamma, sizeof(float) * C);
  if (dbeta) RNN_RANGE(dbeta, sizeof(float) * C);
  RNN_RANGE(gamma, sizeof(float) * C);
  RNN_RANGE(dx, sizeof(float) * (size_t)n * C * hw);
  const size_t total = (size_t)n * C * hw;
  if (vec4_ok(hw, total, {dy, y, relu_out, dx}) && C <= BN_FUSE_MAX_C) {  // finalize fused into dx
    const float4 *d4 = reinterpret_cast<const float4*>(dy), *y4 = reinterpret_cast<const float4*>(y),
                 *r4 = reinterpret_cast<const float4*>(relu_out);
    const unsigned g = ew4_grid(total / 4, ctx->num_sms);
    const size_t shm = 2 * C * sizeof(float);
    // the wgrad's B image of dx: one column tile of exactly C rows, whole
    // 32-pixel K blocks
    char* pk = (pack && pack_bn == C && total % (32 * (size_t)C) == 0) ? reinterpret_cast<char*>(pack) : nullptr;
    if (pk) RNN_RANGE(pk, total * 2 * sizeof(float));
    float4* dx4 = reinterpret_cast<float4*>(dx);
    const unsigned hw4 = (unsigned)(hw / 4), t4 = (unsigned)(total / 4);
    if (relu_mask) {
      RNN_RANGE(relu_mask, total / 8);
      bn_dx4_fin_kernel<2><<<g, 256, shm, ctx->stream>>>(d4, y4, r4, relu_mask, C, hw4, t4, (float)count, gamma,
                                                         mean, invstd, sums, dgamma, dbeta, pscale, dx4, pk,
                                                         pack_bn);
    } else if (relu_out) {
      bn_dx4_fin_kernel<1><<<g, 256, shm, ctx->stream>>>(d4, y4, r4, nullptr, C, hw4, t4, (float)count, gamma,
                                                         mean, invstd, sums, dgamma, dbeta, pscale, dx4, pk,
                                                         pack_bn);
    } else {
      bn_dx4_fin_kernel<0><<<g, 256, shm, ctx->stream>>>(d4, y4, r4, nullptr, C, hw4, t4, (float)count, gamma,
                                                         mean, invstd, sums, dgamma, dbeta, pscale, dx4, pk,
                                                         pack_bn);
    }
    RNN_CHECK_LAUNCH();
    if (packed) *packed = pk != nullptr;
    return RNN_OK;
  }
  bn_bwd_finalize_kernel<<<(C + 127) / 128, 128, 0, ctx->stream>>>(sums, C, dgb, dgb + C, dgamma, dbeta,
                                                                    pscale);
  RNN_CHECK_LAUNCH();
  if (vec4_ok(hw, total, {dy, y, relu_out, dx})) {
    const float4 *d4 = reinterpret_cast<const float4*>(dy), *y4 = reinterpret_cast<const float4*>(y),
                 *r4 = reinterpret_cast<const float4*>(relu_out);
    const unsigned g = ew4_grid(total / 4, ctx->num_sms);
    if (relu_mask)
      bn_dx4_kernel<2><<<g, 256, 0, ctx->stream>>>(d4, y4, r4, relu_mask, C, (unsigned)(hw / 4),
                                                   (unsigned)(total / 4), (float)count, gamma, mean, invstd, dgb,
                                                   dgb + C, reinterpret_cast<float4*>(dx));
    else if (relu_out)
      bn_dx4_kernel<1><<<g, 256, 0, ctx->stream>>>(d4, y4, r4, nullptr, C, (unsigned)(hw / 4),
                                                   (unsigned)(total / 4), (float)count, gamma, mean, invstd, dgb,
                                                   dgb + C, reinterpret_cast<float4*>(dx));
    else
      bn_dx4_kernel<0><<<g, 256, 0, ctx->stream>>>(d4, y4, r4, nullptr, C, (unsigned)(hw / 4),
                                                   (unsigned)(total / 4), (float)count, gamma, mean, invstd, dgb,
                                                   dgb + C, reinterpret_cast<float4*>(dx));
  } else {
    bn_dx_kernel<<<ew_grid(total, ctx->num_sms), 256, 0, ctx->stream>>>(
        dy, y, relu_out, C, hw, total, (float)count, gamma, mean, invstd, dgb, dgb + C, dx);
  }
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

size_t bn_scratch_bytes(int n, int C, int num_sms) {
  const int P = bn_parts(n, C, num_sms);
  // partials + sums + dg/db floats, 256-byte aligned pieces
  size_t a = ((size_t)C * P * 2 * sizeof(double) + 255) & ~(size_t)255;
  size_t b = ((size_t)C * 2 * sizeof(double) + 255) & ~(size_t)255;
  size_t c = ((size_t)C * 2 * sizeof(float) + 255) & ~(size_t)255;
  return a + b + c;
}

}  // namespace rnn

using namespace rnn;

extern "C" int rnn_batchnorm_fwd_dev(rnn_ctx* ctx, const float* y, int n, int c, int hw, const float* gamma,
                                     const float* beta, float* rmean, float* rvar, float mom, float eps,
                                     int relu, float* mean, float* invstd, float* out) {
  RNN_REQUIRE(ctx && y && gamma && beta && mean && invstd && out, "batchnorm_fwd: null argument");
  RNN_REQUIRE(n > 0 && c > 0 && hw > 0, "batchnorm_fwd: bad shape");
  RNN_TRY(ensure_ws(ctx, bn_scratch_bytes(n, c, ctx->num_sms)));
  const int P = bn_parts(n, c, ctx->num_sms);
  double* part = static_cast<double*>(ctx->ws);
  double* sums = reinterpret_cast<double*>(static_cast<char*>(ctx->ws) +
                                           (((size_t)c * P * 2 * sizeof(double) + 255) & ~(size_t)255));
  RNN_TRY(bn_fwd_sums(ctx, y, n, c, hw, part, sums));
  return bn_fwd_finish(ctx, y, n, c, hw, (double)n * hw, sums, gamma, beta, rmean, rvar, mom, eps, relu, mean,
                       invstd, out);
}

extern "C" int rnn_batchnorm_eval_dev(rnn_ctx* ctx, const float* y, int n, int c, int hw, const float* gamma,
                                      const float* beta, const float* rmean, const float* rvar, float eps,
                                      int relu, float* out) {
  RNN_REQUIRE(ctx && y && gamma && beta && rmean && rvar && out, "batchnorm_eval: null argument");
  const size_t total = (size_t)n * c * hw;
  if (total == 0) return RNN_OK;
  RNN_RANGE(y, total * sizeof(float));
  RNN_RANGE(out, total * sizeof(float));
  RNN_RANGE(rmean, c * sizeof(float));
  RNN_RANGE(rvar, c * sizeof(float));
  bn_eval_kernel<<<ew_grid(total, ctx->num_sms), 256, 0, ctx->stream>>>(y, c, hw, total, gamma, beta, rmean,
                                                                         rvar, eps, relu, out);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

extern "C" int rnn_batchnorm_bwd_dev(rnn_ctx* ctx, const float* dy, const float* y, int n, int c, int hw,
                                     const float* gamma, const float* mean, const float* invstd,
                                     const float* relu_out, float* dx, float* dgamma, float* dbeta) {
  RNN_REQUIRE(ctx && dy && y && gamma && mean && invstd && dx, "batchnorm_bwd: null argument");
  RNN_REQUIRE(n > 0 && c > 0 && hw > 0, "batchnorm_bwd: bad shape");
  RNN_TRY(ensure_ws(ctx, bn_scratch_bytes(n, c, ctx->num_sms)));
  const int P = bn_parts(n, c, ctx->num_sms);
  char* base = static_cast<char*>(ctx->ws);
  size_t a = ((size_t)c * P * 2 * sizeof(double) + 255) & ~(size_t)255;
  size_t b = ((size_t)c * 2 * sizeof(double) + 255) & ~(size_t)255;
  double* part = reinterpret_cast<double*>(base);
  double* sums = reinterpret_cast<double*>(base + a);
  float* dgb = reinterpret_cast<float*>(base + a + b);
  RNN_TRY(bn_bwd_sums(ctx, dy, y, relu_out, n, c, hw, mean, invstd, part, sums));
  return bn_bwd_finish(ctx, dy, y, relu_out, n, c, hw, (double)n * hw, sums, gamma, mean, invstd, dgb, dx,
                       dgamma, dbeta, 1.0f);
}

// The SyncBN exchange on its own (the data-parallel ResNet step runs it inside
// its statistics kernels): per-channel forward sums of this rank's y, summed
// with every peer's through the mailboxes in rank order.  For callers that
// map their peers' device memory themselves (CUDA IPC) and for tests of the
// exchange on one device.
extern "C" int rnn_batchnorm_stats_peer_dev(rnn_ctx* ctx, const float* y, int n, int c, int hw, int rank, int world,
                                            void* const* mailboxes, unsigned long long* seq, int cmax, int wait_ms,
                                            double* sums) {
  RNN_REQUIRE(ctx && y && mailboxes && seq && sums, "batchnorm_stats_peer: null argument");
  RNN_REQUIRE(n > 0 && c > 0 && hw > 0 && world >= 1 && rank >= 0 && rank < world && c <= cmax && wait_ms > 0,
              "batchnorm_stats_peer: bad arguments (n %d c %d hw %d rank %d world %d cmax %d wait %d ms)", n, c, hw,
              rank, world, cmax, wait_ms);
  RNN_REQUIRE(vec4_ok(hw, (size_t)n * c * hw, {y}), "batchnorm_stats_peer: hw %% 4 == 0 and a 16-byte aligned y");
  RNN_RANGE(mailboxes, sizeof(void*) * world);
  RNN_RANGE(seq, sizeof(unsigned long long));
  const int P = bn_parts(n, c, ctx->num_sms);
  RNN_TRY(ensure_ws(ctx, sizeof(double) * (size_t)c * P * 2));
  PeerSums ps;
  ps.rank = rank;
  ps.world = world;
  ps.cmax = cmax;
  ps.mail = reinterpret_cast<char* const*>(mailboxes);
  ps.seq = seq;
  ps.dev_error = ctx->dev_error;
  ps.wait_ns = (unsigned long long)wait_ms * 1000000ull;
  return bn_fwd_sums(ctx, y, n, c, hw, static_cast<double*>(ctx->ws), sums, &ps, nullptr);
}

extern "C" size_t rnn_peer_mailbox_bytes(int cmax) { return rnn::peer_mail_bytes(cmax); }
