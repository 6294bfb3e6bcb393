// Column sums of a row-major [rows][c] matrix, out[j] += sum_r a[r][j]
// (times m[r][j] when m is given): the bias, LayerNorm-affine and
// LayerScale gradients.  Two passes in a fixed order (deterministic): CTA
// partials over CS_ROWS-row slabs, then one sum over the partials.
//
// The float4 path (c % 4 == 0, 16-byte aligned operands) gives each warp a
// 128-column strip and a CTA 8 warps over one slab, so a warp reads 512
// contiguous bytes per row and sixteen rows are in flight per lane; the
// partials of the 8 warps are combined in shared memory.  The final pass
// runs 32 warps per 128-column strip (few CTAs: its grid is the column
// strips only), each summing every 32nd partial, then combines the warps in
// shared memory.  Other shapes take the scalar kernels (one thread per
// column).
#pragma once

#include "common.cuh"

namespace rnn {

constexpr int CS_ROWS = 128;  // rows per partial (the callers size `part` as ceil(rows / CS_ROWS) x c)

// the kernels have internal linkage: each translation unit that includes
// this header gets its own copy
namespace {

__device__ __forceinline__ void cs_add4(float4& s, const float4 v) {
  s.x += v.x;
  s.y += v.y;
  s.z += v.z;
  s.w += v.w;
}

template <bool MUL>
__global__ void __launch_bounds__(256) cs_partial4_kernel(const float4* __restrict__ a, const float4* __restrict__ m,
                                                           int rows, int c4, float4* __restrict__ part) {
  __shared__ float4 red[8][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int j = blockIdx.x * 32 + lane;
  const int r0 = blockIdx.y * CS_ROWS;
  float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (j < c4) {
#pragma unroll
    for (int i = 0; i < CS_ROWS / 8; i++) {
      const int r = r0 + w + 8 * i;
      if (r < rows) {
        float4 v = __ldg(a + (size_t)r * c4 + j);
        if (MUL) {
          const float4 q = __ldg(m + (size_t)r * c4 + j);
          v.x *= q.x;
          v.y *= q.y;
          v.z *= q.z;
          v.w *= q.w;
        }
        cs_add4(s, v);
      }
    }
  }
  red[w][lane] = s;
  __syncthreads();
  if (w == 0 && j < c4) {
    float4 t = red[0][lane];
#pragma unroll
    for (int k = 1; k < 8; k++) cs_add4(t, red[k][lane]);
    part[(size_t)blockIdx.y * c4 + j] = t;
  }
}

// One-launch form (float4 path): the CTAs of a column strip count
// themselves in on a device counter after writing their partials; the last
// one adds the strip's partials in slab order (8 warps: warp w takes slabs
// w, w+8, ..., then the warps in order), adds into out and resets the
// counter.  Which CTA finishes last varies, the order of the sums does not.
constexpr int CS_COUNTER0 = 2, CS_COUNTERS = 14;  // ctx->counters slots 2 .. 15
template <bool MUL>
__global__ void __launch_bounds__(256) cs_fused4_kernel(const float4* __restrict__ a, const float4* __restrict__ m,
                                                         int rows, int c4, float4* __restrict__ part,
                                                         float4* __restrict__ out, unsigned* __restrict__ counters) {
  __shared__ float4 red[8][32];
  __shared__ bool last;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int j = blockIdx.x * 32 + lane;
  const int r0 = blockIdx.y * CS_ROWS;
  float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (j < c4) {
#pragma unroll
    for (int i = 0; i < CS_ROWS / 8; i++) {
      const int r = r0 + w + 8 * i;
      if (r < rows) {
        float4 v = __ldg(a + (size_t)r * c4 + j);
        if (MUL) {
          const float4 q = __ldg(m + (size_t)r * c4 + j);
          v.x *= q.x;
          v.y *= q.y;
          v.z *= q.z;
          v.w *= q.w;
        }
        cs_add4(s, v);
      }
    }
  }
  red[w][lane] = s;
  __syncthreads();
  if (w == 0 && j < c4) {
    float4 t = red[0][lane];
#pragma unroll
    for (int k = 1; k < 8; k++) cs_add4(t, red[k][lane]);
    part[(size_t)blockIdx.y * c4 + j] = t;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&counters[blockIdx.x], 1u) == gridDim.y - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int nb = gridDim.y;
  float4 t = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (j < c4)
    for (int b = w; b < nb; b += 8) cs_add4(t, __ldcg(part + (size_t)b * c4 + j));
  __syncthreads();
  red[w][lane] = t;
  __syncthreads();
  if (w == 0) {
    if (j < c4) {
      float4 u = red[0][lane];
#pragma unroll
      for (int k = 1; k < 8; k++) cs_add4(u, red[k][lane]);
      float4 o = out[j];
      cs_add4(o, u);
      out[j] = o;
    }
    if (lane == 0) counters[blockIdx.x] = 0u;
  }
}

constexpr int CS_FINAL_WARPS = 32;

__global__ void __launch_bounds__(CS_FINAL_WARPS * 32) cs_final4_kernel(const float4* __restrict__ part, int nb,
                                                                         int c4, float4* __restrict__ out) {
  __shared__ float4 red[CS_FINAL_WARPS][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int j = blockIdx.x * 32 + lane;
  float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (j < c4) {
#pragma unroll 4
    for (int b = w; b < nb; b += CS_FINAL_WARPS) cs_add4(s, __ldg(part + (size_t)b * c4 + j));
  }
  red[w][lane] = s;
  __syncthreads();
  if (w == 0 && j < c4) {
    float4 t = red[0][lane];
#pragma unroll
    for (int k = 1; k < CS_FINAL_WARPS; k++) cs_add4(t, red[k][lane]);
    float4 o = out[j];
    cs_add4(o, t);
    out[j] = o;
  }
}

// scalar forms: one thread per column
__global__ void cs_partial_kernel(const float* __restrict__ a, const float* __restrict__ m, int rows, int c,
                                  float* __restrict__ part) {
  const int blk = blockIdx.y;
  const int r0 = blk * CS_ROWS, r1 = min(rows, r0 + CS_ROWS);
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < c; j += gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int r = r0; r < r1; r++) s += m ? a[(size_t)r * c + j] * m[(size_t)r * c + j] : a[(size_t)r * c + j];
    part[(size_t)blk * c + j] = s;
  }
}

__global__ void cs_final_kernel(const float* __restrict__ part, int nb, int c, float* __restrict__ out) {
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < c; j += gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int b = 0; b < nb; b++) s += part[(size_t)b * c + j];
    out[j] += s;
  }
}

}  // namespace

inline bool cs_aligned(const void* p) { return ((uintptr_t)p & 15) == 0; }

// out[j] += sum_b part[b][j] over nb partial rows
inline int colsum_final(rnn_ctx* ctx, const float* part, int nb, int c, float* out) {
  if (c % 4 == 0 && cs_aligned(part) && cs_aligned(out)) {
    const int c4 = c / 4;
    cs_final4_kernel<<<(c4 + 31) / 32, CS_FINAL_WARPS * 32, 0, ctx->stream>>>(
        reinterpret_cast<const float4*>(part), nb, c4, reinterpret_cast<float4*>(out));
  } else {
    cs_final_kernel<<<(c + 255) / 256, 256, 0, ctx->stream>>>(part, nb, c, out);
  }
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

// out[j] += sum_r a[r][j] (* m[r][j]); part holds ceil(rows / CS_ROWS) x c floats
inline int colsum_two_pass(rnn_ctx* ctx, const float* a, const float* m, int rows, int c, float* part, float* out) {
  const int nb = (rows + CS_ROWS - 1) / CS_ROWS;
  if (c % 4 == 0 && cs_aligned(a) && (!m || cs_aligned(m)) && cs_aligned(part) && cs_aligned(out) &&
      (c / 4 + 31) / 32 <= CS_COUNTERS) {
    const int c4 = c / 4;
    const dim3 grid((c4 + 31) / 32, nb);
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* m4 = reinterpret_cast<const float4*>(m);
    float4* p4 = reinterpret_cast<float4*>(part);
    float4* o4 = reinterpret_cast<float4*>(out);
    unsigned* cnt = ctx->counters + CS_COUNTER0;
    if (m)
      cs_fused4_kernel<true><<<grid, 256, 0, ctx->stream>>>(a4, m4, rows, c4, p4, o4, cnt);
    else
      cs_fused4_kernel<false><<<grid, 256, 0, ctx->stream>>>(a4, m4, rows, c4, p4, o4, cnt);
    RNN_CHECK_LAUNCH();
    return RNN_OK;
  }
  if (c % 4 == 0 && cs_aligned(a) && (!m || cs_aligned(m)) && cs_aligned(part)) {
    const int c4 = c / 4;
    const dim3 grid((c4 + 31) / 32, nb);
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* m4 = reinterpret_cast<const float4*>(m);
    float4* p4 = reinterpret_cast<float4*>(part);
    if (m)
      cs_partial4_kernel<true><<<grid, 256, 0, ctx->stream>>>(a4, m4, rows, c4, p4);
    else
      cs_partial4_kernel<false><<<grid, 256, 0, ctx->stream>>>(a4, m4, rows, c4, p4);
  } else {
    cs_partial_kernel<<<dim3((c + 255) / 256, nb), 256, 0, ctx->stream>>>(a, m, rows, c, part);
  }
  RNN_CHECK_LAUNCH();
  return colsum_final(ctx, part, nb, c, out);
}

}  // namespace rnn
