// The rustvit step's memory-bound glue on device (norm.rs, vit.rs, tok.rs,
// loss.rs): LayerScale, the SwiGLU gate, the depthwise 3x3 token conv,
// SeqPool attention pooling, DropPath, the 2x2 token merge, the NCHW <->
// token transposes, the taxonomic head's coarse-to-fine combine, and the
// soft-target cross-entropy, distillation and hint losses.
//
// Activations are [n, t, c] row-major (tok.rs:13-21).  Every parameter
// gradient is reduced through per-block partials over fixed ranges summed in
// a fixed order (no float atomics), so results are deterministic.
#include <algorithm>
#include <vector>

#include "colsum.cuh"
#include "ew.cuh"
#include "rng.h"

namespace rnn {

static unsigned gl_grid(size_t n, int sms) {
  return (unsigned)std::max<size_t>(1, std::min<size_t>((n + 255) / 256, (size_t)sms * 16));
}

// ---------------------------------------------------------------- LayerScale

__global__ void chan_scale_kernel(const float* __restrict__ x, size_t total, int c, const float* __restrict__ l,
                                  float* __restrict__ y) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x)
    y[i] = x[i] * l[i % c];
}

// float4 form (c % 4 == 0, all operands 16-byte aligned)
__global__ void chan_scale4_kernel(const float4* __restrict__ x, size_t total4, int c4, const float4* __restrict__ l,
                                   float4* __restrict__ y) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = x[i], q = __ldg(l + i % c4);
    y[i] = make_float4(v.x * q.x, v.y * q.y, v.z * q.z, v.w * q.w);
  }
}
static bool gl_al16(const void* p) { return ((uintptr_t)p & 15) == 0; }
// y = x * l per channel
static int chan_scale(rnn_ctx* ctx, const float* x, size_t total, int c, const float* l, float* y) {
  if (c % 4 == 0 && gl_al16(x) && gl_al16(l) && gl_al16(y))
    chan_scale4_kernel<<<gl_grid(total / 4, ctx->num_sms), 256, 0, ctx->stream>>>(
        reinterpret_cast<const float4*>(x), total / 4, c / 4, reinterpret_cast<const float4*>(l),
        reinterpret_cast<float4*>(y));
  else
    chan_scale_kernel<<<gl_grid(total, ctx->num_sms), 256, 0, ctx->stream>>>(x, total, c, l, y);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

// part[b][j] = sum over rows [b*R, (b+1)*R) of a[r][j] * m[r][j] (m optional)
static int gl_colsum(rnn_ctx* ctx, const float* a, const float* m, int rows, int c, float* out) {
  const int nb = (rows + CS_ROWS - 1) / CS_ROWS;
  RNN_TRY(ensure_aux(ctx, (size_t)nb * c * 4));
  float* part = static_cast<float*>(ctx->aux);
  return colsum_two_pass(ctx, a, m, rows, c, part, out);
}

// ---------------------------------------------------------------- SwiGLU gate

__global__ void swiglu_fwd_kernel(const float* __restrict__ ab, int rows, int h, float* __restrict__ u) {
  const size_t total = (size_t)rows * h;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / h, j = i - r * h;
    const float a = ab[r * 2 * h + j], b = ab[r * 2 * h + h + j];
    const float s = 1.0f / (1.0f + expf(-a));
    u[i] = a * s * b;
  }
}
__global__ void swiglu_bwd_kernel(const float* __restrict__ du, const float* __restrict__ ab, int rows, int h,
                                  float* __restrict__ dab) {
  const size_t total = (size_t)rows * h;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / h, j = i - r * h;
    const float a = ab[r * 2 * h + j], b = ab[r * 2 * h + h + j];
    const float s = 1.0f / (1.0f + expf(-a)), d = du[i];
    dab[r * 2 * h + j] = d * b * s * (1.0f + a * (1.0f - s));  // norm.rs:281-283
    dab[r * 2 * h + h + j] = d * (a * s);
  }
}

// ---------------------------------------------------------------- DwConv3

// y[i, oy, ox, :] = b + sum_taps w[tap] * x[i, oy+ky-1, ox+kx-1, :]
__global__ void dw3_fwd_kernel(const float* __restrict__ x, int n, int th, int tw, int c, const float* __restrict__ w,
                               const float* __restrict__ b, float* __restrict__ y) {
  const size_t total = (size_t)n * th * tw * c;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int j = (int)(e % c);
    const size_t pix = e / c;
    const int ox = (int)(pix % tw), oy = (int)((pix / tw) % th);
    const size_t ibase = (pix / ((size_t)th * tw)) * th * tw;
    float acc = b[j];
    for (int ky = 0; ky < 3; ky++) {
      const int sy = oy + ky - 1;
      if (sy < 0 || sy >= th) continue;
      for (int kx = 0; kx < 3; kx++) {
        const int sx = ox + kx - 1;
        if (sx < 0 || sx >= tw) continue;
        acc += w[(ky * 3 + kx) * c + j] * x[(ibase + (size_t)sy * tw + sx) * c + j];
      }
    }
    y[e] = acc;
  }
}
// dx[i, sy, sx, :] = sum over output pixels that read (sy, sx) of w[tap] dy
__global__ void dw3_dx_kernel(const float* __restrict__ dy, int n, int th, int tw, int c, const float* __restrict__ w,
                              float* __restrict__ dx, int accd) {
  const size_t total = (size_t)n * th * tw * c;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int j = (int)(e % c);
    const size_t pix = e / c;
    const int sx = (int)(pix % tw), sy = (int)((pix / tw) % th);
    const size_t ibase = (pix / ((size_t)th * tw)) * th * tw;
    float acc = 0.0f;
    for (int ky = 0; ky < 3; ky++) {
      const int oy = sy - ky + 1;
      if (oy < 0 || oy >= th) continue;
      for (int kx = 0; kx < 3; kx++) {
        const int ox = sx - kx + 1;
        if (ox < 0 || ox >= tw) continue;
        acc += w[(ky * 3 + kx) * c + j] * dy[(ibase + (size_t)oy * tw + ox) * c + j];
      }
    }
    dx[e] = accd ? dx[e] + acc : acc;
  }
}
// per-image partials of dW [9][c] and dB [c]: part[i][10][c]
__global__ void dw3_dw_partial(const float* __restrict__ dy, const float* __restrict__ x, int th, int tw, int c,
                               float* __restrict__ part) {
  const int i = blockIdx.y;
  const float* dyi = dy + (size_t)i * th * tw * c;
  const float* xi = x + (size_t)i * th * tw * c;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < 10 * c; e += gridDim.x * blockDim.x) {
    const int tap = e / c, j = e - tap * c;
    float s = 0.0f;
    if (tap == 9) {
      for (int p = 0; p < th * tw; p++) s += dyi[(size_t)p * c + j];
    } else {
      const int ky = tap / 3, kx = tap % 3;
      for (int oy = 0; oy < th; oy++) {
        const int sy = oy + ky - 1;
        if (sy < 0 || sy >= th) continue;
        for (int ox = 0; ox < tw; ox++) {
          const int sx = ox + kx - 1;
          if (sx < 0 || sx >= tw) continue;
          s += dyi[((size_t)oy * tw + ox) * c + j] * xi[((size_t)sy * tw + sx) * c + j];
        }
      }
    }
    part[(size_t)i * 10 * c + e] = s;
  }
}
// float4 forms (c % 4 == 0, 16-byte aligned tensors): a thread handles four
// channels of one pixel with 32-bit index arithmetic; each channel's sum
// runs in the same order as the scalar kernels above.
__device__ __forceinline__ void fma4(float4& a, const float4 w, const float4 v) {
  a.x += w.x * v.x;
  a.y += w.y * v.y;
  a.z += w.z * v.z;
  a.w += w.w * v.w;
}
__global__ void dw3_fwd4_kernel(const float4* __restrict__ x, int npix, int th, int tw, int c4,
                                const float4* __restrict__ w, const float4* __restrict__ b, float4* __restrict__ y) {
  const int total = npix * c4, hw = th * tw;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    const int j = e % c4, pix = e / c4;
    const int img = pix / hw, rem = pix - img * hw;
    const int oy = rem / tw, ox = rem - oy * tw;
    float4 acc = __ldg(b + j);
    for (int ky = 0; ky < 3; ky++) {
      const int sy = oy + ky - 1;
      if (sy < 0 || sy >= th) continue;
      for (int kx = 0; kx < 3; kx++) {
        const int sx = ox + kx - 1;
        if (sx < 0 || sx >= tw) continue;
        fma4(acc, __ldg(w + (ky * 3 + kx) * c4 + j), __ldg(x + (size_t)(img * hw + sy * tw + sx) * c4 + j));
      }
    }
    y[e] = acc;
  }
}
__global__ void dw3_dx4_kernel(const float4* __restrict__ dy, int npix, int th, int tw, int c4,
                               const float4* __restrict__ w, float4* __restrict__ dx, int accd) {
  const int total = npix * c4, hw = th * tw;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    const int j = e % c4, pix = e / c4;
    const int img = pix / hw, rem = pix - img * hw;
    const int sy = rem / tw, sx = rem - sy * tw;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int ky = 0; ky < 3; ky++) {
      const int oy = sy - ky + 1;
      if (oy < 0 || oy >= th) continue;
      for (int kx = 0; kx < 3; kx++) {
        const int ox = sx - kx + 1;
        if (ox < 0 || ox >= tw) continue;
        fma4(acc, __ldg(w + (ky * 3 + kx) * c4 + j), __ldg(dy + (size_t)(img * hw + oy * tw + ox) * c4 + j));
      }
    }
    if (accd) {
      const float4 q = dx[e];
      acc = make_float4(q.x + acc.x, q.y + acc.y, q.z + acc.z, q.w + acc.w);
    }
    dx[e] = acc;
  }
}
// Per-image partials of dW and dB, part[i][10][c]: a CTA covers 32 channel
// quads of one image with 8 pixel groups (group g takes pixels g, g+8, ...
// in order) that accumulate all ten sums at once, then adds the 8 groups in
// order in shared memory.
constexpr int DW3_PG = 8;
__global__ void __launch_bounds__(32 * DW3_PG) dw3_dw_partial4(const float4* __restrict__ dy,
                                                                 const float4* __restrict__ x, int th, int tw, int c4,
                                                                 float4* __restrict__ part) {
  __shared__ float4 red[DW3_PG][10][32];
  const int q = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int j = blockIdx.x * 32 + q;
  const int i = blockIdx.y, hw = th * tw;
  float4 acc[10];
#pragma unroll
  for (int t = 0; t < 10; t++) acc[t] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (j < c4) {
    const float4* dyi = dy + (size_t)i * hw * c4 + j;
    const float4* xi = x + (size_t)i * hw * c4 + j;
    for (int p = g; p < hw; p += DW3_PG) {
      const int oy = p / tw, ox = p - oy * tw;
      const float4 d = __ldg(dyi + (size_t)p * c4);
      acc[9].x += d.x;
      acc[9].y += d.y;
      acc[9].z += d.z;
      acc[9].w += d.w;
#pragma unroll
      for (int t = 0; t < 9; t++) {
        const int sy = oy + t / 3 - 1, sx = ox + t % 3 - 1;
        if (sy >= 0 && sy < th && sx >= 0 && sx < tw) fma4(acc[t], d, __ldg(xi + (size_t)(sy * tw + sx) * c4));
      }
    }
  }
#pragma unroll
  for (int t = 0; t < 10; t++) red[g][t][q] = acc[t];
  __syncthreads();
  for (int o = threadIdx.x; o < 10 * 32; o += blockDim.x) {
    const int t = o >> 5, qq = o & 31, jj = blockIdx.x * 32 + qq;
    if (jj >= c4) continue;
    float4 s = red[0][t][qq];
    for (int gg = 1; gg < DW3_PG; gg++) {
      const float4 v = red[gg][t][qq];
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    part[((size_t)i * 10 + t) * c4 + jj] = s;
  }
}
__global__ void dw3_dw_final(const float* __restrict__ part, int n, int c, float* __restrict__ dw,
                             float* __restrict__ db) {
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < 10 * c; e += gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += part[(size_t)i * 10 * c + e];
    if (e < 9 * c) dw[e] += s;
    else db[e - 9 * c] += s;
  }
}

// ---------------------------------------------------------------- SeqPool

// one block per image: w = softmax_t(x_t . p), z = sum_t w_t x_t
__global__ void seqpool_fwd_kernel(const float* __restrict__ x, int t, int c, const float* __restrict__ p,
                                   float* __restrict__ z, float* __restrict__ w) {
  extern __shared__ float sw[];  // [t]
  const int i = blockIdx.x;
  const float* xi = x + (size_t)i * t * c;
  const int wp = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int j = wp; j < t; j += nw) {
    float s = 0.0f;
    for (int k = l; k < c; k += 32) s += xi[(size_t)j * c + k] * p[k];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (l == 0) sw[j] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float mx = -INFINITY;
    for (int j = 0; j < t; j++) mx = sw[j] > mx ? sw[j] : mx;
    float sum = 0.0f;
    for (int j = 0; j < t; j++) {
      sw[j] = expf(sw[j] - mx);
      sum += sw[j];
    }
    const float inv = 1.0f / sum;
    for (int j = 0; j < t; j++) {
      sw[j] *= inv;
      w[(size_t)i * t + j] = sw[j];
    }
  }
  __syncthreads();
  for (int k = threadIdx.x; k < c; k += blockDim.x) {
    float s = 0.0f;
    for (int j = 0; j < t; j++) s += sw[j] * xi[(size_t)j * c + k];
    z[(size_t)i * c + k] = s;
  }
}
// one block per image: dx, and dp partial part[i][c]
__global__ void seqpool_bwd_kernel(const float* __restrict__ dz, const float* __restrict__ x,
                                   const float* __restrict__ w, int t, int c, const float* __restrict__ p,
                                   float* __restrict__ dx, float* __restrict__ part) {
  extern __shared__ float sh[];  // dw[t], ds[t]
  float* dwv = sh;
  float* ds = sh + t;
  const int i = blockIdx.x;
  const float* xi = x + (size_t)i * t * c;
  const float* dzi = dz + (size_t)i * c;
  const float* wi = w + (size_t)i * t;
  const int wp = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int j = wp; j < t; j += nw) {
    float s = 0.0f;
    for (int k = l; k < c; k += 32) s += dzi[k] * xi[(size_t)j * c + k];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (l == 0) dwv[j] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float dot = 0.0f;
    for (int j = 0; j < t; j++) dot += dwv[j] * wi[j];
    for (int j = 0; j < t; j++) ds[j] = wi[j] * (dwv[j] - dot);
  }
  __syncthreads();
  for (int k = threadIdx.x; k < c; k += blockDim.x) {
    float a = 0.0f;
    for (int j = 0; j < t; j++) {
      a += ds[j] * xi[(size_t)j * c + k];
      dx[((size_t)i * t + j) * c + k] = wi[j] * dzi[k] + ds[j] * p[k];
    }
    part[(size_t)i * c + k] = a;
  }
}

// ---------------------------------------------------------------- DropPath / merge / layout

__global__ void row_scale_kernel(float* __restrict__ x, size_t per, size_t total, const float* __restrict__ mask) {
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x)
    x[e] *= mask[e / per];
}
// float4 form (per % 4 == 0, x 16-byte aligned): a float4 never spans two images
__global__ void row_scale4_kernel(float4* __restrict__ x, size_t per4, size_t total4, const float* __restrict__ mask) {
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total4; e += (size_t)gridDim.x * blockDim.x) {
    const float m = __ldg(mask + e / per4);
    float4 v = x[e];
    v.x *= m;
    v.y *= m;
    v.z *= m;
    v.w *= m;
    x[e] = v;
  }
}
static int row_scale(rnn_ctx* ctx, float* x, size_t per, size_t total, const float* mask) {
  if (per % 4 == 0 && ((uintptr_t)x & 15) == 0)
    row_scale4_kernel<<<gl_grid(total / 4, ctx->num_sms), 256, 0, ctx->stream>>>(reinterpret_cast<float4*>(x),
                                                                                per / 4, total / 4, mask);
  else
    row_scale_kernel<<<gl_grid(total, ctx->num_sms), 256, 0, ctx->stream>>>(x, per, total, mask);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

// y[i, (oy,ox), q*c + j] = z[i, (2oy+dy_q, 2ox+dx_q), j]; dir=1 is the inverse copy
__global__ void token_merge_kernel(const float* __restrict__ src, int n, int th, int c, float* __restrict__ dst,
                                   int dir) {
  const int t2 = th / 2;
  const size_t total = (size_t)n * t2 * t2 * 4 * c;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int j = (int)(e % c);
    const size_t r = e / c;
    const int q = (int)(r % 4);
    const size_t cell = r / 4;
    const int ox = (int)(cell % t2), oy = (int)((cell / t2) % t2);
    const size_t i = cell / ((size_t)t2 * t2);
    const size_t zi = ((i * th + 2 * oy + (q >> 1)) * th + 2 * ox + (q & 1)) * c + j;
    if (dir == 0) dst[e] = src[zi];
    else dst[zi] = src[e];
  }
}

// [n, c, hw] <-> [n, hw, c] through 32x32 shared tiles (dir 0: NCHW -> tokens)
__global__ void nchw_tok_kernel(const float* __restrict__ in, int c, int hw, float* __restrict__ out, int dir) {
  __shared__ float tile[32][33];
  const int i = blockIdx.z;
  const int rows = dir == 0 ? c : hw, cols = dir == 0 ? hw : c;  // input viewed as [rows, cols]
  const float* src = in + (size_t)i * c * hw;
  float* dst = out + (size_t)i * c * hw;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int r = r0 + k, cc = c0 + threadIdx.x;
    if (r < rows && cc < cols) tile[k][threadIdx.x] = src[(size_t)r * cols + cc];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int cc = c0 + k, r = r0 + threadIdx.x;
    if (r < rows && cc < cols) dst[(size_t)cc * rows + r] = tile[threadIdx.x][k];
  }
}

// ---------------------------------------------------------------- TaxoHead

__global__ void taxo_fwd_kernel(float* __restrict__ zf, const float* __restrict__ zc, int n, int nf, int nc,
                                const uint32_t* __restrict__ parent) {
  const size_t total = (size_t)n * nf;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const size_t i = e / nf;
    const int k = (int)(e - i * nf);
    zf[e] += zc[i * nc + parent[k]];
  }
}
// dc[i][g] = dzc[i][g] + sum_{k: parent[k]==g} dzf[i][k] (k in increasing order)
__global__ void taxo_bwd_kernel(const float* __restrict__ dzf, const float* __restrict__ dzc, int n, int nf, int nc,
                                const uint32_t* __restrict__ parent, float* __restrict__ dc) {
  const size_t total = (size_t)n * nc;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const size_t i = e / nc;
    const uint32_t g = (uint32_t)(e - i * nc);
    float s = dzc[e];
    for (int k = 0; k < nf; k++)
      if (parent[k] == g) s += dzf[i * nf + k];
    dc[e] = s;
  }
}

// ---------------------------------------------------------------- losses

// one warp per row; row_loss[i], hit[i]  (loss.rs:39-81)
__global__ void ce_soft_rows(const float* __restrict__ z, const float* __restrict__ t, const uint32_t* __restrict__ hard,
                             int n, int nc, float scale, float inv, float* __restrict__ dz, float* __restrict__ row_loss,
                             int* __restrict__ hit) {
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, l = threadIdx.x & 31;
  if (i >= n) return;
  const float* zr = z + (size_t)i * nc;
  const float* tr = t + (size_t)i * nc;
  float* d = dz + (size_t)i * nc;
  float mx = -INFINITY;
  int arg = 0x7fffffff;
  for (int j = l; j < nc; j += 32)
    if (zr[j] > mx || (zr[j] == mx && j < arg)) { mx = zr[j]; arg = j; }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, mx, o);
    const int oa = __shfl_xor_sync(0xffffffffu, arg, o);
    if (om > mx || (om == mx && oa < arg)) { mx = om; arg = oa; }
  }
  float sum = 0.0f;
  for (int j = l; j < nc; j += 32) sum += expf(zr[j] - mx);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float lse = mx + logf(sum);
  float lr = 0.0f;
  for (int j = l; j < nc; j += 32) {
    lr += tr[j] * (lse - zr[j]);
    d[j] = (expf(zr[j] - mx) / sum - tr[j]) * inv * scale;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lr += __shfl_xor_sync(0xffffffffu, lr, o);
  if (l == 0) {
    row_loss[i] = lr;
    hit[i] = (uint32_t)arg == hard[i] ? 1 : 0;
  }
}

// one warp per row (loss.rs:87-130): dz += T (ps - pt) / n * scale
__global__ void kl_rows(const float* __restrict__ zs, const float* __restrict__ zt, int n, int nc, float temp,
                        float scale, float inv, float* __restrict__ dz, float* __restrict__ row_loss) {
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, l = threadIdx.x & 31;
  if (i >= n) return;
  const float it = 1.0f / temp;
  const float* a = zs + (size_t)i * nc;
  const float* b = zt + (size_t)i * nc;
  float ma = -INFINITY, mb = -INFINITY;
  for (int j = l; j < nc; j += 32) {
    ma = fmaxf(ma, a[j]);
    mb = fmaxf(mb, b[j]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ma = fmaxf(ma, __shfl_xor_sync(0xffffffffu, ma, o));
    mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
  }
  float sa = 0.0f, sb = 0.0f;
  for (int j = l; j < nc; j += 32) {
    sa += expf((a[j] - ma) * it);
    sb += expf((b[j] - mb) * it);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sa += __shfl_xor_sync(0xffffffffu, sa, o);
    sb += __shfl_xor_sync(0xffffffffu, sb, o);
  }
  const float ia = 1.0f / sa, ib = 1.0f / sb;
  float lr = 0.0f;
  for (int j = l; j < nc; j += 32) {
    const float ps = expf((a[j] - ma) * it) * ia, pt = expf((b[j] - mb) * it) * ib;
    if (pt > 1e-9f) lr += pt * (logf(fmaxf(pt, 1e-9f)) - logf(fmaxf(ps, 1e-9f)));
    dz[(size_t)i * nc + j] += temp * (ps - pt) * inv * scale;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lr += __shfl_xor_sync(0xffffffffu, lr, o);
  if (l == 0) row_loss[i] = lr * temp * temp;
}

// one warp per row (loss.rs:133-151): dz += 2 e / (n c) * scale
__global__ void hint_rows(const float* __restrict__ p, const float* __restrict__ t, int n, int c, float scale,
                          float inv, float* __restrict__ dz, float* __restrict__ row_loss) {
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, l = threadIdx.x & 31;
  if (i >= n) return;
  float s = 0.0f;
  for (int j = l; j < c; j += 32) {
    const float e = p[(size_t)i * c + j] - t[(size_t)i * c + j];
    s += e * e;
    dz[(size_t)i * c + j] += 2.0f * e * inv * scale;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (l == 0) row_loss[i] = s;
}

// out[0] = factor * sum(row_loss) (fixed-order tree), correct_out = sum(hit)
__global__ void rows_total(const float* __restrict__ row_loss, const int* __restrict__ hit, int n, float factor,
                           float* __restrict__ out, int* __restrict__ correct_out) {
  __shared__ double sl[256];
  __shared__ int sh[256];
  double a = 0.0;
  int h = 0;
  for (int i = threadIdx.x; i < n; i += 256) {
    a += row_loss[i];
    if (hit) h += hit[i];
  }
  sl[threadIdx.x] = a;
  sh[threadIdx.x] = h;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (threadIdx.x < s) {
      sl[threadIdx.x] += sl[threadIdx.x + s];
      sh[threadIdx.x] += sh[threadIdx.x + s];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    if (out) *out = (float)sl[0] * factor;
    if (correct_out) *correct_out = sh[0];
  }
}

static int rows_scratch(rnn_ctx* ctx, int n, float** row_loss, int** hit) {
  RNN_TRY(ensure_aux(ctx, (size_t)n * 8 + 512));
  *row_loss = static_cast<float*>(ctx->aux);
  *hit = reinterpret_cast<int*>(static_cast<char*>(ctx->aux) + (((size_t)n * 4 + 255) & ~(size_t)255));
  return RNN_OK;
}

}  // namespace rnn

using namespace rnn;

// ---------------------------------------------------------------- C ABI

extern "C" int rnn_layerscale_fwd_dev(rnn_ctx* ctx, const float* x, int rows, int c, const float* l, float* y) {
  RNN_REQUIRE(ctx && x && l && y && rows >= 0 && c > 0, "layerscale_fwd: bad arguments");
  const size_t total = (size_t)rows * c;
  if (!total) return RNN_OK;
  RNN_RANGE(x, total * 4); RNN_RANGE(y, total * 4); RNN_RANGE(l, (size_t)c * 4);
  return chan_scale(ctx, x, total, c, l, y);
}

extern "C" int rnn_layerscale_bwd_dev(rnn_ctx* ctx, const float* dy, const float* x, int rows, int c, const float* l,
                                      float* dl, float* dx) {
  RNN_REQUIRE(ctx && dy && x && l && dl && dx && rows >= 0 && c > 0, "layerscale_bwd: bad arguments");
  const size_t total = (size_t)rows * c;
  if (!total) return RNN_OK;
  RNN_RANGE(dy, total * 4); RNN_RANGE(x, total * 4); RNN_RANGE(dx, total * 4); RNN_RANGE(dl, (size_t)c * 4);
  RNN_TRY(gl_colsum(ctx, dy, x, rows, c, dl));
  return chan_scale(ctx, dy, total, c, l, dx);
}

extern "C" int rnn_swiglu_act_fwd_dev(rnn_ctx* ctx, const float* ab, int rows, int h, float* u) {
  RNN_REQUIRE(ctx && ab && u && rows >= 0 && h > 0, "swiglu_fwd: bad arguments");
  const size_t total = (size_t)rows * h;
  if (!total) return RNN_OK;
  RNN_RANGE(ab, total * 8); RNN_RANGE(u, total * 4);
  swiglu_fwd_kernel<<<gl_grid(total, ctx->num_sms), 256, 0, ctx->stream>>>(ab, rows, h, u);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

extern "C" int rnn_swiglu_act_bwd_dev(rnn_ctx* ctx, const float* du, const float* ab, int rows, int h, float* dab) {
  RNN_REQUIRE(ctx && du && ab && dab && rows >= 0 && h > 0, "swiglu_bwd: bad arguments");
  const size_t total = (size_t)rows * h;
  if (!total) return RNN_OK;
  RNN_RANGE(du, total * 4); RNN_RANGE(ab, total * 8); RNN_RANGE(dab, total * 8);
  swiglu_bwd_kernel<<<gl_grid(total, ctx->num_sms), 256, 0, ctx->stream>>>(du, ab, rows, h, dab);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

// The float4 depthwise kernels need c % 4 == 0, 16-byte aligned tensors and
// 32-bit element indices.
static bool dw3_vec_ok(size_t total, int c, std::initializer_list<const void*> ptrs) {
  if (c % 4 != 0 || total / 4 >= (size_t)INT32_MAX) return false;
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) & 15) return false;
  return true;
}

extern "C" int rnn_dwconv3_fwd_dev(rnn_ctx* ctx, const float* x, int n, int th, int tw, int c, const float* w,
                                   const float* b, float* y) {
  RNN_REQUIRE(ctx && x && w && b && y && n >= 0 && th > 0 && tw > 0 && c > 0, "dwconv3_fwd: bad arguments");
  const size_t total = (size_t)n * th * tw * c;
  if (!total) return RNN_OK;
  RNN_RANGE(x, total * 4); RNN_RANGE(y, total * 4); RNN_RANGE(w, (size_t)9 * c * 4); RNN_RANGE(b, (size_t)c * 4);
  if (dw3_vec_ok(total, c, {x, w, b, y})) {
    dw3_fwd4_kernel<<<gl_grid(total / 4, ctx->num_sms), 256, 0, ctx->stream>>>(
        reinterpret_cast<const float4*>(x), n * th * tw, th, tw, c / 4, reinterpret_cast<const float4*>(w),
        reinterpret_cast<const float4*>(b), reinterpret_cast<float4*>(y));
  } else {
    dw3_fwd_kernel<<<gl_grid(total, ctx->num_sms), 256, 0, ctx->stream>>>(x, n, th, tw, c, w, b, y);
  }
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int rnn::dwconv3_bwd(rnn_ctx* ctx, const float* dy, const float* x, int n, int th, int tw, int c, const float* w,
                     float* dw, float* db, float* dx, bool acc_dx) {
  RNN_REQUIRE(ctx && dy && x && w && dw && db && dx && n >= 0 && th > 0 && tw > 0 && c > 0,
              "dwconv3_bwd: bad arguments");
  const size_t total = (size_t)n * th * tw * c;
  if (!total) return RNN_OK;
  RNN_RANGE(dy, total * 4); RNN_RANGE(x, total * 4); RNN_RANGE(dx, total * 4);
  RNN_RANGE(dw, (size_t)9 * c * 4); RNN_RANGE(db, (size_t)c * 4);
  RNN_TRY(ensure_aux(ctx, (size_t)n * 10 * c * 4));
  float* part = static_cast<float*>(ctx->aux);
  const bool vec = dw3_vec_ok(total, c, {dy, x, w, dx, part});
  if (vec) {
    dw3_dw_partial4<<<dim3((c / 4 + 31) / 32, n), 32 * DW3_PG, 0, ctx->stream>>>(
        reinterpret_cast<const float4*>(dy), reinterpret_cast<const float4*>(x), th, tw, c / 4,
        reinterpret_cast<float4*>(part));
  } else {
    dw3_dw_partial<<<dim3((10 * c + 255) / 256, n), 256, 0, ctx->stream>>>(dy, x, th, tw, c, part);
  }
  RNN_CHECK_LAUNCH();
  dw3_dw_final<<<(10 * c + 255) / 256, 256, 0, ctx->stream>>>(part, n, c, dw, db);
  RNN_CHECK_LAUNCH();
  if (vec) {
    dw3_dx4_kernel<<<gl_grid(total / 4, ctx->num_sms), 256, 0, ctx->stream>>>(
        reinterpret_cast<const float4*>(dy), n * th * tw, th, tw, c / 4, reinterpret_cast<const float4*>(w),
        reinterpret_cast<float4*>(dx), acc_dx ? 1 : 0);
  } else {
    dw3_dx_kernel<<<gl_grid(total, ctx->num_sms), 256, 0, ctx->stream>>>(dy, n, th, tw, c, w, dx, acc_dx ? 1 : 0);
  }
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

extern "C" int rnn_dwconv3_bwd_dev(rnn_ctx* ctx, const float* dy, const float* x, int n, int th, int tw, int c,
                                   const float* w, float* dw, float* db, float* dx) {
  return rnn::dwconv3_bwd(ctx, dy, x, n, th, tw, c, w, dw, db, dx, false);
}

extern "C" int rnn_seqpool_fwd_dev(rnn_ctx* ctx, const float* x, int n, int t, int c, const float* p, float* z,
                                   float* w) {
  RNN_REQUIRE(ctx && x && p && z && w && n >= 0 && t > 0 && c > 0, "seqpool_fwd: bad arguments");
  if (!n) return RNN_OK;
  RNN_RANGE(x, (size_t)n * t * c * 4); RNN_RANGE(z, (size_t)n * c * 4); RNN_RANGE(w, (size_t)n * t * 4);
  RNN_RANGE(p, (size_t)c * 4);
  seqpool_fwd_kernel<<<n, 256, (size_t)t * 4, ctx->stream>>>(x, t, c, p, z, w);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

extern "C" int rnn_seqpool_bwd_dev(rnn_ctx* ctx, const float* dz, const float* x, const float* w, int n, int t, int c,
                                   const float* p, float* dp, float* dx) {
  RNN_REQUIRE(ctx && dz && x && w && p && dp && dx && n >= 0 && t > 0 && c > 0, "seqpool_bwd: bad arguments");
  if (!n) return RNN_OK;
  RNN_RANGE(dz, (size_t)n * c * 4); RNN_RANGE(x, (size_t)n * t * c * 4); RNN_RANGE(w, (size_t)n * t * 4);
  RNN_RANGE(dx, (size_t)n * t * c * 4); RNN_RANGE(dp, (size_t)c * 4); RNN_RANGE(p, (size_t)c * 4);
  RNN_TRY(ensure_aux(ctx, (size_t)n * c * 4 + (size_t)CS_ROWS * c * 4 * 4));
  float* part = static_cast<float*>(ctx->aux);
  seqpool_bwd_kernel<<<n, 256, (size_t)2 * t * 4, ctx->stream>>>(dz, x, w, t, c, p, dx, part);
  RNN_CHECK_LAUNCH();
  return colsum_final(ctx, part, n, c, dp);
}

// DropPath (vit.rs:40-73): the per-image keep mask comes from Rng::new(seed)
// exactly like the reference.  One device thread draws the n uniforms in
// order (the stream is sequential and n is a batch size), so the mask needs
// no host round trip and the call stays asynchronous.
__global__ void droppath_mask_kernel(uint64_t seed, int n, float keep, float* __restrict__ mask) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  Rng rng(seed);
  for (int i = 0; i < n; i++) mask[i] = rng.uniform() < keep ? 1.0f / keep : 0.0f;
}

extern "C" int rnn_droppath_fwd_dev(rnn_ctx* ctx, float* x, int n, size_t per_image, float p, uint64_t seed,
                                    float* mask) {
  RNN_REQUIRE(ctx && x && mask && n >= 0 && p >= 0.0f && p < 1.0f, "droppath_fwd: bad arguments");
  if (!n) return RNN_OK;
  RNN_RANGE(x, (size_t)n * per_image * 4);
  RNN_RANGE(mask, (size_t)n * 4);
  droppath_mask_kernel<<<1, 32, 0, ctx->stream>>>(seed, n, 1.0f - p, mask);
  RNN_CHECK_LAUNCH();
  const size_t total = (size_t)n * per_image;
  return row_scale(ctx, x, per_image, total, mask);
}

extern "C" int rnn_droppath_bwd_dev(rnn_ctx* ctx, float* dy, int n, size_t per_image, const float* mask) {
  RNN_REQUIRE(ctx && dy && mask && n >= 0, "droppath_bwd: bad arguments");
  if (!n) return RNN_OK;
  RNN_RANGE(dy, (size_t)n * per_image * 4);
  RNN_RANGE(mask, (size_t)n * 4);
  const size_t total = (size_t)n * per_image;
  return row_scale(ctx, dy, per_image, total, mask);
}

extern "C" int rnn_token_merge_dev(rnn_ctx* ctx, const float* src, int n, int th, int c, float* dst, int backward) {
  RNN_REQUIRE(ctx && src && dst && n >= 0 && th > 0 && th % 2 == 0 && c > 0, "token_merge: bad arguments");
  const size_t total = (size_t)n * th * th * c;
  if (!total) return RNN_OK;
  RNN_RANGE(src, total * 4);
  RNN_RANGE(dst, total * 4);
  token_merge_kernel<<<gl_grid(total, ctx->num_sms), 256, 0, ctx->stream>>>(src, n, th, c, dst, backward ? 1 : 0);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

extern "C" int rnn_tok_layout_dev(rnn_ctx* ctx, const float* in, int n, int c, int hw, float* out, int to_nchw) {
  RNN_REQUIRE(ctx && in && out && n >= 0 && c > 0 && hw > 0, "tok_layout: bad arguments");
  if (!n) return RNN_OK;
  RNN_RANGE(in, (size_t)n * c * hw * 4);
  RNN_RANGE(out, (size_t)n * c * hw * 4);
  const int rows = to_nchw ? hw : c, cols = to_nchw ? c : hw;
  dim3 grid((cols + 31) / 32, (rows + 31) / 32, n), block(32, 8);
  nchw_tok_kernel<<<grid, block, 0, ctx->stream>>>(in, c, hw, out, to_nchw ? 1 : 0);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

extern "C" int rnn_taxo_combine_fwd_dev(rnn_ctx* ctx, float* zf, const float* zc, int n, int nf, int nc,
                                        const uint32_t* parent) {
  RNN_REQUIRE(ctx && zf && zc && parent && n >= 0 && nf > 0 && nc > 0, "taxo_fwd: bad arguments");
  if (!n) return RNN_OK;
  RNN_RANGE(zf, (size_t)n * nf * 4); RNN_RANGE(zc, (size_t)n * nc * 4); RNN_RANGE(parent, (size_t)nf * 4);
  taxo_fwd_kernel<<<gl_grid((size_t)n * nf, ctx->num_sms), 256, 0, ctx->stream>>>(zf, zc, n, nf, nc, parent);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

extern "C" int rnn_taxo_combine_bwd_dev(rnn_ctx* ctx, const float* dzf, const float* dzc, int n, int nf, int nc,
                                        const uint32_t* parent, float* dc) {
  RNN_REQUIRE(ctx && dzf && dzc && parent && dc && n >= 0 && nf > 0 && nc > 0, "taxo_bwd: bad arguments");
  if (!n) return RNN_OK;
  RNN_RANGE(dzf, (size_t)n * nf * 4); RNN_RANGE(dzc, (size_t)n * nc * 4); RNN_RANGE(dc, (size_t)n * nc * 4);
  RNN_RANGE(parent, (size_t)nf * 4);
  taxo_bwd_kernel<<<gl_grid((size_t)n * nc, ctx->num_sms), 256, 0, ctx->stream>>>(dzf, dzc, n, nf, nc, parent, dc);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

extern "C" int rnn_ce_soft_dev(rnn_ctx* ctx, const float* logits, const float* target, const uint32_t* hard, int n,
                               int nclass, float scale, float* dz, float* loss_out, int* correct_out) {
  RNN_REQUIRE(ctx && logits && target && hard && dz && n >= 0 && nclass > 0, "ce_soft: bad arguments");
  if (!n) return RNN_OK;
  const size_t e = (size_t)n * nclass;
  RNN_RANGE(logits, e * 4); RNN_RANGE(target, e * 4); RNN_RANGE(dz, e * 4); RNN_RANGE(hard, (size_t)n * 4);
  float* rl;
  int* hit;
  RNN_TRY(rows_scratch(ctx, n, &rl, &hit));
  const float inv = 1.0f / (float)n;
  ce_soft_rows<<<(n * 32 + 255) / 256, 256, 0, ctx->stream>>>(logits, target, hard, n, nclass, scale, inv, dz, rl, hit);
  RNN_CHECK_LAUNCH();
  rows_total<<<1, 256, 0, ctx->stream>>>(rl, hit, n, inv, loss_out, correct_out);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

extern "C" int rnn_kl_distill_dev(rnn_ctx* ctx, const float* student, const float* teacher, int n, int nclass,
                                  float temp, float scale, float* dz, float* loss_out) {
  RNN_REQUIRE(ctx && student && teacher && dz && n >= 0 && nclass > 0 && temp > 0, "kl_distill: bad arguments");
  if (!n) return RNN_OK;
  const size_t e = (size_t)n * nclass;
  RNN_RANGE(student, e * 4); RNN_RANGE(teacher, e * 4); RNN_RANGE(dz, e * 4);
  float* rl;
  int* hit;
  RNN_TRY(rows_scratch(ctx, n, &rl, &hit));
  const float inv = 1.0f / (float)n;
  kl_rows<<<(n * 32 + 255) / 256, 256, 0, ctx->stream>>>(student, teacher, n, nclass, temp, scale, inv, dz, rl);
  RNN_CHECK_LAUNCH();
  rows_total<<<1, 256, 0, ctx->stream>>>(rl, nullptr, n, inv, loss_out, nullptr);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

extern "C" int rnn_hint_mse_dev(rnn_ctx* ctx, const float* pred, const float* target, int n, int c, float scale,
                                float* dz, float* loss_out) {
  RNN_REQUIRE(ctx && pred && target && dz && n >= 0 && c > 0, "hint_mse: bad arguments");
  if (!n) return RNN_OK;
  const size_t e = (size_t)n * c;
  RNN_RANGE(pred, e * 4); RNN_RANGE(target, e * 4); RNN_RANGE(dz, e * 4);
  float* rl;
  int* hit;
  RNN_TRY(rows_scratch(ctx, n, &rl, &hit));
  const float inv = 1.0f / (float)e;
  hint_rows<<<(n * 32 + 255) / 256, 256, 0, ctx->stream>>>(pred, target, n, c, scale, inv, dz, rl);
  RNN_CHECK_LAUNCH();
  rows_total<<<1, 256, 0, ctx->stream>>>(rl, nullptr, n, inv * scale, loss_out, nullptr);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}
