// Token-space layers on [rows, c] row-major activations (tok.rs layout):
// LayerNorm (norm.rs:38-137) and the Linear layer (linear.rs:44-96).
//
// LayerNorm: one warp per row; per-row mean/variance from f64 sums like the
// reference; xhat and invstd are stored for the backward (norm.rs:53-66).
// Column reductions (dgamma, dbeta, Linear's bias gradient) use per-block
// partials over fixed row ranges summed in order: deterministic.
// Linear's three products are GEMMs on the tcgen05 engine.
#include <algorithm>

#include "colsum.cuh"
#include "ew.cuh"

namespace rnn {

static __device__ __forceinline__ double wsum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
static __device__ __forceinline__ float wsum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void ln_fwd_kernel(const float* __restrict__ x, int rows, int c, const float* __restrict__ g,
                              const float* __restrict__ b, float eps, float* __restrict__ y, float* __restrict__ xhat,
                              float* __restrict__ invstd) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, l = threadIdx.x & 31;
  if (r >= rows) return;
  const float* xr = x + (size_t)r * c;
  double s = 0.0, s2 = 0.0;
  for (int j = l; j < c; j += 32) {
    const double v = xr[j];
    s += v;
    s2 += v * v;
  }
  s = wsum_d(s);
  s2 = wsum_d(s2);
  const double m = (double)c, mu = s / m;
  const double va = s2 / m - mu * mu;
  const float var = (float)(va > 0.0 ? va : 0.0);
  const float is = 1.0f / sqrtf(var + eps);
  const float muf = (float)mu;
  if (l == 0 && invstd) invstd[r] = is;
  for (int j = l; j < c; j += 32) {
    const float h = (xr[j] - muf) * is;
    if (xhat) xhat[(size_t)r * c + j] = h;
    y[(size_t)r * c + j] = g[j] * h + b[j];
  }
}

// dx per row (norm.rs:120-135): d = dy*g; dx = invstd (d - mean(d) - xhat mean(d xhat))
__global__ void ln_dx_kernel(const float* __restrict__ dy, const float* __restrict__ xhat,
                             const float* __restrict__ invstd, int rows, int c, const float* __restrict__ g,
                             float* __restrict__ dx, int acc) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, l = threadIdx.x & 31;
  if (r >= rows) return;
  const float* dyr = dy + (size_t)r * c;
  const float* xh = xhat + (size_t)r * c;
  float m1 = 0.0f, m2 = 0.0f;
  for (int j = l; j < c; j += 32) {
    const float d = dyr[j] * g[j];
    m1 += d;
    m2 += d * xh[j];
  }
  m1 = wsum_f(m1);
  m2 = wsum_f(m2);
  const float inv = 1.0f / (float)c, is = invstd[r];
  for (int j = l; j < c; j += 32) {
    const float d = dyr[j] * g[j];
    const float o = is * (d - m1 * inv - xh[j] * m2 * inv);
    dx[(size_t)r * c + j] = acc ? dx[(size_t)r * c + j] + o : o;
  }
}

// The whole LayerNorm backward in one pass over dy and xhat (c a multiple of
// 128 up to 512, 16-byte aligned tensors): a CTA of 8 warps takes a slab of
// LN_SLAB rows, warp w rows w, w+8, ... of it, each row's loads issued while
// the previous row is computed.  Lane l holds the float4 column groups l,
// l+32, ... of the row: it computes dx as ln_dx_kernel does
// (norm.rs:120-135) and adds dy*xhat and dy into per-lane column partials,
// which the CTA combines over its warps in order into the slab's partial
// dgamma / dbeta (part[0][slab][c], part[1][slab][c]); colsum_final adds the
// slabs in order.  dy and xhat are read once instead of three times.
constexpr int LN_SLAB = 64;
template <int NC4>
__global__ void __launch_bounds__(256) ln_bwd4_kernel(const float4* __restrict__ dy, const float4* __restrict__ xhat,
                                                      const float* __restrict__ invstd, int rows,
                                                      const float4* __restrict__ g, float4* __restrict__ dx,
                                                      float4* __restrict__ part, int nb, int acc) {
  constexpr int C4 = 32 * NC4;
  __shared__ float4 red[8][2][C4];
  const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int slab = blockIdx.x;
  float4 gv[NC4], pg[NC4], pb[NC4];
#pragma unroll
  for (int k = 0; k < NC4; k++) {
    gv[k] = __ldg(g + l + 32 * k);
    pg[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    pb[k] = pg[k];
  }
  const float inv = 1.0f / (float)(4 * C4);
  const int r0 = slab * LN_SLAB + w;
  const int r_end = min(rows, (slab + 1) * LN_SLAB);
  float4 dn[NC4], xn[NC4];  // the next row's operands, loaded ahead
  if (r0 < r_end) {
#pragma unroll
    for (int k = 0; k < NC4; k++) {
      dn[k] = __ldg(dy + (size_t)r0 * C4 + l + 32 * k);
      xn[k] = __ldg(xhat + (size_t)r0 * C4 + l + 32 * k);
    }
  }
  for (int r = r0; r < r_end; r += 8) {
    float4 dv[NC4], xv[NC4];
#pragma unroll
    for (int k = 0; k < NC4; k++) {
      dv[k] = dn[k];
      xv[k] = xn[k];
    }
    if (r + 8 < r_end) {
#pragma unroll
      for (int k = 0; k < NC4; k++) {
        dn[k] = __ldg(dy + (size_t)(r + 8) * C4 + l + 32 * k);
        xn[k] = __ldg(xhat + (size_t)(r + 8) * C4 + l + 32 * k);
      }
    }
    float m1 = 0.0f, m2 = 0.0f;
#pragma unroll
    for (int k = 0; k < NC4; k++) {
      const float d0 = dv[k].x * gv[k].x, d1 = dv[k].y * gv[k].y, d2 = dv[k].z * gv[k].z, d3 = dv[k].w * gv[k].w;
      m1 += d0;
      m1 += d1;
      m1 += d2;
      m1 += d3;
      m2 += d0 * xv[k].x;
      m2 += d1 * xv[k].y;
      m2 += d2 * xv[k].z;
      m2 += d3 * xv[k].w;
      pg[k].x += dv[k].x * xv[k].x;
      pg[k].y += dv[k].y * xv[k].y;
      pg[k].z += dv[k].z * xv[k].z;
      pg[k].w += dv[k].w * xv[k].w;
      pb[k].x += dv[k].x;
      pb[k].y += dv[k].y;
      pb[k].z += dv[k].z;
      pb[k].w += dv[k].w;
    }
    m1 = wsum_f(m1);
    m2 = wsum_f(m2);
    const float is = __ldg(invstd + r), a = m1 * inv, b = m2 * inv;
#pragma unroll
    for (int k = 0; k < NC4; k++) {
      float4 o;
      o.x = is * (dv[k].x * gv[k].x - a - xv[k].x * b);
      o.y = is * (dv[k].y * gv[k].y - a - xv[k].y * b);
      o.z = is * (dv[k].z * gv[k].z - a - xv[k].z * b);
      o.w = is * (dv[k].w * gv[k].w - a - xv[k].w * b);
      if (acc) {
        const float4 q = dx[(size_t)r * C4 + l + 32 * k];
        o = make_float4(q.x + o.x, q.y + o.y, q.z + o.z, q.w + o.w);
      }
      dx[(size_t)r * C4 + l + 32 * k] = o;
    }
  }
#pragma unroll
  for (int k = 0; k < NC4; k++) {
    red[w][0][l + 32 * k] = pg[k];
    red[w][1][l + 32 * k] = pb[k];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 2 * C4; e += blockDim.x) {
    const int which = e / C4, j = e - which * C4;
    float4 t = red[0][which][j];
    for (int ww = 1; ww < 8; ww++) {
      const float4 v = red[ww][which][j];
      t.x += v.x;
      t.y += v.y;
      t.z += v.z;
      t.w += v.w;
    }
    part[((size_t)which * nb + slab) * C4 + j] = t;
  }
}

// out[c] += sum_r a[r][c] (* bm[r][c]); part is scratch of ceil(rows / CS_ROWS) * c floats
static int colsum(rnn_ctx* ctx, const float* a, const float* bm, int rows, int c, float* part, float* out) {
  return colsum_two_pass(ctx, a, bm, rows, c, part, out);
}

// float4 form (c % 4 == 0, y and b 16-byte aligned)
__global__ void bias_add4_kernel(float4* __restrict__ y, const float4* __restrict__ b, size_t total4, int c4) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total4; i += (size_t)gridDim.x * blockDim.x) {
    float4 v = y[i];
    const float4 q = __ldg(b + i % c4);
    v.x += q.x;
    v.y += q.y;
    v.z += q.z;
    v.w += q.w;
    y[i] = v;
  }
}
__global__ void bias_add_kernel(float* __restrict__ y, const float* __restrict__ b, size_t rows, int c) {
  const size_t total = rows * (size_t)c;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x)
    y[i] += b[i % c];
}

}  // namespace rnn

using namespace rnn;

extern "C" int rnn_layernorm_fwd_dev(rnn_ctx* ctx, const float* x, int rows, int c, const float* g, const float* b,
                                     float eps, float* y, float* xhat, float* invstd) {
  RNN_REQUIRE(ctx && x && g && b && y, "layernorm_fwd: null argument");
  RNN_REQUIRE(rows >= 0 && c > 0, "layernorm_fwd: bad shape");
  if (rows == 0) return RNN_OK;
  const size_t n = (size_t)rows * c;
  RNN_RANGE(x, n * 4);
  RNN_RANGE(y, n * 4);
  if (xhat) RNN_RANGE(xhat, n * 4);
  if (invstd) RNN_RANGE(invstd, (size_t)rows * 4);
  RNN_RANGE(g, (size_t)c * 4);
  RNN_RANGE(b, (size_t)c * 4);
  ln_fwd_kernel<<<(rows * 32 + 255) / 256, 256, 0, ctx->stream>>>(x, rows, c, g, b, eps, y, xhat, invstd);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int rnn::layernorm_bwd(rnn_ctx* ctx, const float* dy, const float* xhat, const float* invstd, int rows, int c,
                       const float* g, float* dx, float* dg, float* db, bool acc_dx) {
  RNN_REQUIRE(ctx && dy && xhat && invstd && g && dx && dg && db, "layernorm_bwd: null argument");
  RNN_REQUIRE(rows >= 0 && c > 0, "layernorm_bwd: bad shape");
  if (rows == 0) return RNN_OK;
  const size_t n = (size_t)rows * c;
  RNN_RANGE(dy, n * 4);
  RNN_RANGE(xhat, n * 4);
  RNN_RANGE(dx, n * 4);
  RNN_RANGE(invstd, (size_t)rows * 4);
  RNN_RANGE(dg, (size_t)c * 4);
  RNN_RANGE(db, (size_t)c * 4);
  const int nblk = (rows + CS_ROWS - 1) / CS_ROWS;
  const bool al = ((uintptr_t)dy & 15) == 0 && ((uintptr_t)xhat & 15) == 0 && ((uintptr_t)dx & 15) == 0 &&
                  ((uintptr_t)g & 15) == 0 && ((uintptr_t)dg & 15) == 0 && ((uintptr_t)db & 15) == 0;
  if (al && c % 128 == 0 && c <= 512) {
    const int nsl = (rows + LN_SLAB - 1) / LN_SLAB;
    RNN_TRY(ensure_ws(ctx, (size_t)2 * nsl * c * 4));
    float* part = static_cast<float*>(ctx->ws);
    const float4* dy4 = reinterpret_cast<const float4*>(dy);
    const float4* xh4 = reinterpret_cast<const float4*>(xhat);
    const float4* g4 = reinterpret_cast<const float4*>(g);
    float4* dx4 = reinterpret_cast<float4*>(dx);
    float4* p4 = reinterpret_cast<float4*>(part);
    switch (c / 128) {
      case 1: ln_bwd4_kernel<1><<<nsl, 256, 0, ctx->stream>>>(dy4, xh4, invstd, rows, g4, dx4, p4, nsl, acc_dx ? 1 : 0); break;
      case 2: ln_bwd4_kernel<2><<<nsl, 256, 0, ctx->stream>>>(dy4, xh4, invstd, rows, g4, dx4, p4, nsl, acc_dx ? 1 : 0); break;
      case 3: ln_bwd4_kernel<3><<<nsl, 256, 0, ctx->stream>>>(dy4, xh4, invstd, rows, g4, dx4, p4, nsl, acc_dx ? 1 : 0); break;
      default: ln_bwd4_kernel<4><<<nsl, 256, 0, ctx->stream>>>(dy4, xh4, invstd, rows, g4, dx4, p4, nsl, acc_dx ? 1 : 0); break;
    }
    RNN_CHECK_LAUNCH();
    // dgamma, dbeta (norm.rs:96-117)
    RNN_TRY(colsum_final(ctx, part, nsl, c, dg));
    return colsum_final(ctx, part + (size_t)nsl * c, nsl, c, db);
  }
  RNN_TRY(ensure_ws(ctx, (size_t)nblk * c * 4));
  float* part = static_cast<float*>(ctx->ws);
  // dgamma, dbeta (norm.rs:96-117)
  RNN_TRY(colsum(ctx, dy, xhat, rows, c, part, dg));
  RNN_TRY(colsum(ctx, dy, nullptr, rows, c, part, db));
  ln_dx_kernel<<<(rows * 32 + 255) / 256, 256, 0, ctx->stream>>>(dy, xhat, invstd, rows, c, g, dx, acc_dx ? 1 : 0);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

extern "C" int rnn_layernorm_bwd_dev(rnn_ctx* ctx, const float* dy, const float* xhat, const float* invstd, int rows,
                                     int c, const float* g, float* dx, float* dg, float* db) {
  return rnn::layernorm_bwd(ctx, dy, xhat, invstd, rows, c, g, dx, dg, db, false);
}

extern "C" int rnn_linear_fwd_dev(rnn_ctx* ctx, const float* x, int rows, int fin, int fout, const float* w,
                                  const float* b, float* y) {
  // linear.rs:44-63: y = x W^T (+ b)
  RNN_REQUIRE(ctx && x && w && y, "linear_fwd: null argument");
  RNN_TRY(tc::gemm_dev(ctx, rows, fout, fin, x, false, w, true, y, false, false));
  if (b && rows > 0) {
    RNN_RANGE(b, (size_t)fout * 4);
    const size_t total = (size_t)rows * fout;
    if (fout % 4 == 0 && ((uintptr_t)y & 15) == 0 && ((uintptr_t)b & 15) == 0)
      bias_add4_kernel<<<(unsigned)std::min<size_t>((total / 4 + 255) / 256, (size_t)ctx->num_sms * 16), 256, 0,
                         ctx->stream>>>(reinterpret_cast<float4*>(y), reinterpret_cast<const float4*>(b),
                                        total / 4, fout / 4);
    else
      bias_add_kernel<<<(unsigned)std::min<size_t>((total + 255) / 256, (size_t)ctx->num_sms * 16), 256, 0,
                        ctx->stream>>>(y, b, rows, fout);
    RNN_CHECK_LAUNCH();
  }
  return RNN_OK;
}

int rnn::linear_bwd(rnn_ctx* ctx, const float* x, const float* dy, int rows, int fin, int fout, const float* w,
                    float* dw, float* db, float* dx, bool acc_dx) {
  // linear.rs:66-96: dW += dY^T X; db += colsum dY; dX = dY W
  RNN_REQUIRE(ctx && x && dy && w && dw && dx, "linear_bwd: null argument");
  if (rows == 0) return RNN_OK;
  RNN_TRY(tc::gemm_dev(ctx, fout, fin, rows, dy, true, x, false, dw, true, true));
  if (db) {
    RNN_RANGE(db, (size_t)fout * 4);
    const int nblk = (rows + CS_ROWS - 1) / CS_ROWS;
    RNN_TRY(ensure_aux(ctx, (size_t)nblk * fout * 4));
    RNN_TRY(colsum(ctx, dy, nullptr, rows, fout, static_cast<float*>(ctx->aux), db));
  }
  return tc::gemm_dev(ctx, rows, fin, fout, dy, false, w, false, dx, acc_dx, false);
}

extern "C" int rnn_linear_bwd_dev(rnn_ctx* ctx, const float* x, const float* dy, int rows, int fin, int fout,
                                  const float* w, float* dw, float* db, float* dx) {
  return rnn::linear_bwd(ctx, x, dy, rows, fin, fout, w, dw, db, dx, false);
}
