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
                             float* __restrict__ dx) {
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
    dx[(size_t)r * c + j] = is * (d - m1 * inv - xh[j] * m2 * inv);
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

extern "C" int rnn_layernorm_bwd_dev(rnn_ctx* ctx, const float* dy, const float* xhat, const float* invstd, int rows,
                                     int c, const float* g, float* dx, float* dg, float* db) {
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
  RNN_TRY(ensure_ws(ctx, (size_t)nblk * c * 4));
  float* part = static_cast<float*>(ctx->ws);
  // dgamma, dbeta (norm.rs:96-117)
  RNN_TRY(colsum(ctx, dy, xhat, rows, c, part, dg));
  RNN_TRY(colsum(ctx, dy, nullptr, rows, c, part, db));
  ln_dx_kernel<<<(rows * 32 + 255) / 256, 256, 0, ctx->stream>>>(dy, xhat, invstd, rows, c, g, dx);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
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

extern "C" int rnn_linear_bwd_dev(rnn_ctx* ctx, const float* x, const float* dy, int rows, int fin, int fout,
                                  const float* w, float* dw, float* db, float* dx) {
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
  return tc::gemm_dev(ctx, rows, fin, fout, dy, false, w, false, dx, false, false);
}
