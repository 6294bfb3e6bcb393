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

#include "bn.cuh"

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

constexpr int BN_NT = 256;

// grid (C, P): block (c, p) sums images [n*p/P, n*(p+1)/P) of channel c.
__global__ void __launch_bounds__(BN_NT) bn_fwd_partial_kernel(const float* __restrict__ y, int n, int C,
                                                             int hw, int P, double* __restrict__ part) {
  const int c = blockIdx.x, p = blockIdx.y;
  const int i0 = (int)((long)n * p / P), i1 = (int)((long)n * (p + 1) / P);
  double s = 0.0, s2 = 0.0;
  const bool vec = (hw & 3) == 0;
  for (int img = i0; img < i1; img++) {
    const float* plane = y + ((size_t)img * C + c) * hw;
    if (vec) {
      const float4* p4 = reinterpret_cast<const float4*>(plane);
      for (int q = threadIdx.x; q < hw / 4; q += BN_NT) {
        float4 v = __ldg(p4 + q);
        s += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
        s2 += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
      }
    } else {
      for (int q = threadIdx.x; q < hw; q += BN_NT) {
        double v = __ldg(plane + q);
        s += v;
        s2 += v * v;
      }
    }
  }
  block_sum2<BN_NT>(s, s2, part + ((size_t)c * P + p) * 2);
}

// Backward partials: sum dy_eff and dy_eff * xhat.
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
                                float* __restrict__ out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)((i / hw) % C);
    const float xh = (y[i] - mean[c]) * invstd[c];
    float v = gamma[c] * xh + beta[c];
    out[i] = relu ? fmaxf(v, 0.0f) : v;
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

static int bn_parts(int n, int C, int num_sms) {
  int P = (4 * num_sms + C - 1) / C;
  if (P > n) P = n;
  if (P < 1) P = 1;
  return P;
}

static unsigned ew_grid(size_t total, int num_sms) {
  size_t g = (total + 255) / 256;
  size_t cap = (size_t)num_sms * 16;
  return (unsigned)std::max<size_t>(1, std::min(g, cap));
}

int bn_fwd_sums(rnn_ctx* ctx, const float* y, int n, int C, int hw, double* part, double* sums) {
  const int P = bn_parts(n, C, ctx->num_sms);
  RNN_RANGE(y, sizeof(float) * (size_t)n * C * hw);
  RNN_RANGE(part, sizeof(double) * (size_t)C * P * 2);
  RNN_RANGE(sums, sizeof(double) * (size_t)C * 2);
  bn_fwd_partial_kernel<<<dim3(C, P), BN_NT, 0, ctx->stream>>>(y, n, C, hw, P, part);
  RNN_CHECK_LAUNCH();
  bn_combine_kernel<<<(C + 127) / 128, 128, 0, ctx->stream>>>(part, C, P, sums);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int bn_fwd_finish(rnn_ctx* ctx, const float* y, int n, int C, int hw, double count, const double* sums,
                  const float* gamma, const float* beta, float* rmean, float* rvar, float mom, float eps,
                  int relu, float* mean, float* invstd, float* out) {
  RNN_RANGE(sums, sizeof(double) * (size_t)C * 2);
  RNN_RANGE(mean, sizeof(float) * C);
  RNN_RANGE(invstd, sizeof(float) * C);
  if (rmean) RNN_RANGE(rmean, sizeof(float) * C);
  if (rvar) RNN_RANGE(rvar, sizeof(float) * C);
  RNN_RANGE(gamma, sizeof(float) * C);
  RNN_RANGE(beta, sizeof(float) * C);
  RNN_RANGE(y, sizeof(float) * (size_t)n * C * hw);
  RNN_RANGE(out, sizeof(float) * (size_t)n * C * hw);
  bn_finalize_kernel<<<(C + 127) / 128, 128, 0, ctx->stream>>>(sums, C, count, mom, eps, mean, invstd,
                                                                rmean, rvar);
  RNN_CHECK_LAUNCH();
  const size_t total = (size_t)n * C * hw;
  bn_apply_kernel<<<ew_grid(total, ctx->num_sms), 256, 0, ctx->stream>>>(y, C, hw, total, gamma, beta,
                                                                          mean, invstd, relu, out);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int bn_bwd_sums(rnn_ctx* ctx, const float* dy, const float* y, const float* relu_out, int n, int C, int hw,
                const float* mean, const float* invstd, double* part, double* sums) {
  const int P = bn_parts(n, C, ctx->num_sms);
  RNN_RANGE(dy, sizeof(float) * (size_t)n * C * hw);
  RNN_RANGE(y, sizeof(float) * (size_t)n * C * hw);
  if (relu_out) RNN_RANGE(relu_out, sizeof(float) * (size_t)n * C * hw);
  RNN_RANGE(mean, sizeof(float) * C);
  RNN_RANGE(invstd, sizeof(float) * C);
  RNN_RANGE(part, sizeof(double) * (size_t)C * P * 2);
  RNN_RANGE(sums, sizeof(double) * (size_t)C * 2);
  bn_bwd_partial_kernel<<<dim3(C, P), BN_NT, 0, ctx->stream>>>(dy, y, relu_out, n, C, hw, P, mean,
                                                               invstd, part);
  RNN_CHECK_LAUNCH();
  bn_combine_kernel<<<(C + 127) / 128, 128, 0, ctx->stream>>>(part, C, P, sums);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int bn_bwd_finish(rnn_ctx* ctx, const float* dy, const float* y, const float* relu_out, int n, int C, int hw,
                  double count, const double* sums, const float* gamma, const float* mean,
                  const float* invstd, float* dgb /* [2C] scratch */, float* dx, float* dgamma,
                  float* dbeta, float pscale) {
  RNN_RANGE(sums, sizeof(double) * (size_t)C * 2);
  RNN_RANGE(dgb, sizeof(float) * (size_t)C * 2);
  if (dgamma) RNN_RANGE(dgamma, sizeof(float) * C);
  if (dbeta) RNN_RANGE(dbeta, sizeof(float) * C);
  RNN_RANGE(gamma, sizeof(float) * C);
  RNN_RANGE(dx, sizeof(float) * (size_t)n * C * hw);
  bn_bwd_finalize_kernel<<<(C + 127) / 128, 128, 0, ctx->stream>>>(sums, C, dgb, dgb + C, dgamma, dbeta,
                                                                    pscale);
  RNN_CHECK_LAUNCH();
  const size_t total = (size_t)n * C * hw;
  bn_dx_kernel<<<ew_grid(total, ctx->num_sms), 256, 0, ctx->stream>>>(
      dy, y, relu_out, C, hw, total, (float)count, gamma, mean, invstd, dgb, dgb + C, dx);
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
