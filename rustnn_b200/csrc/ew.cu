// Memory-bound glue of the ResNet step (nn.rs): relu_back_, add_, add_relu_,
// global average pooling, the scalar classifier nn::Linear, softmax_ce and
// the SGD-Nesterov parameter update.  All grid-stride, 16-byte vectorised
// where the length allows; reductions use fixed partitions so every result
// is deterministic.
#include <algorithm>

#include "ew.cuh"

namespace rnn {

static unsigned grid_for(size_t n, int num_sms, int per_sm = 16) {
  size_t g = (n + 255) / 256;
  return (unsigned)std::max<size_t>(1, std::min(g, (size_t)num_sms * per_sm));
}

// ---------------------------------------------------------------- elementwise

__global__ void relu_back_kernel(float* __restrict__ d, const float* __restrict__ y, size_t n) {
  // nn.rs:433-439
  const size_t n4 = n / 4;
  float4* d4 = reinterpret_cast<float4*>(d);
  const float4* y4 = reinterpret_cast<const float4*>(y);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    float4 a = d4[i], b = y4[i];
    if (b.x <= 0.0f) a.x = 0.0f;
    if (b.y <= 0.0f) a.y = 0.0f;
    if (b.z <= 0.0f) a.z = 0.0f;
    if (b.w <= 0.0f) a.w = 0.0f;
    d4[i] = a;
  }
  for (size_t i = n4 * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    if (y[i] <= 0.0f) d[i] = 0.0f;
}

__global__ void add_kernel(float* __restrict__ a, const float* __restrict__ b, size_t n, int relu) {
  // nn.rs:441-450
  const size_t n4 = n / 4;
  float4* a4 = reinterpret_cast<float4*>(a);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    float4 x = a4[i], y = b4[i];
    x.x += y.x; x.y += y.y; x.z += y.z; x.w += y.w;
    if (relu) {
      x.x = fmaxf(x.x, 0.0f); x.y = fmaxf(x.y, 0.0f); x.z = fmaxf(x.z, 0.0f); x.w = fmaxf(x.w, 0.0f);
    }
    a4[i] = x;
  }
  for (size_t i = n4 * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float v = a[i] + b[i];
    a[i] = relu ? fmaxf(v, 0.0f) : v;
  }
}

// a += (y <= 0 ? 0 : b): the identity shortcut's gradient with the join's
// relu_back_ folded in (nn.rs:433-450, relu_back_ then add_)
__global__ void add_masked_kernel(float* __restrict__ a, const float* __restrict__ b,
                                  const float* __restrict__ y, size_t n) {
  const size_t n4 = n / 4;
  float4* a4 = reinterpret_cast<float4*>(a);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  const float4* y4 = reinterpret_cast<const float4*>(y);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    float4 x = a4[i], d = __ldg(b4 + i), m = __ldg(y4 + i);
    x.x += m.x <= 0.0f ? 0.0f : d.x;
    x.y += m.y <= 0.0f ? 0.0f : d.y;
    x.z += m.z <= 0.0f ? 0.0f : d.z;
    x.w += m.w <= 0.0f ? 0.0f : d.w;
    a4[i] = x;
  }
  for (size_t i = n4 * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    a[i] += y[i] <= 0.0f ? 0.0f : b[i];
}

// a += (mask bit <= 0 ? 0 : b) with the ReLU outcome as bits (bit e of word
// e/32); float4 i covers bits 4*(i%8)..+3 of word i/8
__global__ void add_masked_bits_kernel(float* __restrict__ a, const float* __restrict__ b,
                                       const uint32_t* __restrict__ m, size_t n4) {
  float4* a4 = reinterpret_cast<float4*>(a);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t w = __ldg(m + (i >> 3)) >> (4 * (unsigned)(i & 7));
    float4 x = a4[i];
    const float4 d = __ldg(b4 + i);
    x.x += (w & 1u) ? d.x : 0.0f;
    x.y += (w & 2u) ? d.y : 0.0f;
    x.z += (w & 4u) ? d.z : 0.0f;
    x.w += (w & 8u) ? d.w : 0.0f;
    a4[i] = x;
  }
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int relu_back(rnn_ctx* ctx, float* d, const float* y, size_t n) {
  if (n == 0) return RNN_OK;
  RNN_REQUIRE(al16(d) && al16(y), "relu_back: pointers must be 16-byte aligned");
  RNN_RANGE(d, n * sizeof(float));
  RNN_RANGE(y, n * sizeof(float));
  relu_back_kernel<<<grid_for(n / 4 + 1, ctx->num_sms), 256, 0, ctx->stream>>>(d, y, n);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int add(rnn_ctx* ctx, float* a, const float* b, size_t n, bool relu) {
  if (n == 0) return RNN_OK;
  RNN_REQUIRE(al16(a) && al16(b), "add: pointers must be 16-byte aligned");
  RNN_RANGE(a, n * sizeof(float));
  RNN_RANGE(b, n * sizeof(float));
  add_kernel<<<grid_for(n / 4 + 1, ctx->num_sms), 256, 0, ctx->stream>>>(a, b, n, relu ? 1 : 0);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int add_masked(rnn_ctx* ctx, float* a, const float* b, const float* y, size_t n, const uint32_t* mask) {
  if (n == 0) return RNN_OK;
  if (mask && n % 4 == 0 && al16(a) && al16(b)) {
    RNN_RANGE(a, n * sizeof(float));
    RNN_RANGE(b, n * sizeof(float));
    RNN_RANGE(mask, (n + 7) / 8);
    add_masked_bits_kernel<<<grid_for(n / 4 + 1, ctx->num_sms), 256, 0, ctx->stream>>>(a, b, mask, n / 4);
    RNN_CHECK_LAUNCH();
    return RNN_OK;
  }
  RNN_REQUIRE(al16(a) && al16(b) && al16(y), "add_masked: pointers must be 16-byte aligned");
  RNN_RANGE(a, n * sizeof(float));
  RNN_RANGE(b, n * sizeof(float));
  RNN_RANGE(y, n * sizeof(float));
  add_masked_kernel<<<grid_for(n / 4 + 1, ctx->num_sms), 256, 0, ctx->stream>>>(a, b, y, n);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

// ---------------------------------------------------------------- pooling

// one warp per (image, channel) plane; nn.rs:455-463
__global__ void gap_fwd_kernel(const float* __restrict__ x, int nc, int hw, float* __restrict__ y) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, l = threadIdx.x & 31;
  if (w >= nc) return;
  const float* p = x + (size_t)w * hw;
  float s = 0.0f;
  for (int q = l; q < hw; q += 32) s += p[q];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (l == 0) y[w] = s / (float)hw;
}

__global__ void gap_bwd_kernel(const float* __restrict__ dy, int nc, int hw, float* __restrict__ dx) {
  // nn.rs:465-473
  const size_t total = (size_t)nc * hw;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x)
    dx[i] = dy[i / hw] / (float)hw;
}

int gap_fwd(rnn_ctx* ctx, const float* x, int nc, int hw, float* y) {
  if (nc == 0) return RNN_OK;
  RNN_RANGE(x, sizeof(float) * (size_t)nc * hw);
  RNN_RANGE(y, sizeof(float) * (size_t)nc);
  gap_fwd_kernel<<<(nc * 32 + 255) / 256, 256, 0, ctx->stream>>>(x, nc, hw, y);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int gap_bwd(rnn_ctx* ctx, const float* dy, int nc, int hw, float* dx) {
  if (nc == 0) return RNN_OK;
  RNN_RANGE(dy, sizeof(float) * (size_t)nc);
  RNN_RANGE(dx, sizeof(float) * (size_t)nc * hw);
  gap_bwd_kernel<<<grid_for((size_t)nc * hw, ctx->num_sms), 256, 0, ctx->stream>>>(dy, nc, hw, dx);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

// ---------------------------------------------------------------- classifier

// y[i,o] = b[o] + sum_j w[o,j] x[i,j]   (nn.rs:501-520): one warp per output
__global__ void fc_fwd_kernel(const float* __restrict__ x, int n, int fin, int fout, const float* __restrict__ w,
                              const float* __restrict__ b, float* __restrict__ y) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, l = threadIdx.x & 31;
  if (gw >= n * fout) return;
  const int i = gw / fout, o = gw - i * fout;
  const float* xr = x + (size_t)i * fin;
  const float* wr = w + (size_t)o * fin;
  float s = 0.0f;
  for (int j = l; j < fin; j += 32) s += wr[j] * xr[j];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (l == 0) y[gw] = b[o] + s;
}

// Classifier backward (nn.rs:524-539): dW[o,j] += sum_i dy[i,o] x[i,j] runs
// on the GEMM engine (fc_bwd); db[o] += sum_i dy[i,o] here, one warp per
// output, lanes striding the batch, fixed-order shuffle reduction.
__global__ void fc_bwd_b_kernel(const float* __restrict__ dy, int n, int fout, float* __restrict__ db) {
  const int o = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, l = threadIdx.x & 31;
  if (o >= fout) return;
  float s = 0.0f;
  for (int i = l; i < n; i += 32) s += dy[(size_t)i * fout + o];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (l == 0) db[o] += s;
}

// dx[i,j] = sum_o dy[i,o] w[o,j]  (nn.rs:541-557)
__global__ void fc_bwd_x_kernel(const float* __restrict__ dy, int n, int fin, int fout, const float* __restrict__ w,
                                float* __restrict__ dx) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * fin) return;
  const int i = idx / fin, j = idx - i * fin;
  float s = 0.0f;
  for (int o = 0; o < fout; o++) s += dy[(size_t)i * fout + o] * w[(size_t)o * fin + j];
  dx[idx] = s;
}

int fc_fwd(rnn_ctx* ctx, const float* x, int n, int fin, int fout, const float* w, const float* b, float* y) {
  const long warps = (long)n * fout;
  if (warps == 0) return RNN_OK;
  RNN_RANGE(x, sizeof(float) * (size_t)n * fin);
  RNN_RANGE(w, sizeof(float) * (size_t)fout * fin);
  RNN_RANGE(b, sizeof(float) * (size_t)fout);
  RNN_RANGE(y, sizeof(float) * (size_t)n * fout);
  fc_fwd_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, ctx->stream>>>(x, n, fin, fout, w, b, y);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int fc_bwd(rnn_ctx* ctx, const float* x, const float* dy, int n, int fin, int fout, const float* w, float* dw,
           float* db, float* dx) {
  RNN_RANGE(x, sizeof(float) * (size_t)n * fin);
  RNN_RANGE(dy, sizeof(float) * (size_t)n * fout);
  RNN_RANGE(w, sizeof(float) * (size_t)fout * fin);
  RNN_RANGE(dw, sizeof(float) * (size_t)fout * fin);
  RNN_RANGE(db, sizeof(float) * (size_t)fout);
  if (dx) RNN_RANGE(dx, sizeof(float) * (size_t)n * fin);
  // dW[fout][fin] += dy^T x on the tensor-core engine (nn.rs:524-539)
  RNN_TRY(tc::gemm_dev(ctx, fout, fin, n, dy, true, x, false, dw, true, false));
  fc_bwd_b_kernel<<<(fout * 32 + 255) / 256, 256, 0, ctx->stream>>>(dy, n, fout, db);
  RNN_CHECK_LAUNCH();
  if (dx) {
    fc_bwd_x_kernel<<<(n * fin + 255) / 256, 256, 0, ctx->stream>>>(dy, n, fin, fout, w, dx);
    RNN_CHECK_LAUNCH();
  }
  return RNN_OK;
}

// ---------------------------------------------------------------- softmax_ce

// one warp per example; nn.rs:588-613.  row_loss[i], hit[i] written.
__global__ void softmax_ce_rows_kernel(const float* __restrict__ logits, const uint32_t* __restrict__ labels,
                                       int n, int nclass, float smooth, float inv, float* __restrict__ d,
                                       float* __restrict__ row_loss, int* __restrict__ hit, int* dev_error) {
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, l = threadIdx.x & 31;
  if (i >= n) return;
  const float* z = logits + (size_t)i * nclass;
  float* dr = d + (size_t)i * nclass;
  const uint32_t yl = labels[i];
  if (yl >= (uint32_t)nclass) {
    // out-of-range label: the reference panics on the slice index; flag it
    // (RNN_ERR_DEVICE at the next synchronise) and contribute nothing
    if (l == 0) {
      atomicOr(dev_error, 2);
      row_loss[i] = NAN;
      hit[i] = 0;
    }
    for (int j = l; j < nclass; j += 32) dr[j] = NAN;
    return;
  }
  const int y = (int)yl;
  // argmax with the lowest index on ties (nn.rs:573-583 keeps the first max)
  float mx = -INFINITY;
  int arg = 0x7fffffff;
  for (int j = l; j < nclass; j += 32) {
    const float v = z[j];
    if (v > mx || (v == mx && j < arg)) { mx = v; arg = j; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, mx, o);
    const int oa = __shfl_xor_sync(0xffffffffu, arg, o);
    if (om > mx || (om == mx && oa < arg)) { mx = om; arg = oa; }
  }
  float sum = 0.0f, zsum = 0.0f;
  for (int j = l; j < nclass; j += 32) {
    sum += expf(z[j] - mx);
    zsum += z[j];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    zsum += __shfl_xor_sync(0xffffffffu, zsum, o);
  }
  const float lse = mx + logf(sum);
  const float on = 1.0f - smooth, off = smooth / (float)nclass;
  for (int j = l; j < nclass; j += 32) {
    const float t = (j == y) ? on + off : off;
    dr[j] = (expf(z[j] - mx) / sum - t) * inv;
  }
  if (l == 0) {
    float loss = on * (lse - z[y]);
    // sum_j (lse - z_j) = nclass * lse - sum_j z_j
    if (smooth > 0.0f) loss += off * ((float)nclass * lse - zsum);
    row_loss[i] = loss;
    hit[i] = (arg == y) ? 1 : 0;
  }
}

// single block: fixed-order tree sum of the row losses and hits
__global__ void softmax_ce_total_kernel(const float* __restrict__ row_loss, const int* __restrict__ hit, int n,
                                        float inv, float* __restrict__ loss_out, int* __restrict__ correct_out) {
  __shared__ double sl[256];
  __shared__ int sh[256];
  double a = 0.0;
  int h = 0;
  for (int i = threadIdx.x; i < n; i += 256) {
    a += row_loss[i];
    h += hit[i];
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
    if (loss_out) *loss_out = (float)sl[0] * inv;
    if (correct_out) *correct_out = sh[0];
  }
}

int softmax_ce(rnn_ctx* ctx, const float* logits, const uint32_t* labels, int n, int nclass, float smooth,
               float* dlogits, float* row_loss, int* hit, float* loss_out, int* correct_out) {
  if (n == 0) return RNN_OK;
  RNN_RANGE(logits, sizeof(float) * (size_t)n * nclass);
  RNN_RANGE(labels, sizeof(uint32_t) * (size_t)n);
  RNN_RANGE(dlogits, sizeof(float) * (size_t)n * nclass);
  RNN_RANGE(row_loss, sizeof(float) * (size_t)n);
  RNN_RANGE(hit, sizeof(int) * (size_t)n);
  if (loss_out) RNN_RANGE(loss_out, sizeof(float));
  if (correct_out) RNN_RANGE(correct_out, sizeof(int));
  const float inv = 1.0f / (float)n;
  softmax_ce_rows_kernel<<<(n * 32 + 255) / 256, 256, 0, ctx->stream>>>(logits, labels, n, nclass, smooth, inv,
                                                                        dlogits, row_loss, hit, ctx->dev_error);
  RNN_CHECK_LAUNCH();
  softmax_ce_total_kernel<<<1, 256, 0, ctx->stream>>>(row_loss, hit, n, inv, loss_out, correct_out);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

// ---------------------------------------------------------------- SGD

// Param::step (nn.rs:102-110) over a flat buffer.  decay_mask (1 byte per
// element) selects weight decay; gscale pre-scales the gradient (1/world for
// the data-parallel mean).
__global__ void sgd_kernel(float* __restrict__ v, float* __restrict__ g, float* __restrict__ m,
                           const uint8_t* __restrict__ decay_mask, int decay_all, size_t n, float lr, float mom,
                           float wd, float gscale) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int dec = decay_mask ? decay_mask[i] : decay_all;
    const float w = dec ? wd : 0.0f;
    const float gg = g[i] * gscale + w * v[i];
    const float mm = mom * m[i] + gg;
    m[i] = mm;
    v[i] -= lr * (gg + mom * mm);
    g[i] = 0.0f;
  }
}

int sgd_nesterov(rnn_ctx* ctx, float* v, float* g, float* m, const uint8_t* decay_mask, int decay_all, size_t n,
                 float lr, float mom, float wd, float gscale) {
  if (n == 0) return RNN_OK;
  RNN_RANGE(v, n * sizeof(float));
  RNN_RANGE(g, n * sizeof(float));
  RNN_RANGE(m, n * sizeof(float));
  if (decay_mask) RNN_RANGE(decay_mask, n);
  sgd_kernel<<<grid_for(n, ctx->num_sms, 8), 256, 0, ctx->stream>>>(v, g, m, decay_mask, decay_all, n, lr, mom,
                                                                     wd, gscale);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

}  // namespace rnn

using namespace rnn;

extern "C" int rnn_relu_back_dev(rnn_ctx* ctx, float* d, const float* y, size_t len) {
  RNN_REQUIRE(ctx && d && y, "relu_back: null argument");
  return relu_back(ctx, d, y, len);
}
extern "C" int rnn_add_dev(rnn_ctx* ctx, float* a, const float* b, size_t len) {
  RNN_REQUIRE(ctx && a && b, "add: null argument");
  return add(ctx, a, b, len, false);
}
extern "C" int rnn_add_relu_dev(rnn_ctx* ctx, float* a, const float* b, size_t len) {
  RNN_REQUIRE(ctx && a && b, "add_relu: null argument");
  return add(ctx, a, b, len, true);
}
extern "C" int rnn_gap_fwd_dev(rnn_ctx* ctx, const float* x, int nc, int hw, float* y) {
  RNN_REQUIRE(ctx && x && y, "gap_fwd: null argument");
  return gap_fwd(ctx, x, nc, hw, y);
}
extern "C" int rnn_gap_bwd_dev(rnn_ctx* ctx, const float* dy, int nc, int hw, float* dx) {
  RNN_REQUIRE(ctx && dy && dx, "gap_bwd: null argument");
  return gap_bwd(ctx, dy, nc, hw, dx);
}
extern "C" int rnn_softmax_ce_dev(rnn_ctx* ctx, const float* logits, const uint32_t* labels, int n, int nclass,
                                  float smooth, float* dlogits, float* loss_out, int* correct_out) {
  RNN_REQUIRE(ctx && logits && labels && dlogits, "softmax_ce: null argument");
  RNN_REQUIRE(n >= 0 && nclass > 0, "softmax_ce: bad shape");
  RNN_TRY(ensure_ws(ctx, (size_t)n * 8 + 256));
  float* row_loss = static_cast<float*>(ctx->ws);
  int* hit = reinterpret_cast<int*>(static_cast<char*>(ctx->ws) + (((size_t)n * 4 + 255) & ~(size_t)255));
  return softmax_ce(ctx, logits, labels, n, nclass, smooth, dlogits, row_loss, hit, loss_out, correct_out);
}
extern "C" int rnn_sgd_nesterov_dev(rnn_ctx* ctx, float* v, float* g, float* m, size_t len, float lr, float mom,
                                    float wd, int decay) {
  RNN_REQUIRE(ctx && v && g && m, "sgd: null argument");
  return sgd_nesterov(ctx, v, g, m, nullptr, decay ? 1 : 0, len, lr, mom, wd, 1.0f);
}
