// The rustvit step's fusions that the reference lists as identified and not
// done (README.md:549-552): the residual add fused into LayerNorm, LayerNorm
// writing its output straight into the packed A operand of the GEMM that
// follows, and the SiLU gate in the epilogue of the SwiGLU's first GEMM.
//
//   rnn_layernorm_res_fwd_dev  s = x (+ r1) (+ r2); y = LN(s)   vit.rs:141-178 + norm.rs:38-100
//                              and, optionally, the [hi | lo] shared-memory
//                              image of y that the tcgen05 engine's producers
//                              would otherwise build (the GEMM bulk-copies it)
//   rnn_linear_fwd_packed_dev  y = x W^T + b from that image, the bias added in
//                              the epilogue                   linear.rs:44-63
//   rnn_swiglu_fwd_dev         ab = x Wg^T + bg and u = silu(a) * g in one GEMM
//                              (norm.rs:250-268): the weight rows are taken
//                              in an order that puts 16 value columns and
//                              their 16 gate columns in every 32-column
//                              accumulator chunk, so the epilogue has both
//
// Numerics are those of the unfused sequence: the sums are the same f32
// additions in the same order, the LayerNorm statistics are f64, the
// contractions are the engine's 3xTF32, and silu(a) * g is a * (1 / (1 +
// exp(-a))) * g as norm.rs:256-259 writes it.
#include <algorithm>

#include "tc_launch.cuh"

namespace rnn {
namespace {

__device__ __forceinline__ double wsum_dbl(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

// Bytes of the packed A image of `rows` x `k`: per 128-row tile and 32-deep
// K block one [hi | lo] pair of 16 KB SWIZZLE_128B tiles.
__host__ __device__ inline size_t aimg_tile_floats() { return 2 * (size_t)tc::BM * tc::BK; }

// One warp per row; lane l holds float4 chunks l, l + 32, ... (c % 128 == 0).
template <int NR>
__global__ void ln_res_fwd_kernel(const float* __restrict__ x, const float* __restrict__ r1,
                                  const float* __restrict__ r2, int rows, int c, const float* __restrict__ g,
                                  const float* __restrict__ b, float eps, float* __restrict__ sum_out,
                                  float* __restrict__ y, float* __restrict__ xhat, float* __restrict__ invstd,
                                  float* __restrict__ aimg) {
  constexpr int MAXQ = 4;  // c <= 512
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, l = threadIdx.x & 31;
  if (r >= rows) return;
  const int nq = c / 128;
  float4 v[MAXQ];
  double s = 0.0, s2 = 0.0;
#pragma unroll
  for (int i = 0; i < MAXQ; i++) {
    if (i >= nq) break;
    const size_t o = (size_t)r * c + 4 * (l + 32 * i);
    float4 t = __ldg(reinterpret_cast<const float4*>(x + o));
    // vit.rs:160-176: y = x; y += branch; y += branch (one rounding each)
    if (NR >= 1) t = add4(t, __ldg(reinterpret_cast<const float4*>(r1 + o)));
    if (NR >= 2) t = add4(t, __ldg(reinterpret_cast<const float4*>(r2 + o)));
    if (sum_out) *reinterpret_cast<float4*>(sum_out + o) = t;
    v[i] = t;
    s += (double)t.x + (double)t.y + (double)t.z + (double)t.w;
    s2 += (double)t.x * t.x + (double)t.y * t.y + (double)t.z * t.z + (double)t.w * t.w;
  }
  s = wsum_dbl(s);
  s2 = wsum_dbl(s2);
  // norm.rs:53-66: f64 mean and biased variance, eps inside the root
  const double m = (double)c, mu = s / m;
  const double va = s2 / m - mu * mu;
  const float var = (float)(va > 0.0 ? va : 0.0);
  const float is = 1.0f / sqrtf(var + eps);
  const float muf = (float)mu;
  if (l == 0 && invstd) invstd[r] = is;
  const int kblocks = c / tc::BK;
#pragma unroll
  for (int i = 0; i < MAXQ; i++) {
    if (i >= nq) break;
    const int q = l + 32 * i;  // float4 chunk of the row: columns 4q .. 4q+3
    const size_t o = (size_t)r * c + 4 * q;
    const float4 gg = __ldg(reinterpret_cast<const float4*>(g + 4 * q));
    const float4 bb = __ldg(reinterpret_cast<const float4*>(b + 4 * q));
    const float h0 = (v[i].x - muf) * is, h1 = (v[i].y - muf) * is, h2 = (v[i].z - muf) * is,
                h3 = (v[i].w - muf) * is;
    if (xhat) *reinterpret_cast<float4*>(xhat + o) = make_float4(h0, h1, h2, h3);
    const float4 out = make_float4(gg.x * h0 + bb.x, gg.y * h1 + bb.y, gg.z * h2 + bb.z, gg.w * h3 + bb.w);
    *reinterpret_cast<float4*>(y + o) = out;
    if (aimg) {
      // element (r, 4q..4q+3) is chunk q % 8 of row r % 128 in the tile of
      // (row tile r / 128, K block q / 8)
      char* tile = reinterpret_cast<char*>(aimg + ((size_t)(r >> 7) * kblocks + (q >> 3)) * aimg_tile_floats());
      const uint32_t off = tc::sw128_offset(r & 127, q & 7);
      const float o0 = tc::tf32_round(out.x), o1 = tc::tf32_round(out.y), o2 = tc::tf32_round(out.z),
                  o3 = tc::tf32_round(out.w);
      *reinterpret_cast<float4*>(tile + off) = make_float4(o0, o1, o2, o3);
      *reinterpret_cast<float4*>(tile + tc::BM * tc::BK * 4 + off) =
          make_float4(out.x - o0, out.y - o1, out.z - o2, out.w - o3);
    }
  }
}

}  // namespace

namespace tc {

// y = A W^T + b with A bulk-copied from the packed image.
template <int BN>
struct LinPackedProb {
  static constexpr bool B_BULK = false;
  static constexpr bool A_BULK = true;
  const float* aimg;
  const float* w;  // [N][K]
  const float* bias;
  float* y;        // [M][N]
  int M, N, K, kblocks;
  bool y_vec;
  struct TS {
    int n0;
  };
  __device__ __forceinline__ void tile_begin(TS& ts, int, int n0, int) const { ts.n0 = n0; }
  __device__ __forceinline__ const void* a_src(int mt, int kb) const {
    return aimg + ((size_t)mt * kblocks + kb) * (2 * (size_t)BM * BK);
  }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) { r = (gt >> 3) + 16 * j; c = gt & 7; }
  static __device__ __forceinline__ void b_slot(int gt, int j, int& r, int& c) {
    const int idx = gt + 128 * j;
    r = idx >> 3;
    c = idx & 7;
  }
  __device__ __forceinline__ void load_a(const TS&, int, int, float (&)[32]) const {}
  template <int NB>
  __device__ __forceinline__ void load_b(const TS& ts, int kb, int gt, float (&v)[NB]) const {
#pragma unroll
    for (int j = 0; j < NB / 4; j++) {
      int r, c;
      b_slot(gt, j, r, c);
      const int row = ts.n0 + r;
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (row < N) t = __ldg(reinterpret_cast<const float4*>(w + (size_t)row * K + kb * BK + 4 * c));
      v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
    }
  }
  __device__ __forceinline__ const void* b_src(int, int) const { return nullptr; }
  __device__ __forceinline__ void store(int row, int col0, int, const float (&v)[32]) const {
    if (row >= M || col0 >= N) return;
    float o[32];
#pragma unroll
    for (int e = 0; e < 32; e++) o[e] = v[e] + (bias && col0 + e < N ? __ldg(bias + col0 + e) : 0.0f);
    store_row32(y + (size_t)row * N + col0, N - col0, o, false, y_vec);
  }
};

// ab = A Wg^T + bg and u = silu(a) * g.  Engine column n of chunk q = n / 32
// is value column 16q + (n % 32) for n % 32 < 16, else gate column
// h + 16q + (n % 32 - 16).  A comes from the packed image (ABULK) or from the
// row-major [M][K] input.
template <int BN, bool ABULK>
struct SwigluProb {
  static constexpr bool B_BULK = false;
  static constexpr bool A_BULK = ABULK;
  const float* aimg;  // ABULK
  const float* x;     // !ABULK: [M][K]
  const float* w;     // [2h][K]
  const float* bias;  // [2h]
  float* ab;          // [M][2h]
  float* u;           // [M][h]
  int M, N, K, h, kblocks;
  struct TS {
    int m0, n0;
  };
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int n0, int) const {
    ts.m0 = m0;
    ts.n0 = n0;
  }
  __device__ __forceinline__ const void* a_src(int mt, int kb) const {
    return aimg + ((size_t)mt * kblocks + kb) * (2 * (size_t)BM * BK);
  }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) { r = (gt >> 3) + 16 * j; c = gt & 7; }
  static __device__ __forceinline__ void b_slot(int gt, int j, int& r, int& c) {
    const int idx = gt + 128 * j;
    r = idx >> 3;
    c = idx & 7;
  }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int gt, float (&v)[32]) const {
#pragma unroll
    for (int j = 0; j < 8; j++) {
      int r, c;
      a_slot(gt, j, r, c);
      const int row = ts.m0 + r;
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (row < M) t = __ldg(reinterpret_cast<const float4*>(x + (size_t)row * K + kb * BK + 4 * c));
      v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
    }
  }
  static __device__ __forceinline__ int wrow(int n, int h) {
    const int q = n >> 5, e = n & 31;
    return e < 16 ? 16 * q + e : h + 16 * q + (e - 16);
  }
  template <int NB>
  __device__ __forceinline__ void load_b(const TS& ts, int kb, int gt, float (&v)[NB]) const {
#pragma unroll
    for (int j = 0; j < NB / 4; j++) {
      int r, c;
      b_slot(gt, j, r, c);
      const int n = ts.n0 + r;
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (n < N) t = __ldg(reinterpret_cast<const float4*>(w + (size_t)wrow(n, h) * K + kb * BK + 4 * c));
      v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
    }
  }
  __device__ __forceinline__ const void* b_src(int, int) const { return nullptr; }
  __device__ __forceinline__ void store(int row, int col0, int, const float (&v)[32]) const {
    if (row >= M || col0 >= N) return;
    const int j0 = col0 / 2;  // 16 value / gate columns of this chunk
    float a[16], gt[16], uu[16];
#pragma unroll
    for (int e = 0; e < 16; e++) {
      a[e] = v[e] + __ldg(bias + j0 + e);            // linear.rs:58-61: y = x W^T + b
      gt[e] = v[16 + e] + __ldg(bias + h + j0 + e);
      const float s = 1.0f / (1.0f + expf(-a[e]));   // norm.rs:221-223
      uu[e] = a[e] * s * gt[e];                      // norm.rs:256-259
    }
    float* abr = ab + (size_t)row * 2 * h;
    float* ur = u + (size_t)row * h + j0;
#pragma unroll
    for (int e = 0; e < 16; e += 4) {
      *reinterpret_cast<float4*>(abr + j0 + e) = make_float4(a[e], a[e + 1], a[e + 2], a[e + 3]);
      *reinterpret_cast<float4*>(abr + h + j0 + e) = make_float4(gt[e], gt[e + 1], gt[e + 2], gt[e + 3]);
      *reinterpret_cast<float4*>(ur + e) = make_float4(uu[e], uu[e + 1], uu[e + 2], uu[e + 3]);
    }
  }
};

template <int BN, class P>
static int run_dense(rnn_ctx* ctx, P p) {
  Sched s = make_sched(p.M, p.N, p.K, BN, 1);
  return launch<BN>(ctx, p, s);
}

template <template <int> class L, class... A>
static int by_bn(int bn, A&&... args) {
  switch (bn) {
    case 32: return L<32>::run(args...);
    case 64: return L<64>::run(args...);
    case 128: return L<128>::run(args...);
    default: return L<256>::run(args...);
  }
}

}  // namespace tc
}  // namespace rnn

using namespace rnn;

static inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

extern "C" int rnn_layernorm_res_fwd_dev(rnn_ctx* ctx, const float* x, const float* r1, const float* r2, int rows,
                                         int c, const float* g, const float* b, float eps, float* sum_out, float* y,
                                         float* xhat, float* invstd, float* a_image) {
  RNN_REQUIRE(ctx && x && g && b && y, "layernorm_res_fwd: null argument");
  RNN_REQUIRE(rows >= 0 && c > 0 && c % 128 == 0 && c <= 512,
              "layernorm_res_fwd: c = %d (a multiple of 128 up to 512)", c);
  RNN_REQUIRE(r1 || !r2, "layernorm_res_fwd: r2 without r1");
  if (rows == 0) return RNN_OK;
  for (const void* p : {(const void*)x, (const void*)r1, (const void*)r2, (const void*)sum_out, (const void*)y,
                        (const void*)xhat, (const void*)g, (const void*)b, (const void*)a_image})
    RNN_REQUIRE(!p || al16(p), "layernorm_res_fwd: every tensor must be 16-byte aligned");
  const size_t n = (size_t)rows * c;
  RNN_RANGE(x, n * 4);
  if (r1) RNN_RANGE(r1, n * 4);
  if (r2) RNN_RANGE(r2, n * 4);
  if (sum_out) RNN_RANGE(sum_out, n * 4);
  RNN_RANGE(y, n * 4);
  if (xhat) RNN_RANGE(xhat, n * 4);
  if (invstd) RNN_RANGE(invstd, (size_t)rows * 4);
  RNN_RANGE(g, (size_t)c * 4);
  RNN_RANGE(b, (size_t)c * 4);
  if (a_image) RNN_RANGE(a_image, (size_t)(rows + tc::BM - 1) / tc::BM * (c / tc::BK) * aimg_tile_floats() * 4);
  const unsigned grid = (unsigned)(((size_t)rows * 32 + 255) / 256);
  if (!r1)
    ln_res_fwd_kernel<0><<<grid, 256, 0, ctx->stream>>>(x, r1, r2, rows, c, g, b, eps, sum_out, y, xhat, invstd,
                                                        a_image);
  else if (!r2)
    ln_res_fwd_kernel<1><<<grid, 256, 0, ctx->stream>>>(x, r1, r2, rows, c, g, b, eps, sum_out, y, xhat, invstd,
                                                        a_image);
  else
    ln_res_fwd_kernel<2><<<grid, 256, 0, ctx->stream>>>(x, r1, r2, rows, c, g, b, eps, sum_out, y, xhat, invstd,
                                                        a_image);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

namespace rnn {
namespace tc {
template <int BN>
struct LinPackedL {
  static int run(rnn_ctx* ctx, const float* img, int rows, int fin, int fout, const float* w, const float* b,
                 float* y) {
    LinPackedProb<BN> p;
    p.aimg = img; p.w = w; p.bias = b; p.y = y;
    p.M = rows; p.N = fout; p.K = fin; p.kblocks = fin / BK;
    p.y_vec = fout % 4 == 0 && al16(y);
    return run_dense<BN>(ctx, p);
  }
};
template <int BN>
struct SwigluL {
  static int run(rnn_ctx* ctx, const float* x, const float* img, int rows, int c, int h, const float* w,
                 const float* b, float* ab, float* u) {
    if (img) {
      SwigluProb<BN, true> p;
      p.aimg = img; p.x = nullptr; p.w = w; p.bias = b; p.ab = ab; p.u = u;
      p.M = rows; p.N = 2 * h; p.K = c; p.h = h; p.kblocks = c / BK;
      return run_dense<BN>(ctx, p);
    }
    SwigluProb<BN, false> p;
    p.aimg = nullptr; p.x = x; p.w = w; p.bias = b; p.ab = ab; p.u = u;
    p.M = rows; p.N = 2 * h; p.K = c; p.h = h; p.kblocks = c / BK;
    return run_dense<BN>(ctx, p);
  }
};
}  // namespace tc
}  // namespace rnn

extern "C" int rnn_linear_fwd_packed_dev(rnn_ctx* ctx, const float* a_image, int rows, int fin, int fout,
                                         const float* w, const float* b, float* y) {
  RNN_REQUIRE(ctx && a_image && w && y, "linear_fwd_packed: null argument");
  RNN_REQUIRE(rows >= 0 && fin > 0 && fin % tc::BK == 0 && fout > 0,
              "linear_fwd_packed: fin = %d (a multiple of 32)", fin);
  RNN_REQUIRE(al16(a_image) && al16(w) && (!b || al16(b)), "linear_fwd_packed: 16-byte aligned operands");
  if (rows == 0) return RNN_OK;
  RNN_RANGE(a_image, (size_t)(rows + tc::BM - 1) / tc::BM * (fin / tc::BK) * aimg_tile_floats() * 4);
  RNN_RANGE(w, (size_t)fout * fin * 4);
  if (b) RNN_RANGE(b, (size_t)fout * 4);
  RNN_RANGE(y, (size_t)rows * fout * 4);
  const int bn = tc::pick_bn(fout, (rows + tc::BM - 1) / tc::BM, ctx->num_sms);
  return tc::by_bn<tc::LinPackedL>(bn, ctx, a_image, rows, fin, fout, w, b, y);
}

extern "C" int rnn_swiglu_fwd_dev(rnn_ctx* ctx, const float* x, const float* a_image, int rows, int c, int h,
                                  const float* wg, const float* bg, float* ab, float* u) {
  RNN_REQUIRE(ctx && (x || a_image) && wg && bg && ab && u, "swiglu_fwd: null argument");
  RNN_REQUIRE(rows >= 0 && c > 0 && c % tc::BK == 0 && h > 0 && h % 16 == 0,
              "swiglu_fwd: c = %d (a multiple of 32), h = %d (a multiple of 16)", c, h);
  for (const void* p : {(const void*)x, (const void*)a_image, (const void*)wg, (const void*)bg, (const void*)ab,
                        (const void*)u})
    RNN_REQUIRE(!p || al16(p), "swiglu_fwd: 16-byte aligned operands");
  if (rows == 0) return RNN_OK;
  if (a_image) RNN_RANGE(a_image, (size_t)(rows + tc::BM - 1) / tc::BM * (c / tc::BK) * aimg_tile_floats() * 4);
  else RNN_RANGE(x, (size_t)rows * c * 4);
  RNN_RANGE(wg, (size_t)2 * h * c * 4);
  RNN_RANGE(bg, (size_t)2 * h * 4);
  RNN_RANGE(ab, (size_t)rows * 2 * h * 4);
  RNN_RANGE(u, (size_t)rows * h * 4);
  const int bn = tc::pick_bn(2 * h, (rows + tc::BM - 1) / tc::BM, ctx->num_sms);
  return tc::by_bn<tc::SwigluL>(bn, ctx, x, a_image, rows, c, h, wg, bg, ab, u);
}
