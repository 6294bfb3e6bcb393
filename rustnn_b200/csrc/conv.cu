// Implicit-GEMM convolutions on the tcgen05 3xTF32 engine.  No im2col /
// col2im matrix ever exists in HBM: the producer warps gather the operand
// tile straight from the NCHW tensors into shared memory, the way
// conv.rs:75-120 (gather_span) builds its B panel straight from the image.
//
//   fwd    M = n*oh*ow output pixels, N = cout, K = cin*k*k   conv.rs:169 forward_image
//   dgrad  M = n*h*w   input pixels,  N = cin,  K = cout*k*k  conv.rs:207 dx_image
//   wgrad  M = cin*k*k,               N = cout, K = n*oh*ow   conv.rs:283 dw_image
//
// The K ordering (ci, kh, kw) matches RowMap (conv.rs:49-58) and the weight
// layout [cout][cin][kh][kw] of nn.rs:116.  dgrad handles stride 2 by
// testing divisibility of (i + pad - kh) by the stride (the transposed
// convolution of scatter_span, conv.rs:124-165).
#include <cuda.h>

#include "bn.cuh"
#include "ew.cuh"
#include "tc_launch.cuh"

namespace rnn {
namespace tc {

// cuTensorMapEncodeTiled through the runtime's driver entry point (the
// library does not link libcuda directly).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled_fn() {
  static const EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(p);
    return static_cast<EncodeTiledFn>(nullptr);
  }();
  return fn;
}

// Tensor map of an NCHW f32 tensor [n][c][h][w] read in boxes of
// box_w x box_h x box_c pixels of one image (zero fill outside); with
// CU_TENSOR_MAP_SWIZZLE_128B (box_w = 32) the 16-byte chunk j of box row r
// lands at chunk j ^ (r % 8) of its 128-byte row.
static int encode_nchw_map(CUtensorMap* m, const float* t, int n, int c, int h, int w, int box_w, int box_h,
                           int box_c, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
  EncodeTiledFn fn = encode_tiled_fn();
  RNN_REQUIRE(fn != nullptr, "conv: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[4] = {(cuuint64_t)w, (cuuint64_t)h, (cuuint64_t)c, (cuuint64_t)n};
  const cuuint64_t strides[3] = {(cuuint64_t)w * 4, (cuuint64_t)h * w * 4, (cuuint64_t)c * h * w * 4};
  const cuuint32_t box[4] = {(cuuint32_t)box_w, (cuuint32_t)box_h, (cuuint32_t)box_c, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(t), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  RNN_REQUIRE(r == CUDA_SUCCESS, "conv: cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return RNN_OK;
}

struct ConvGeom {
  int n, cin, h, w, cout, stride, pad, oh, ow;
};

// Epilogue store of 32 consecutive output channels of one pixel into a
// channel-planar tensor: out[o0 + j*plane], j < nvalid, becomes v or, with
// acc, out + v.  When accumulating, the loads of each group of 8 channels
// are issued before its stores, so the warp waits on memory 4 times per call
// rather than once per channel (the compiler may not hoist a load above a
// store to the same array).
__device__ __forceinline__ void store_planes32(float* out, size_t o0, size_t plane, int nvalid,
                                               const float (&v)[32], int acc) {
#pragma unroll
  for (int g = 0; g < 32; g += 8) {
    float add[8];
#pragma unroll
    for (int e = 0; e < 8; e++) add[e] = (acc && g + e < nvalid) ? out[o0 + (size_t)(g + e) * plane] : 0.0f;
#pragma unroll
    for (int e = 0; e < 8; e++)
      if (g + e < nvalid) out[o0 + (size_t)(g + e) * plane] = acc ? add[e] + v[g + e] : v[g + e];
  }
}

// BatchNorm statistics of a forward convolution's output, summed in its
// epilogue (the engine's STATS hook) so the BN layer that follows does not
// re-read y: per-channel (sum y, sum y^2) in f64.
struct ConvStatsDev {
  double* part = nullptr;    // [gridDim.x][N][2] per-CTA partials; nullptr = off
  unsigned* counter = nullptr;
  double* sums = nullptr;    // [N][2] totals (over ranks when ps.world > 1)
  PeerSums ps;
};

// After the CTA's last tile (all threads): fold the four epilogue warps'
// sums of each column in order into this CTA's partial; the last CTA to
// finish adds the partials in CTA order (deterministic), runs the
// cross-rank exchange when there are peers, and rearms the counter.
__device__ inline void conv_stats_flush(const double* sm, const ConvStatsDev& st, int N) {
  for (int col = threadIdx.x; col < N; col += blockDim.x) {
    const int c = col >> 5, l = col & 31;
    double s = 0.0, q = 0.0;
#pragma unroll
    for (int w = 0; w < 4; w++) {
      s += sm[(2 * c) * 128 + w * 32 + l];
      q += sm[(2 * c + 1) * 128 + w * 32 + l];
    }
    st.part[((size_t)blockIdx.x * N + col) * 2] = s;
    st.part[((size_t)blockIdx.x * N + col) * 2 + 1] = q;
    __threadfence();
  }
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(st.counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int col = threadIdx.x; col < N; col += blockDim.x) {
    double s = 0.0, q = 0.0;
    for (unsigned p = 0; p < gridDim.x; p++) {
      s += __ldcg(st.part + ((size_t)p * N + col) * 2);
      q += __ldcg(st.part + ((size_t)p * N + col) * 2 + 1);
    }
    st.sums[col * 2] = s;
    st.sums[col * 2 + 1] = q;
  }
  if (st.ps.world > 1) {
    __syncthreads();
    peer_exchange(st.ps, st.sums, N);
  }
  if (threadIdx.x == 0) *st.counter = 0u;
}

// ---------------------------------------------------------------- forward

template <int KS>
struct ConvFwdProb {
  static constexpr bool A_KMAJOR = false;  // lanes walk output pixels
  static constexpr bool B_KMAJOR = true;   // weights [cout][cin*KS*KS]
  static constexpr int KK = KS * KS;
  const float* x;
  const float* w;
  float* y;
  ConvGeom g;
  int M, N, K;
  int acc;
  int splits;
  bool w_vec;

  __device__ __forceinline__ void load_a(int row, int k4, float (&v)[4]) const {
    const int ohw = g.oh * g.ow;
    if (row >= M) {
      v[0] = v[1] = v[2] = v[3] = 0.0f;
      return;
    }
    const int img = row / ohw, rem = row - img * ohw;
    const int oy = rem / g.ow, ox = rem - oy * g.ow;
    const int iy0 = oy * g.stride - g.pad, ix0 = ox * g.stride - g.pad;
    const float* xi = x + (size_t)img * g.cin * g.h * g.w;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int k = k4 + i;
      float val = 0.0f;
      if (k < K) {
        const int ci = k / KK, kk = k - ci * KK;
        const int kh = kk / KS, kw = kk - kh * KS;
        const int iy = iy0 + kh, ix = ix0 + kw;
        if (iy >= 0 && iy < g.h && ix >= 0 && ix < g.w)
          val = __ldg(xi + ((size_t)ci * g.h + iy) * g.w + ix);
      }
      v[i] = val;
    }
  }

  __device__ __forceinline__ void load_b(int row, int k4, float (&v)[4]) const {
    if (row < N && w_vec && k4 + 3 < K) {
      float4 t = __ldg(reinterpret_cast<const float4*>(w + (size_t)row * K + k4));
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
#pragma unroll
      for (int i = 0; i < 4; i++)
        v[i] = (row < N && k4 + i < K) ? __ldg(w + (size_t)row * K + k4 + i) : 0.0f;
    }
  }

  __device__ __forceinline__ void store(int row, int col0, int, const float (&v)[32]) const {
    if (row >= M) return;
    const int ohw = g.oh * g.ow;
    const int img = row / ohw, rem = row - img * ohw;
    float* yp = y + ((size_t)img * g.cout) * ohw + rem;
#pragma unroll
    for (int j = 0; j < 32; j++) {
      const int co = col0 + j;
      if (co < N) {
        float* p = yp + (size_t)co * ohw;
        *p = acc ? *p + v[j] : v[j];
      }
    }
  }
};

// ---------------------------------------------------------------- dgrad

template <int KS>
struct ConvDgradProb {
  static constexpr bool A_KMAJOR = false;  // lanes walk input pixels
  static constexpr bool B_KMAJOR = true;   // rows = ci, K = (co, kh, kw)
  static constexpr int KK = KS * KS;
  const float* dy;
  const float* w;
  float* dx;
  ConvGeom g;
  int M, N, K;
  int acc;
  int splits;

  __device__ __forceinline__ void load_a(int row, int k4, float (&v)[4]) const {
    const int hw = g.h * g.w;
    if (row >= M) {
      v[0] = v[1] = v[2] = v[3] = 0.0f;
      return;
    }
    const int img = row / hw, rem = row - img * hw;
    const int iy = rem / g.w, ix = rem - iy * g.w;
    const float* dyi = dy + (size_t)img * g.cout * g.oh * g.ow;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int k = k4 + i;
      float val = 0.0f;
      if (k < K) {
        const int co = k / KK, kk = k - co * KK;
        const int kh = kk / KS, kw = kk - kh * KS;
        const int ty = iy + g.pad - kh, tx = ix + g.pad - kw;
        if (ty >= 0 && tx >= 0) {
          int oy, ox;
          bool ok;
          if (g.stride == 1) {
            oy = ty; ox = tx; ok = true;
          } else {
            oy = ty / g.stride; ox = tx / g.stride;
            ok = (oy * g.stride == ty) && (ox * g.stride == tx);
          }
          if (ok && oy < g.oh && ox < g.ow)
            val = __ldg(dyi + ((size_t)co * g.oh + oy) * g.ow + ox);
        }
      }
      v[i] = val;
    }
  }

  __device__ __forceinline__ void load_b(int row, int k4, float (&v)[4]) const {
    // B(ci, (co,kh,kw)) = W[co][ci][kh][kw]
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int k = k4 + i;
      float val = 0.0f;
      if (row < N && k < K) {
        const int co = k / KK, kk = k - co * KK;
        val = __ldg(w + ((size_t)co * g.cin + row) * KK + kk);
      }
      v[i] = val;
    }
  }

  __device__ __forceinline__ void store(int row, int col0, int, const float (&v)[32]) const {
    if (row >= M) return;
    const int hw = g.h * g.w;
    const int img = row / hw, rem = row - img * hw;
    float* xp = dx + ((size_t)img * g.cin) * hw + rem;
#pragma unroll
    for (int j = 0; j < 32; j++) {
      const int ci = col0 + j;
      if (ci < N) {
        float* p = xp + (size_t)ci * hw;
        *p = acc ? *p + v[j] : v[j];
      }
    }
  }
};

// ---------------------------------------------------------------- wgrad

template <int KS>
struct ConvWgradProb {
  static constexpr bool A_KMAJOR = true;  // lanes walk pixels (K)
  static constexpr bool B_KMAJOR = true;
  static constexpr int KK = KS * KS;
  const float* x;
  const float* dy;
  float* dw;  // [cout][cin*KK], accumulated
  float* ws;  // split partials [splits][M][N]
  ConvGeom g;
  int M, N, K;
  int splits;
  bool dy_vec;

  __device__ __forceinline__ void load_a(int row, int k4, float (&v)[4]) const {
    // A((ci,kh,kw), pixel) = X[img, ci, oy*s - pad + kh, ox*s - pad + kw]
    if (row >= M) {
      v[0] = v[1] = v[2] = v[3] = 0.0f;
      return;
    }
    const int ci = row / KK, kk = row - ci * KK;
    const int kh = kk / KS, kw = kk - kh * KS;
    const int ohw = g.oh * g.ow;
    int img = k4 / ohw, rem = k4 - img * ohw;
    int oy = rem / g.ow, ox = rem - oy * g.ow;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float val = 0.0f;
      if (k4 + i < K) {
        const int iy = oy * g.stride - g.pad + kh, ix = ox * g.stride - g.pad + kw;
        if (iy >= 0 && iy < g.h && ix >= 0 && ix < g.w)
          val = __ldg(x + (((size_t)img * g.cin + ci) * g.h + iy) * g.w + ix);
      }
      v[i] = val;
      // next pixel
      if (++ox == g.ow) {
        ox = 0;
        if (++oy == g.oh) {
          oy = 0;
          ++img;
        }
      }
    }
  }

  __device__ __forceinline__ void load_b(int row, int k4, float (&v)[4]) const {
    // B(co, pixel) = dY[img, co, oy, ox]
    const int ohw = g.oh * g.ow;
    if (row >= N) {
      v[0] = v[1] = v[2] = v[3] = 0.0f;
      return;
    }
    if (dy_vec && k4 + 3 < K) {  // ohw % 4 == 0: the 4 pixels share an image
      const int img = k4 / ohw, rem = k4 - img * ohw;
      float4 t = __ldg(reinterpret_cast<const float4*>(dy + ((size_t)img * g.cout + row) * ohw + rem));
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
      return;
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int p = k4 + i;
      float val = 0.0f;
      if (p < K) {
        const int img = p / ohw, rem = p - img * ohw;
        val = __ldg(dy + ((size_t)img * g.cout + row) * ohw + rem);
      }
      v[i] = val;
    }
  }

  __device__ __forceinline__ void store(int row, int col0, int split, const float (&v)[32]) const {
    if (row >= M || col0 >= N) return;
    if (splits > 1) {
      store_row32(ws + ((size_t)split * M + row) * N + col0, N - col0, v, false, (N % 4) == 0);
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++) {
        const int co = col0 + j;
        if (co < N) dw[(size_t)co * M + row] += v[j];
      }
    }
  }
};

// ---------------------------------------------------------------- fast paths
//
// When the contracted channel count is a multiple of 32, fwd and dgrad order
// K tap-major: k = tap * C + c, so one 32-wide K block is one (kh, kw) tap
// over 32 consecutive channels.  A producer thread owns one output row
// (pixel); per K block it resolves the tap's input position and validity
// once and then issues 32 loads strided by one channel plane (each warp load
// covers 32 consecutive pixels).  The weights go through pack_b_kernel into
// the MMA's shared-memory image and are streamed with cp.async.bulk.

template <int KS, int BN>
struct FastConvFwd {
  static constexpr bool B_BULK = true;
  static constexpr bool STATS = true;
  static constexpr int KK = KS * KS;
  const float* x;
  float* y;
  const float* bpack;
  ConvStatsDev st;
  ConvGeom g;
  int M, N;
  int CB;  // channel blocks of 32 per tap
  int kblocks;
  int acc;
  int splits;

  struct TS {
    const float* xb;
    int iy0, ix0;
    bool ok;
  };
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int, int gt) const {
    const int row = m0 + gt;
    ts.ok = row < M;
    const int ohw = g.oh * g.ow;
    const int r = ts.ok ? row : 0;
    const int img = r / ohw, rem = r - img * ohw;
    const int oy = rem / g.ow, ox = rem - oy * g.ow;
    ts.iy0 = oy * g.stride - g.pad;
    ts.ix0 = ox * g.stride - g.pad;
    ts.xb = x + (size_t)img * g.cin * g.h * g.w;
  }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) { r = gt; c = j; }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int, float (&v)[32]) const {
    const int tap = kb / CB, cb = kb - tap * CB;
    const int kh = tap / KS, kw = tap - kh * KS;
    const int iy = ts.iy0 + kh, ix = ts.ix0 + kw;
    const bool valid = ts.ok && iy >= 0 && iy < g.h && ix >= 0 && ix < g.w;
    const int hw = g.h * g.w;
    const float* p = ts.xb + (size_t)(cb * 32) * hw + (valid ? iy * g.w + ix : 0);
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = valid ? __ldg(p + (size_t)j * hw) : 0.0f;
  }
  __device__ __forceinline__ const void* b_src(int nt, int kb) const {
    return bpack + ((size_t)nt * kblocks + kb) * (2 * BN * BK);
  }
  __device__ __forceinline__ void store(int row, int col0, int, const float (&v)[32]) const {
    if (row >= M) return;
    const int ohw = g.oh * g.ow;
    const int img = row / ohw, rem = row - img * ohw;
    store_planes32(y, ((size_t)img * g.cout + col0) * ohw + rem, ohw, N - col0, v, acc);
  }
  __device__ __forceinline__ bool stats_on() const { return st.part != nullptr; }
  __device__ __forceinline__ void stats_flush(const double* sm) const { conv_stats_flush(sm, st, N); }
};

// B(co, k = tap*cin + ci) = W[co][ci][tap]
struct PackFwdSrc {
  const float* w;
  int cout, cin, kk;
  __device__ __forceinline__ float operator()(int co, int k) const {
    const int tap = k / cin, ci = k - tap * cin;
    return (co < cout && tap < kk) ? __ldg(w + ((size_t)co * cin + ci) * kk + tap) : 0.0f;
  }
};

template <int KS, int BN>
struct FastConvDgrad {
  static constexpr bool B_BULK = true;
  static constexpr int KK = KS * KS;
  const float* dy;
  float* dx;
  const float* bpack;
  ConvGeom g;
  int M, N;
  int CB;  // cout blocks of 32 per tap
  int kblocks;
  int acc;
  int splits;

  struct TS {
    const float* dyb;
    int ty0, tx0;  // iy + pad, ix + pad
    bool ok;
  };
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int, int gt) const {
    const int row = m0 + gt;
    ts.ok = row < M;
    const int hw = g.h * g.w;
    const int r = ts.ok ? row : 0;
    const int img = r / hw, rem = r - img * hw;
    const int iy = rem / g.w, ix = rem - iy * g.w;
    ts.ty0 = iy + g.pad;
    ts.tx0 = ix + g.pad;
    ts.dyb = dy + (size_t)img * g.cout * g.oh * g.ow;
  }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) { r = gt; c = j; }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int, float (&v)[32]) const {
    const int tap = kb / CB, cb = kb - tap * CB;
    const int kh = tap / KS, kw = tap - kh * KS;
    const int ty = ts.ty0 - kh, tx = ts.tx0 - kw;
    int oy, ox;
    bool valid = ts.ok && ty >= 0 && tx >= 0;
    if (g.stride == 1) {
      oy = ty; ox = tx;
    } else {
      oy = ty / g.stride; ox = tx / g.stride;
      valid = valid && oy * g.stride == ty && ox * g.stride == tx;
    }
    valid = valid && oy < g.oh && ox < g.ow;
    const int ohw = g.oh * g.ow;
    const float* p = ts.dyb + (size_t)(cb * 32) * ohw + (valid ? oy * g.ow + ox : 0);
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = valid ? __ldg(p + (size_t)j * ohw) : 0.0f;
  }
  __device__ __forceinline__ const void* b_src(int nt, int kb) const {
    return bpack + ((size_t)nt * kblocks + kb) * (2 * BN * BK);
  }
  __device__ __forceinline__ void store(int row, int col0, int, const float (&v)[32]) const {
    if (row >= M) return;
    const int hw = g.h * g.w;
    const int img = row / hw, rem = row - img * hw;
    store_planes32(dx, ((size_t)img * g.cin + col0) * hw + rem, hw, N - col0, v, acc);
  }
};

// dgrad of a 1x1 convolution with stride s > 1 and no padding (the
// projection shortcut): only the input pixels (s*oy, s*ox) receive gradient,
// so the GEMM runs over the n*oh*ow output pixels (rows), reads dY like the
// 1x1 forward reads x, and scatters each row into dX; the other pixels are
// zeroed by the caller (or keep their value when accumulating).
template <int BN>
struct FastDgrad1x1Strided {
  static constexpr bool B_BULK = true;
  const float* dy;
  float* dx;
  const float* bpack;
  ConvGeom g;
  int M, N;
  int kblocks;  // cout / 32
  int acc;
  int splits;

  struct TS {
    const float* p;
    bool ok;
  };
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int, int gt) const {
    const int row = m0 + gt;
    ts.ok = row < M;
    const int ohw = g.oh * g.ow;
    const int r = ts.ok ? row : 0;
    const int img = r / ohw, rem = r - img * ohw;
    ts.p = dy + (size_t)img * g.cout * ohw + rem;
  }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) { r = gt; c = j; }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int, float (&v)[32]) const {
    const size_t ohw = (size_t)g.oh * g.ow;
    const float* p = ts.p + (size_t)(kb * 32) * ohw;
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = ts.ok ? __ldg(p + (size_t)j * ohw) : 0.0f;
  }
  __device__ __forceinline__ const void* b_src(int nt, int kb) const {
    return bpack + ((size_t)nt * kblocks + kb) * (2 * BN * BK);
  }
  __device__ __forceinline__ void store(int row, int col0, int, const float (&v)[32]) const {
    if (row >= M) return;
    const int ohw = g.oh * g.ow, hw = g.h * g.w;
    const int img = row / ohw, rem = row - img * ohw;
    const int oy = rem / g.ow, ox = rem - oy * g.ow;
    store_planes32(dx, ((size_t)img * g.cin + col0) * hw + (size_t)(oy * g.stride) * g.w + ox * g.stride, hw,
                   N - col0, v, acc);
  }
};

// 3x3, stride 1, pad 1 convolution over W = 32 (or 16) pixel-wide images
// whose height is a multiple of 128/W (the 32x32 and 16x16 stages of the
// CIFAR networks), as forward (src = x, out = y) or as dgrad (src = dY,
// out = dX, taps flipped in the packed weights).  A row tile is 128/W whole
// image rows; K is ordered (32-channel block cb, tap, channel), and for each
// cb the producers stage the tile's halo -- 32 channels x (128/W + 2) rows x
// (W + 8) columns (columns -4 .. W+3, so every 16-byte chunk is either
// inside the row or all padding) -- in shared memory with cp.async, then
// build all nine tap-shifted A tiles from it: one global read of the input
// per channel block instead of nine.  At W = 16 a warp reads two image rows
// per load, so halo rows are stored in pairs interleaved by 16-byte chunk
// (row pair, column chunk, row parity, column % 4): the half-warp reading
// an even row and the one reading the odd row use disjoint banks.
constexpr bool HALO_A_TMEM = true;

template <int BN, int W_ = 32>
struct HaloConv3x3 {
  static constexpr bool B_BULK = true;
  static constexpr int TAPS = 9;
  static constexpr int W = W_;
  static_assert(W == 32 || W == 16, "halo widths");
  static constexpr int TR = BM / W;      // image rows per tile
  static constexpr int HR = TR + 2;      // halo rows
  static constexpr int HX = W + 8;       // halo columns (-4 .. W+3)
  static constexpr int HCH = HX / 4;     // 16-byte chunks per halo row
  static constexpr bool PAIRS = W < 32;
  static constexpr int CSTR = PAIRS ? ((HR + 1) / 2) * 2 * HX : HR * HX;  // floats per channel
  static constexpr int HALO_FLOATS = 32 * CSTR;
  static constexpr int HALO_BYTES = 2 * HALO_FLOATS * 4;
  // 32-wide images: a halo buffer is the dense box [32 channels][HR rows][HX
  // columns] of the source, filled by one tensor copy (columns -4 .. W+3 and
  // the rows above and below the image come back as zeros).  16-wide images
  // store rows in interleaved pairs, which a box copy cannot produce: they
  // keep the per-thread cp.async.
  static constexpr bool HALO_TMA = !PAIRS;
  // the producers write the split A tile into tensor memory (tcgen05.st):
  // shared memory then carries only the halo and the B images
  static constexpr bool A_TMEM = HALO_A_TMEM;
  static constexpr bool STATS = true;
  // float offset of halo row r, halo column x (0 .. HX-1) within a channel
  static __device__ __forceinline__ int pos(int r, int x) {
    if constexpr (PAIRS) return (r >> 1) * (2 * HX) + (x >> 2) * 8 + (r & 1) * 4 + (x & 3);
    return r * HX + x;
  }
  CUtensorMap tmap;  // src as [n][CS][H][W], boxes of [32][HR][HX] (HALO_TMA)
  const float* src;  // [n][CS][H][W]
  float* out;        // [n][N][H][W]
  const float* bpack;
  ConvStatsDev st;
  int CS, H;
  int M, N;
  int kblocks;
  int acc;
  int splits;

  struct TS {
    int unused;
  };
  __device__ __forceinline__ void tile_begin(TS&, int, int, int) const {}
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) { r = gt; c = j; }
  __device__ __forceinline__ void halo_issue(uint32_t halo, int buf, int mt, int kbs, int ptid, int npt) const {
    const int cb = kbs / TAPS;  // 32-channel block
    const int hw = H * W;
    const int m0 = mt * BM;
    const int img = m0 / hw, oy0 = (m0 - img * hw) / W;
    const float* base = src + ((size_t)img * CS + cb * 32) * hw;
    const uint32_t dst0 = halo + (uint32_t)(buf * HALO_FLOATS * 4);
    for (int q = ptid; q < 32 * HR * HCH; q += npt) {
      const int c = q / (HR * HCH), rem = q - c * (HR * HCH);
      const int r = rem / HCH, xc = rem - r * HCH;
      const int iy = oy0 - 1 + r, ix = xc * 4 - 4;
      const bool in = iy >= 0 && iy < H && ix >= 0 && ix < W;
      const float* g = in ? base + ((size_t)c * H + iy) * W + ix : src;
      cp_async16(dst0 + (uint32_t)((c * CSTR + pos(r, xc * 4)) * 4), g, in ? 16u : 0u);
    }
  }
  __device__ __forceinline__ void halo_tma(uint32_t halo, int buf, uint64_t* bar, int mt, int kbs) const {
    const int cb = kbs / TAPS;  // 32-channel block
    const int hw = H * W;
    const int m0 = mt * BM;
    const int img = m0 / hw, oy0 = (m0 - img * hw) / W;
    mbar_arrive_expect_tx(bar, (uint32_t)(HALO_FLOATS * 4));
    // x starts at column -4: -16 bytes, a multiple of 16
    tma_load_4d(halo + (uint32_t)(buf * HALO_FLOATS * 4), &tmap, -4, oy0 - 1, cb * 32, img, bar);
  }
  __device__ __forceinline__ void load_a_halo(uint32_t halo, int buf, const TS&, int tap, int gt,
                                              float (&v)[32]) const {
    const int kh = tap / 3, kw = tap - kh * 3;
    const int oyl = gt / W, ox = gt - oyl * W;
    const uint32_t a = halo + (uint32_t)((buf * HALO_FLOATS + pos(oyl + kh, ox + kw + 3)) * 4);
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = ld_shared_f32(a + (uint32_t)(j * CSTR * 4));
  }
  __device__ __forceinline__ const void* b_src(int nt, int kb) const {
    return bpack + ((size_t)nt * kblocks + kb) * (2 * BN * BK);
  }
  __device__ __forceinline__ void store(int row, int col0, int, const float (&v)[32]) const {
    if (row >= M) return;
    const int hw = H * W;
    const int img = row / hw, rem = row - img * hw;
    store_planes32(out, ((size_t)img * N + col0) * hw + rem, hw, N - col0, v, acc);
  }
  __device__ __forceinline__ bool stats_on() const { return st.part != nullptr; }
  __device__ __forceinline__ void stats_flush(const double* sm) const { conv_stats_flush(sm, st, N); }
};

// K = (32-channel block, tap, channel) for the halo kernels.
// forward: B(co, k) = W[co][cb*32 + c][tap]
struct PackHaloFwdSrc {
  const float* w;
  int cout, cin;
  __device__ __forceinline__ float operator()(int co, int k) const {
    const int cb = k / 288, r = k - cb * 288, tap = r >> 5, ci = cb * 32 + (r & 31);
    return (co < cout && ci < cin) ? __ldg(w + ((size_t)co * cin + ci) * 9 + tap) : 0.0f;
  }
};
// dgrad: B(ci, k) = W[cb*32 + c][ci][8 - tap] (the flipped kernel)
struct PackHaloDgradSrc {
  const float* w;
  int cout, cin;
  __device__ __forceinline__ float operator()(int ci, int k) const {
    const int cb = k / 288, r = k - cb * 288, tap = r >> 5, co = cb * 32 + (r & 31);
    return (ci < cin && co < cout) ? __ldg(w + ((size_t)co * cin + ci) * 9 + (8 - tap)) : 0.0f;
  }
};

// B(ci, k = tap*cout + co) = W[co][ci][tap]
struct PackDgradSrc {
  const float* w;
  int cout, cin, kk;
  __device__ __forceinline__ float operator()(int ci, int k) const {
    const int tap = k / cout, co = k - tap * cout;
    return (ci < cin && tap < kk) ? __ldg(w + ((size_t)co * cin + ci) * kk + tap) : 0.0f;
  }
};

// dgrad of a 3x3, stride-2, pad-1 convolution split by input-pixel parity
// (py, px): pixel (2a+py, 2b+px) only receives taps with kh = 1 (py = 0) or
// kh in {0, 2} (py = 1), the same for kw, at dY position (a + (py+1-kh)/2,
// b + (px+1-kw)/2).  One launch per class runs M = n*A*B pixels of the
// class against K = taps(class)*cout (1, 2, 2 and 4 taps): 9 taps in all
// instead of the 36 a stride-blind gather multiplies by zero.
template <int BN>
struct FastDgradS2 {
  static constexpr bool B_BULK = true;
  const float* dy;
  float* dx;
  const float* bpack;
  ConvGeom g;
  int M, N;
  int CB;        // cout blocks of 32 per tap
  int kblocks;   // ntaps * CB
  int acc;
  int splits;
  int py, px, A, B;  // class parity and its rows / columns per image
  int dyo[4], dxo[4];  // per class tap: dY row / column offset (a + dyo, b + dxo)

  struct TS {
    const float* dyb;
    int a, b;
    bool ok;
  };
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int, int gt) const {
    const int row = m0 + gt;
    ts.ok = row < M;
    const int ab = A * B;
    const int r = ts.ok ? row : 0;
    const int img = r / ab, rem = r - img * ab;
    ts.a = rem / B;
    ts.b = rem - ts.a * B;
    ts.dyb = dy + (size_t)img * g.cout * g.oh * g.ow;
  }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) { r = gt; c = j; }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int, float (&v)[32]) const {
    const int t = kb / CB, cb = kb - t * CB;
    const int oy = ts.a + dyo[t], ox = ts.b + dxo[t];
    const bool valid = ts.ok && oy >= 0 && oy < g.oh && ox >= 0 && ox < g.ow;
    const int ohw = g.oh * g.ow;
    const float* p = ts.dyb + (size_t)(cb * 32) * ohw + (valid ? oy * g.ow + ox : 0);
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = valid ? __ldg(p + (size_t)j * ohw) : 0.0f;
  }
  __device__ __forceinline__ const void* b_src(int nt, int kb) const {
    return bpack + ((size_t)nt * kblocks + kb) * (2 * BN * BK);
  }
  __device__ __forceinline__ void store(int row, int col0, int, const float (&v)[32]) const {
    if (row >= M) return;
    const int ab = A * B, hw = g.h * g.w;
    const int img = row / ab, rem = row - img * ab;
    const int a = rem / B, b = rem - a * B;
    store_planes32(dx, ((size_t)img * g.cin + col0) * hw + (size_t)(2 * a + py) * g.w + 2 * b + px, hw, N - col0,
                   v, acc);
  }
};

// B(ci, k = t*cout + co) = W[co][ci][tap[t]] for the class's taps
struct PackDgradS2Src {
  const float* w;
  int cout, cin, ntaps;
  int tap[4];
  __device__ __forceinline__ float operator()(int ci, int k) const {
    const int t = k / cout, co = k - t * cout;
    return (ci < cin && t < ntaps) ? __ldg(w + ((size_t)co * cin + ci) * 9 + tap[t]) : 0.0f;
  }
};

// wgrad: M = (ci, kh, kw) rows, N = cout, K = pixels, when every group of 4
// consecutive pixels lies in one output row (ow % 4 == 0).  A producer
// thread owns 4 consecutive pixels of 8 rows; it decodes the pixel block once
// per K block and the 8 rows once per tile.  dY is read with 16-byte loads.
template <int KS>
struct FastConvWgrad {
  static constexpr bool B_BULK = false;
  static constexpr int KK = KS * KS;
  const float* x;
  const float* dy;
  float* dw;
  float* ws;
  ConvGeom g;
  int M, N, K;
  int splits;

  struct TS {
    int rowoff[8];  // ci*H*W + (kh-pad)*W + (kw-pad)
    int dkh[8], dkw[8];
    uint32_t rok;   // bit j: row j in range
    int n0;
  };
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int n0, int gt) const {
    ts.rok = 0;
    ts.n0 = n0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int row = m0 + (gt >> 3) + 16 * j;
      const int r = row < M ? row : 0;
      const int ci = r / KK, kk = r - ci * KK;
      const int kh = kk / KS, kw = kk - kh * KS;
      ts.dkh[j] = kh - g.pad;
      ts.dkw[j] = kw - g.pad;
      ts.rowoff[j] = ci * g.h * g.w + ts.dkh[j] * g.w + ts.dkw[j];
      if (row < M) ts.rok |= 1u << j;
    }
  }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) {
    r = (gt >> 3) + 16 * j;
    c = gt & 7;
  }
  static __device__ __forceinline__ void b_slot(int gt, int j, int& r, int& c) {
    const int idx = gt + 128 * j;
    r = idx >> 3;
    c = idx & 7;
  }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int gt, float (&v)[32]) const {
    const int p0 = kb * BK + 4 * (gt & 7);
    const int ohw = g.oh * g.ow;
    if (p0 >= K) {
#pragma unroll
      for (int j = 0; j < 32; j++) v[j] = 0.0f;
      return;
    }
    const int img = p0 / ohw, rem = p0 - img * ohw;
    const int oy = rem / g.ow, ox = rem - oy * g.ow;
    const int ys = oy * g.stride, xs = ox * g.stride;
    const float* base = x + (size_t)img * g.cin * g.h * g.w + ys * g.w + xs;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int iy = ys + ts.dkh[j];
      const bool rv = ((ts.rok >> j) & 1u) && iy >= 0 && iy < g.h;
      const float* p = base + (rv ? ts.rowoff[j] : 0);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int ix = xs + i * g.stride + ts.dkw[j];
        const bool ok = rv && ix >= 0 && ix < g.w;
        v[4 * j + i] = ok ? __ldg(p + i * g.stride) : 0.0f;
      }
    }
  }
  template <int NB>
  __device__ __forceinline__ void load_b(const TS& ts, int kb, int gt, float (&v)[NB]) const {
    const int p0 = kb * BK + 4 * (gt & 7);
    const int ohw = g.oh * g.ow;
    const bool pin = p0 < K;
    const int img = pin ? p0 / ohw : 0, rem = pin ? p0 - img * ohw : 0;
    const float* base = dy + ((size_t)img * g.cout) * ohw + rem;
#pragma unroll
    for (int j = 0; j < NB / 4; j++) {
      const int co = ts.n0 + ((gt + 128 * j) >> 3);
      if (pin && co < N) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(base + (size_t)co * ohw));
        v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
      } else {
        v[4 * j] = v[4 * j + 1] = v[4 * j + 2] = v[4 * j + 3] = 0.0f;
      }
    }
  }
  __device__ __forceinline__ const void* b_src(int, int) const { return nullptr; }
  __device__ __forceinline__ void store(int row, int col0, int split, const float (&v)[32]) const {
    if (row >= M || col0 >= N) return;
    if (splits > 1) {
      store_row32(ws + ((size_t)split * M + row) * N + col0, N - col0, v, false, (N % 4) == 0);
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++) {
        const int co = col0 + j;
        if (co < N) dw[(size_t)co * M + row] += v[j];
      }
    }
  }
};

// wgrad with dY pre-packed (B_BULK): pack_b_kernel writes the hi/lo image
// of every (cout tile, 32-pixel K block) of dY once, and the producers only
// gather the im2col operand; the B tile, which every row tile of the
// launch re-reads, then arrives by bulk copy like the weights of fwd/dgrad.
template <int KS, int BN>
struct FastConvWgradPacked : FastConvWgrad<KS> {
  static constexpr bool B_BULK = true;
  const float* bpack;
  int kblocks;
  __device__ __forceinline__ const void* b_src(int nt, int kb) const {
    return bpack + ((size_t)nt * kblocks + kb) * (2 * BN * BK);
  }
};

// Pixels 4q + kw - 1 .. 4q + kw + 2 of an image row whose pixels 4q .. 4q+3
// are m, with `left` = pixel 4q - 1 and `right` = pixel 4q + 4 (zero past
// the row ends): the kw-shifted window of a 3x3 wgrad row.  Selects, not
// branches: the three kw rows of a (ci, kh) sit in adjacent lanes, so a
// branch on kw would run all three paths one after another.
__device__ __forceinline__ void kw_shift4(const float4 m, float left, float right, int kw, float* v) {
  const bool k0 = kw == 0, k2 = kw == 2;
  v[0] = k0 ? left : (k2 ? m.y : m.x);
  v[1] = k0 ? m.x : (k2 ? m.z : m.y);
  v[2] = k0 ? m.y : (k2 ? m.w : m.z);
  v[3] = k0 ? m.z : (k2 ? right : m.w);
}

// wgrad of a 3x3/s1/p1 convolution over W in {8, 16, 32} pixel-wide images
// (W*H a multiple of 32, so a K block is 32/W whole rows of one image) with
// A in tensor memory: a producer thread owns one (ci, kh, kw) row and builds
// its 32 pixels of the K block from eight aligned 16-byte loads of the
// input rows, shifting by kw - 1 across neighbouring chunks (zero at the
// row ends); the three kw rows of a (ci, kh) sit in adjacent lanes and read
// the same addresses.  dY is pre-packed and bulk-copied as B.
template <int BN, int W, bool ATM = true>
struct FastConvWgradT : FastConvWgradPacked<3, BN> {
  // A in tensor memory (ATM) unless the tile's accumulators fill it (BN 256)
  static constexpr bool A_TMEM = ATM;
  static_assert(W == 8 || W == 16 || W == 32, "row widths");
  static constexpr int R = 32 / W;  // image rows per K block
  struct TS {
    const float* xc;  // channel ci's plane of image 0
    int kh, kw;
    bool ok;
  };
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int, int gt) const {
    const int row = m0 + gt;
    ts.ok = row < this->M;
    const int r = ts.ok ? row : 0;
    const int ci = r / 9, kk = r - ci * 9;
    ts.kh = kk / 3;
    ts.kw = kk - ts.kh * 3;
    ts.xc = this->x + (size_t)ci * this->g.h * W;
  }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) { r = gt; c = j; }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int, float (&v)[32]) const {
    const int h = this->g.h, hw = h * W;
    const int p0 = kb * BK;
    const bool pin = ts.ok && p0 < this->K;
    const int pp = pin ? p0 : 0;
    const int img = pp / hw, oy0 = (pp - img * hw) / W;
    const float* base = ts.xc + (size_t)img * this->g.cin * hw;
    float4 c[8];
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const int r = (4 * q) / W, px0 = (4 * q) % W;
      const int iy = oy0 + r + ts.kh - 1;
      c[q] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (pin && iy >= 0 && iy < h) c[q] = __ldg(reinterpret_cast<const float4*>(base + iy * W + px0));
    }
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const int px0 = (4 * q) % W;
      const float left = px0 > 0 ? c[q - (px0 > 0 ? 1 : 0)].w : 0.0f;       // pixel px0 - 1 of the row
      const float right = px0 + 4 < W ? c[q + (px0 + 4 < W ? 1 : 0)].x : 0.0f;  // pixel px0 + 4
      kw_shift4(c[q], left, right, ts.kw, &v[4 * q]);
    }
  }
};

// wgrad of a 3x3/s1/p1 convolution over 32- or 16-wide images with the
// input rows staged by tensor copies.  A K block is R = 32/W image rows;
// K runs in groups of TAPS = 8 K blocks, 8R rows of one image (H a multiple
// of 8R); one 4-D tensor copy per group brings image rows oy0-1 ..
// oy0+8R+1 of the (at most 16) channels a 128-row tile touches into shared
// memory as [16 channels][HROWS rows][W columns] of W*4-byte lines,
// swizzled over the line width (128-byte swizzle at W = 32, 64-byte at
// W = 16), zeros above and below the image and past the last channel.  A
// producer thread owns one (ci, kh, kw) row, as in FastConvWgradT, and
// reads its 32 pixels of a K block as eight 16-byte shared loads, shifting
// by kw - 1 across neighbouring chunks of each image row.  Each input row
// crosses L2 once per group instead of being fetched by every producer warp
// per K block, and the producers no longer wait on global loads.
template <int BN, int W_ = 32>
struct FastConvWgradHalo : FastConvWgradPacked<3, BN> {
  static constexpr bool A_TMEM = true;
  static constexpr int W = W_;
  static_assert(W == 32 || W == 16, "tensor-copy wgrad widths");
  static constexpr int R = 32 / W;            // image rows per K block
  static constexpr int TAPS = 8;              // K blocks per halo group
  static constexpr int LINE = W * 4;          // bytes per image row in a buffer
  static constexpr int CPL = W / 4;           // 16-byte chunks per line
  // Under either swizzle a line's chunks land on the banks that line % 8
  // selects; the lines one load phase reads, (c, kh..kh+2) and
  // (c+1, kh'..kh'+2), are all distinct mod 8 when HROWS % 8 is 3.
  static constexpr int HROWS = (8 * R + 2 + 5) / 8 * 8 + 3;  // rows oy0-1 .. oy0+8R (+ unused)
  static_assert(HROWS >= 8 * R + 2 && HROWS % 8 == 3, "halo rows");
  static constexpr int SWM = W == 32 ? 7 : 3;  // swizzle: chunk ^= (byte offset >> 7) & SWM
  static constexpr int HCH = 16;               // channels a 128-row tile touches, at most
  static constexpr int BUF_BYTES = HCH * HROWS * LINE;
  static_assert(BUF_BYTES % 1024 == 0, "swizzled buffers start on 1024-byte boundaries");
  static constexpr int HALO_BYTES = 2 * BUF_BYTES;
  static constexpr bool HALO_TMA = true;
  CUtensorMap tmap;  // x as [n][cin][H][W], boxes of [16][HROWS][W], swizzled
  struct TS {
    int line;  // line of (channel - first channel of the tile, kh) in a buffer
    int kw;
    bool ok;
  };
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int, int gt) const {
    const int row = m0 + gt;
    ts.ok = row < this->M;
    const int r = ts.ok ? row : m0;
    const int ci = r / 9, kk = r - ci * 9, kh = kk / 3;
    ts.kw = kk - kh * 3;
    ts.line = (ci - m0 / 9) * HROWS + kh;
  }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) { r = gt; c = j; }
  __device__ __forceinline__ void halo_tma(uint32_t halo, int buf, uint64_t* bar, int mt, int kbs) const {
    const int kbi = this->g.h / R;  // K blocks per image
    const int img = kbs / kbi, oy0 = (kbs - img * kbi) * R;
    mbar_arrive_expect_tx(bar, (uint32_t)BUF_BYTES);
    tma_load_4d(halo + (uint32_t)(buf * BUF_BYTES), &tmap, 0, oy0 - 1, (mt * BM) / 9, img, bar);
  }
  __device__ __forceinline__ void load_a_halo(uint32_t halo, int buf, const TS& ts, int tap, int,
                                              float (&v)[32]) const {
    const uint32_t base = halo + (uint32_t)(buf * BUF_BYTES);
    float4 c[8];
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const uint32_t off = (uint32_t)((ts.line + R * tap + q / CPL) * LINE + (q % CPL) * 16);
      c[q] = ld_shared_v4(base + (off ^ (((off >> 7) & SWM) << 4)));
    }
    if (!ts.ok) {
#pragma unroll
      for (int q = 0; q < 8; q++) c[q] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const int cq = q % CPL;  // chunk within its image row
      const float left = cq > 0 ? c[q > 0 ? q - 1 : 0].w : 0.0f;          // pixel 4cq - 1 of the row
      const float right = cq < CPL - 1 ? c[q < 7 ? q + 1 : 7].x : 0.0f;  // pixel 4cq + 4
      kw_shift4(c[q], left, right, ts.kw, &v[4 * q]);
    }
  }
};

// B(co, k = pixel) = dY[img][co][pixel]
struct PackWgradDySrc {
  const float* dy;
  int cout, ohw, K;
  __device__ __forceinline__ float operator()(int co, int p) const {
    if (co >= cout || p >= K) return 0.0f;
    const int img = p / ohw, rem = p - img * ohw;
    return __ldg(dy + ((size_t)img * cout + co) * ohw + rem);
  }
};

// ---------------------------------------------------------------- launch

// Device bytes each conv operand spans (range checks).
struct ConvSpans {
  size_t x, w, y;
};
static inline ConvSpans spans(const ConvGeom& g, int k) {
  return {sizeof(float) * (size_t)g.n * g.cin * g.h * g.w, sizeof(float) * (size_t)g.cout * g.cin * k * k,
          sizeof(float) * (size_t)g.n * g.cout * g.oh * g.ow};
}

template <int BN>
struct ConvLauncher {
  template <class P>
  static int run(rnn_ctx* ctx, P prob, int splits) {
    Sched s = make_sched(prob.M, prob.N, prob.K, BN, splits);
    prob.splits = s.splits;
    return launch<BN>(ctx, prob, s);
  }
};

template <int BN>
struct WgradLauncher {
  template <class P>
  static int run(rnn_ctx* ctx, P prob, int splits) {
    Sched s = make_sched(prob.M, prob.N, prob.K, BN, splits);
    prob.splits = s.splits;
    if (s.splits > 1) {
      RNN_TRY(ensure_ws(ctx, sizeof(float) * (size_t)s.splits * prob.M * prob.N));
      prob.ws = static_cast<float*>(ctx->ws);
      RNN_RANGE(prob.ws, sizeof(float) * (size_t)s.splits * prob.M * prob.N);
    }
    RNN_TRY(launch<BN>(ctx, prob, s));
    if (s.splits > 1)
      RNN_TRY(launch_splitk_reduce(ctx, prob.ws, prob.dw, prob.M, prob.N, s.splits, true, true));
    return RNN_OK;
  }
};

// The packed dY image (B of the wgrad kernels): made here, or handed in by
// the caller (`dy_packed`, written by the BatchNorm backward that produced
// dY) when it has this tile width and one column tile.
template <int BN, class P>
static int wgrad_dy_image(rnn_ctx* ctx, P& p, const ConvGeom& g, int N, int K, const float* dy,
                          const float* dy_packed) {
  p.kblocks = (K + BK - 1) / BK;
  const int n_tiles = (N + BN - 1) / BN;
  const size_t bytes = (size_t)n_tiles * p.kblocks * 2 * BN * BK * sizeof(float);
  if (dy_packed) {
    RNN_RANGE(dy_packed, bytes);
    p.bpack = dy_packed;
    return RNN_OK;
  }
  RNN_TRY(ensure_pack(ctx, bytes));
  p.bpack = static_cast<const float*>(ctx->pack);
  RNN_RANGE(ctx->pack, bytes);
  PackWgradDySrc src{dy, g.cout, g.oh * g.ow, K};
  return launch_pack<BN>(ctx, src, n_tiles, p.kblocks, static_cast<float*>(ctx->pack));
}

template <int KS, int BN>
static int wgrad_packed(rnn_ctx* ctx, const float* x, const float* dy, float* dw, const ConvGeom& g, int M, int N,
                        int K, int splits, const float* dy_packed) {
  FastConvWgradPacked<KS, BN> p;
  p.x = x; p.dy = dy; p.dw = dw; p.ws = nullptr; p.g = g; p.M = M; p.N = N; p.K = K; p.splits = 1;
  RNN_TRY(wgrad_dy_image<BN>(ctx, p, g, N, K, dy, dy_packed));
  return WgradLauncher<BN>::run(ctx, p, splits);
}

template <int BN, int W>
static int wgrad_t(rnn_ctx* ctx, const float* x, const float* dy, float* dw, const ConvGeom& g, int M, int N,
                   int K, int splits, const float* dy_packed) {
  FastConvWgradT<BN, W, (BN <= 128)> p;
  p.x = x; p.dy = dy; p.dw = dw; p.ws = nullptr; p.g = g; p.M = M; p.N = N; p.K = K; p.splits = 1;
  RNN_TRY(wgrad_dy_image<BN>(ctx, p, g, N, K, dy, dy_packed));
  return WgradLauncher<BN>::run(ctx, p, splits);
}

// 32- and 16-wide 3x3 wgrads take the tensor-copy kernel when each split runs at
// least WGRAD_HALO_MIN_KB K blocks (image rows); shorter splits pay more for
// the first halo copy and the group barriers than the row loads cost
// (measured, dY pack included, against FastConvWgradT with the branch-free
// shift: 64 channels at batch 1024, 1,136 blocks per split, 0.678 -> 0.615
// ms; 32 channels at batch 128, 88 blocks, 0.0494 -> 0.0507 ms, so the
// short splits stay on the row loads).  RNN_WGRAD_HALO=0 keeps every call on
// FastConvWgradT, =1 sends every eligible call to the tensor-copy kernel
// (A/B runs).
constexpr int WGRAD_HALO_MIN_KB = 512;
static bool wgrad_halo_on(int kb_per_split) {
  const char* v = getenv("RNN_WGRAD_HALO");
  if (v && v[0]) return v[0] != '0';
  return kb_per_split >= WGRAD_HALO_MIN_KB;
}

// The tensor-copy wgrad (FastConvWgradHalo): every split's K range is a
// whole number of 8-row groups, so the split count from pick_splits is
// rounded to that.
template <int BN, int W>
static int wgrad_halo(rnn_ctx* ctx, const float* x, const float* dy, float* dw, const ConvGeom& g, int M, int N,
                      int K, int splits, const float* dy_packed) {
  using P = FastConvWgradHalo<BN, W>;
  P p;
  p.x = x; p.dy = dy; p.dw = dw; p.ws = nullptr; p.g = g; p.M = M; p.N = N; p.K = K; p.splits = 1;
  RNN_TRY(encode_nchw_map(&p.tmap, x, g.n, g.cin, g.h, P::W, P::W, P::HROWS, P::HCH,
                          W == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B));
  RNN_TRY(wgrad_dy_image<BN>(ctx, p, g, N, K, dy, dy_packed));
  Sched s = make_sched(M, N, K, BN, splits);
  s.kb_per_split = (s.kb_per_split + P::TAPS - 1) / P::TAPS * P::TAPS;
  s.splits = (s.kblocks + s.kb_per_split - 1) / s.kb_per_split;
  s.num_tiles = s.m_tiles * s.n_tiles * s.splits;
  p.splits = s.splits;
  if (s.splits > 1) {
    RNN_TRY(ensure_ws(ctx, sizeof(float) * (size_t)s.splits * M * N));
    p.ws = static_cast<float*>(ctx->ws);
    RNN_RANGE(p.ws, sizeof(float) * (size_t)s.splits * M * N);
  }
  RNN_TRY(launch<BN>(ctx, p, s));
  if (s.splits > 1) RNN_TRY(launch_splitk_reduce(ctx, p.ws, dw, M, N, s.splits, true, true));
  return RNN_OK;
}

template <int W>
static int wgrad_t_bn(rnn_ctx* ctx, int bn, const float* x, const float* dy, float* dw, const ConvGeom& g, int M,
                      int N, int K, int splits, const float* dy_packed) {
  switch (bn) {
    case 32: return wgrad_t<32, W>(ctx, x, dy, dw, g, M, N, K, splits, dy_packed);
    case 64: return wgrad_t<64, W>(ctx, x, dy, dw, g, M, N, K, splits, dy_packed);
    case 128: return wgrad_t<128, W>(ctx, x, dy, dw, g, M, N, K, splits, dy_packed);
    default: return wgrad_t<256, W>(ctx, x, dy, dw, g, M, N, K, splits, dy_packed);
  }
}

// Widest tile the thread-per-row wgrad gather serves.
constexpr int WGRAD_T_MAX_BN = 256;

// Every 3x3 wgrad pre-packs dY (the B operand every row tile re-reads);
// measured at batch 1024 against gathering it per tile: 64ch 1.00 -> 0.91
// ms, 128ch 0.63 -> 0.50, 256ch 0.55 -> 0.35 (pack included).

template <template <int> class L, class P>
static int run_bn(rnn_ctx* ctx, int bn, const P& p, int splits) {
  switch (bn) {
    case 32: return L<32>::run(ctx, p, splits);
    case 64: return L<64>::run(ctx, p, splits);
    case 128: return L<128>::run(ctx, p, splits);
    default: return L<256>::run(ctx, p, splits);
  }
}

static int check_geom(int n, int cin, int h, int w, int cout, int k, int stride, int pad,
                      ConvGeom* g) {
  RNN_REQUIRE(n >= 0 && cin > 0 && h > 0 && w > 0 && cout > 0, "conv: bad shape");
  RNN_REQUIRE(k == 1 || k == 3, "conv: kernel size %d unsupported (1 or 3)", k);
  RNN_REQUIRE(stride >= 1 && pad >= 0, "conv: bad stride/pad");
  g->n = n; g->cin = cin; g->h = h; g->w = w; g->cout = cout; g->stride = stride; g->pad = pad;
  g->oh = (h + 2 * pad - k) / stride + 1;  // nn.rs:148-150
  g->ow = (w + 2 * pad - k) / stride + 1;
  RNN_REQUIRE(g->oh > 0 && g->ow > 0, "conv: empty output");
  RNN_REQUIRE((size_t)n * cin * h * w < (1ull << 31) && (size_t)n * cout * g->oh * g->ow < (1ull << 31),
              "conv: tensor exceeds 2^31 elements");
  return RNN_OK;
}

// Arms the epilogue statistics of a forward problem when they were asked
// for and one column tile covers every channel.
template <class P>
static int setup_stats(rnn_ctx* ctx, P& p, const Sched& s, ConvStats* stats) {
  if (!stats || !stats->sums || s.n_tiles != 1) return RNN_OK;
  const int grid = std::min(s.num_tiles, ctx->num_sms);
  const size_t bytes = (size_t)grid * p.N * 2 * sizeof(double);
  RNN_TRY(ensure_statp(ctx, bytes));
  RNN_RANGE(stats->sums, (size_t)p.N * 2 * sizeof(double));
  p.st.part = static_cast<double*>(ctx->statp);
  p.st.counter = ctx->counters + COUNTER_CONV_STATS;
  p.st.sums = stats->sums;
  const PeerSums* ps = stats->ps;
  p.st.ps = (ps && ps->world > 1 && p.N <= ps->cmax) ? *ps : PeerSums{};
  stats->fused = true;
  stats->reduced = p.st.ps.world > 1;
  return RNN_OK;
}

template <int KS, int BN>
static int fast_fwd(rnn_ctx* ctx, const float* x, const float* wt, float* y, const ConvGeom& g, bool acc,
                    ConvStats* stats) {
  constexpr int KK = KS * KS;
  FastConvFwd<KS, BN> p;
  p.x = x; p.y = y; p.g = g; p.acc = acc ? 1 : 0; p.splits = 1;
  p.M = g.n * g.oh * g.ow; p.N = g.cout;
  p.CB = g.cin / 32;
  p.kblocks = KK * p.CB;
  Sched s = make_sched(p.M, p.N, p.kblocks * BK, BN, 1);
  const size_t bytes = (size_t)s.n_tiles * p.kblocks * 2 * BN * BK * sizeof(float);
  RNN_TRY(ensure_pack(ctx, bytes));
  p.bpack = static_cast<const float*>(ctx->pack);
  RNN_RANGE(ctx->pack, bytes);
  PackFwdSrc src{wt, g.cout, g.cin, KK};
  RNN_TRY(launch_pack<BN>(ctx, src, s.n_tiles, p.kblocks, static_cast<float*>(ctx->pack)));
  RNN_TRY(setup_stats(ctx, p, s, stats));
  return launch<BN>(ctx, p, s);
}

template <int KS, int BN>
static int fast_dgrad(rnn_ctx* ctx, const float* dy, const float* wt, float* dx, const ConvGeom& g, bool acc) {
  constexpr int KK = KS * KS;
  FastConvDgrad<KS, BN> p;
  p.dy = dy; p.dx = dx; p.g = g; p.acc = acc ? 1 : 0; p.splits = 1;
  p.M = g.n * g.h * g.w; p.N = g.cin;
  p.CB = g.cout / 32;
  p.kblocks = KK * p.CB;
  Sched s = make_sched(p.M, p.N, p.kblocks * BK, BN, 1);
  const size_t bytes = (size_t)s.n_tiles * p.kblocks * 2 * BN * BK * sizeof(float);
  RNN_TRY(ensure_pack(ctx, bytes));
  p.bpack = static_cast<const float*>(ctx->pack);
  RNN_RANGE(ctx->pack, bytes);
  PackDgradSrc src{wt, g.cout, g.cin, KK};
  RNN_TRY(launch_pack<BN>(ctx, src, s.n_tiles, p.kblocks, static_cast<float*>(ctx->pack)));
  return launch<BN>(ctx, p, s);
}

// True when the halo kernels cover a 3x3/s1/p1 convolution whose gathered
// operand has cs channels over h x w pixels.
static bool halo_ok(int cs, int h, int w, int k, int stride, int pad, const void* src) {
  return k == 3 && stride == 1 && pad == 1 && (w == 32 || w == 16) && h % (BM / w) == 0 && cs % 32 == 0 &&
         (reinterpret_cast<uintptr_t>(src) & 15) == 0;
}
// Widest tile for 16-pixel-wide images.  The halo leaves room for 2 ring
// stages at BN = 128 and 3 at BN = 64; measured at 128 channels, batch 1024:
// BN = 128 fwd/dgrad 0.405/0.393 ms (0.407/0.405 without the halo), BN = 64
// (two column tiles each rebuilding A) 0.60/0.59 ms.
constexpr int HALO16_MAX_BN = 128;

// fwd (dgrad = false): src = x [n][cin], out = y [n][cout];
// dgrad: src = dY [n][cout], out = dX [n][cin].
template <int BN, int W>
static int halo_conv(rnn_ctx* ctx, const float* src, const float* wt, float* out, const ConvGeom& g, bool dgrad,
                     bool acc, ConvStats* stats) {
  HaloConv3x3<BN, W> p;
  p.src = src; p.out = out;
  p.CS = dgrad ? g.cout : g.cin;
  p.H = g.h;
  if constexpr (HaloConv3x3<BN, W>::HALO_TMA) {
    RNN_TRY(encode_nchw_map(&p.tmap, src, g.n, p.CS, g.h, W, HaloConv3x3<BN, W>::HX, HaloConv3x3<BN, W>::HR, 32));
  } else {
    memset(&p.tmap, 0, sizeof(p.tmap));
  }
  p.M = g.n * g.h * g.w;
  p.N = dgrad ? g.cin : g.cout;
  p.kblocks = 9 * (p.CS / 32);
  p.acc = acc ? 1 : 0;
  p.splits = 1;
  Sched s = make_sched(p.M, p.N, p.kblocks * BK, BN, 1);
  const size_t bytes = (size_t)s.n_tiles * p.kblocks * 2 * BN * BK * sizeof(float);
  RNN_TRY(ensure_pack(ctx, bytes));
  p.bpack = static_cast<const float*>(ctx->pack);
  RNN_RANGE(ctx->pack, bytes);
  if (dgrad) {
    PackHaloDgradSrc ps{wt, g.cout, g.cin};
    RNN_TRY(launch_pack<BN>(ctx, ps, s.n_tiles, p.kblocks, static_cast<float*>(ctx->pack)));
  } else {
    PackHaloFwdSrc ps{wt, g.cout, g.cin};
    RNN_TRY(launch_pack<BN>(ctx, ps, s.n_tiles, p.kblocks, static_cast<float*>(ctx->pack)));
    RNN_TRY(setup_stats(ctx, p, s, stats));
  }
  return launch<BN>(ctx, p, s);
}

static int halo_dispatch(rnn_ctx* ctx, const float* src, const float* wt, float* out, const ConvGeom& g,
                         bool dgrad, bool acc, ConvStats* stats = nullptr) {
  const int N = dgrad ? g.cin : g.cout;
  const int M = g.n * g.h * g.w;
  // 256-wide tiles leave no room for a ring next to the halo buffers
  int bn = pick_bn(N, (M + BM - 1) / BM, ctx->num_sms);
  if (bn > 128) bn = 128;
  if (g.w == 16) {
    if (bn > HALO16_MAX_BN) bn = HALO16_MAX_BN;
    switch (bn) {
      case 32: return halo_conv<32, 16>(ctx, src, wt, out, g, dgrad, acc, stats);
      case 64: return halo_conv<64, 16>(ctx, src, wt, out, g, dgrad, acc, stats);
      default: return halo_conv<128, 16>(ctx, src, wt, out, g, dgrad, acc, stats);
    }
  }
  switch (bn) {
    case 32: return halo_conv<32, 32>(ctx, src, wt, out, g, dgrad, acc, stats);
    case 64: return halo_conv<64, 32>(ctx, src, wt, out, g, dgrad, acc, stats);
    default: return halo_conv<128, 32>(ctx, src, wt, out, g, dgrad, acc, stats);
  }
}

// The four parity classes of a 3x3/s2/p1 dgrad, one launch each; together
// they write every pixel of dX exactly once.
template <int BN>
static int dgrad_s2(rnn_ctx* ctx, const float* dy, const float* wt, float* dx, const ConvGeom& g, bool acc) {
  // the pack buffer is sized once for the widest class (4 taps): growing it
  // between the launches would free memory a queued launch still reads
  const size_t max_bytes = (size_t)((g.cin + BN - 1) / BN) * (4 * (g.cout / 32)) * 2 * BN * BK * sizeof(float);
  RNN_TRY(ensure_pack(ctx, max_bytes));
  for (int cls = 0; cls < 4; cls++) {
    FastDgradS2<BN> p;
    p.dy = dy; p.dx = dx; p.g = g; p.acc = acc ? 1 : 0; p.splits = 1;
    p.py = cls >> 1;
    p.px = cls & 1;
    p.A = (g.h + 1 - p.py) / 2;
    p.B = (g.w + 1 - p.px) / 2;
    if (p.A <= 0 || p.B <= 0) continue;
    // taps of the class: kh = 1 for even rows, {0, 2} for odd rows (same for kw)
    int khs[2], kws[2], nkh = 0, nkw = 0;
    if (p.py == 0) khs[nkh++] = 1; else { khs[nkh++] = 0; khs[nkh++] = 2; }
    if (p.px == 0) kws[nkw++] = 1; else { kws[nkw++] = 0; kws[nkw++] = 2; }
    PackDgradS2Src src{wt, g.cout, g.cin, 0, {0, 0, 0, 0}};
    for (int i = 0; i < nkh; i++)
      for (int j = 0; j < nkw; j++) {
        const int t = src.ntaps++;
        src.tap[t] = khs[i] * 3 + kws[j];
        p.dyo[t] = (p.py + 1 - khs[i]) / 2;  // iy = 2a + py = 2*oy - 1 + kh
        p.dxo[t] = (p.px + 1 - kws[j]) / 2;
      }
    for (int t = src.ntaps; t < 4; t++) { p.dyo[t] = 0; p.dxo[t] = 0; }
    p.M = g.n * p.A * p.B;
    p.N = g.cin;
    p.CB = g.cout / 32;
    p.kblocks = src.ntaps * p.CB;
    Sched s = make_sched(p.M, p.N, p.kblocks * BK, BN, 1);
    const size_t bytes = (size_t)s.n_tiles * p.kblocks * 2 * BN * BK * sizeof(float);
    p.bpack = static_cast<const float*>(ctx->pack);
    RNN_RANGE(ctx->pack, bytes);
    RNN_TRY(launch_pack<BN>(ctx, src, s.n_tiles, p.kblocks, static_cast<float*>(ctx->pack)));
    RNN_TRY(launch<BN>(ctx, p, s));
  }
  return RNN_OK;
}

template <int BN>
static int fast_dgrad_1x1_strided(rnn_ctx* ctx, const float* dy, const float* wt, float* dx, const ConvGeom& g,
                                  bool acc) {
  if (!acc) RNN_CUDA(cudaMemsetAsync(dx, 0, sizeof(float) * (size_t)g.n * g.cin * g.h * g.w, ctx->stream));
  FastDgrad1x1Strided<BN> p;
  p.dy = dy; p.dx = dx; p.g = g; p.acc = acc ? 1 : 0; p.splits = 1;
  p.M = g.n * g.oh * g.ow; p.N = g.cin;
  p.kblocks = g.cout / 32;
  Sched s = make_sched(p.M, p.N, p.kblocks * BK, BN, 1);
  const size_t bytes = (size_t)s.n_tiles * p.kblocks * 2 * BN * BK * sizeof(float);
  RNN_TRY(ensure_pack(ctx, bytes));
  p.bpack = static_cast<const float*>(ctx->pack);
  RNN_RANGE(ctx->pack, bytes);
  PackDgradSrc src{wt, g.cout, g.cin, 1};
  RNN_TRY(launch_pack<BN>(ctx, src, s.n_tiles, p.kblocks, static_cast<float*>(ctx->pack)));
  return launch<BN>(ctx, p, s);
}

int conv_fwd(rnn_ctx* ctx, const float* x, int n, int cin, int h, int w, const float* wt, int cout,
             int k, int stride, int pad, float* y, bool acc, ConvStats* stats) {
  if (stats) stats->fused = stats->reduced = false;
  ConvGeom g;
  RNN_TRY(check_geom(n, cin, h, w, cout, k, stride, pad, &g));
  if (n == 0) return RNN_OK;
  const ConvSpans sp = spans(g, k);
  RNN_RANGE(x, sp.x);
  RNN_RANGE(wt, sp.w);
  RNN_RANGE(y, sp.y);
  const int M = n * g.oh * g.ow, N = cout, K = cin * k * k;
  const int bn = pick_bn(N, (M + BM - 1) / BM, ctx->num_sms);
  auto fill = [&](auto& p) {
    p.x = x; p.w = wt; p.y = y; p.g = g; p.M = M; p.N = N; p.K = K; p.acc = acc ? 1 : 0;
    p.splits = 1;
    p.w_vec = (K % 4 == 0) && ((reinterpret_cast<uintptr_t>(wt) & 15) == 0);
  };
  if (halo_ok(cin, h, w, k, stride, pad, x)) return halo_dispatch(ctx, x, wt, y, g, false, acc, stats);
  if (cin % 32 == 0) {
    switch (bn) {
      case 32:
        return k == 3 ? fast_fwd<3, 32>(ctx, x, wt, y, g, acc, stats) : fast_fwd<1, 32>(ctx, x, wt, y, g, acc, stats);
      case 64:
        return k == 3 ? fast_fwd<3, 64>(ctx, x, wt, y, g, acc, stats) : fast_fwd<1, 64>(ctx, x, wt, y, g, acc, stats);
      case 128:
        return k == 3 ? fast_fwd<3, 128>(ctx, x, wt, y, g, acc, stats)
                      : fast_fwd<1, 128>(ctx, x, wt, y, g, acc, stats);
      default:
        return k == 3 ? fast_fwd<3, 256>(ctx, x, wt, y, g, acc, stats)
                      : fast_fwd<1, 256>(ctx, x, wt, y, g, acc, stats);
    }
  }
  if (k == 3) {
    ConvFwdProb<3> p; fill(p);
    return run_bn<ConvLauncher>(ctx, bn, p, 1);
  }
  ConvFwdProb<1> p; fill(p);
  return run_bn<ConvLauncher>(ctx, bn, p, 1);
}

int conv_dgrad(rnn_ctx* ctx, const float* dy, int n, int cin, int h, int w, const float* wt,
               int cout, int k, int stride, int pad, float* dx, bool acc) {
  ConvGeom g;
  RNN_TRY(check_geom(n, cin, h, w, cout, k, stride, pad, &g));
  if (n == 0) return RNN_OK;
  const ConvSpans sp = spans(g, k);
  RNN_RANGE(dy, sp.y);
  RNN_RANGE(wt, sp.w);
  RNN_RANGE(dx, sp.x);
  const int M = n * h * w, N = cin, K = cout * k * k;
  const int bn = pick_bn(N, (M + BM - 1) / BM, ctx->num_sms);
  auto fill = [&](auto& p) {
    p.dy = dy; p.w = wt; p.dx = dx; p.g = g; p.M = M; p.N = N; p.K = K; p.acc = acc ? 1 : 0;
    p.splits = 1;
  };
  if (cout % 32 == 0 && k == 1 && stride > 1 && pad == 0) {
    // the GEMM covers the n*oh*ow pixels that receive gradient
    switch (pick_bn(N, (n * g.oh * g.ow + BM - 1) / BM, ctx->num_sms)) {
      case 32: return fast_dgrad_1x1_strided<32>(ctx, dy, wt, dx, g, acc);
      case 64: return fast_dgrad_1x1_strided<64>(ctx, dy, wt, dx, g, acc);
      case 128: return fast_dgrad_1x1_strided<128>(ctx, dy, wt, dx, g, acc);
      default: return fast_dgrad_1x1_strided<256>(ctx, dy, wt, dx, g, acc);
    }
  }
  if (halo_ok(cout, h, w, k, stride, pad, dy)) return halo_dispatch(ctx, dy, wt, dx, g, true, acc);
  if (cout % 32 == 0 && k == 3 && stride == 2 && pad == 1) {
    // per parity class M = n*h*w/4: choose the tile width for that
    switch (pick_bn(N, (n * ((h + 1) / 2) * ((w + 1) / 2) + BM - 1) / BM, ctx->num_sms)) {
      case 32: return dgrad_s2<32>(ctx, dy, wt, dx, g, acc);
      case 64: return dgrad_s2<64>(ctx, dy, wt, dx, g, acc);
      case 128: return dgrad_s2<128>(ctx, dy, wt, dx, g, acc);
      default: return dgrad_s2<256>(ctx, dy, wt, dx, g, acc);
    }
  }
  if (cout % 32 == 0) {
    switch (bn) {
      case 32: return k == 3 ? fast_dgrad<3, 32>(ctx, dy, wt, dx, g, acc) : fast_dgrad<1, 32>(ctx, dy, wt, dx, g, acc);
      case 64: return k == 3 ? fast_dgrad<3, 64>(ctx, dy, wt, dx, g, acc) : fast_dgrad<1, 64>(ctx, dy, wt, dx, g, acc);
      case 128:
        return k == 3 ? fast_dgrad<3, 128>(ctx, dy, wt, dx, g, acc) : fast_dgrad<1, 128>(ctx, dy, wt, dx, g, acc);
      default:
        return k == 3 ? fast_dgrad<3, 256>(ctx, dy, wt, dx, g, acc) : fast_dgrad<1, 256>(ctx, dy, wt, dx, g, acc);
    }
  }
  if (k == 3) {
    ConvDgradProb<3> p; fill(p);
    return run_bn<ConvLauncher>(ctx, bn, p, 1);
  }
  ConvDgradProb<1> p; fill(p);
  return run_bn<ConvLauncher>(ctx, bn, p, 1);
}

int wgrad_dy_pack_bn(int n, int cout, int k, int oh, int ow, const void* dy) {
  const int bn = cout <= 32 ? 32 : cout <= 64 ? 64 : cout <= 128 ? 128 : 256;
  const bool packed = k == 3 && ow % 4 == 0 && (reinterpret_cast<uintptr_t>(dy) & 15) == 0;
  return (packed && bn == cout && ((long)n * oh * ow) % BK == 0) ? bn : 0;
}

int conv_wgrad(rnn_ctx* ctx, const float* x, const float* dy, int n, int cin, int h, int w,
               int cout, int k, int stride, int pad, float* dw, int force_splits, const float* dy_packed) {
  ConvGeom g;
  RNN_TRY(check_geom(n, cin, h, w, cout, k, stride, pad, &g));
  if (n == 0) return RNN_OK;
  const ConvSpans sp = spans(g, k);
  RNN_RANGE(x, sp.x);
  RNN_RANGE(dy, sp.y);
  RNN_RANGE(dw, sp.w);
  const int M = cin * k * k, N = cout, K = n * g.oh * g.ow;
  // The im2col operand (A) is the expensive one to gather; each gathered
  // element feeds BN multiply-adds, so use the widest tile that covers cout
  // and let split-K supply the parallelism.
  const int bn = N <= 32 ? 32 : N <= 64 ? 64 : N <= 128 ? 128 : 256;
  const int splits = force_splits > 0 ? force_splits : pick_splits(M, N, K, bn, ctx->num_sms);
  auto fill = [&](auto& p) {
    p.x = x; p.dy = dy; p.dw = dw; p.ws = nullptr; p.g = g; p.M = M; p.N = N; p.K = K;
    p.splits = 1;
    p.dy_vec = ((g.oh * g.ow) % 4 == 0) && ((reinterpret_cast<uintptr_t>(dy) & 15) == 0);
  };
  if (g.ow % 4 == 0 && (reinterpret_cast<uintptr_t>(dy) & 15) == 0) {  // dY read as float4
    auto ffill = [&](auto& p) {
      p.x = x; p.dy = dy; p.dw = dw; p.ws = nullptr; p.g = g; p.M = M; p.N = N; p.K = K; p.splits = 1;
    };
    // thread-per-row gather: 3x3/s1/p1 over 8/16/32-wide rows, whole-row K
    // blocks; A in tensor memory up to 128-wide tiles (256-wide tiles'
    // accumulators fill it, they keep A in shared memory)
    if (k == 3 && stride == 1 && pad == 1 && (h * w) % 32 == 0 && bn <= WGRAD_T_MAX_BN &&
        (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
      // tensor-copy staging: groups of 8 K blocks (8 * 32/w rows) within one image
      if ((w == 32 || w == 16) && h % (8 * (32 / w)) == 0 && bn <= 128 &&
          wgrad_halo_on(make_sched(M, N, K, bn, splits).kb_per_split)) {
        if (w == 32) {
          switch (bn) {
            case 32: return wgrad_halo<32, 32>(ctx, x, dy, dw, g, M, N, K, splits, dy_packed);
            case 64: return wgrad_halo<64, 32>(ctx, x, dy, dw, g, M, N, K, splits, dy_packed);
            default: return wgrad_halo<128, 32>(ctx, x, dy, dw, g, M, N, K, splits, dy_packed);
          }
        }
        switch (bn) {
          case 32: return wgrad_halo<32, 16>(ctx, x, dy, dw, g, M, N, K, splits, dy_packed);
          case 64: return wgrad_halo<64, 16>(ctx, x, dy, dw, g, M, N, K, splits, dy_packed);
          default: return wgrad_halo<128, 16>(ctx, x, dy, dw, g, M, N, K, splits, dy_packed);
        }
      }
      if (w == 32) return wgrad_t_bn<32>(ctx, bn, x, dy, dw, g, M, N, K, splits, dy_packed);
      if (w == 16) return wgrad_t_bn<16>(ctx, bn, x, dy, dw, g, M, N, K, splits, dy_packed);
      if (w == 8) return wgrad_t_bn<8>(ctx, bn, x, dy, dw, g, M, N, K, splits, dy_packed);
    }
    if (k == 3) {  // other 3x3 shapes (stride 2, other widths): 4 pixels x 8 rows per thread, dY packed
      switch (bn) {
        case 32: return wgrad_packed<3, 32>(ctx, x, dy, dw, g, M, N, K, splits, dy_packed);
        case 64: return wgrad_packed<3, 64>(ctx, x, dy, dw, g, M, N, K, splits, dy_packed);
        case 128: return wgrad_packed<3, 128>(ctx, x, dy, dw, g, M, N, K, splits, dy_packed);
        default: return wgrad_packed<3, 256>(ctx, x, dy, dw, g, M, N, K, splits, dy_packed);
      }
    }
    FastConvWgrad<1> p; ffill(p);
    return run_bn<WgradLauncher>(ctx, bn, p, splits);
  }
  if (k == 3) {
    ConvWgradProb<3> p; fill(p);
    return run_bn<WgradLauncher>(ctx, bn, p, splits);
  }
  ConvWgradProb<1> p; fill(p);
  return run_bn<WgradLauncher>(ctx, bn, p, splits);
}

}  // namespace tc
}  // namespace rnn

using namespace rnn;

extern "C" int rnn_conv2d_fwd_dev(rnn_ctx* ctx, const float* x, int n, int cin, int h, int w,
                                  const float* wt, int cout, int k, int stride, int pad, float* y,
                                  int acc) {
  RNN_REQUIRE(ctx && x && wt && y, "conv2d_fwd: null argument");
  return tc::conv_fwd(ctx, x, n, cin, h, w, wt, cout, k, stride, pad, y, acc != 0);
}

extern "C" int rnn_conv2d_dgrad_dev(rnn_ctx* ctx, const float* dy, int n, int cin, int h, int w,
                                    const float* wt, int cout, int k, int stride, int pad,
                                    float* dx, int acc) {
  RNN_REQUIRE(ctx && dy && wt && dx, "conv2d_dgrad: null argument");
  return tc::conv_dgrad(ctx, dy, n, cin, h, w, wt, cout, k, stride, pad, dx, acc != 0);
}

extern "C" int rnn_conv2d_wgrad_dev(rnn_ctx* ctx, const float* x, const float* dy, int n, int cin,
                                    int h, int w, int cout, int k, int stride, int pad, float* dw) {
  RNN_REQUIRE(ctx && x && dy && dw, "conv2d_wgrad: null argument");
  return tc::conv_wgrad(ctx, x, dy, n, cin, h, w, cout, k, stride, pad, dw, 0);
}
