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
#include "tc_launch.cuh"

namespace rnn {
namespace tc {

struct ConvGeom {
  int n, cin, h, w, cout, stride, pad, oh, ow;
};

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

int conv_fwd(rnn_ctx* ctx, const float* x, int n, int cin, int h, int w, const float* wt, int cout,
             int k, int stride, int pad, float* y, bool acc) {
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
  if (k == 3) {
    ConvDgradProb<3> p; fill(p);
    return run_bn<ConvLauncher>(ctx, bn, p, 1);
  }
  ConvDgradProb<1> p; fill(p);
  return run_bn<ConvLauncher>(ctx, bn, p, 1);
}

int conv_wgrad(rnn_ctx* ctx, const float* x, const float* dy, int n, int cin, int h, int w,
               int cout, int k, int stride, int pad, float* dw, int force_splits) {
  ConvGeom g;
  RNN_TRY(check_geom(n, cin, h, w, cout, k, stride, pad, &g));
  if (n == 0) return RNN_OK;
  const ConvSpans sp = spans(g, k);
  RNN_RANGE(x, sp.x);
  RNN_RANGE(dy, sp.y);
  RNN_RANGE(dw, sp.w);
  const int M = cin * k * k, N = cout, K = n * g.oh * g.ow;
  const int bn = pick_bn(N, (M + BM - 1) / BM, ctx->num_sms);
  const int splits = force_splits > 0 ? force_splits : pick_splits(M, N, K, bn, ctx->num_sms);
  auto fill = [&](auto& p) {
    p.x = x; p.dy = dy; p.dw = dw; p.ws = nullptr; p.g = g; p.M = M; p.N = N; p.K = K;
    p.splits = 1;
    p.dy_vec = ((g.oh * g.ow) % 4 == 0) && ((reinterpret_cast<uintptr_t>(dy) & 15) == 0);
  };
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
