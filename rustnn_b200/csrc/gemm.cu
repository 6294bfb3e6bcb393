// Dense GEMM entry points on the tcgen05 3xTF32 engine.
//
//   rnn_gemm_dev     C (+)= op(A) op(B)           gemm.rs:434 matmul / :500 gemm_small
//   rnn_gemm_dw_dev  C  += A^T B  (split over K)  gemm.rs:555 matmul_dw
//
// Operand A rows are the M index and operand B rows the N index of the
// engine; K-contiguous operands use the K-major producer mapping (lanes walk
// K, 16-byte loads when K is a multiple of 4), M/N-contiguous operands the
// MN-major mapping (lanes walk rows, each warp load covers 32 consecutive
// floats).
#include "tc_launch.cuh"

namespace rnn {
namespace tc {

template <bool AT, bool BT>
struct DenseProb {
  static constexpr bool A_KMAJOR = !AT;  // A [m x k] row-major: K contiguous
  static constexpr bool B_KMAJOR = BT;   // B [n x k] row-major: K contiguous
  const float* a;
  const float* b;
  float* c;
  float* ws;  // split-K partials [splits][M][N] (splits > 1)
  int M, N, K;
  int acc;
  int splits;
  bool a_vec, b_vec, c_vec;

  __device__ __forceinline__ void load_a(int row, int k4, float (&v)[4]) const {
    if (!AT) {
      if (row < M && a_vec && k4 + 3 < K) {
        float4 t = __ldg(reinterpret_cast<const float4*>(a + (size_t)row * K + k4));
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; i++)
          v[i] = (row < M && k4 + i < K) ? __ldg(a + (size_t)row * K + k4 + i) : 0.0f;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; i++)
        v[i] = (row < M && k4 + i < K) ? __ldg(a + (size_t)(k4 + i) * M + row) : 0.0f;
    }
  }

  __device__ __forceinline__ void load_b(int row, int k4, float (&v)[4]) const {
    if (BT) {
      if (row < N && b_vec && k4 + 3 < K) {
        float4 t = __ldg(reinterpret_cast<const float4*>(b + (size_t)row * K + k4));
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; i++)
          v[i] = (row < N && k4 + i < K) ? __ldg(b + (size_t)row * K + k4 + i) : 0.0f;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; i++)
        v[i] = (row < N && k4 + i < K) ? __ldg(b + (size_t)(k4 + i) * N + row) : 0.0f;
    }
  }

  __device__ __forceinline__ void store(int row, int col0, int split, const float (&v)[32]) const {
    if (row >= M || col0 >= N) return;
    const int nvalid = N - col0;
    if (splits > 1) {
      store_row32(ws + ((size_t)split * M + row) * N + col0, nvalid, v, false, c_vec);
    } else {
      store_row32(c + (size_t)row * N + col0, nvalid, v, acc != 0, c_vec);
    }
  }
};

// DenseProb on the engine's native interface.  K-major operands keep the
// per-chunk mapping (8 threads per row, 16-byte loads along K).  An
// M/N-contiguous operand (A with at, B without bt) is gathered in 4 x 4
// blocks: a thread loads 4 consecutive rows at each of 4 consecutive K with
// one 16-byte load per K (a warp covers 512 contiguous bytes) and transposes
// the block in registers into the 4 rows' K chunks, instead of 16 scalar
// loads.  For A the thread owns rows 4*(gt % 32) .. +3 in chunks
// 2*(gt / 32) and +1; for B (tiles of 64 columns and more) block
// gt + 128*t covers rows 4*(b % (BN/4)) .. +3 in chunk b / (BN/4).  Ragged
// or unaligned operands fall back to bounds-checked scalar loads.
template <bool AT, bool BT, int BN>
struct DenseNative : DenseProb<AT, BT> {
  using Base = DenseProb<AT, BT>;
  static constexpr bool B_BULK = false;
  static constexpr bool B_BLOCKS = !BT && BN >= 64;
  struct TS {
    int m0, n0;
  };
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int n0, int) const {
    ts.m0 = m0;
    ts.n0 = n0;
  }
  // A thread's 4-row block is stored one row per step, rotated by
  // (block / 2) % 4: across a warp the rows of one step then differ in row % 8
  // (8 values), so the 16-byte stores hit all eight positions of the
  // 128-byte swizzle row (the minimum of four wavefronts per warp store).
  static __device__ __forceinline__ int rot(int rb) { return (rb >> 1) & 3; }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) {
    if (!AT) { r = (gt >> 3) + 16 * j; c = gt & 7; }
    else {
      const int rb = gt & 31;
      r = 4 * rb + (((j & 3) + rot(rb)) & 3);
      c = 2 * (gt >> 5) + (j >> 2);
    }
  }
  static __device__ __forceinline__ void b_slot(int gt, int j, int& r, int& c) {
    if (BT) {
      const int idx = gt + 128 * j;
      r = idx >> 3; c = idx & 7;
    } else if (B_BLOCKS) {
      const int b = gt + 128 * (j >> 2), rb = b % (BN / 4);
      r = 4 * rb + (((j & 3) + rot(rb)) & 3);
      c = b / (BN / 4);
    } else {
      const int idx = gt + 128 * j;
      r = idx % BN; c = idx / BN;
    }
  }
  // rows r0..r0+3 of an operand stored [K][rows] (row index contiguous), at
  // K values k0..k0+3, in slot order: out[4*jj + kk] = X[k0 + kk][r0 + ((jj + s) & 3)]
  // (each loaded float4 rotated by s with two conditional swaps)
  static __device__ __forceinline__ void block4(const float* __restrict__ x, int rows, int K, int r0, int k0,
                                                bool vec, int s, float* __restrict__ out) {
    const bool full = vec && r0 + 3 < rows && k0 + 3 < K;
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      float a, b, c, d;
      if (full) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(x + (size_t)(k0 + kk) * rows + r0));
        a = t.x; b = t.y; c = t.z; d = t.w;
      } else {
        const bool kin = k0 + kk < K;
        const float* row = x + (size_t)(k0 + kk) * rows + r0;
        a = kin && r0 < rows ? __ldg(row) : 0.0f;
        b = kin && r0 + 1 < rows ? __ldg(row + 1) : 0.0f;
        c = kin && r0 + 2 < rows ? __ldg(row + 2) : 0.0f;
        d = kin && r0 + 3 < rows ? __ldg(row + 3) : 0.0f;
      }
      if (s & 2) {
        const float t0 = a, t1 = b;
        a = c; b = d; c = t0; d = t1;
      }
      if (s & 1) {
        const float t0 = a;
        a = b; b = c; c = d; d = t0;
      }
      out[kk] = a; out[4 + kk] = b; out[8 + kk] = c; out[12 + kk] = d;
    }
  }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int gt, float (&v)[32]) const {
    if constexpr (!AT) {
#pragma unroll
      for (int j = 0; j < 8; j++) {
        int r, c;
        a_slot(gt, j, r, c);
        float t[4];
        Base::load_a(ts.m0 + r, kb * BK + 4 * c, t);
        v[4 * j] = t[0]; v[4 * j + 1] = t[1]; v[4 * j + 2] = t[2]; v[4 * j + 3] = t[3];
      }
    } else {
#pragma unroll
      for (int jc = 0; jc < 2; jc++)
        block4(this->a, this->M, this->K, ts.m0 + 4 * (gt & 31), kb * BK + 4 * (2 * (gt >> 5) + jc), this->a_vec,
               rot(gt & 31), v + 16 * jc);
    }
  }
  template <int NB>
  __device__ __forceinline__ void load_b(const TS& ts, int kb, int gt, float (&v)[NB]) const {
    if constexpr (B_BLOCKS) {
#pragma unroll
      for (int t = 0; t < NB / 16; t++) {
        const int b = gt + 128 * t;
        block4(this->b, this->N, this->K, ts.n0 + 4 * (b % (BN / 4)), kb * BK + 4 * (b / (BN / 4)), this->b_vec,
               rot(b % (BN / 4)), v + 16 * t);
      }
    } else {
#pragma unroll
      for (int j = 0; j < NB / 4; j++) {
        int r, c;
        b_slot(gt, j, r, c);
        float t[4];
        Base::load_b(ts.n0 + r, kb * BK + 4 * c, t);
        v[4 * j] = t[0]; v[4 * j + 1] = t[1]; v[4 * j + 2] = t[2]; v[4 * j + 3] = t[3];
      }
    }
  }
  __device__ __forceinline__ const void* b_src(int, int) const { return nullptr; }
};

template <int BN, bool AT, bool BT>
static DenseNative<AT, BT, BN> native(const DenseProb<AT, BT>& p) {
  DenseNative<AT, BT, BN> n;
  static_cast<DenseProb<AT, BT>&>(n) = p;
  return n;
}

template <int BN>
struct DenseLauncher {
  template <class P>
  static int run(rnn_ctx* ctx, P prob, int splits) {
    Sched s = make_sched(prob.M, prob.N, prob.K, BN, splits);
    prob.splits = s.splits;
    if (s.splits > 1) {
      RNN_TRY(ensure_ws(ctx, sizeof(float) * (size_t)s.splits * prob.M * prob.N));
      prob.ws = static_cast<float*>(ctx->ws);
      RNN_RANGE(prob.ws, sizeof(float) * (size_t)s.splits * prob.M * prob.N);
    }
    RNN_RANGE(prob.a, sizeof(float) * (size_t)prob.M * prob.K);
    RNN_RANGE(prob.b, sizeof(float) * (size_t)prob.N * prob.K);
    RNN_RANGE(prob.c, sizeof(float) * (size_t)prob.M * prob.N);
    RNN_TRY(launch<BN>(ctx, native<BN>(prob), s));
    if (s.splits > 1)
      RNN_TRY(launch_splitk_reduce(ctx, prob.ws, prob.c, prob.M, prob.N, s.splits, prob.acc != 0,
                                   false));
    return RNN_OK;
  }
};

static inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <bool AT, bool BT>
static int gemm_typed(rnn_ctx* ctx, int m, int n, int k, const float* a, const float* b, float* c,
                      bool acc, bool force_split) {
  DenseProb<AT, BT> p;
  p.a = a; p.b = b; p.c = c; p.ws = nullptr;
  p.M = m; p.N = n; p.K = k; p.acc = acc ? 1 : 0; p.splits = 1;
  // 16-byte loads: along K for a K-major operand, along the rows for an
  // M/N-contiguous one (DenseNative's 4 x 4 blocks)
  p.a_vec = (AT ? m % 4 == 0 : k % 4 == 0) && al16(a);
  p.b_vec = (BT ? k % 4 == 0 : n % 4 == 0) && al16(b);
  p.c_vec = (n % 4 == 0) && al16(c);
  const int m_tiles = (m + BM - 1) / BM;
  int bn = pick_bn(n, m_tiles, ctx->num_sms);
  // Few output tiles and a long K (the weight-gradient shapes: M x N a few
  // hundred squared, K the token count): the SMs are filled by splitting K
  // anyway, so narrow tiles only multiply the re-reads of the A strips (one
  // per column tile) and issue narrower MMAs.  Take 128-column tiles there:
  // rustvit qkv dW (768 x 256 x 16384) 112 -> 53 us, step 12.53 -> 12.03 ms.
  if (bn < 128 && n >= 64 && pick_splits(m, n, k, bn, ctx->num_sms) > 1 && (long)m * n * k >= (1L << 22))
    bn = n >= 128 ? 128 : 64;
  if (AT && !BT) {  // the matmul_dw layout: RNN_DW_BN=32|64|128|256 forces the tile width (A/B runs)
    const char* e = getenv("RNN_DW_BN");
    const int f = e ? atoi(e) : 0;
    if (f == 32 || f == 64 || f == 128 || f == 256) bn = f;
  }
  int splits = pick_splits(m, n, k, bn, ctx->num_sms);
  if (!force_split && splits > 1 && (long)m * n * k < (1L << 22)) splits = 1;
  switch (bn) {
    case 32: return DenseLauncher<32>::run(ctx, p, splits);
    case 64: return DenseLauncher<64>::run(ctx, p, splits);
    case 128: return DenseLauncher<128>::run(ctx, p, splits);
    default: return DenseLauncher<256>::run(ctx, p, splits);
  }
}

// A batch of same-shape GEMMs in one launch: C_i (+)= op(A_i) op(B_i) for
// i < batch, the operands of item i at a + i*sa, b + i*sb, c + i*sc.  The
// M dimension of the schedule stacks the items, each padded to whole
// 128-row tiles (mp rows), so a tile never spans two items; the tile's item
// selects the A and B operands and the C block.  No split over K: the items
// fill the SMs.
template <bool AT, bool BT, int BN>
struct BatchedDenseProb {
  static constexpr bool A_KMAJOR = !AT;
  static constexpr bool B_KMAJOR = BT;
  static constexpr bool B_BULK = false;
  const float* a;
  const float* b;
  float* c;
  size_t sa, sb, sc;
  int M, N, K, mp;
  int acc;
  bool a_vec, b_vec, c_vec;

  struct TS {
    int item, m0, n0;
  };
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int n0, int) const {
    ts.item = m0 / mp;
    ts.m0 = m0 - ts.item * mp;
    ts.n0 = n0;
  }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) {
    if (A_KMAJOR) { r = (gt >> 3) + 16 * j; c = gt & 7; }
    else { r = gt; c = j; }
  }
  static __device__ __forceinline__ void b_slot(int gt, int j, int& r, int& c) {
    const int idx = gt + 128 * j;
    if (B_KMAJOR) { r = idx >> 3; c = idx & 7; }
    else { r = idx % BN; c = idx / BN; }
  }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int gt, float (&v)[32]) const {
    const float* ai = a + (size_t)ts.item * sa;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      int r, cc;
      a_slot(gt, j, r, cc);
      const int row = ts.m0 + r, k4 = kb * BK + 4 * cc;
      if (!AT && row < M && a_vec && k4 + 3 < K) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(ai + (size_t)row * K + k4));
        v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; i++)
          v[4 * j + i] = (row < M && k4 + i < K)
                             ? __ldg(AT ? ai + (size_t)(k4 + i) * M + row : ai + (size_t)row * K + k4 + i)
                             : 0.0f;
      }
    }
  }
  template <int NB>
  __device__ __forceinline__ void load_b(const TS& ts, int kb, int gt, float (&v)[NB]) const {
    const float* bi = b + (size_t)ts.item * sb;
#pragma unroll
    for (int j = 0; j < NB / 4; j++) {
      int r, cc;
      b_slot(gt, j, r, cc);
      const int row = ts.n0 + r, k4 = kb * BK + 4 * cc;
      if (BT && row < N && b_vec && k4 + 3 < K) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(bi + (size_t)row * K + k4));
        v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; i++)
          v[4 * j + i] = (row < N && k4 + i < K)
                             ? __ldg(BT ? bi + (size_t)row * K + k4 + i : bi + (size_t)(k4 + i) * N + row)
                             : 0.0f;
      }
    }
  }
  __device__ __forceinline__ const void* b_src(int, int) const { return nullptr; }
  __device__ __forceinline__ void store(int row, int col0, int, const float (&v)[32]) const {
    const int item = row / mp, r = row - item * mp;
    if (r >= M || col0 >= N) return;
    store_row32(c + (size_t)item * sc + (size_t)r * N + col0, N - col0, v, acc != 0, c_vec);
  }
};

template <int BN, bool AT, bool BT>
static int gemm_batched_bn(rnn_ctx* ctx, int batch, int m, int n, int k, const float* a, size_t sa, const float* b,
                           size_t sb, float* c, size_t sc, bool acc) {
  BatchedDenseProb<AT, BT, BN> p;
  p.a = a; p.b = b; p.c = c;
  p.sa = sa; p.sb = sb; p.sc = sc;
  p.M = m; p.N = n; p.K = k;
  const int m_tiles = (m + BM - 1) / BM;
  p.mp = m_tiles * BM;
  p.acc = acc ? 1 : 0;
  p.a_vec = (k % 4 == 0) && al16(a) && sa % 4 == 0;
  p.b_vec = (k % 4 == 0) && al16(b) && sb % 4 == 0;
  p.c_vec = (n % 4 == 0) && al16(c) && sc % 4 == 0;
  const Sched s = make_sched(batch * p.mp, n, k, BN, 1);
  return launch_native<BN>(ctx, p, s);
}

template <bool AT, bool BT>
static int gemm_batched_typed(rnn_ctx* ctx, int batch, int m, int n, int k, const float* a, size_t sa,
                              const float* b, size_t sb, float* c, size_t sc, bool acc) {
  const int bn = pick_bn(n, batch * ((m + BM - 1) / BM), ctx->num_sms);
  switch (bn) {
    case 32: return gemm_batched_bn<32, AT, BT>(ctx, batch, m, n, k, a, sa, b, sb, c, sc, acc);
    case 64: return gemm_batched_bn<64, AT, BT>(ctx, batch, m, n, k, a, sa, b, sb, c, sc, acc);
    case 128: return gemm_batched_bn<128, AT, BT>(ctx, batch, m, n, k, a, sa, b, sb, c, sc, acc);
    default: return gemm_batched_bn<256, AT, BT>(ctx, batch, m, n, k, a, sa, b, sb, c, sc, acc);
  }
}

int gemm_batched_dev(rnn_ctx* ctx, int batch, int m, int n, int k, const float* a, size_t sa, bool at,
                     const float* b, size_t sb, bool bt, float* c, size_t sc, bool acc) {
  RNN_REQUIRE(batch >= 0 && m >= 0 && n >= 0 && k > 0, "gemm_batched: bad size batch=%d m=%d n=%d k=%d", batch, m,
              n, k);
  if (batch == 0 || m == 0 || n == 0) return RNN_OK;
  RNN_REQUIRE(a && b && c, "gemm_batched: null operand");
  RNN_REQUIRE(sa >= (size_t)m * k && sb >= (size_t)n * k && sc >= (size_t)m * n,
              "gemm_batched: item strides overlap");
  RNN_RANGE(a, sizeof(float) * ((size_t)(batch - 1) * sa + (size_t)m * k));
  RNN_RANGE(b, sizeof(float) * ((size_t)(batch - 1) * sb + (size_t)n * k));
  RNN_RANGE(c, sizeof(float) * ((size_t)(batch - 1) * sc + (size_t)m * n));
  if (!at && !bt) return gemm_batched_typed<false, false>(ctx, batch, m, n, k, a, sa, b, sb, c, sc, acc);
  if (!at && bt) return gemm_batched_typed<false, true>(ctx, batch, m, n, k, a, sa, b, sb, c, sc, acc);
  if (at && !bt) return gemm_batched_typed<true, false>(ctx, batch, m, n, k, a, sa, b, sb, c, sc, acc);
  return gemm_batched_typed<true, true>(ctx, batch, m, n, k, a, sa, b, sb, c, sc, acc);
}

__global__ void zero_kernel(float* c, size_t len) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (; i < len; i += stride) c[i] = 0.0f;
}

int gemm_dev(rnn_ctx* ctx, int m, int n, int k, const float* a, bool at, const float* b, bool bt,
             float* c, bool acc, bool force_split) {
  RNN_REQUIRE(m >= 0 && n >= 0 && k >= 0, "gemm: negative size m=%d n=%d k=%d", m, n, k);
  if (m == 0 || n == 0) return RNN_OK;
  RNN_REQUIRE(c != nullptr, "gemm: null C");
  if (k == 0) {  // gemm.rs:449-453
    if (!acc) {
      size_t len = (size_t)m * n;
      RNN_RANGE(c, len * sizeof(float));
      zero_kernel<<<(unsigned)std::min<size_t>((len + 255) / 256, 4096), 256, 0, ctx->stream>>>(c, len);
      RNN_CHECK_LAUNCH();
    }
    return RNN_OK;
  }
  RNN_REQUIRE(a != nullptr && b != nullptr, "gemm: null operand");
  if (!at && !bt) return gemm_typed<false, false>(ctx, m, n, k, a, b, c, acc, force_split);
  if (!at && bt) return gemm_typed<false, true>(ctx, m, n, k, a, b, c, acc, force_split);
  if (at && !bt) return gemm_typed<true, false>(ctx, m, n, k, a, b, c, acc, force_split);
  return gemm_typed<true, true>(ctx, m, n, k, a, b, c, acc, force_split);
}

// ---------------------------------------------------------------- split-K

__global__ void splitk_reduce_kernel(const float* __restrict__ ws, float* __restrict__ out, int rows,
                                     int cols, int splits, int acc, int transpose) {
  const size_t total = (size_t)rows * cols;
  const size_t plane = total;
  if (!transpose) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
      float s = 0.0f;
      for (int p = 0; p < splits; p++) s += ws[p * plane + i];
      out[i] = acc ? out[i] + s : s;
    }
  } else {
    // 32x32 tiles through shared memory so that both the partial reads
    // (row-major [rows][cols]) and the transposed writes are coalesced.
    __shared__ float tile[32][33];
    const int tr = (rows + 31) / 32, tcn = (cols + 31) / 32;
    for (int t = blockIdx.x; t < tr * tcn; t += gridDim.x) {
      const int r0 = (t % tr) * 32, c0 = (t / tr) * 32;
      // each of the 256 threads sums 4 elements of the tile together, so
      // 4 (x 4 unrolled) independent partial loads are in flight at once;
      // every element still adds its splits in order 0, 1, ...
      float s[4];
      size_t off[4];
      bool in[4];
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const int e = threadIdx.x + q * 256;
        const int r = r0 + e / 32, c = c0 + e % 32;
        in[q] = r < rows && c < cols;
        off[q] = in[q] ? (size_t)r * cols + c : 0;
        s[q] = 0.0f;
      }
#pragma unroll 4
      for (int p = 0; p < splits; p++)
#pragma unroll
        for (int q = 0; q < 4; q++) s[q] += in[q] ? ws[p * plane + off[q]] : 0.0f;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const int e = threadIdx.x + q * 256;
        tile[e / 32][e % 32] = s[q];
      }
      __syncthreads();
      for (int e = threadIdx.x; e < 1024; e += blockDim.x) {
        const int cc = e / 32, rr = e % 32;
        const int r = r0 + rr, c = c0 + cc;
        if (r < rows && c < cols) {
          float* o = out + (size_t)c * rows + r;
          *o = acc ? *o + tile[rr][cc] : tile[rr][cc];
        }
      }
      __syncthreads();
    }
  }
}

// Row-major form over float4 groups (total % 4 == 0, 16-byte aligned): the
// partials of four splits are loaded together and then added in split order,
// so every element gets the same sum as in the scalar form.
__global__ void splitk_reduce4_kernel(const float4* __restrict__ ws, float4* __restrict__ out, size_t total4,
                                      int splits, int acc) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total4; i += (size_t)gridDim.x * blockDim.x) {
    float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    int p = 0;
    for (; p + 4 <= splits; p += 4) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; u++) v[u] = __ldg(ws + (size_t)(p + u) * total4 + i);
#pragma unroll
      for (int u = 0; u < 4; u++) {
        s.x += v[u].x;
        s.y += v[u].y;
        s.z += v[u].z;
        s.w += v[u].w;
      }
    }
    for (; p < splits; p++) {
      const float4 v = __ldg(ws + (size_t)p * total4 + i);
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    if (acc) {
      const float4 o = out[i];
      s = make_float4(o.x + s.x, o.y + s.y, o.z + s.z, o.w + s.w);
    }
    out[i] = s;
  }
}

// Transposed form for many splits (the convolution weight gradients: 29
// splits and more): a CTA of 1024 threads covers 8 rows x 32 columns, and
// four thread groups sum four contiguous ranges of the splits (in order)
// before group 0 adds the four range sums in order -- each thread's chain
// of dependent loads is a quarter as long.  Deterministic.
constexpr int SKR_ROWS = 8, SKR_GROUPS = 4;
__global__ void __launch_bounds__(256 * SKR_GROUPS) splitk_reduce_t4_kernel(const float* __restrict__ ws,
                                                                          float* __restrict__ out, int rows,
                                                                          int cols, int splits, int acc) {
  __shared__ float red[SKR_GROUPS][SKR_ROWS][33];
  const int e = threadIdx.x & 255, q = threadIdx.x >> 8;
  const int rr = e >> 5, cc = e & 31;
  const int r = blockIdx.x * SKR_ROWS + rr, c = blockIdx.y * 32 + cc;
  const size_t plane = (size_t)rows * cols;
  const int per = (splits + SKR_GROUPS - 1) / SKR_GROUPS;
  const int s0 = q * per, s1 = min(splits, s0 + per);
  float s = 0.0f;
  if (r < rows && c < cols) {
    const float* p = ws + (size_t)r * cols + c;
#pragma unroll 4
    for (int sp = s0; sp < s1; sp++) s += __ldg(p + (size_t)sp * plane);
  }
  red[q][rr][cc] = s;
  __syncthreads();
  if (q == 0) {
    // write out[c][r]: consecutive threads take consecutive rows of a column
    const int wc = threadIdx.x >> 3, wr = threadIdx.x & 7;
    const int orow = blockIdx.x * SKR_ROWS + wr, ocol = blockIdx.y * 32 + wc;
    if (orow < rows && ocol < cols) {
      float t = red[0][wr][wc];
#pragma unroll
      for (int g = 1; g < SKR_GROUPS; g++) t += red[g][wr][wc];
      float* o = out + (size_t)ocol * rows + orow;
      *o = acc ? *o + t : t;
    }
  }
}

int launch_splitk_reduce(rnn_ctx* ctx, const float* ws, float* out, int rows, int cols, int splits,
                         bool acc, bool transpose) {
  size_t total = (size_t)rows * cols;
  RNN_RANGE(ws, total * splits * sizeof(float));
  RNN_RANGE(out, total * sizeof(float));
  if (transpose && splits >= 8) {
    const dim3 grid((rows + SKR_ROWS - 1) / SKR_ROWS, (cols + 31) / 32);
    splitk_reduce_t4_kernel<<<grid, 256 * SKR_GROUPS, 0, ctx->stream>>>(ws, out, rows, cols, splits, acc ? 1 : 0);
    RNN_CHECK_LAUNCH();
    return RNN_OK;
  }
  if (!transpose && total % 4 == 0 && al16(ws) && al16(out)) {
    const size_t total4 = total / 4;
    const unsigned g4 = (unsigned)std::max<size_t>(1, std::min<size_t>((total4 + 255) / 256, (size_t)ctx->num_sms * 8));
    splitk_reduce4_kernel<<<g4, 256, 0, ctx->stream>>>(reinterpret_cast<const float4*>(ws),
                                                       reinterpret_cast<float4*>(out), total4, splits, acc ? 1 : 0);
    RNN_CHECK_LAUNCH();
    return RNN_OK;
  }
  unsigned grid;
  if (transpose) grid = (unsigned)std::min<size_t>(((rows + 31) / 32) * (size_t)((cols + 31) / 32), 4096);
  else grid = (unsigned)std::min<size_t>((total + 255) / 256, (size_t)ctx->num_sms * 8);
  if (grid == 0) return RNN_OK;
  // the transposed form assumes 256 threads (4 tile elements each)
  splitk_reduce_kernel<<<grid, 256, 0, ctx->stream>>>(ws, out, rows, cols, splits, acc ? 1 : 0,
                                                      transpose ? 1 : 0);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

}  // namespace tc
}  // namespace rnn

using namespace rnn;

extern "C" int rnn_gemm_dev(rnn_ctx* ctx, int m, int n, int k, const float* a, int at,
                            const float* b, int bt, float* c, int acc) {
  RNN_REQUIRE(ctx != nullptr, "null context");
  return tc::gemm_dev(ctx, m, n, k, a, at != 0, b, bt != 0, c, acc != 0, false);
}

extern "C" int rnn_gemm_dw_dev(rnn_ctx* ctx, int m, int n, int k, const float* a, const float* b,
                               float* c) {
  RNN_REQUIRE(ctx != nullptr, "null context");
  if (m == 0 || n == 0 || k == 0) return RNN_OK;  // gemm.rs:556-558
  // C[m x n] += A^T B with A [k x m], B [k x n]: op(A) = A^T (at), op(B) = B
  return tc::gemm_dev(ctx, m, n, k, a, true, b, false, c, true, true);
}

// ---------------------------------------------------------------- no-alloc variant
//
// rnn_gemm_dw_noalloc_dev is matmul_dw (C += A^T B) for callers that must not
// allocate device memory at all: for example a host framework that has
// reserved the device's memory for its own caching pool (a cudaMalloc from a
// library could fail or fragment that pool), or a latency-critical loop that
// cannot pay cudaMalloc's implicit device synchronisation.  It needs no
// context: the split-K partial sums go to a fixed file-scope device array of
// NOALLOC_SCRATCH_BYTES (16 MiB), which every GPU that loads this library
// holds until the process exits.  All calls share that array, so two calls
// whose kernels overlap on a GPU race; issue them on one stream or order them.
// The partials it holds are fully rewritten by each call before they are read,
// so nothing in it has to start at zero.
#include <mutex>

namespace rnn {
namespace tc {

constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(16) << 20;
constexpr size_t NOALLOC_SCRATCH_FLOATS = NOALLOC_SCRATCH_BYTES / sizeof(float);
constexpr int NOALLOC_MAX_DEVICES = 64;

static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_SCRATCH_FLOATS];
static __device__ int g_noalloc_error;  // pipeline-wait timeouts of these launches

struct NoAllocDevice {
  float* scratch = nullptr;  // device address of g_noalloc_scratch on this device
  int* error = nullptr;
  int num_sms = 0;
  bool ready = false;
};
static NoAllocDevice g_noalloc_devices[NOALLOC_MAX_DEVICES];
static std::mutex g_noalloc_mutex;

// Once per device, with that device current: host code only holds a
// stand-in for the array's name, so the device address has to be looked up.
static int noalloc_setup(int device, NoAllocDevice** out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  RNN_REQUIRE(device >= 0 && device < NOALLOC_MAX_DEVICES, "gemm_dw_noalloc: device %d out of range", device);
  NoAllocDevice& d = g_noalloc_devices[device];
  if (!d.ready) {
    RNN_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&d.scratch), g_noalloc_scratch));
    RNN_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&d.error), g_noalloc_error));
    RNN_CUDA(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, device));
    d.ready = true;
  }
  *out = &d;
  return RNN_OK;
}

template <int BN>
static int noalloc_run(rnn_ctx* ctx, DenseProb<true, false> p, int splits) {
  Sched s = make_sched(p.M, p.N, p.K, BN, splits);
  p.splits = s.splits;
  p.ws = s.splits > 1 ? static_cast<float*>(ctx->ws) : nullptr;
  RNN_TRY(launch<BN>(ctx, native<BN>(p), s));
  if (s.splits > 1) {
    const size_t total = (size_t)p.M * p.N;
    const unsigned grid = (unsigned)std::min<size_t>((total + 255) / 256, (size_t)ctx->num_sms * 8);
    splitk_reduce_kernel<<<grid, 256, 0, ctx->stream>>>(p.ws, p.c, p.M, p.N, s.splits, 1, 0);
    RNN_CHECK_LAUNCH();
  }
  return RNN_OK;
}

}  // namespace tc
}  // namespace rnn

extern "C" int rnn_gemm_dw_noalloc_dev(int m, int n, int k, const float* a, const float* b, float* c,
                                       void* stream) {
  using namespace rnn::tc;
  RNN_REQUIRE(m >= 0 && n >= 0 && k >= 0, "gemm_dw_noalloc: negative size m=%d n=%d k=%d", m, n, k);
  if (m == 0 || n == 0 || k == 0) return RNN_OK;
  RNN_REQUIRE(a && b && c, "gemm_dw_noalloc: null operand");
  // at least two partial planes must fit: m*n <= scratch / 2
  RNN_REQUIRE((size_t)m * n <= NOALLOC_SCRATCH_FLOATS / 2,
              "gemm_dw_noalloc: m*n = %zu exceeds this entry point's limit of %zu elements (its fixed %zu-MiB "
              "scratch holds at least two partial results); use rnn_gemm_dw_dev",
              (size_t)m * n, NOALLOC_SCRATCH_FLOATS / 2, NOALLOC_SCRATCH_BYTES >> 20);
  RNN_RANGE(a, sizeof(float) * (size_t)k * m);
  RNN_RANGE(b, sizeof(float) * (size_t)k * n);
  RNN_RANGE(c, sizeof(float) * (size_t)m * n);
  int device = 0;
  RNN_CUDA(cudaGetDevice(&device));
  NoAllocDevice* d = nullptr;
  RNN_TRY(noalloc_setup(device, &d));
  rnn_ctx ctx;  // on the stack: nothing is allocated
  ctx.device = device;
  ctx.num_sms = d->num_sms;
  ctx.stream = static_cast<cudaStream_t>(stream);
  ctx.ws = d->scratch;
  ctx.ws_bytes = NOALLOC_SCRATCH_BYTES;
  ctx.dev_error = d->error;
  DenseProb<true, false> p;
  p.a = a; p.b = b; p.c = c; p.ws = nullptr;
  p.M = m; p.N = n; p.K = k; p.acc = 1; p.splits = 1;
  p.a_vec = (m % 4 == 0) && ((reinterpret_cast<uintptr_t>(a) & 15) == 0);
  p.b_vec = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(b) & 15) == 0);
  p.c_vec = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(c) & 15) == 0);
  const int bn = pick_bn(n, (m + BM - 1) / BM, ctx.num_sms);
  int splits = pick_splits(m, n, k, bn, ctx.num_sms);
  const int cap = (int)std::min<size_t>(NOALLOC_SCRATCH_FLOATS / ((size_t)m * n), 1 << 20);
  if (splits > cap) splits = cap;
  switch (bn) {
    case 32: return noalloc_run<32>(&ctx, p, splits);
    case 64: return noalloc_run<64>(&ctx, p, splits);
    case 128: return noalloc_run<128>(&ctx, p, splits);
    default: return noalloc_run<256>(&ctx, p, splits);
  }
}

// The allocation-free entry has no context whose synchronise could report a
// kernel that gave up waiting on its pipeline, so its kernels OR that into
// g_noalloc_error and this query reports it: it waits for `stream`, reads the
// word of the current device, clears it, and returns RNN_ERR_DEVICE when it
// was set (the C written by the calls since the last query is then not to be
// trusted).  Nothing is allocated; the read goes to a host stack variable.
extern "C" int rnn_gemm_dw_noalloc_status(void* stream) {
  using namespace rnn::tc;
  int device = 0;
  RNN_CUDA(cudaGetDevice(&device));
  NoAllocDevice* d = nullptr;
  RNN_TRY(noalloc_setup(device, &d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int err = 0;
  RNN_CUDA(cudaMemcpyAsync(&err, d->error, sizeof(int), cudaMemcpyDeviceToHost, s));
  RNN_CUDA(cudaStreamSynchronize(s));
  if (err == 0) return RNN_OK;
  RNN_CUDA(cudaMemsetAsync(d->error, 0, sizeof(int), s));
  RNN_CUDA(cudaStreamSynchronize(s));
  return rnn::set_error(RNN_ERR_DEVICE,
                        "gemm_dw_noalloc: device error 0x%x (a kernel gave up waiting on a pipeline barrier); "
                        "C of the calls since the last status query is not valid", err);
}
