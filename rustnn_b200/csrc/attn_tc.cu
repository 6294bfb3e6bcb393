// Tensor-core attention on the tcgen05 3xTF32 engine.
//
// attn.rs runs Core::forward / Core::backward (:148-343) as small GEMMs per
// (image, head) through gemm_small.  Here every product of a call is one
// launch of the persistent engine over all pairs, with two heads of one image
// per 128-row tile: the 64 query rows of head 2p and those of head 2p+1.
// Their products with the keys of the same image use a block-diagonal
// operand along K: rows of head 2p carry Q in K columns [0, dh) and zeros in
// [dh, 2dh), rows of head 2p+1 the other way round, and the key operand is
// the natural [K_2p | K_2p+1] slice of a kv row, so one 128 x tk x 2dh MMA
// chain yields both heads' scores and every accumulator row is a real query
// row.  Products whose output columns are per head (O = P V, dQ = dS K) run
// over N = 2dh columns and keep each row's own head block.
//
//   forward   AttnScoreProb   S = Q K^T; epilogue: tau*S + bias (the
//                             per-head table rel[relidx] with the diagonal
//                             mask folded in, built once per call), row
//                             softmax -> P (HBM, as attn.rs:186-211 stores it)
//             AttnPVProb      O = P V
//   backward  AttnDSProb      dP = dO V^T; epilogue: dS = P (dP - rowsum(dP P))
//                             -> workspace (attn.rs:276-291)
//             AttnDQProb      G = dS K; epilogue: dq += tau G and the dtau
//                             partial sum_i Q_i . G_i, which equals the
//                             reference's sum dS * (Q K^T) (attn.rs:292-308)
//                             without recomputing the scores
//             AttnDKVProb     dV = P^T dO and dK = tau dS^T Q per head (two
//                             items of one launch), += into dkv
//             attn_drel       drel (attn.rs:309-315): the image sum of dS,
//                             then per relative index a fixed-order gather
// dtau partials are per (image, half of a head's rows) and reduced in a fixed
// order afterwards (attn.cu), so the backward is deterministic and uses no
// atomics.
#include <cmath>

#include "attn_tc.cuh"
#include "tc_launch.cuh"

namespace rnn {
namespace tc {

namespace {

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ void put4(float (&v)[32], int j, float4 t) {
  v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
}

// K-major producer mapping (8 threads per row, 16 rows per step) shared by
// the head-pair problems.
__device__ __forceinline__ void kmajor_a_slot(int gt, int j, int& r, int& c) {
  r = (gt >> 3) + 16 * j;
  c = gt & 7;
}
__device__ __forceinline__ void kmajor_b_slot(int gt, int j, int& r, int& c) {
  const int idx = gt + 128 * j;
  r = idx >> 3;
  c = idx & 7;
}
template <int BN>
__device__ __forceinline__ void mnmajor_b_slot(int gt, int j, int& r, int& c) {
  const int idx = gt + 128 * j;
  r = idx % BN;
  c = idx / BN;
}

// Head-pair tile: image and pair of a 128-row tile; row r of it is query
// (r & 63) of head 2*pair + (r >> 6).
struct PairTS {
  int img, pr;
};
__device__ __forceinline__ void pair_of(const AttnTC& a, int mt, PairTS& ts) {
  ts.img = mt / a.hp;
  ts.pr = mt - ts.img * a.hp;
}

// Block-diagonal A over the two heads: K block kb of [0, 2*DH) belongs to
// head part kb*32/DH; rows of the other head part read nothing.  `src` row
// (img, i) of head hd starts at src + (img*tq + i)*stride + off + hd*DH.
template <int DH>
__device__ __forceinline__ void load_blockdiag(const AttnTC& a, const PairTS& ts, int kb, int gt, const float* src,
                                               int stride, int off, float (&v)[32]) {
  const int kh = (kb * BK) / DH;
  const int d0 = kb * BK - kh * DH;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    int r, c;
    kmajor_a_slot(gt, j, r, c);
    const int hl = r >> 6, i = r & 63;
    if (hl == kh) {
      const float* row = src + (size_t)(ts.img * a.tq + i) * stride + off + (2 * ts.pr + hl) * DH;
      put4(v, j, ldg4(row + d0 + 4 * c));
    } else {
      put4(v, j, make_float4(0.f, 0.f, 0.f, 0.f));
    }
  }
}

// Key rows of the pair, K = [0, 2*DH) along the kv row from column off.
template <int NB, int DH>
__device__ __forceinline__ void load_keyrows(const AttnTC& a, const PairTS& ts, int kb, int gt, int off,
                                             float (&v)[NB]) {
#pragma unroll
  for (int j = 0; j < NB / 4; j++) {
    int r, c;
    kmajor_b_slot(gt, j, r, c);
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < a.tk)
      t = ldg4(a.kv + (size_t)(ts.img * a.tk + r) * a.kvstride + off + 2 * ts.pr * DH + kb * BK + 4 * c);
    v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
  }
}

// Rows of a [n][h][tq][tk] tensor (P or dS) as the K-major A of the pair.
__device__ __forceinline__ void load_scorerows(const AttnTC& a, const PairTS& ts, int kb, int gt, const float* src,
                                               float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 8; j++) {
    int r, c;
    kmajor_a_slot(gt, j, r, c);
    const int hl = r >> 6, i = r & 63;
    const float* row = src + ((size_t)(ts.img * a.h + 2 * ts.pr + hl) * a.tq + i) * a.tk;
    put4(v, j, ldg4(row + kb * BK + 4 * c));
  }
}

// The pair's value (or key) columns as an MN-major B: B[col][k] = kv row k,
// column off + 2*pair*DH + col, for col < 2*DH and key k.
template <int NB, int BN, int DH>
__device__ __forceinline__ void load_kvcols(const AttnTC& a, const PairTS& ts, int kb, int gt, int off,
                                            float (&v)[NB]) {
#pragma unroll
  for (int j = 0; j < NB / 4; j++) {
    int r, c;
    mnmajor_b_slot<BN>(gt, j, r, c);
    const float* col = a.kv + (size_t)(ts.img * a.tk) * a.kvstride + off + 2 * ts.pr * DH + r;
    const int k0 = kb * BK + 4 * c;
#pragma unroll
    for (int e = 0; e < 4; e++) v[4 * j + e] = __ldg(col + (size_t)(k0 + e) * a.kvstride);
  }
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// The row epilogues give lane l accumulator row l of its warp, and the 32
// rows of a warp are consecutive rows (stride ld floats) of P, dS, q or the
// bias table.  A row-per-lane access would make every warp instruction touch
// 32 lines; these move a 32 x 32 chunk through a padded shared-memory buffer
// (32 x 33 floats per warp, conflict-free both ways) so each global access is
// one row's 128 contiguous bytes.
constexpr int STAGE_LD = 33;
constexpr int STAGE_WARP_BYTES = 32 * STAGE_LD * 4;

// out[e] = base[lane * ld + c0 + e], e < 32
__device__ __forceinline__ void stage_load(const float* __restrict__ base, size_t ld, int c0, float* buf, int lane,
                                           float (&out)[32]) {
  float t[32];
#pragma unroll
  for (int rr = 0; rr < 32; rr++) t[rr] = __ldg(base + rr * ld + c0 + lane);
#pragma unroll
  for (int rr = 0; rr < 32; rr++) buf[rr * STAGE_LD + lane] = t[rr];
  __syncwarp();
#pragma unroll
  for (int e = 0; e < 32; e++) out[e] = buf[lane * STAGE_LD + e];
  __syncwarp();
}

// base[lane * ld + c0 + e] = v[e] (acc: +=)
__device__ __forceinline__ void stage_store(float* __restrict__ base, size_t ld, int c0, float* buf, int lane,
                                            const float (&v)[32], bool acc = false) {
#pragma unroll
  for (int e = 0; e < 32; e++) buf[lane * STAGE_LD + e] = v[e];
  __syncwarp();
#pragma unroll
  for (int rr = 0; rr < 32; rr++) {
    float* p = base + rr * ld + c0 + lane;
    *p = acc ? *p + buf[rr * STAGE_LD + lane] : buf[rr * STAGE_LD + lane];
  }
  __syncwarp();
}

}  // namespace

// ---------------------------------------------------------------- forward

// S = Q K^T for the pair; the epilogue turns each row into P (attn.rs:181-211):
// z_j = tau * S_ij + rel[relidx[i][j]], z_ii = -inf under the diagonal mask,
// P_ij = exp(z_j - max z) / sum, with the same operation order as the SIMT
// kernel (expf, one reciprocal, a product).
template <int DH>
struct AttnScoreProb {
  static constexpr bool B_BULK = false;
  static constexpr int ROW_EPI_WARP_BYTES = STAGE_WARP_BYTES;
  AttnTC a;
  int M, N;
  using TS = PairTS;
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int, int) const { pair_of(a, m0 / BM, ts); }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) { kmajor_a_slot(gt, j, r, c); }
  static __device__ __forceinline__ void b_slot(int gt, int j, int& r, int& c) { kmajor_b_slot(gt, j, r, c); }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int gt, float (&v)[32]) const {
    load_blockdiag<DH>(a, ts, kb, gt, a.q, a.qstride, a.qoff, v);
  }
  template <int NB>
  __device__ __forceinline__ void load_b(const TS& ts, int kb, int gt, float (&v)[NB]) const {
    load_keyrows<NB, DH>(a, ts, kb, gt, a.koff, v);
  }
  __device__ __forceinline__ const void* b_src(int, int) const { return nullptr; }

  // Two passes over the row in TMEM.  Pass 1: z = tau * S + bias per
  // 32-column chunk (bias is -inf on a masked diagonal, so z is too), z
  // written back over the chunk, the running maximum and the sum of
  // exp(z - max) (rescaled when a chunk raises the maximum).  Pass 2: P from
  // z.  The warp's 32 rows are queries i0 .. i0+31 of one head, consecutive
  // rows of the bias table and of P, staged through shared memory.
  template <int BN, bool STACK>
  __device__ __forceinline__ void epi_row(int mt, int, int q, int lane, uint32_t taddr, uint8_t* wsm) const {
    PairTS ts;
    pair_of(a, mt, ts);
    const int hd = 2 * ts.pr + (q >> 1), i0 = (q & 1) * 32;
    const float t = __ldg(a.tau + hd);
    float* buf = reinterpret_cast<float*>(wsm);
    const float* bias0 = a.bias + ((size_t)hd * a.tq + i0) * a.tk;
    const int nch = a.tk / 32;
    float mx = -INFINITY, sum = 0.0f;
#pragma unroll 1
    for (int c = 0; c < nch; c++) {
      float b[32], v[32];
      stage_load(bias0, a.tk, c * 32, buf, lane, b);
      acc_ld32<BN, STACK>(taddr, c, v);
      uint32_t zu[32];
      float cm = -INFINITY;
#pragma unroll
      for (int e = 0; e < 32; e++) {
        const float z = t * v[e] + b[e];
        zu[e] = __float_as_uint(z);
        cm = fmaxf(cm, z);
      }
      tmem_st32(taddr + c * 32, zu);
      if (cm == -INFINITY) continue;  // every key of the chunk masked
      if (cm > mx) {
        sum = mx == -INFINITY ? 0.0f : sum * expf(mx - cm);
        mx = cm;
      }
#pragma unroll
      for (int e = 0; e < 32; e++) sum += expf(__uint_as_float(zu[e]) - mx);
    }
    tmem_wait_st();
    const float inv = 1.0f / sum;
    float* p0 = a.p + ((size_t)(ts.img * a.h + hd) * a.tq + i0) * a.tk;
#pragma unroll 1
    for (int c = 0; c < nch; c++) {
      float z[32];
      tmem_ld32(taddr + c * 32, z);
#pragma unroll
      for (int e = 0; e < 32; e++) z[e] = expf(z[e] - mx) * inv;
      stage_store(p0, a.tk, c * 32, buf, lane, z);
    }
  }
};

// O = P V over N = 2*DH columns (both heads' value columns); a row keeps the
// columns of its own head (attn.rs:214-220).
template <int DH>
struct AttnPVProb {
  static constexpr bool B_BULK = false;
  static constexpr int BN = 2 * DH;
  AttnTC a;
  int M, N;
  using TS = PairTS;
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int, int) const { pair_of(a, m0 / BM, ts); }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) { kmajor_a_slot(gt, j, r, c); }
  static __device__ __forceinline__ void b_slot(int gt, int j, int& r, int& c) { mnmajor_b_slot<BN>(gt, j, r, c); }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int gt, float (&v)[32]) const {
    load_scorerows(a, ts, kb, gt, a.p, v);
  }
  template <int NB>
  __device__ __forceinline__ void load_b(const TS& ts, int kb, int gt, float (&v)[NB]) const {
    load_kvcols<NB, BN, DH>(a, ts, kb, gt, a.voff, v);
  }
  __device__ __forceinline__ const void* b_src(int, int) const { return nullptr; }
  __device__ __forceinline__ void store(int row, int col0, int, const float (&v)[32]) const {
    PairTS ts;
    pair_of(a, row / BM, ts);
    const int r = row & (BM - 1), hl = r >> 6, i = r & 63;
    if (col0 / DH != hl) return;
    float* dst = a.o + (size_t)(ts.img * a.tq + i) * (a.h * DH) + (2 * ts.pr + hl) * DH + (col0 - hl * DH);
    store_row32(dst, 32, v, false, true);
  }
};

// ---------------------------------------------------------------- backward

// dP = dO V^T for the pair; the epilogue forms dS = P (dP - sum_j dP_j P_j)
// (attn.rs:280-291) and writes it to the workspace; drel is formed from the
// workspace afterwards (attn_drel).
template <int DH>
struct AttnDSProb {
  static constexpr bool B_BULK = false;
  static constexpr int ROW_EPI_WARP_BYTES = 0;
  AttnTC a;
  int M, N;
  using TS = PairTS;
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int, int) const { pair_of(a, m0 / BM, ts); }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) { kmajor_a_slot(gt, j, r, c); }
  static __device__ __forceinline__ void b_slot(int gt, int j, int& r, int& c) { kmajor_b_slot(gt, j, r, c); }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int gt, float (&v)[32]) const {
    load_blockdiag<DH>(a, ts, kb, gt, a.dout, a.h * DH, 0, v);
  }
  template <int NB>
  __device__ __forceinline__ void load_b(const TS& ts, int kb, int gt, float (&v)[NB]) const {
    load_keyrows<NB, DH>(a, ts, kb, gt, a.voff, v);
  }
  __device__ __forceinline__ const void* b_src(int, int) const { return nullptr; }

  template <int BN, bool STACK>
  __device__ __forceinline__ void epi_row(int mt, int, int q, int lane, uint32_t taddr, uint8_t*) const {
    PairTS ts;
    pair_of(a, mt, ts);
    const int row = q * 32 + lane, hl = row >> 6, i = row & 63, hd = 2 * ts.pr + hl;
    const size_t prow = ((size_t)(ts.img * a.h + hd) * a.tq + i) * a.tk;
    const float* pg = a.pin + prow;
    float* dsg = a.ds + prow;
    const int nch = a.tk / 32;
    // request the whole P row into L2 first (one 128-byte line per chunk, no
    // registers held), so that the chunk loads below wait on L2, not DRAM
    for (int c = 0; c < nch; c++) asm volatile("prefetch.global.L2 [%0];" ::"l"(pg + c * 32));
    float dot = 0.0f;
#pragma unroll 1
    for (int c = 0; c < nch; c++) {
      float4 p4[8];
#pragma unroll
      for (int e = 0; e < 8; e++) p4[e] = ldg4(pg + c * 32 + 4 * e);
      float v[32];
      acc_ld32<BN, STACK>(taddr, c, v);
#pragma unroll
      for (int e = 0; e < 8; e++) {
        dot = fmaf(v[4 * e], p4[e].x, dot);
        dot = fmaf(v[4 * e + 1], p4[e].y, dot);
        dot = fmaf(v[4 * e + 2], p4[e].z, dot);
        dot = fmaf(v[4 * e + 3], p4[e].w, dot);
      }
    }
#pragma unroll 1
    for (int c = 0; c < nch; c++) {
      float4 p4[8];
#pragma unroll
      for (int e = 0; e < 8; e++) p4[e] = ldg4(pg + c * 32 + 4 * e);
      float v[32];
      acc_ld32<BN, STACK>(taddr, c, v);
#pragma unroll
      for (int e = 0; e < 8; e++)
        *reinterpret_cast<float4*>(dsg + c * 32 + 4 * e) =
            make_float4(p4[e].x * (v[4 * e] - dot), p4[e].y * (v[4 * e + 1] - dot), p4[e].z * (v[4 * e + 2] - dot),
                        p4[e].w * (v[4 * e + 3] - dot));
    }
  }
};

// G = dS K for the pair over N = 2*DH columns; a row keeps its own head's
// block: dq += tau * G (attn.rs:316-321) and the row's share of
// dtau = sum_i Q_i . G_i.
template <int DH>
struct AttnDQProb {
  static constexpr bool B_BULK = false;
  static constexpr int ROW_EPI_WARP_BYTES = 0;
  static constexpr int BN = 2 * DH;
  AttnTC a;
  int M, N;
  using TS = PairTS;
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int, int) const { pair_of(a, m0 / BM, ts); }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) { kmajor_a_slot(gt, j, r, c); }
  static __device__ __forceinline__ void b_slot(int gt, int j, int& r, int& c) { mnmajor_b_slot<BN>(gt, j, r, c); }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int gt, float (&v)[32]) const {
    load_scorerows(a, ts, kb, gt, a.ds, v);
  }
  template <int NB>
  __device__ __forceinline__ void load_b(const TS& ts, int kb, int gt, float (&v)[NB]) const {
    load_kvcols<NB, BN, DH>(a, ts, kb, gt, a.koff, v);
  }
  __device__ __forceinline__ const void* b_src(int, int) const { return nullptr; }

  template <int BN_, bool STACK>
  __device__ __forceinline__ void epi_row(int mt, int, int q, int lane, uint32_t taddr, uint8_t*) const {
    PairTS ts;
    pair_of(a, mt, ts);
    const int row = q * 32 + lane, hl = row >> 6, i = row & 63, hd = 2 * ts.pr + hl;
    const float t = __ldg(a.tau + hd);
    const size_t qrow = (size_t)(ts.img * a.tq + i) * a.qstride + a.qoff + hd * DH;
    const float* qg = a.q + qrow;
    float* dqg = a.dq + qrow;
    float tacc = 0.0f;
#pragma unroll 1
    for (int c = hl * (DH / 32); c < (hl + 1) * (DH / 32); c++) {
      float v[32];
      acc_ld32<BN_, STACK>(taddr, c, v);
      const int d0 = c * 32 - hl * DH;
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        const float4 q4 = ldg4(qg + d0 + e);
        tacc = fmaf(q4.x, v[e], tacc);
        tacc = fmaf(q4.y, v[e + 1], tacc);
        tacc = fmaf(q4.z, v[e + 2], tacc);
        tacc = fmaf(q4.w, v[e + 3], tacc);
        float4* d4 = reinterpret_cast<float4*>(dqg + d0 + e);
        float4 o = *d4;
        o.x += t * v[e];
        o.y += t * v[e + 1];
        o.z += t * v[e + 2];
        o.w += t * v[e + 3];
        *d4 = o;
      }
    }
    tacc = warp_sum_f(tacc);
    if (lane == 0) a.part[(size_t)(ts.img * 2 + (q & 1)) * a.h + hd] = tacc;
  }
};

// dV = P^T dO (item 2*pair_item) and dK = tau dS^T Q (item + 1) for one
// (image, head), M = the tk keys in 128-row tiles, K = tq queries, N = DH
// (attn.rs:270-274, 322-327); += into dkv.
template <int DH>
struct AttnDKVProb {
  static constexpr bool B_BULK = false;
  static constexpr int BN = DH;
  AttnTC a;
  int M, N, mtp;  // mtp: 128-row tiles per item
  struct TS {
    int img, hd, which, j0;
  };
  __device__ __forceinline__ void item_of(int mt, TS& ts) const {
    const int item = mt / mtp;
    ts.j0 = (mt - item * mtp) * BM;
    ts.which = item & 1;
    const int ih = item >> 1;
    ts.img = ih / a.h;
    ts.hd = ih - ts.img * a.h;
  }
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int, int) const { item_of(m0 / BM, ts); }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) { r = gt; c = j; }
  static __device__ __forceinline__ void b_slot(int gt, int j, int& r, int& c) { mnmajor_b_slot<BN>(gt, j, r, c); }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int gt, float (&v)[32]) const {
    const int key = ts.j0 + gt;
    const float* src = (ts.which ? a.ds : a.pin) + (size_t)(ts.img * a.h + ts.hd) * a.tq * a.tk + key;
    const bool ok = key < a.tk;
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = ok ? __ldg(src + (size_t)(kb * BK + j) * a.tk) : 0.0f;
  }
  template <int NB>
  __device__ __forceinline__ void load_b(const TS& ts, int kb, int gt, float (&v)[NB]) const {
    const float* base;
    size_t stride;
    if (ts.which) {
      base = a.q + (size_t)ts.img * a.tq * a.qstride + a.qoff + ts.hd * DH;
      stride = a.qstride;
    } else {
      base = a.dout + (size_t)ts.img * a.tq * (a.h * DH) + ts.hd * DH;
      stride = (size_t)a.h * DH;
    }
#pragma unroll
    for (int j = 0; j < NB / 4; j++) {
      int r, c;
      mnmajor_b_slot<BN>(gt, j, r, c);
      const int k0 = kb * BK + 4 * c;
#pragma unroll
      for (int e = 0; e < 4; e++) v[4 * j + e] = __ldg(base + (size_t)(k0 + e) * stride + r);
    }
  }
  __device__ __forceinline__ const void* b_src(int, int) const { return nullptr; }
  __device__ __forceinline__ void store(int row, int col0, int, const float (&v)[32]) const {
    TS ts;
    item_of(row / BM, ts);
    const int key = ts.j0 + (row & (BM - 1));
    if (key >= a.tk) return;
    float* dst = a.dkv + (size_t)(ts.img * a.tk + key) * a.kvstride + (ts.which ? a.koff : a.voff) + ts.hd * DH + col0;
    if (ts.which) {
      const float t = __ldg(a.tau + ts.hd);
      float w[32];
#pragma unroll
      for (int e = 0; e < 32; e++) w[e] = t * v[e];
      store_row32(dst, 32, w, true, true);
    } else {
      store_row32(dst, 32, v, true, true);
    }
  }
};

// ---------------------------------------------------------------- small kernels

__global__ void attn_bias_kernel(const float* __restrict__ rel, const uint32_t* __restrict__ relidx, int h, int tq,
                                 int tk, int nrel, int mask, float* __restrict__ bias) {
  const int total = h * tq * tk;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    const int hd = e / (tq * tk), ij = e - hd * tq * tk, i = ij / tk, j = ij - i * tk;
    bias[e] = (mask && i == j) ? -INFINITY : rel[(size_t)hd * nrel + relidx[ij]];
  }
}

// dssum[e] = sum_n ds[n][e] over the n images, n ascending.
__global__ void attn_image_sum_kernel(const float* __restrict__ ds, int n, int per, float* __restrict__ dssum) {
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < per; e += gridDim.x * blockDim.x) {
    float s = 0.0f;
    int k = 0;
    for (; k + 8 <= n; k += 8) {  // eight images' loads in flight, added in order
      float a[8];
#pragma unroll
      for (int u = 0; u < 8; u++) a[u] = __ldg(ds + (size_t)(k + u) * per + e);
#pragma unroll
      for (int u = 0; u < 8; u++) s += a[u];
    }
    for (; k < n; k++) s += __ldg(ds + (size_t)k * per + e);
    dssum[e] = s;
  }
}

// drel[h][r] += sum_i dssum[h][i][inv[i][r]]: one warp per (h, r), lane l
// sums queries l, l+32, ... in ascending order, then a fixed shuffle tree
// over the lanes (deterministic; the queries' loads are in flight together
// instead of one dependent index-then-value pair after another).
__global__ void attn_drel_gather_kernel(const float* __restrict__ dssum, const int* __restrict__ inv, int h, int tq,
                                        int tk, int nrel, float* __restrict__ drel) {
  const int total = h * nrel;
  const int lane = threadIdx.x & 31;
  const int wstride = (gridDim.x * blockDim.x) >> 5;
  for (int e = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; e < total; e += wstride) {
    const int hd = e / nrel, r = e - hd * nrel;
    float s = 0.0f;
    for (int i = lane; i < tq; i += 32) {
      const int j = __ldg(inv + (size_t)i * nrel + r);
      if (j >= 0) s += __ldg(dssum + ((size_t)hd * tq + i) * tk + j);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
    if (lane == 0) drel[e] += s;
  }
}

// ---------------------------------------------------------------- host

static inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int attn_bias_build(rnn_ctx* ctx, const AttnTC& a, float* bias) {
  const int total = a.h * a.tq * a.tk;
  const int grid = std::min((total + 255) / 256, ctx->num_sms * 8);
  attn_bias_kernel<<<grid, 256, 0, ctx->stream>>>(a.rel, a.relidx, a.h, a.tq, a.tk, a.nrel, a.mask, bias);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int attn_drel(rnn_ctx* ctx, const AttnTC& a, const int* inv, float* dssum, float* drel) {
  const int per = a.h * a.tq * a.tk;
  attn_image_sum_kernel<<<std::min((per + 255) / 256, ctx->num_sms * 8), 256, 0, ctx->stream>>>(a.ds, a.n, per,
                                                                                                dssum);
  RNN_CHECK_LAUNCH();
  const int total = a.h * a.nrel;
  attn_drel_gather_kernel<<<std::min((total + 7) / 8, ctx->num_sms * 8), 256, 0, ctx->stream>>>(
      dssum, inv, a.h, a.tq, a.tk, a.nrel, drel);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

bool attn_tc_ok(const AttnTC& a, bool backward) {
  if (a.tq != 64 || a.h % 2 != 0 || !(a.dh == 32 || a.dh == 64)) return false;
  if (a.tk % 32 != 0 || a.tk < 32 || a.tk > 256) return false;
  if (a.qstride % 4 || a.qoff % 4 || a.kvstride % 4 || a.koff % 4 || a.voff % 4) return false;
  if (!al16(a.q) || !al16(a.kv)) return false;
  if (!backward) return al16(a.p) && al16(a.o);
  return al16(a.pin) && al16(a.dout) && al16(a.dq) && al16(a.dkv);
}

template <int BN, class P>
static int run_pair(rnn_ctx* ctx, P p, int K) {
  p.M = p.a.n * p.a.hp * BM;
  Sched s = make_sched(p.M, p.N, K, BN, 1);
  return launch<BN>(ctx, p, s);
}

template <template <int> class P, int DH>
static int run_keys(rnn_ctx* ctx, const AttnTC& a) {
  P<DH> p;
  p.a = a;
  p.N = a.tk;
  const int K = 2 * DH;
  if (a.tk <= 32) return run_pair<32>(ctx, p, K);
  if (a.tk <= 64) return run_pair<64>(ctx, p, K);
  if (a.tk <= 128) return run_pair<128>(ctx, p, K);
  return run_pair<256>(ctx, p, K);
}

template <int DH>
static int fwd_dh(rnn_ctx* ctx, const AttnTC& a) {
  RNN_TRY((run_keys<AttnScoreProb, DH>(ctx, a)));
  AttnPVProb<DH> pv;
  pv.a = a;
  pv.N = 2 * DH;
  return run_pair<2 * DH>(ctx, pv, a.tk);
}

template <int DH>
static int bwd_dh(rnn_ctx* ctx, const AttnTC& a) {
  RNN_TRY((run_keys<AttnDSProb, DH>(ctx, a)));
  AttnDQProb<DH> dq;
  dq.a = a;
  dq.N = 2 * DH;
  RNN_TRY(run_pair<2 * DH>(ctx, dq, a.tk));
  AttnDKVProb<DH> kv;
  kv.a = a;
  kv.N = DH;
  kv.mtp = (a.tk + BM - 1) / BM;
  kv.M = a.n * a.h * 2 * kv.mtp * BM;
  Sched s = make_sched(kv.M, kv.N, a.tq, DH, 1);
  return launch<DH>(ctx, kv, s);
}

int attn_tc_fwd(rnn_ctx* ctx, const AttnTC& a) {
  return a.dh == 32 ? fwd_dh<32>(ctx, a) : fwd_dh<64>(ctx, a);
}

int attn_tc_bwd(rnn_ctx* ctx, const AttnTC& a) {
  return a.dh == 32 ? bwd_dh<32>(ctx, a) : bwd_dh<64>(ctx, a);
}

}  // namespace tc
}  // namespace rnn
