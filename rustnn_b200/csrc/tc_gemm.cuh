// Persistent tcgen05 GEMM engine for sm_100a with a 3xTF32 split.
//
// One kernel template drives every contraction of the library: the dense
// GEMM (gemm.rs:434 matmul / gemm_small), the weight-gradient GEMM
// (gemm.rs:555 matmul_dw) and the three implicit-GEMM convolutions
// (conv.rs:169 forward_image, :207 dx_image, :283 dw_image).  What differs
// between them is only how a tile of each operand is fetched from global
// memory and how the accumulator tile is written back; that is supplied by a
// `Prob` type (see gemm.cu / conv.cu).
//
// Accuracy: f32 operands are split in registers as x = hi + lo with
// hi = x rounded to TF32 (11 significant bits) and lo = x - hi (exact).  Each
// K step issues three tcgen05.mma.kind::tf32: lo*hi, hi*lo, hi*hi into one
// f32 TMEM accumulator (the lo*lo term, ~2^-22 relative, is dropped).  This
// is the split-TF32 scheme of Ootomo & Yokota (2022).
//
// CTA layout (288 threads, one CTA per SM, persistent over output tiles):
//   warps 0-3  producers: global -> registers -> hi/lo split -> shared memory
//              in the canonical K-major SWIZZLE_128B layout, STAGES-deep ring
//   warp  4    TMEM allocator + single-thread tcgen05.mma issuer
//   warps 5-8  epilogue: tcgen05.ld from a double-buffered TMEM accumulator
//              (2 x BN columns), so the epilogue of tile i overlaps the
//              main loop of tile i+1
// Tiles are BM=128 rows (TMEM lanes) x BN columns, BK=32 f32 (128 bytes) of K
// per pipeline stage.  Every wait is bounded: on timeout the CTA raises an
// abort flag, all roles drain, TMEM is freed and an error word is set.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rnn {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 32;  // f32 elements of K per stage = one 128-byte swizzle row
constexpr int NUM_PRODUCER_WARPS = 4;
constexpr int MMA_WARP = 4;
constexpr int FIRST_EPI_WARP = 5;
constexpr int NUM_THREADS = 9 * 32;
constexpr unsigned long long WAIT_TIMEOUT_NS = 2000000000ull;  // 2 s

// ------------------------------------------------------------------ PTX

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait.  Returns false when the CTA is aborting (another role timed
// out) or when this wait itself ran past WAIT_TIMEOUT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* dev_error) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(a, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > WAIT_TIMEOUT_NS) {
      *abort_flag = 1;
      if (dev_error) atomicOr(dev_error, 1);
      return false;
    }
  }
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D(tmem) (+)= A(smem) * B(smem)^T, kind::tf32, one CTA.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every previously issued tcgen05.mma of this thread
// has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 TMEM lanes x 32 consecutive f32 columns; thread i of the warp receives
// lane (base_lane + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major operand, SWIZZLE_128B, 8-row
// groups 1024 bytes apart (SBO), sm_100 descriptor version 1.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address, bits 0-13
  d |= static_cast<uint64_t>(1) << 16;                   // LBO (unused for SW128 K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;           // SBO, bits 32-45
  d |= static_cast<uint64_t>(1) << 46;                   // version
  d |= static_cast<uint64_t>(2) << 61;                   // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::tf32: D f32, A/B tf32, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// Round to the nearest TF32 value (ties away from zero) by integer arithmetic
// on the f32 bit pattern; the 13 low mantissa bits are cleared.
__device__ __forceinline__ float tf32_round(float x) {
  uint32_t u = __float_as_uint(x);
  u = (u + 0x1000u) & 0xFFFFE000u;
  return __uint_as_float(u);
}

// Byte offset of the 16-byte chunk `c` (K elements 4c..4c+3) of row `r`
// inside a K-major SWIZZLE_128B tile whose rows are 128 bytes.
__device__ __forceinline__ uint32_t sw128_offset(int r, int c) {
  return static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// Splits 4 values and stores hi and lo chunks.
__device__ __forceinline__ void store_split(uint32_t hi_base, uint32_t lo_base, uint32_t off,
                                            const float (&v)[4]) {
  float h0 = tf32_round(v[0]), h1 = tf32_round(v[1]), h2 = tf32_round(v[2]),
        h3 = tf32_round(v[3]);
  st_shared_v4(hi_base + off, h0, h1, h2, h3);
  st_shared_v4(lo_base + off, v[0] - h0, v[1] - h1, v[2] - h2, v[3] - h3);
}

// ------------------------------------------------------------------ config

template <int BN_>
struct Cfg {
  static constexpr int BN = BN_;
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
  static constexpr int A_BYTES = BM * BK * 4;  // 16 KB
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE_BYTES = 2 * (A_BYTES + B_BYTES);  // hi + lo
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 4 ? 4 : (200 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128
                                   : (2 * BN <= 256) ? 256 : 512;
  // 1024 bytes of alignment slack + barriers
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr uint32_t IDESC = idesc_tf32(BM, BN);
};

// Work decomposition shared by the host launcher and the kernel.
struct Sched {
  int m_tiles, n_tiles, splits;
  int kblocks;         // total K blocks of BK
  int kb_per_split;    // K blocks per split (last split may get fewer)
  int num_tiles;       // m_tiles * n_tiles * splits
};

// ------------------------------------------------------------------ kernel

// Prob concept:
//   static constexpr bool A_KMAJOR, B_KMAJOR;   producer thread mapping
//   int M, N;                                  problem rows / columns
//   __device__ void begin_tile(int m0, int n0, int split, TileState&) (optional
//       per-thread precomputation; see the Prob types)
//   __device__ void load_a(int row, int k4, float (&v)[4]) const
//   __device__ void load_b(int row, int k4, float (&v)[4]) const
//       rows are global row indices, k4 the first of 4 consecutive K indices;
//       must return 0 for out-of-range rows / K
//   __device__ void store(int row, int col0, int split, const float (&v)[32]) const
//       col0 is a multiple of 32; row may be >= M (ignore), cols may exceed N
template <int BN, class Prob>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    tc3_gemm_kernel(const Prob prob, const Sched sched, int* dev_error) {
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned operand ring
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t ring = (raw_addr + 1023u) & ~1023u;
  uint8_t* ring_ptr = smem_raw + (ring - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring_ptr + C::STAGES * C::STAGE_BYTES);
  uint64_t* full = bars;                      // [STAGES] producers -> MMA
  uint64_t* empty = bars + C::STAGES;         // [STAGES] MMA commit -> producers
  uint64_t* acc_full = bars + 2 * C::STAGES;  // [2] MMA commit -> epilogue
  uint64_t* acc_empty = acc_full + 2;         // [2] epilogue -> MMA
  uint64_t* drain = acc_empty + 2;            // [1] abort path
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      mbar_init(&full[s], NUM_PRODUCER_WARPS * 32);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4 * 32);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles_mn = sched.m_tiles * sched.n_tiles;

  if (warp < NUM_PRODUCER_WARPS) {
    // ---------------------------------------------------------- producers
    const int t = threadIdx.x;  // 0..127
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < sched.num_tiles && ok; tile += gridDim.x) {
      const int split = tile / tiles_mn;
      const int mn = tile - split * tiles_mn;
      const int mt = mn % sched.m_tiles, nt = mn / sched.m_tiles;
      const int m0 = mt * BM, n0 = nt * BN;
      const int kb0 = split * sched.kb_per_split;
      int kb1 = kb0 + sched.kb_per_split;
      if (kb1 > sched.kblocks) kb1 = sched.kblocks;
      for (int kb = kb0; kb < kb1; kb++, it++) {
        const int stage = it % C::STAGES;
        const uint32_t phase = (it / C::STAGES) & 1;
        const int k0 = kb * BK;
        // A: 128 rows x 8 chunks, 8 chunks per thread
        float va[8][4];
#pragma unroll
        for (int j = 0; j < 8; j++) {
          int r, c;
          if (Prob::A_KMAJOR) { r = (t >> 3) + 16 * j; c = t & 7; }
          else { r = t; c = j; }
          prob.load_a(m0 + r, k0 + 4 * c, va[j]);
        }
        // B: BN rows x 8 chunks, BN/16 chunks per thread
        constexpr int BJ = BN / 16;
        float vb[BJ][4];
#pragma unroll
        for (int j = 0; j < BJ; j++) {
          int idx = t + 128 * j, r, c;
          if (Prob::B_KMAJOR) { r = idx >> 3; c = idx & 7; }
          else { r = idx % BN; c = idx / BN; }
          prob.load_b(n0 + r, k0 + 4 * c, vb[j]);
        }
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, dev_error)) { ok = false; break; }
        const uint32_t a_hi = ring + stage * C::STAGE_BYTES;
        const uint32_t a_lo = a_hi + C::A_BYTES;
        const uint32_t b_hi = a_lo + C::A_BYTES;
        const uint32_t b_lo = b_hi + C::B_BYTES;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          int r, c;
          if (Prob::A_KMAJOR) { r = (t >> 3) + 16 * j; c = t & 7; }
          else { r = t; c = j; }
          store_split(a_hi, a_lo, sw128_offset(r, c), va[j]);
        }
#pragma unroll
        for (int j = 0; j < BJ; j++) {
          int idx = t + 128 * j, r, c;
          if (Prob::B_KMAJOR) { r = idx >> 3; c = idx & 7; }
          else { r = idx % BN; c = idx / BN; }
          store_split(b_hi, b_lo, sw128_offset(r, c), vb[j]);
        }
        fence_async_smem();
        mbar_arrive(&full[stage]);
      }
    }
  } else if (warp == MMA_WARP) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      uint32_t it = 0, tcount = 0;
      bool ok = true;
      bool issued = false;
      for (int tile = blockIdx.x; tile < sched.num_tiles && ok; tile += gridDim.x, tcount++) {
        const int split = tile / tiles_mn;
        const int kb0 = split * sched.kb_per_split;
        int kb1 = kb0 + sched.kb_per_split;
        if (kb1 > sched.kblocks) kb1 = sched.kblocks;
        const uint32_t buf = tcount & 1;
        const uint32_t aphase = (tcount >> 1) & 1;
        if (!mbar_wait(&acc_empty[buf], aphase ^ 1, abort_flag, dev_error)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = kb0; kb < kb1; kb++, it++) {
          const int stage = it % C::STAGES;
          const uint32_t phase = (it / C::STAGES) & 1;
          if (!mbar_wait(&full[stage], phase, abort_flag, dev_error)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_hi = ring + stage * C::STAGE_BYTES;
          const uint32_t a_lo = a_hi + C::A_BYTES;
          const uint32_t b_hi = a_lo + C::A_BYTES;
          const uint32_t b_lo = b_hi + C::B_BYTES;
#pragma unroll
          for (int j = 0; j < BK / 8; j++) {
            const uint32_t koff = j * 32;  // 8 tf32 = 32 bytes along K
            const uint64_t dah = sdesc_sw128(a_hi + koff), dal = sdesc_sw128(a_lo + koff);
            const uint64_t dbh = sdesc_sw128(b_hi + koff), dbl = sdesc_sw128(b_lo + koff);
            const uint32_t first = (kb == kb0 && j == 0) ? 0u : 1u;
            mma_tf32(d_tmem, dal, dbh, C::IDESC, first);
            mma_tf32(d_tmem, dah, dbl, C::IDESC, 1u);
            mma_tf32(d_tmem, dah, dbh, C::IDESC, 1u);
            issued = true;
          }
          mma_commit(&empty[stage]);
        }
        if (!ok) break;
        mma_commit(&acc_full[buf]);
      }
      if (!ok && issued) {
        // make sure no MMA still writes TMEM before it is released
        mma_commit(drain);
        const uint32_t a = smem_u32(drain);
        const unsigned long long t0 = globaltimer();
        while (!mbar_try_wait(a, 0) && globaltimer() - t0 < WAIT_TIMEOUT_NS) {
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint32_t tcount = 0;
    for (int tile = blockIdx.x; tile < sched.num_tiles; tile += gridDim.x, tcount++) {
      const int split = tile / tiles_mn;
      const int mn = tile - split * tiles_mn;
      const int mt = mn % sched.m_tiles, nt = mn / sched.m_tiles;
      const uint32_t buf = tcount & 1;
      const uint32_t aphase = (tcount >> 1) & 1;
      if (!mbar_wait(&acc_full[buf], aphase, abort_flag, dev_error)) break;
      tc_fence_after();
      const int row = mt * BM + q * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; c++) {
        float v[32];
        tmem_ld32(taddr + c * 32, v);
        prob.store(row, nt * BN + c * 32, split, v);
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == MMA_WARP) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

}  // namespace tc
}  // namespace rnn
