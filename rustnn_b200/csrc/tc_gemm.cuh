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
// CTA layout (one CTA per SM, persistent over output tiles):
//   warps 0..4G-1  producers in G groups of four (G = 3 when the ring has
//              at least three stages, else 2) that take K blocks round-robin,
//              so G blocks' global loads are in flight at once:
//              global -> registers -> hi/lo split -> shared memory in the
//              canonical K-major SWIZZLE_128B layout, STAGES-deep ring.  When
//              the B operand is a weight tensor it is pre-packed once per call
//              into that exact shared-memory image (hi and lo) and one thread
//              streams it with cp.async.bulk instead (no register traffic)
//   warp 4G    TMEM allocator + MMA issuer (one elected lane issues)
//   next four  epilogue: tcgen05.ld from a double-buffered TMEM accumulator,
//              so the epilogue of tile i overlaps the main loop of tile i+1
// Tiles are BM=128 rows (TMEM lanes) x BN columns, BK=32 f32 (128 bytes) of K
// per pipeline stage.  Every wait is bounded: on timeout the CTA raises an
// abort flag, all roles drain, TMEM is freed and an error word is set.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>
#include <utility>

namespace rnn {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 32;  // f32 elements of K per stage = one 128-byte swizzle row
constexpr int GROUP_THREADS = 128;  // one producer group = four warps, one A row per thread
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

// One arrival that also announces `bytes` of incoming bulk-copy traffic.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// 1-D bulk copy global -> shared (TMA engine, no tensor map, no multicast);
// completes `bytes` of transaction count on `bar`.  16-byte aligned, size a
// multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst_smem),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 4-D tiled tensor copy global -> shared through a tensor map (TMA, no
// multicast); coordinates innermost first, elements outside the tensor
// (negative included) are filled with zeros.  The innermost coordinate times
// the element size must be a multiple of 16 bytes.  `tmap` is the generic
// address of a __grid_constant__ kernel parameter.
__device__ __forceinline__ void tma_load_4d(uint32_t dst_smem, const void* tmap, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(dst_smem),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// 16-byte asynchronous copy global -> shared through L2 (cp.async.cg, not
// the bulk/TMA engine); src_bytes = 0 zero-fills the 16 bytes and reads
// nothing.  Completion: cp_async_wait_all() in the issuing thread.
__device__ __forceinline__ void cp_async16(uint32_t dst_smem, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst_smem), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ float ld_shared_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ float4 ld_shared_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
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

// try_wait that lets the hardware park the thread for up to `ns`
// nanoseconds; it resumes as soon as the phase completes.
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Bounded wait.  Returns false when the CTA is aborting (another role timed
// out) or when this wait itself ran past WAIT_TIMEOUT_NS.  Waiting threads
// are parked by the suspend hint instead of spinning, so they do not take
// issue slots from the producer warps on the same sub-partition; the abort
// flag and the clock are polled between parks.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* dev_error) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait_hint(a, parity, 20000u)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > WAIT_TIMEOUT_NS) {
      *abort_flag = 1;
      if (dev_error) atomicOr(dev_error, 1);
      return false;
    }
  }
}

// One lane of a converged warp (elect.sync); true in exactly one lane.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
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
// D(tmem) (+)= A(tmem) * B(smem)^T, kind::tf32, one CTA.
__device__ __forceinline__ void mma_tf32_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive columns from registers; thread i of the warp
// writes lane (base lane + i).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

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

// Columns [32c, 32c + 32) of this lane's accumulator row; narrow (STACK)
// tiles hold A*B_hi and A*B_lo in two halves BN columns apart, added here
// exactly as the engine's own epilogue adds them.
template <int BN, bool STACK>
__device__ __forceinline__ void acc_ld32(uint32_t taddr, int c, float (&v)[32]) {
  tmem_ld32(taddr + c * 32, v);
  if constexpr (STACK) {
    float w[32];
    tmem_ld32(taddr + BN + c * 32, w);
#pragma unroll
    for (int e = 0; e < 32; e++) v[e] += w[e];
  }
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

// EXTRA: bytes of problem-owned shared memory after the ring (the halo
// buffers of HALO problems); the ring gets what is left of the budget.
template <int BN_, int EXTRA_ = 0, bool ATM_ = false, bool STACKABLE_ = true>
struct Cfg {
  static constexpr int BN = BN_;
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
  static constexpr int EXTRA = EXTRA_;
  static_assert(EXTRA % 1024 == 0, "EXTRA keeps the barriers 8-byte and the ring 1024-byte aligned");
  // Tiles of up to 64 columns issue each 8-deep K step as two MMAs: one of
  // width 2*BN, A_hi over the stacked [B_hi; B_lo] image (the lo tile follows
  // the hi tile in shared memory, so one descriptor covers both), and one of
  // width BN, A_lo over B_hi.  Columns [0, BN) collect hi*B_hi + lo*B_hi,
  // columns [BN, 2BN) hi*B_lo, and the epilogue adds the halves.  Two MMA
  // instructions instead of three, and no more B read from shared memory
  // than the three plain ones.  (An earlier form, lo and hi each over the
  // whole stacked image, computed the unused lo*lo product and read a third
  // more B; on the 64-channel halo kernels it measured 5 % slower than three
  // plain MMAs; this form is 5 % faster than them: 0.419 -> 0.400 ms.)
  // Problems whose row epilogue reads the accumulator rows themselves
  // (attention) keep the plain form: stacking doubles their TMEM reads and
  // they are epilogue-bound (dh-64 score kernel 0.0253 -> 0.0275 ms stacked).
  static constexpr bool STACK = BN <= 64 && STACKABLE_;
  static constexpr int ACC_COLS = STACK ? 2 * BN : BN;  // columns per accumulator buffer
  // ATM: the A operand (hi and lo) lives in tensor memory: the producers
  // write it with tcgen05.st and the MMA reads it from there, so shared
  // memory carries only B.  TMEM: [0, 2*ACC_COLS) accumulators, then one
  // 64-column slot (32 hi + 32 lo, lane = A row) per ring stage.
  static constexpr bool ATM = ATM_;
  static constexpr int A_COL0 = 2 * ACC_COLS;
  static constexpr int A_BYTES = BM * BK * 4;  // 16 KB
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int A_SMEM = ATM ? 0 : 2 * A_BYTES;     // A hi + lo in the stage, unless in TMEM
  static constexpr int STAGE_BYTES = A_SMEM + 2 * B_BYTES;  // [A hi | A lo |] B hi | B lo
  // 227 KB per CTA minus the alignment slack and barriers below
  static constexpr int RING_BUDGET = 227 * 1024 - 1024 - 256 - EXTRA;
  static constexpr int STAGES_SMEM = RING_BUDGET / STAGE_BYTES;
  static constexpr int STAGES_TMEM = ATM ? (512 - A_COL0) / 64 : 4;
  static constexpr int STAGES_MIN = STAGES_SMEM < STAGES_TMEM ? STAGES_SMEM : STAGES_TMEM;
  static constexpr int STAGES = STAGES_MIN > 4 ? 4 : STAGES_MIN;
  static_assert(STAGES >= 2, "the ring needs two stages");
  static constexpr int TMEM_COLS = ATM ? 512 : (2 * ACC_COLS <= 32) ? 32 : (2 * ACC_COLS <= 64) ? 64
                                   : (2 * ACC_COLS <= 128) ? 128 : (2 * ACC_COLS <= 256) ? 256 : 512;
  // 1024 bytes of alignment slack + barriers
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EXTRA + 1024 + 256;
  static constexpr uint32_t IDESC = idesc_tf32(BM, BN);
  static constexpr uint32_t IDESC2 = idesc_tf32(BM, 2 * BN);  // stacked-B MMA (STACK)
  // Producer groups take K blocks round-robin (block it -> group it % GROUPS),
  // so GROUPS blocks' global loads are in flight.  A group's next block is
  // GROUPS ahead of its last one; its wait on the stage's empty barrier can
  // only tell the awaited phase from the one before it, so a group must never
  // run more than one ring lap ahead: GROUPS <= STAGES.
  static constexpr int GROUPS = STAGES >= 3 ? 3 : 2;
  static_assert(GROUPS <= STAGES, "producer groups may not outrun the stage ring");
  static constexpr int PRODUCER_WARPS = 4 * GROUPS;
  static constexpr int MMA_WARP = PRODUCER_WARPS;     // TMEM allocator + MMA issuer
  static constexpr int FIRST_EPI_WARP = MMA_WARP + 1;  // four epilogue warps follow
  static constexpr int THREADS = (PRODUCER_WARPS + 5) * 32;
  static constexpr int BCH = BN / 16;  // B chunks (4 K values) per producer thread
};

// Work decomposition shared by the host launcher and the kernel.
struct Sched {
  int m_tiles, n_tiles, splits;
  int kblocks;         // total K blocks of BK
  int kb_per_split;    // K blocks per split (last split may get fewer)
  int num_tiles;       // m_tiles * n_tiles * splits
};

// ------------------------------------------------------------------ Prob
//
// A problem type supplies, for one producer thread `gt` (0..127 within its
// group):
//   static constexpr bool B_BULK;          B arrives pre-packed by bulk copy
//   struct TS;                             per-thread tile state
//   void tile_begin(TS&, int m0, int n0, int gt) const;
//   void load_a(const TS&, int kb, int gt, float (&v)[32]) const;
//        the thread's 8 A chunks; chunk j = K values 4c..4c+3 of row r with
//        (r, c) = a_slot(gt, j); zero outside the problem
//   static void a_slot(int gt, int j, int& r, int& c);
//   void load_b(const TS&, int kb, int gt, float (&v)[BCH*4]) const;   (!B_BULK)
//   static void b_slot(int gt, int j, int& r, int& c);                   (!B_BULK)
//   const void* b_src(int n_tile, int kb) const;  packed (hi, lo) image (B_BULK)
//   void store(int row, int col0, int split, const float (&v)[32]) const;
//        epilogue: 32 consecutive accumulator columns of one row
//   int M, N;

// Adapter for problems written against the per-chunk interface
//   A_KMAJOR / B_KMAJOR, load_a(row, k4, v4), load_b(row, k4, v4), store.
template <class P, int BN>
struct ChunkProb : P {
  static constexpr bool B_BULK = false;
  struct TS {
    int m0, n0;
  };
  __device__ __forceinline__ void tile_begin(TS& ts, int m0, int n0, int) const {
    ts.m0 = m0;
    ts.n0 = n0;
  }
  static __device__ __forceinline__ void a_slot(int gt, int j, int& r, int& c) {
    if (P::A_KMAJOR) { r = (gt >> 3) + 16 * j; c = gt & 7; }
    else { r = gt; c = j; }
  }
  static __device__ __forceinline__ void b_slot(int gt, int j, int& r, int& c) {
    const int idx = gt + 128 * j;
    if (P::B_KMAJOR) { r = idx >> 3; c = idx & 7; }
    else { r = idx % BN; c = idx / BN; }
  }
  __device__ __forceinline__ void load_a(const TS& ts, int kb, int gt, float (&v)[32]) const {
#pragma unroll
    for (int j = 0; j < 8; j++) {
      int r, c;
      a_slot(gt, j, r, c);
      float t[4];
      P::load_a(ts.m0 + r, kb * BK + 4 * c, t);
      v[4 * j] = t[0]; v[4 * j + 1] = t[1]; v[4 * j + 2] = t[2]; v[4 * j + 3] = t[3];
    }
  }
  template <int NB>
  __device__ __forceinline__ void load_b(const TS& ts, int kb, int gt, float (&v)[NB]) const {
#pragma unroll
    for (int j = 0; j < NB / 4; j++) {
      int r, c;
      b_slot(gt, j, r, c);
      float t[4];
      P::load_b(ts.n0 + r, kb * BK + 4 * c, t);
      v[4 * j] = t[0]; v[4 * j + 1] = t[1]; v[4 * j + 2] = t[2]; v[4 * j + 3] = t[3];
    }
  }
  __device__ __forceinline__ const void* b_src(int, int) const { return nullptr; }
};

// Problems that stage a halo of the gathered operand in shared memory
// declare HALO_BYTES (both buffers) and TAPS, and supply
//   void halo_issue(uint32_t halo, int buf, int m_tile, int kbs, int ptid, int npt) const;
//        cp.async the halo of the K-block group that starts at K block kbs
//        (TAPS consecutive K blocks) of row tile m_tile into buffer buf;
//        producer thread ptid of npt
//   void load_a_halo(uint32_t halo, int buf, const TS&, int tap, int gt, float (&v)[32]) const;
// A HALO problem may set HALO_TMA: one producer thread then fills a halo
// buffer with a tensor copy instead of every producer issuing cp.async,
//   void halo_tma(uint32_t halo, int buf, uint64_t* bar, int m_tile, int kbs) const;
//        arrive.expect_tx on bar and start the copy of buffer buf,
// and the producers wait on that buffer's barrier before reading it.  Under
// split-K the launcher makes every split's K range a whole number of groups
// (kb_per_split a multiple of TAPS); groups start at the split's first block.
template <class P, class = void>
struct prob_halo {
  static constexpr int value = 0;
};
template <class P>
struct prob_halo<P, std::void_t<decltype(P::HALO_BYTES)>> {
  static constexpr int value = P::HALO_BYTES;
};
template <class P, class = void>
struct prob_halo_tma {
  static constexpr bool value = false;
};
template <class P>
struct prob_halo_tma<P, std::void_t<decltype(P::HALO_TMA)>> {
  static constexpr bool value = P::HALO_TMA;
};
// Problems with STATS = true can have the epilogue sum every output column
// over the rows (f64, per CTA, in shared memory after the halo) and supply
//   bool stats_on() const;                       runtime switch
//   void stats_flush(const double* sm) const;    all threads, after the tiles
// sm = [BN/32 chunks][2 (sum, sum of squares)][128 epilogue threads]
template <class P, class = void>
struct prob_stats {
  static constexpr bool value = false;
};
template <class P>
struct prob_stats<P, std::void_t<decltype(P::STATS)>> {
  static constexpr bool value = P::STATS;
};
template <int BN>
constexpr int stats_bytes() { return (BN / 32) * 2 * 128 * 8; }
// Problems that need a whole accumulator row at once (a row softmax, a row
// dot product) declare ROW_EPI_WARP_BYTES (shared memory per epilogue warp,
// possibly 0) and supply
//   template <int BN, bool STACK>
//   void epi_row(int m_tile, int n_tile, int q, int lane, uint32_t taddr, uint8_t* wsm) const;
// called by all 32 lanes of epilogue warp q (0..3) in place of store(): the
// warp owns accumulator rows q*32 + lane of the tile at TMEM address taddr
// (lane quarter and buffer applied) and reads them with acc_ld32 (warp-wide,
// .sync.aligned); wsm is the warp's own shared memory.
template <class P, class = void>
struct prob_rowepi {
  static constexpr bool value = false;
  static constexpr int bytes = 0;
};
template <class P>
struct prob_rowepi<P, std::void_t<decltype(P::ROW_EPI_WARP_BYTES)>> {
  static constexpr bool value = true;
  static constexpr int bytes = (4 * P::ROW_EPI_WARP_BYTES + 1023) / 1024 * 1024;
};
template <class P, int BN>
struct prob_extra_bn {
  static constexpr int value =
      prob_halo<P>::value + (prob_stats<P>::value ? stats_bytes<BN>() : 0) + prob_rowepi<P>::bytes;
};
// Problems with A_BULK = true supply the A operand pre-packed, like a bulk
// B: const void* a_src(int m_tile, int kb) const returns the [hi | lo] image
// of that 128-row tile and K block (K-major SWIZZLE_128B rows), and load_a
// is not called.
template <class P, class = void>
struct prob_abulk {
  static constexpr bool value = false;
};
template <class P>
struct prob_abulk<P, std::void_t<decltype(P::A_BULK)>> {
  static constexpr bool value = P::A_BULK;
};
// HALO problems may set A_TMEM: their producers write A into tensor memory.
template <class P, class = void>
struct prob_atm {
  static constexpr bool value = false;
};
template <class P>
struct prob_atm<P, std::void_t<decltype(P::A_TMEM)>> {
  static constexpr bool value = P::A_TMEM;
};

// ------------------------------------------------------------------ kernel

template <class Prob, int BN>
using CfgOf = Cfg<BN, prob_extra_bn<Prob, BN>::value, prob_atm<Prob>::value, !prob_rowepi<Prob>::value>;

// Column sums over the warp's 32 rows: v holds this lane's row; lane l
// returns (sum, sum of squares) of column l.  Recursive halving: at each of
// the five levels a lane keeps the half of its columns that its lane bit
// selects and adds the partner's copy; the first two levels in f32 (sums of
// at most four rows), the last three in f64.
__device__ __forceinline__ void warp_colsum2(const float (&v)[32], double& s_out, double& q_out) {
  const int lane = threadIdx.x & 31;
  float a[16], b[16];
  {
    const bool up = lane & 16;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const float lo = v[i], hi = v[i + 16];
      a[i] = (up ? hi : lo) + __shfl_xor_sync(0xffffffffu, up ? lo : hi, 16);
      const float lo2 = lo * lo, hi2 = hi * hi;
      b[i] = (up ? hi2 : lo2) + __shfl_xor_sync(0xffffffffu, up ? lo2 : hi2, 16);
    }
  }
  double da[8], db[8];
  {
    const bool up = lane & 8;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float ka = up ? a[i + 8] : a[i], sa = up ? a[i] : a[i + 8];
      const float kb = up ? b[i + 8] : b[i], sb = up ? b[i] : b[i + 8];
      da[i] = (double)ka + (double)__shfl_xor_sync(0xffffffffu, sa, 8);
      db[i] = (double)kb + (double)__shfl_xor_sync(0xffffffffu, sb, 8);
    }
  }
#pragma unroll
  for (int k = 4; k >= 1; k >>= 1) {
    const bool up = lane & k;
#pragma unroll
    for (int i = 0; i < k; i++) {
      const double ka = up ? da[i + k] : da[i], sa = up ? da[i] : da[i + k];
      const double kb = up ? db[i + k] : db[i], sb = up ? db[i] : db[i + k];
      da[i] = ka + __shfl_xor_sync(0xffffffffu, sa, k);
      db[i] = kb + __shfl_xor_sync(0xffffffffu, sb, k);
    }
  }
  s_out = da[0];
  q_out = db[0];
}

template <int BN, class Prob>
__global__ void __launch_bounds__(CfgOf<Prob, BN>::THREADS, 1)
    tc3_gemm_kernel(const __grid_constant__ Prob prob, const Sched sched, int* dev_error) {
  using C = CfgOf<Prob, BN>;
  constexpr bool HALO = prob_halo<Prob>::value > 0;
  constexpr bool HTMA = HALO && prob_halo_tma<Prob>::value;
  constexpr bool STATS = prob_stats<Prob>::value;
  constexpr bool ROWEPI = prob_rowepi<Prob>::value;
  static_assert(!C::ATM || Prob::B_BULK, "A in tensor memory needs a bulk-copied B");
  constexpr bool A_BULK = prob_abulk<Prob>::value;
  static_assert(!(A_BULK && (C::ATM || HALO)), "a bulk-copied A lives in shared memory");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned operand ring
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t ring = (raw_addr + 1023u) & ~1023u;
  uint8_t* ring_ptr = smem_raw + (ring - raw_addr);
  const uint32_t halo = ring + C::STAGES * C::STAGE_BYTES;  // HALO problems' buffers
  // STATS problems' per-thread column sums follow the halo
  double* stats_sm = reinterpret_cast<double*>(ring_ptr + C::STAGES * C::STAGE_BYTES + prob_halo<Prob>::value);
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring_ptr + C::STAGES * C::STAGE_BYTES + C::EXTRA);
  uint64_t* full = bars;                      // [STAGES] producers -> MMA
  uint64_t* empty = bars + C::STAGES;         // [STAGES] MMA commit -> producers
  uint64_t* acc_full = bars + 2 * C::STAGES;  // [2] MMA commit -> epilogue
  uint64_t* acc_empty = acc_full + 2;         // [2] epilogue -> MMA
  uint64_t* drain = acc_empty + 2;            // [1] abort path
  uint64_t* halo_bar = drain + 1;             // [1] all producers: a halo buffer is filled / released
  uint64_t* halo_full = halo_bar + 1;         // [2] HALO_TMA: the tensor copy of a halo buffer landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(halo_full + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      // one group's 128 threads, plus the bulk-copy thread's expect_tx arrival
      mbar_init(&full[s], GROUP_THREADS + ((Prob::B_BULK || A_BULK) ? 1 : 0));
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4 * 32);
    }
    mbar_init(drain, 1);
    mbar_init(halo_bar, C::PRODUCER_WARPS * 32);
    mbar_init(&halo_full[0], 1);
    mbar_init(&halo_full[1], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == C::MMA_WARP) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles_mn = sched.m_tiles * sched.n_tiles;

  if (warp < C::PRODUCER_WARPS) {
   if constexpr (HALO) {
    // ---------------------------------------------------- halo producers
    // Each tile's K range [kb0, kb1) runs in groups of TAPS blocks from kb0
    // (the conv fwd/dgrad: one 32-channel block, every tap; the wgrad: TAPS
    // image rows).  All producer threads fill the halo of the next group
    // into the spare buffer while the current one is read, and meet on
    // halo_bar at every group boundary: it publishes the landed halo and
    // releases the buffer the next prefetch overwrites.  Groups keep taking
    // K blocks round-robin as below.
    const int group = warp >> 2;
    const int gt = threadIdx.x & (GROUP_THREADS - 1);
    const int ptid = threadIdx.x;
    constexpr int NPT = C::PRODUCER_WARPS * 32;
    constexpr int TAPS = Prob::TAPS;
    auto mt_of = [&](int tile) { return (tile % tiles_mn) % sched.m_tiles; };
    auto kb0_of = [&](int tile) { return (tile / tiles_mn) * sched.kb_per_split; };
    uint32_t it = 0, hc = 0;
    bool ok = true;
    // HALO_TMA: sequence numbers of the last halo copy started and the last
    // one waited for (copy s fills buffer s & 1 for the (s >> 1)-th time)
    int tma_issued = -1, tma_waited = -1;
    if (blockIdx.x < sched.num_tiles) {
      if constexpr (HTMA) {
        if (ptid == 0) prob.halo_tma(halo, 0, &halo_full[0], mt_of(blockIdx.x), kb0_of(blockIdx.x));
        tma_issued = 0;
      } else {
        prob.halo_issue(halo, 0, mt_of(blockIdx.x), kb0_of(blockIdx.x), ptid, NPT);
      }
    }
    if constexpr (!HTMA) cp_async_commit();
    for (int tile = blockIdx.x; tile < sched.num_tiles && ok; tile += gridDim.x) {
      const int mn = tile % tiles_mn;
      const int mt = mn % sched.m_tiles, nt = mn / sched.m_tiles;
      const int kb0 = kb0_of(tile);
      const int kb1 = kb0 + sched.kb_per_split < sched.kblocks ? kb0 + sched.kb_per_split : sched.kblocks;
      typename Prob::TS ts;
      prob.tile_begin(ts, mt * BM, nt * BN, gt);
      for (int kb = kb0; kb < kb1; kb++, it++) {
        const int tap = (kb - kb0) % TAPS;
        if (tap == 0) {
          if constexpr (!HTMA) cp_async_wait_all();
          // every producer is done with the buffer the next copy overwrites
          mbar_arrive(halo_bar);
          if (!mbar_wait(halo_bar, hc & 1, abort_flag, dev_error)) { ok = false; break; }
          // the next group: the rest of this tile's K range, else the next tile's first
          int ntile = tile, nkbs = kb + TAPS;
          if (nkbs >= kb1) {
            ntile = tile + gridDim.x;
            nkbs = ntile < sched.num_tiles ? kb0_of(ntile) : 0;
          }
          if constexpr (HTMA) {
            if (ntile < sched.num_tiles) {
              if (ptid == 0) prob.halo_tma(halo, (hc + 1) & 1, &halo_full[(hc + 1) & 1], mt_of(ntile), nkbs);
              tma_issued = (int)hc + 1;
            }
            // this group's halo (copy hc) has landed
            if (!mbar_wait(&halo_full[hc & 1], (hc >> 1) & 1, abort_flag, dev_error)) { ok = false; break; }
            tma_waited = (int)hc;
          } else {
            if (ntile < sched.num_tiles) {
              prob.halo_issue(halo, (hc + 1) & 1, mt_of(ntile), nkbs, ptid, NPT);
            }
            cp_async_commit();
          }
          hc++;
        }
        if ((int)(it % C::GROUPS) != group) continue;
        const int stage = it % C::STAGES;
        const uint32_t phase = (it / C::STAGES) & 1;
        float va[32];
        prob.load_a_halo(halo, (hc - 1) & 1, ts, tap, gt, va);
        // warp-uniform outcome: tcgen05.st below is .sync.aligned
        if (!__all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1, abort_flag, dev_error))) {
          ok = false;
          break;
        }
        const uint32_t a_hi = ring + stage * C::STAGE_BYTES;
        const uint32_t a_lo = a_hi + C::A_BYTES;
        const uint32_t b_hi = a_hi + C::A_SMEM;
        if (gt == 0) {
          mbar_arrive_expect_tx(&full[stage], 2 * C::B_BYTES);
          bulk_g2s(b_hi, prob.b_src(nt, kb), 2 * C::B_BYTES, &full[stage]);
        }
        if constexpr (C::ATM) {
          // thread gt owns A row gt = TMEM lane gt (warp w of a group
          // reaches lanes 32*(w%4) ..; groups are 4 warps)
          uint32_t hi[32], lo[32];
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const float h = tf32_round(va[j]);
            hi[j] = __float_as_uint(h);
            lo[j] = __float_as_uint(va[j] - h);
          }
          const uint32_t acol = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16) + C::A_COL0 + stage * 64;
          tmem_st32(acol, hi);
          tmem_st32(acol + 32, lo);
          tmem_wait_st();
          tc_fence_before();
          (void)a_lo;
        } else {
#pragma unroll
          for (int j = 0; j < 8; j++) {
            int r, c;
            Prob::a_slot(gt, j, r, c);
            const float t[4] = {va[4 * j], va[4 * j + 1], va[4 * j + 2], va[4 * j + 3]};
            store_split(a_hi, a_lo, sw128_offset(r, c), t);
          }
          fence_async_smem();
        }
        mbar_arrive(&full[stage]);
      }
    }
    if constexpr (HTMA) {
      // on an abort, let the copies still in flight (at most two) land
      // before the CTA exits
      if (!ok && ptid == 0) {
        for (int sq = tma_waited + 1; sq <= tma_issued; sq++) {
          const uint32_t a = smem_u32(&halo_full[sq & 1]);
          const unsigned long long t0 = globaltimer();
          while (!mbar_try_wait(a, (sq >> 1) & 1) && globaltimer() - t0 < WAIT_TIMEOUT_NS) {
          }
        }
      }
    } else {
      cp_async_wait_all();
    }
   } else {
    // ---------------------------------------------------------- producers
    const int group = warp >> 2;                 // 0 .. GROUPS-1
    const int gt = threadIdx.x & (GROUP_THREADS - 1);
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < sched.num_tiles && ok; tile += gridDim.x) {
      const int split = tile / tiles_mn;
      const int mn = tile - split * tiles_mn;
      const int mt = mn % sched.m_tiles, nt = mn / sched.m_tiles;
      const int kb0 = split * sched.kb_per_split;
      int kb1 = kb0 + sched.kb_per_split;
      if (kb1 > sched.kblocks) kb1 = sched.kblocks;
      typename Prob::TS ts;
      prob.tile_begin(ts, mt * BM, nt * BN, gt);
      for (int kb = kb0; kb < kb1; kb++, it++) {
        if ((int)(it % C::GROUPS) != group) continue;
        const int stage = it % C::STAGES;
        const uint32_t phase = (it / C::STAGES) & 1;
        float va[32];
        if constexpr (!A_BULK) prob.load_a(ts, kb, gt, va);
        constexpr int NB = Prob::B_BULK ? 4 : C::BCH * 4;
        float vb[NB];
        if constexpr (!Prob::B_BULK) prob.template load_b<NB>(ts, kb, gt, vb);
        // warp-uniform outcome: the ATM path's tcgen05.st is .sync.aligned
        if (!__all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1, abort_flag, dev_error))) {
          ok = false;
          break;
        }
        const uint32_t a_hi = ring + stage * C::STAGE_BYTES;
        const uint32_t a_lo = a_hi + C::A_BYTES;
        const uint32_t b_hi = a_hi + C::A_SMEM;
        const uint32_t b_lo = b_hi + C::B_BYTES;
        if constexpr (Prob::B_BULK || A_BULK) {
          if (gt == 0) {
            mbar_arrive_expect_tx(&full[stage], (Prob::B_BULK ? 2 * C::B_BYTES : 0) + (A_BULK ? 2 * C::A_BYTES : 0));
            if constexpr (Prob::B_BULK) bulk_g2s(b_hi, prob.b_src(nt, kb), 2 * C::B_BYTES, &full[stage]);
            if constexpr (A_BULK) bulk_g2s(a_hi, prob.a_src(mt, kb), 2 * C::A_BYTES, &full[stage]);
          }
        }
        if constexpr (A_BULK) {
          (void)a_lo;
        } else if constexpr (C::ATM) {
          // load_a returned the thread's own A row (a_slot(gt, j) == (gt, j)):
          // row gt = TMEM lane gt
          uint32_t hi[32], lo[32];
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const float h = tf32_round(va[j]);
            hi[j] = __float_as_uint(h);
            lo[j] = __float_as_uint(va[j] - h);
          }
          const uint32_t acol = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16) + C::A_COL0 + stage * 64;
          tmem_st32(acol, hi);
          tmem_st32(acol + 32, lo);
          tmem_wait_st();
          tc_fence_before();
          (void)a_lo;
        } else {
#pragma unroll
          for (int j = 0; j < 8; j++) {
            int r, c;
            Prob::a_slot(gt, j, r, c);
            const float t[4] = {va[4 * j], va[4 * j + 1], va[4 * j + 2], va[4 * j + 3]};
            store_split(a_hi, a_lo, sw128_offset(r, c), t);
          }
        }
        if constexpr (!Prob::B_BULK) {
#pragma unroll
          for (int j = 0; j < NB / 4; j++) {
            int r, c;
            Prob::b_slot(gt, j, r, c);
            const float t[4] = {vb[4 * j], vb[4 * j + 1], vb[4 * j + 2], vb[4 * j + 3]};
            store_split(b_hi, b_lo, sw128_offset(r, c), t);
          }
        }
        if constexpr (!C::ATM) fence_async_smem();
        mbar_arrive(&full[stage]);
      }
    }
    (void)lane;
   }
  } else if (warp == C::MMA_WARP) {
    // ---------------------------------------------------------- MMA issuer
    // The whole warp walks the schedule, waits and builds the descriptors
    // (warp-uniform values); one elected lane issues the MMAs and commits.
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
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_empty[buf], aphase ^ 1, abort_flag, dev_error))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * C::ACC_COLS;
      for (int kb = kb0; kb < kb1; kb++, it++) {
        const int stage = it % C::STAGES;
        const uint32_t phase = (it / C::STAGES) & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort_flag, dev_error))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_hi = ring + stage * C::STAGE_BYTES;
        const uint32_t a_lo = a_hi + C::A_BYTES;
        const uint32_t b_hi = a_hi + C::A_SMEM;
        const uint32_t b_lo = b_hi + C::B_BYTES;
        if (elect_one()) {
#pragma unroll
          for (int j = 0; j < BK / 8; j++) {
            const uint32_t koff = j * 32;  // 8 tf32 = 32 bytes along K
            const uint64_t dah = sdesc_sw128(a_hi + koff), dal = sdesc_sw128(a_lo + koff);
            const uint64_t dbh = sdesc_sw128(b_hi + koff), dbl = sdesc_sw128(b_lo + koff);
            const uint32_t first = (kb == kb0 && j == 0) ? 0u : 1u;
            if constexpr (C::ATM) {
              // A hi at columns [stage*64, +32), lo at [+32, +64); 8 columns per K step
              const uint32_t tah = tmem_base + C::A_COL0 + stage * 64 + j * 8, tal = tah + 32;
              if constexpr (C::STACK) {
                mma_tf32_ta(d_tmem, tah, dbh, C::IDESC2, first);  // hi * [hi; lo]
                mma_tf32_ta(d_tmem, tal, dbh, C::IDESC, 1u);      // lo * hi (first BN columns)
              } else {
                mma_tf32_ta(d_tmem, tal, dbh, C::IDESC, first);  // lo * hi
                mma_tf32_ta(d_tmem, tah, dbl, C::IDESC, 1u);     // hi * lo
                mma_tf32_ta(d_tmem, tah, dbh, C::IDESC, 1u);     // hi * hi
              }
              (void)dah;
              (void)dal;
            } else if constexpr (C::STACK) {
              mma_tf32(d_tmem, dah, dbh, C::IDESC2, first);  // hi * [hi; lo]
              mma_tf32(d_tmem, dal, dbh, C::IDESC, 1u);      // lo * hi (first BN columns)
              (void)dbl;
            } else {
              mma_tf32(d_tmem, dal, dbh, C::IDESC, first);  // lo * hi
              mma_tf32(d_tmem, dah, dbl, C::IDESC, 1u);     // hi * lo
              mma_tf32(d_tmem, dah, dbh, C::IDESC, 1u);     // hi * hi
            }
          }
          mma_commit(&empty[stage]);
        }
        __syncwarp();
        issued = true;
      }
      if (!ok) break;
      if (elect_one()) mma_commit(&acc_full[buf]);
      __syncwarp();
    }
    if (!ok && issued) {
      // make sure no MMA still writes TMEM before it is released
      if (elect_one()) {
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
    const int et = (warp - C::FIRST_EPI_WARP) * 32 + lane;
    bool stats = false;
    if constexpr (STATS) {
      stats = prob.stats_on();
      if (stats)
        for (int c = 0; c < 2 * (BN / 32); c++) stats_sm[c * 128 + et] = 0.0;
    }
    uint32_t tcount = 0;
    for (int tile = blockIdx.x; tile < sched.num_tiles; tile += gridDim.x, tcount++) {
      const int split = tile / tiles_mn;
      const int mn = tile - split * tiles_mn;
      const int mt = mn % sched.m_tiles, nt = mn / sched.m_tiles;
      const uint32_t buf = tcount & 1;
      const uint32_t aphase = (tcount >> 1) & 1;
      // warp-uniform outcome: tcgen05.ld below is .sync.aligned
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], aphase, abort_flag, dev_error))) break;
      tc_fence_after();
      const int row = mt * BM + q * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * C::ACC_COLS;
      if constexpr (ROWEPI) {
        uint8_t* wsm = ring_ptr + C::STAGES * C::STAGE_BYTES + prob_halo<Prob>::value +
                       (STATS ? stats_bytes<BN>() : 0) + (warp - C::FIRST_EPI_WARP) * Prob::ROW_EPI_WARP_BYTES;
        prob.template epi_row<BN, C::STACK>(mt, nt, q, lane, taddr, wsm);
        (void)row;
      }
      if constexpr (!ROWEPI) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; c++) {
          float v[32];
          tmem_ld32(taddr + c * 32, v);
          if constexpr (C::STACK) {
            float w[32];
            tmem_ld32(taddr + BN + c * 32, w);
#pragma unroll
            for (int e = 0; e < 32; e++) v[e] += w[e];
          }
          prob.store(row, nt * BN + c * 32, split, v);
          if constexpr (STATS) {
            if (stats) {
              double cs, cq;
              warp_colsum2(v, cs, cq);
              stats_sm[(2 * c) * 128 + et] += cs;
              stats_sm[(2 * c + 1) * 128 + et] += cq;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == C::MMA_WARP) tmem_dealloc(tmem_base, C::TMEM_COLS);
  if constexpr (STATS) {
    if (prob.stats_on()) prob.stats_flush(stats_sm);
  }
}

// ------------------------------------------------------------------ packing
//
// Writes the B operand of every (n tile, K block) as the shared-memory image
// the MMA reads: [hi tile | lo tile], each BN rows x 128 bytes in the
// K-major SWIZZLE_128B layout.  `Src` maps (row, k) of the B operand to a
// value (zero outside).  One thread per 16-byte chunk.
template <int BN, class Src>
__global__ void pack_b_kernel(const Src src, int n_tiles, int kblocks, float* __restrict__ out) {
  const long total = (long)n_tiles * kblocks * BN * 8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int c = (int)(i & 7);
    const long rest = i >> 3;
    const int r = (int)(rest % BN);
    const long tk = rest / BN;  // n_tile * kblocks + kb
    const int kb = (int)(tk % kblocks), nt = (int)(tk / kblocks);
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; e++) v[e] = src(nt * BN + r, kb * BK + 4 * c + e);
    float h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      h[e] = tf32_round(v[e]);
      l[e] = v[e] - h[e];
    }
    char* img = reinterpret_cast<char*>(out) + tk * (2L * BN * BK * 4);
    const uint32_t off = static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
    *reinterpret_cast<float4*>(img + off) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(img + BN * BK * 4 + off) = make_float4(l[0], l[1], l[2], l[3]);
  }
}

}  // namespace tc
}  // namespace rnn
