// Fused batched attention: attn.rs Core::forward (:148-223) and
// Core::backward (:226-343) for every (image, head) in one launch.
//
// One CTA per (head, image, query chunk).  K and V of the (image, head) and
// the chunk's Q / dO rows live in shared memory (rows padded to dh+1 floats
// so column walks are bank-conflict free), next to the chunk's score block.
// The contractions are register-tiled f32 FFMA: a warp owns 8 rows, a lane
// owns columns lane + 32*j, so A reads are warp broadcasts and B reads hit 32
// distinct banks.  Softmax is one warp per row.
//
// Outputs follow the reference exactly: P is written to HBM (the backward
// reads it, attn.rs:186-211), O goes to [n, tq, h*dh], and the backward
// accumulates (+=) into strided dq / dkv (attn.rs:274, 323, 327) and into
// dtau / drel.  dtau and drel are reduced without atomics: each CTA writes a
// partial (drel built row by row: within one query row every key maps to a
// distinct relative-position index), and a second kernel sums the partials
// in a fixed order.  The query-chunked backward runs one launch per chunk so
// the += into dK / dV never races.
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "common.cuh"

namespace rnn {

// ---------------------------------------------------------------- rel_index

// attn.rs:23-72: the relative-position bias index of every (query, key) pair.
static int rel_index_host(int th, int tw, int mh, int mw, std::vector<uint32_t>* idx) {
  int sy, sx, scale, oy, ox;
  if (mh == th) {
    sy = 2 * th - 1; sx = 2 * tw - 1; scale = 1; oy = th - 1; ox = tw - 1;
  } else {
    sy = 2 * (th - 1) + mh; sx = 2 * (tw - 1) + mw; scale = 2; oy = mh - 1; ox = mw - 1;
  }
  if (idx) {
    idx->clear();
    idx->reserve((size_t)th * tw * mh * mw);
    for (int qy = 0; qy < th; qy++)
      for (int qx = 0; qx < tw; qx++)
        for (int my = 0; my < mh; my++)
          for (int mx = 0; mx < mw; mx++)
            idx->push_back((uint32_t)((scale * qy - my + oy) * sx + (scale * qx - mx + ox)));
  }
  return sy * sx;
}

// Device copies of the index table, one per (device, geometry), built once.
static std::mutex g_rel_mu;
static std::map<std::tuple<int, int, int, int, int>, uint32_t*> g_rel_tables;

static int rel_table(rnn_ctx* ctx, int th, int tw, int mh, int mw, const uint32_t** out, int* nrel) {
  std::vector<uint32_t> idx;
  *nrel = rel_index_host(th, tw, mh, mw, &idx);
  std::lock_guard<std::mutex> lock(g_rel_mu);
  auto key = std::make_tuple(ctx->device, th, tw, mh, mw);
  auto it = g_rel_tables.find(key);
  if (it == g_rel_tables.end()) {
    uint32_t* d = nullptr;
    RNN_CUDA(cudaMalloc(&d, idx.size() * sizeof(uint32_t)));
    RNN_CUDA(cudaMemcpy(d, idx.data(), idx.size() * sizeof(uint32_t), cudaMemcpyHostToDevice));
    it = g_rel_tables.emplace(key, d).first;
  }
  *out = it->second;
  return RNN_OK;
}

// ---------------------------------------------------------------- kernels

struct AttnArgs {
  int n, h, tq, tk, nrel, mask;
  const uint32_t* relidx;
  const float* q;
  int qstride, qoff;
  const float* kv;
  int kvstride, koff, voff;
  const float* tau;
  const float* rel;
  float* p;        // forward writes P
  const float* pin;  // backward reads P
  float* o;
  const float* dout;
  float* dq;
  float* dkv;
  float* part;  // backward partials [n][nchunk][h][1 + nrel]
  int tqc, nchunk, chunk;
};

constexpr int ATT_THREADS = 256;
constexpr int ATT_WARPS = ATT_THREADS / 32;

// out(i, j) = sum_k fa(i, k) * fb(k, j) for i < M, j < N.  Warp w owns rows
// w*TM.. (stepping by 8*TM), lane l owns columns l + 32*jj (jj < TN).
template <int TM, int TN, class FA, class FB, class FO>
__device__ __forceinline__ void tile_mm(int M, int N, int K, FA fa, FB fb, FO fo) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  for (int i0 = w * TM; i0 < M; i0 += ATT_WARPS * TM)
    for (int jb = 0; jb < N; jb += 32 * TN) {
      float acc[TM][TN];
#pragma unroll
      for (int ii = 0; ii < TM; ii++)
#pragma unroll
        for (int jj = 0; jj < TN; jj++) acc[ii][jj] = 0.0f;
      for (int k = 0; k < K; k++) {
        float av[TM], bv[TN];
#pragma unroll
        for (int ii = 0; ii < TM; ii++) av[ii] = (i0 + ii < M) ? fa(i0 + ii, k) : 0.0f;
#pragma unroll
        for (int jj = 0; jj < TN; jj++) {
          const int j = jb + l + 32 * jj;
          bv[jj] = (j < N) ? fb(k, j) : 0.0f;
        }
#pragma unroll
        for (int ii = 0; ii < TM; ii++)
#pragma unroll
          for (int jj = 0; jj < TN; jj++) acc[ii][jj] = fmaf(av[ii], bv[jj], acc[ii][jj]);
      }
#pragma unroll
      for (int ii = 0; ii < TM; ii++)
#pragma unroll
        for (int jj = 0; jj < TN; jj++) {
          const int i = i0 + ii, j = jb + l + 32 * jj;
          if (i < M && j < N) fo(i, j, acc[ii][jj]);
        }
    }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int DH>
__global__ void __launch_bounds__(ATT_THREADS) attn_fwd_kernel(const AttnArgs a) {
  extern __shared__ float sm[];
  constexpr int LD = DH + 1;
  constexpr int TND = DH >= 32 ? DH / 32 : 1;
  const int hd = blockIdx.x, img = blockIdx.y;
  const int q0 = blockIdx.z * a.tqc;
  const int tqc = min(a.tqc, a.tq - q0);
  const int tk = a.tk, c = a.h * DH;
  float* Qs = sm;
  float* Ks = Qs + a.tqc * LD;
  float* Vs = Ks + tk * LD;
  float* Ss = Vs + tk * LD;
  for (int e = threadIdx.x; e < tqc * DH; e += ATT_THREADS) {
    const int r = e / DH, d = e - r * DH;
    Qs[r * LD + d] = a.q[((size_t)img * a.tq + q0 + r) * a.qstride + a.qoff + hd * DH + d];
  }
  for (int e = threadIdx.x; e < tk * DH; e += ATT_THREADS) {
    const int r = e / DH, d = e - r * DH;
    const float* row = a.kv + ((size_t)img * tk + r) * a.kvstride + hd * DH + d;
    Ks[r * LD + d] = row[a.koff];
    Vs[r * LD + d] = row[a.voff];
  }
  __syncthreads();
  // S = tau * Q K^T + rel[relidx], diagonal masked (attn.rs:181-195)
  const float t = a.tau[hd];
  const float* rb = a.rel + (size_t)hd * a.nrel;
  tile_mm<8, 2>(
      tqc, tk, DH, [&](int i, int k) { return Qs[i * LD + k]; }, [&](int k, int j) { return Ks[j * LD + k]; },
      [&](int i, int j, float v) {
        const int qi = q0 + i;
        float val = t * v + rb[a.relidx[(size_t)qi * tk + j]];
        if (a.mask && j == qi) val = -INFINITY;
        Ss[i * tk + j] = val;
      });
  __syncthreads();
  // row softmax (attn.rs:191-211); P to HBM for the backward
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  for (int i = w; i < tqc; i += ATT_WARPS) {
    float* row = Ss + i * tk;
    float mx = -INFINITY;
    for (int j = l; j < tk; j += 32) mx = fmaxf(mx, row[j]);
    mx = warp_max(mx);
    float sum = 0.0f;
    for (int j = l; j < tk; j += 32) {
      const float e = row[j] == -INFINITY ? 0.0f : expf(row[j] - mx);
      row[j] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    const float inv = 1.0f / sum;
    float* prow = a.p + (((size_t)img * a.h + hd) * a.tq + q0 + i) * tk;
    for (int j = l; j < tk; j += 32) {
      const float pv = row[j] * inv;
      row[j] = pv;
      prow[j] = pv;
    }
  }
  __syncthreads();
  // O = P V (attn.rs:213-220)
  tile_mm<8, TND>(
      tqc, DH, tk, [&](int i, int k) { return Ss[i * tk + k]; }, [&](int k, int j) { return Vs[k * LD + j]; },
      [&](int i, int j, float v) { a.o[((size_t)img * a.tq + q0 + i) * c + hd * DH + j] = v; });
}

template <int DH>
__global__ void __launch_bounds__(ATT_THREADS) attn_bwd_kernel(const AttnArgs a) {
  extern __shared__ float sm[];
  constexpr int LD = DH + 1;
  constexpr int TND = DH >= 32 ? DH / 32 : 1;
  const int hd = blockIdx.x, img = blockIdx.y;
  const int q0 = a.chunk * a.tqc;
  const int tqc = min(a.tqc, a.tq - q0);
  const int tk = a.tk, c = a.h * DH, nrel = a.nrel;
  float* Ks = sm;
  float* Vs = Ks + tk * LD;
  float* Qs = Vs + tk * LD;
  float* Ds = Qs + a.tqc * LD;  // dO chunk
  float* Ps = Ds + a.tqc * LD;  // P chunk
  float* Gs = Ps + a.tqc * tk;  // dP -> dS
  float* Rs = Gs + a.tqc * tk;  // drel partial [nrel]
  __shared__ float red[ATT_WARPS];
  for (int e = threadIdx.x; e < tk * DH; e += ATT_THREADS) {
    const int r = e / DH, d = e - r * DH;
    const float* row = a.kv + ((size_t)img * tk + r) * a.kvstride + hd * DH + d;
    Ks[r * LD + d] = row[a.koff];
    Vs[r * LD + d] = row[a.voff];
  }
  for (int e = threadIdx.x; e < tqc * DH; e += ATT_THREADS) {
    const int r = e / DH, d = e - r * DH;
    Qs[r * LD + d] = a.q[((size_t)img * a.tq + q0 + r) * a.qstride + a.qoff + hd * DH + d];
    Ds[r * LD + d] = a.dout[((size_t)img * a.tq + q0 + r) * c + hd * DH + d];
  }
  const float* pbase = a.pin + (((size_t)img * a.h + hd) * a.tq + q0) * tk;
  for (int e = threadIdx.x; e < tqc * tk; e += ATT_THREADS) Ps[e] = pbase[e];
  for (int e = threadIdx.x; e < nrel; e += ATT_THREADS) Rs[e] = 0.0f;
  __syncthreads();
  // dV += P^T dO (attn.rs:270-274)
  tile_mm<8, TND>(
      tk, DH, tqc, [&](int kj, int i) { return Ps[i * tk + kj]; }, [&](int i, int d) { return Ds[i * LD + d]; },
      [&](int kj, int d, float v) { a.dkv[((size_t)img * tk + kj) * a.kvstride + a.voff + hd * DH + d] += v; });
  // dP = dO V^T (attn.rs:276-279)
  tile_mm<8, 2>(
      tqc, tk, DH, [&](int i, int d) { return Ds[i * LD + d]; }, [&](int d, int kj) { return Vs[kj * LD + d]; },
      [&](int i, int kj, float v) { Gs[i * tk + kj] = v; });
  __syncthreads();
  // dS = P (dP - sum_k dP P) (attn.rs:280-290)
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  for (int i = w; i < tqc; i += ATT_WARPS) {
    float* g = Gs + i * tk;
    const float* pr = Ps + i * tk;
    float dot = 0.0f;
    for (int j = l; j < tk; j += 32) dot += g[j] * pr[j];
    dot = warp_sum(dot);
    for (int j = l; j < tk; j += 32) g[j] = pr[j] * (g[j] - dot);
  }
  __syncthreads();
  // dtau partial: sum dS * (Q K^T), raw scores recomputed (attn.rs:292-308)
  float tacc = 0.0f;
  tile_mm<8, 2>(
      tqc, tk, DH, [&](int i, int k) { return Qs[i * LD + k]; }, [&](int k, int j) { return Ks[j * LD + k]; },
      [&](int i, int j, float v) { tacc += Gs[i * tk + j] * v; });
  tacc = warp_sum(tacc);
  if (l == 0) red[w] = tacc;
  // drel partial, one query row at a time (distinct indices within a row)
  for (int i = 0; i < tqc; i++) {
    const uint32_t* ridx = a.relidx + (size_t)(q0 + i) * tk;
    for (int j = threadIdx.x; j < tk; j += ATT_THREADS) Rs[ridx[j]] += Gs[i * tk + j];
    __syncthreads();
  }
  float* part = a.part + (((size_t)img * a.nchunk + a.chunk) * a.h + hd) * (1 + nrel);
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int k = 0; k < ATT_WARPS; k++) s += red[k];
    part[0] = s;
  }
  for (int e = threadIdx.x; e < nrel; e += ATT_THREADS) part[1 + e] = Rs[e];
  // dS *= tau (attn.rs:316)
  const float t = a.tau[hd];
  for (int e = threadIdx.x; e < tqc * tk; e += ATT_THREADS) Gs[e] *= t;
  __syncthreads();
  // dQ += dS K, dK += dS^T Q (attn.rs:318-327)
  tile_mm<8, TND>(
      tqc, DH, tk, [&](int i, int kj) { return Gs[i * tk + kj]; }, [&](int kj, int d) { return Ks[kj * LD + d]; },
      [&](int i, int d, float v) { a.dq[((size_t)img * a.tq + q0 + i) * a.qstride + a.qoff + hd * DH + d] += v; });
  tile_mm<8, TND>(
      tk, DH, tqc, [&](int kj, int i) { return Gs[i * tk + kj]; }, [&](int i, int d) { return Qs[i * LD + d]; },
      [&](int kj, int d, float v) { a.dkv[((size_t)img * tk + kj) * a.kvstride + a.koff + hd * DH + d] += v; });
}

// dtau[hd] += sum over (image, chunk) of part[..][0]; drel[hd*nrel+r] +=
// sum of part[..][1+r]; images then chunks, in order.
__global__ void attn_reduce_kernel(const float* __restrict__ part, int n, int nchunk, int h, int nrel,
                                   float* __restrict__ dtau, float* __restrict__ drel) {
  const int total = h * (1 + nrel);
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    const int hd = e / (1 + nrel), r = e - hd * (1 + nrel);
    float s = 0.0f;
    for (int i = 0; i < n; i++)
      for (int ch = 0; ch < nchunk; ch++) s += part[(((size_t)i * nchunk + ch) * h + hd) * (1 + nrel) + r];
    if (r == 0) dtau[hd] += s;
    else drel[(size_t)hd * nrel + r - 1] += s;
  }
}

// ---------------------------------------------------------------- host

static size_t fwd_smem(int dh, int tqc, int tk) {
  return sizeof(float) * ((size_t)tqc * (dh + 1) + 2 * (size_t)tk * (dh + 1) + (size_t)tqc * tk);
}
static size_t bwd_smem(int dh, int tqc, int tk, int nrel) {
  return sizeof(float) *
         (2 * (size_t)tk * (dh + 1) + 2 * (size_t)tqc * (dh + 1) + 2 * (size_t)tqc * tk + (size_t)nrel);
}
constexpr size_t ATT_SMEM_CAP = 220 * 1024;

template <int DH>
static int launch_fwd(rnn_ctx* ctx, AttnArgs a) {
  int tqc = 64;
  while (tqc > 1 && fwd_smem(DH, tqc, a.tk) > ATT_SMEM_CAP) tqc /= 2;
  if (tqc > a.tq) tqc = a.tq;
  const size_t smem = fwd_smem(DH, tqc, a.tk);
  RNN_REQUIRE(smem <= ATT_SMEM_CAP, "attention: %d keys of head dim %d do not fit in shared memory", a.tk, DH);
  a.tqc = tqc;
  RNN_CUDA(cudaFuncSetAttribute(attn_fwd_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid(a.h, a.n, (a.tq + tqc - 1) / tqc);
  attn_fwd_kernel<DH><<<grid, ATT_THREADS, smem, ctx->stream>>>(a);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

template <int DH>
static int launch_bwd(rnn_ctx* ctx, AttnArgs a, float* dtau, float* drel) {
  int tqc = 64;
  while (tqc > 1 && bwd_smem(DH, tqc, a.tk, a.nrel) > ATT_SMEM_CAP) tqc /= 2;
  if (tqc > a.tq) tqc = a.tq;
  const size_t smem = bwd_smem(DH, tqc, a.tk, a.nrel);
  RNN_REQUIRE(smem <= ATT_SMEM_CAP, "attention backward: %d keys of head dim %d do not fit in shared memory",
              a.tk, DH);
  a.tqc = tqc;
  a.nchunk = (a.tq + tqc - 1) / tqc;
  const size_t part_floats = (size_t)a.n * a.nchunk * a.h * (1 + a.nrel);
  RNN_TRY(ensure_ws(ctx, part_floats * sizeof(float)));
  a.part = static_cast<float*>(ctx->ws);
  RNN_RANGE(a.part, part_floats * sizeof(float));
  RNN_CUDA(cudaFuncSetAttribute(attn_bwd_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  for (int ch = 0; ch < a.nchunk; ch++) {  // chunks in stream order: dK/dV += never race
    a.chunk = ch;
    attn_bwd_kernel<DH><<<dim3(a.h, a.n, 1), ATT_THREADS, smem, ctx->stream>>>(a);
    RNN_CHECK_LAUNCH();
  }
  const int total = a.h * (1 + a.nrel);
  attn_reduce_kernel<<<(total + 255) / 256, 256, 0, ctx->stream>>>(a.part, a.n, a.nchunk, a.h, a.nrel, dtau, drel);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

static int check_args(int n, int h, int dh, int th, int tw, int mh, int mw, int qstride, int qoff, int kvstride,
                      int koff, int voff) {
  RNN_REQUIRE(n > 0 && h > 0 && th > 0 && tw > 0 && mh > 0 && mw > 0, "attention: bad shape");
  RNN_REQUIRE(dh == 4 || dh == 6 || dh == 8 || dh == 12 || dh == 16 || dh == 24 || dh == 32 || dh == 48 ||
                  dh == 64,
              "attention: head dim %d unsupported (4, 6, 8, 12, 16, 24, 32, 48 or 64)", dh);
  RNN_REQUIRE(qoff >= 0 && qoff + h * dh <= qstride, "attention: q columns exceed its row stride");
  RNN_REQUIRE(koff >= 0 && voff >= 0 && koff + h * dh <= kvstride && voff + h * dh <= kvstride,
              "attention: k/v columns exceed the kv row stride");
  return RNN_OK;
}

#define ATTN_DISPATCH(fn, dh, ...)                           \
  switch (dh) {                                              \
    case 4: return fn<4>(__VA_ARGS__);                       \
    case 6: return fn<6>(__VA_ARGS__);                       \
    case 8: return fn<8>(__VA_ARGS__);                       \
    case 12: return fn<12>(__VA_ARGS__);                     \
    case 16: return fn<16>(__VA_ARGS__);                     \
    case 24: return fn<24>(__VA_ARGS__);                     \
    case 32: return fn<32>(__VA_ARGS__);                     \
    case 48: return fn<48>(__VA_ARGS__);                     \
    default: return fn<64>(__VA_ARGS__);                     \
  }

}  // namespace rnn

using namespace rnn;

extern "C" int rnn_rel_index(int th, int tw, int mh, int mw, uint32_t* idx, int* nrel) {
  RNN_REQUIRE(th > 0 && tw > 0 && mh > 0 && mw > 0 && nrel, "rel_index: bad arguments");
  std::vector<uint32_t> v;
  *nrel = rel_index_host(th, tw, mh, mw, idx ? &v : nullptr);
  if (idx) std::copy(v.begin(), v.end(), idx);
  return RNN_OK;
}

extern "C" int rnn_attn_fwd_dev(rnn_ctx* ctx, int n, int h, int dh, int th, int tw, int mh, int mw, int mask_diag,
                                const float* q, int qstride, int qoff, const float* kv, int kvstride, int koff,
                                int voff, const float* tau, const float* rel, float* p, float* o) {
  RNN_REQUIRE(ctx && q && kv && tau && rel && p && o, "attn_fwd: null argument");
  RNN_TRY(check_args(n, h, dh, th, tw, mh, mw, qstride, qoff, kvstride, koff, voff));
  AttnArgs a{};
  a.n = n; a.h = h; a.tq = th * tw; a.tk = mh * mw; a.mask = mask_diag ? 1 : 0;
  RNN_REQUIRE(!a.mask || a.tq == a.tk, "attn_fwd: the diagonal mask needs tq == tk");
  RNN_TRY(rel_table(ctx, th, tw, mh, mw, &a.relidx, &a.nrel));
  a.q = q; a.qstride = qstride; a.qoff = qoff;
  a.kv = kv; a.kvstride = kvstride; a.koff = koff; a.voff = voff;
  a.tau = tau; a.rel = rel; a.p = p; a.o = o;
  RNN_RANGE(q, sizeof(float) * (size_t)n * a.tq * qstride);
  RNN_RANGE(kv, sizeof(float) * (size_t)n * a.tk * kvstride);
  RNN_RANGE(tau, sizeof(float) * h);
  RNN_RANGE(rel, sizeof(float) * (size_t)h * a.nrel);
  RNN_RANGE(p, sizeof(float) * (size_t)n * h * a.tq * a.tk);
  RNN_RANGE(o, sizeof(float) * (size_t)n * a.tq * h * dh);
  ATTN_DISPATCH(launch_fwd, dh, ctx, a)
}

extern "C" int rnn_attn_bwd_dev(rnn_ctx* ctx, int n, int h, int dh, int th, int tw, int mh, int mw,
                                const float* q, int qstride, int qoff, const float* kv, int kvstride, int koff,
                                int voff, const float* tau, const float* p, const float* dout, float* dq,
                                float* dkv, float* dtau, float* drel) {
  RNN_REQUIRE(ctx && q && kv && tau && p && dout && dq && dkv && dtau && drel, "attn_bwd: null argument");
  RNN_TRY(check_args(n, h, dh, th, tw, mh, mw, qstride, qoff, kvstride, koff, voff));
  AttnArgs a{};
  a.n = n; a.h = h; a.tq = th * tw; a.tk = mh * mw;
  RNN_TRY(rel_table(ctx, th, tw, mh, mw, &a.relidx, &a.nrel));
  a.q = q; a.qstride = qstride; a.qoff = qoff;
  a.kv = kv; a.kvstride = kvstride; a.koff = koff; a.voff = voff;
  a.tau = tau; a.pin = p; a.dout = dout; a.dq = dq; a.dkv = dkv;
  RNN_RANGE(q, sizeof(float) * (size_t)n * a.tq * qstride);
  RNN_RANGE(kv, sizeof(float) * (size_t)n * a.tk * kvstride);
  RNN_RANGE(dq, sizeof(float) * (size_t)n * a.tq * qstride);
  RNN_RANGE(dkv, sizeof(float) * (size_t)n * a.tk * kvstride);
  RNN_RANGE(p, sizeof(float) * (size_t)n * h * a.tq * a.tk);
  RNN_RANGE(dout, sizeof(float) * (size_t)n * a.tq * h * dh);
  RNN_RANGE(dtau, sizeof(float) * h);
  RNN_RANGE(drel, sizeof(float) * (size_t)h * a.nrel);
  ATTN_DISPATCH(launch_bwd, dh, ctx, a, dtau, drel)
}
