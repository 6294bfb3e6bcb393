// Fused batched attention: attn.rs Core::forward (:148-223) and
// Core::backward (:226-343) for every (image, head) in one launch.
//
// Forward: one CTA per (head, image, chunk of query rows) holds K and V of
// the pair in shared memory (rows padded to dh+1 floats so a lane walking its
// own key row hits its own bank); each warp streams query rows: lane l scores
// keys l+32k against the row held in registers, the softmax is two warp
// reductions, P goes to HBM (the backward reads it, attn.rs:186-211) and to a
// per-warp row buffer, and lane d forms O[i][d].
//
// Backward in two phases.  Row phase (per query chunk): dP = dO V^T and the
// raw scores Q K^T are recomputed per key, dS = P (dP - sum dP P), dtau and
// drel partials (drel in a warp-private buffer: within one query row every
// key maps to a distinct relative index), tau*dS to a workspace, and dQ +=
// tau dS K.  Column phase (per key chunk): dV += P^T dO and dK += (tau dS)^T
// Q from shared-memory copies of the chunk's columns.  The per-CTA partials
// are summed in a fixed order by a warp-per-output kernel, so the whole
// backward is deterministic and uses no atomics.  dq / dkv / dtau / drel
// accumulate (+=) like attn.rs:274, 323, 327.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "attn_tc.cuh"
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

// Inverse of the index table, one per (device, geometry): inv[i][r] = the key
// j with relidx[i][j] == r, or -1 (within a query row the indices are
// distinct, so there is at most one).
static std::map<std::tuple<int, int, int, int, int>, int*> g_inv_tables;

static int rel_inv_table(rnn_ctx* ctx, int th, int tw, int mh, int mw, const int** out) {
  std::vector<uint32_t> idx;
  const int nrel = rel_index_host(th, tw, mh, mw, &idx);
  const int tq = th * tw, tk = mh * mw;
  std::lock_guard<std::mutex> lock(g_rel_mu);
  auto key = std::make_tuple(ctx->device, th, tw, mh, mw);
  auto it = g_inv_tables.find(key);
  if (it == g_inv_tables.end()) {
    std::vector<int> inv((size_t)tq * nrel, -1);
    for (int i = 0; i < tq; i++)
      for (int j = 0; j < tk; j++) inv[(size_t)i * nrel + idx[(size_t)i * tk + j]] = j;
    int* d = nullptr;
    RNN_CUDA(cudaMalloc(&d, inv.size() * sizeof(int)));
    RNN_CUDA(cudaMemcpy(d, inv.data(), inv.size() * sizeof(int), cudaMemcpyHostToDevice));
    it = g_inv_tables.emplace(key, d).first;
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
  float* p;          // forward writes P
  const float* pin;  // backward reads P
  float* o;
  const float* dout;
  float* dq;
  float* dkv;
  float* ds;    // backward: tau * dS [n][h][tq][tk]
  float* part;  // backward partials [n][nchunk][h][1 + nrel]
  int qc, nchunk;
};

constexpr int AT_THREADS = 256;
constexpr int AT_WARPS = AT_THREADS / 32;
constexpr int AT_MAXK = 8;   // keys per lane: tk <= 256
constexpr int AT_QC = 64;    // query rows per CTA (row kernels)
constexpr int AT_KC = 32;    // keys per CTA (column kernel)

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

// sum_j w[j] * col[j * ld] with four independent accumulators (j mod 4),
// combined as (a0 + a1) + (a2 + a3): a tk-long dependent FMA chain becomes
// four chains a quarter as long
__device__ __forceinline__ float row_dot4(const float* __restrict__ w, const float* __restrict__ col, int ld, int tk) {
  float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
  int j = 0;
  for (; j + 3 < tk; j += 4) {
    a0 = fmaf(w[j], col[j * ld], a0);
    a1 = fmaf(w[j + 1], col[(j + 1) * ld], a1);
    a2 = fmaf(w[j + 2], col[(j + 2) * ld], a2);
    a3 = fmaf(w[j + 3], col[(j + 3) * ld], a3);
  }
  for (; j < tk; j++) a0 = fmaf(w[j], col[j * ld], a0);
  return (a0 + a1) + (a2 + a3);
}

// Row length of K and V in the forward kernel's shared memory.  A lane walks
// its own key row, so the rows are padded: with DH a multiple of 4 the rows are read as float4
// and hold an odd number of 16-byte units (DH, or DH + 4), which keeps the
// eight lanes of each quarter-warp LDS.128 phase on distinct banks; other
// head dims are read as floats from rows of DH + 1.
__host__ __device__ constexpr int attn_ld(int dh) {
  return dh % 4 != 0 ? dh + 1 : ((dh / 4) % 2 == 1 ? dh : dh + 4);
}
// The backward's row kernel reads its rows as float4 only from head dim 64
// up (measured: faster at 64, slower at 32, where the wider rows cost
// occupancy); below that it keeps scalar walks over rows of DH + 1.
__host__ __device__ constexpr bool attn_bwd_vec(int dh) { return dh >= 64 && dh % 4 == 0; }
__host__ __device__ constexpr int attn_bwd_ld(int dh) { return attn_bwd_vec(dh) ? attn_ld(dh) : dh + 1; }

// K and V of one (image, head) into shared memory, rows of LD floats.
template <int DH, int LD>
__device__ __forceinline__ void load_kv(const AttnArgs& a, int img, int hd, float* Ks, float* Vs) {
  for (int e = threadIdx.x; e < a.tk * DH; e += AT_THREADS) {
    const int r = e / DH, d = e - r * DH;
    const float* row = a.kv + ((size_t)img * a.tk + r) * a.kvstride + hd * DH + d;
    Ks[r * LD + d] = row[a.koff];
    Vs[r * LD + d] = row[a.voff];
  }
}

// Forward (attn.rs:167-221), one CTA per (head, image, chunk of AT_QC query
// rows), one warp per query row at a time: lane l scores keys l + 32k
// against the row (held in registers), the row softmax is two warp
// reductions, P goes to HBM and to a per-warp row buffer, and lane d forms
// O[i][d] = sum_j P[i][j] V[j][d].
template <int DH>
__global__ void __launch_bounds__(AT_THREADS) attn_fwd_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) float sm[];
  constexpr int LD = attn_ld(DH);
  const int hd = blockIdx.x, img = blockIdx.y, q0 = blockIdx.z * a.qc;
  const int rows = min(a.qc, a.tq - q0), tk = a.tk, c = a.h * DH;
  float* Ks = sm;
  float* Vs = Ks + tk * LD;
  float* Pw = Vs + tk * LD;  // [AT_WARPS][tk]
  load_kv<DH, LD>(a, img, hd, Ks, Vs);
  __syncthreads();
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const float t = a.tau[hd];
  const float* rb = a.rel + (size_t)hd * a.nrel;
  float* prow = Pw + w * tk;
  for (int i = w; i < rows; i += AT_WARPS) {
    const int qi = q0 + i;
    float qr[DH];
    const float* qg = a.q + ((size_t)img * a.tq + qi) * a.qstride + a.qoff + hd * DH;
#pragma unroll
    for (int d = 0; d < DH; d++) qr[d] = __ldg(qg + d);
    const uint32_t* ridx = a.relidx + (size_t)qi * tk;
    float sv[AT_MAXK];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < AT_MAXK; k++) {
      const int j = l + 32 * k;
      float val = -INFINITY;
      if (j < tk) {
        const float* kr = Ks + j * LD;
        float acc = 0.0f;
        if constexpr (DH % 4 == 0) {
#pragma unroll
          for (int d = 0; d < DH; d += 4) {
            const float4 k4 = *reinterpret_cast<const float4*>(kr + d);
            acc = fmaf(qr[d], k4.x, acc);
            acc = fmaf(qr[d + 1], k4.y, acc);
            acc = fmaf(qr[d + 2], k4.z, acc);
            acc = fmaf(qr[d + 3], k4.w, acc);
          }
        } else {
#pragma unroll
          for (int d = 0; d < DH; d++) acc = fmaf(qr[d], kr[d], acc);
        }
        val = t * acc + rb[ridx[j]];  // attn.rs:181-190
        if (a.mask && j == qi) val = -INFINITY;  // attn.rs:194
      }
      sv[k] = val;
      mx = fmaxf(mx, val);
    }
    mx = warp_max(mx);
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < AT_MAXK; k++) {
      const float e = sv[k] == -INFINITY ? 0.0f : expf(sv[k] - mx);
      sv[k] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    const float inv = 1.0f / sum;
    float* pg = a.p + (((size_t)img * a.h + hd) * a.tq + qi) * tk;
#pragma unroll
    for (int k = 0; k < AT_MAXK; k++) {
      const int j = l + 32 * k;
      if (j < tk) {
        const float pv = sv[k] * inv;
        pg[j] = pv;
        prow[j] = pv;
      }
    }
    __syncwarp();
    float* og = a.o + ((size_t)img * a.tq + qi) * c + hd * DH;
    for (int d = l; d < DH; d += 32) og[d] = row_dot4(prow, Vs + d, LD, tk);
    __syncwarp();
  }
}

// Backward, row phase (attn.rs:276-321), one CTA per (head, image, chunk of
// query rows), a warp per row: dP = dO V^T and the raw scores Q K^T are
// recomputed per key, dS = P (dP - sum_k dP P); dtau accumulates dS * QK^T,
// drel accumulates dS at the row's relative indices (distinct within a row,
// so a warp-private buffer takes them without atomics), tau * dS goes to HBM
// for the column phase, and lane d adds tau * sum_j dS[i][j] K[j][d] to dQ.
// Partials (dtau, drel) per CTA are summed in a fixed order afterwards.
template <int DH>
__global__ void __launch_bounds__(AT_THREADS) attn_bwd_rows_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) float sm[];
  constexpr int LD = attn_bwd_ld(DH);
  const int hd = blockIdx.x, img = blockIdx.y, chunk = blockIdx.z, q0 = chunk * a.qc;
  const int rows = min(a.qc, a.tq - q0), tk = a.tk, c = a.h * DH, nrel = a.nrel;
  float* Ks = sm;
  float* Vs = Ks + tk * LD;
  float* Dw = Vs + tk * LD;              // [AT_WARPS][tk] tau * dS row
  float* Rw = Dw + AT_WARPS * tk;        // [AT_WARPS][nrel] drel per warp
  __shared__ float red[AT_WARPS];
  load_kv<DH, LD>(a, img, hd, Ks, Vs);
  for (int e = threadIdx.x; e < AT_WARPS * nrel; e += AT_THREADS) Rw[e] = 0.0f;
  __syncthreads();
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const float t = a.tau[hd];
  float* dsrow = Dw + w * tk;
  float* rw = Rw + w * nrel;
  float tacc = 0.0f;
  for (int i = w; i < rows; i += AT_WARPS) {
    const int qi = q0 + i;
    float qr[DH], dr[DH];
    const float* qg = a.q + ((size_t)img * a.tq + qi) * a.qstride + a.qoff + hd * DH;
    const float* dg = a.dout + ((size_t)img * a.tq + qi) * c + hd * DH;
#pragma unroll
    for (int d = 0; d < DH; d++) {
      qr[d] = __ldg(qg + d);
      dr[d] = __ldg(dg + d);
    }
    const float* pg = a.pin + (((size_t)img * a.h + hd) * a.tq + qi) * tk;
    float pv[AT_MAXK], dp[AT_MAXK], raw[AT_MAXK];
    float dot = 0.0f;
#pragma unroll
    for (int k = 0; k < AT_MAXK; k++) {
      const int j = l + 32 * k;
      pv[k] = dp[k] = raw[k] = 0.0f;
      if (j < tk) {
        const float* kr = Ks + j * LD;
        const float* vr = Vs + j * LD;
        float s1 = 0.0f, s2 = 0.0f;
        if constexpr (attn_bwd_vec(DH)) {
#pragma unroll
          for (int d = 0; d < DH; d += 4) {
            const float4 v4 = *reinterpret_cast<const float4*>(vr + d);
            const float4 k4 = *reinterpret_cast<const float4*>(kr + d);
            s1 = fmaf(dr[d], v4.x, s1);
            s2 = fmaf(qr[d], k4.x, s2);
            s1 = fmaf(dr[d + 1], v4.y, s1);
            s2 = fmaf(qr[d + 1], k4.y, s2);
            s1 = fmaf(dr[d + 2], v4.z, s1);
            s2 = fmaf(qr[d + 2], k4.z, s2);
            s1 = fmaf(dr[d + 3], v4.w, s1);
            s2 = fmaf(qr[d + 3], k4.w, s2);
          }
        } else {
#pragma unroll
          for (int d = 0; d < DH; d++) {
            s1 = fmaf(dr[d], vr[d], s1);
            s2 = fmaf(qr[d], kr[d], s2);
          }
        }
        dp[k] = s1;
        raw[k] = s2;
        pv[k] = __ldg(pg + j);
        dot = fmaf(s1, pv[k], dot);
      }
    }
    dot = warp_sum(dot);
    const uint32_t* ridx = a.relidx + (size_t)qi * tk;
    float* dsg = a.ds + (((size_t)img * a.h + hd) * a.tq + qi) * tk;
#pragma unroll
    for (int k = 0; k < AT_MAXK; k++) {
      const int j = l + 32 * k;
      if (j < tk) {
        const float ds = pv[k] * (dp[k] - dot);
        tacc = fmaf(ds, raw[k], tacc);
        rw[ridx[j]] += ds;
        const float dst = ds * t;
        dsrow[j] = dst;
        dsg[j] = dst;
      }
    }
    __syncwarp();
    float* dqg = a.dq + ((size_t)img * a.tq + qi) * a.qstride + a.qoff + hd * DH;
    for (int d = l; d < DH; d += 32) dqg[d] += row_dot4(dsrow, Ks + d, LD, tk);
    __syncwarp();
  }
  tacc = warp_sum(tacc);
  if (l == 0) red[w] = tacc;
  __syncthreads();
  float* part = a.part + (((size_t)img * a.nchunk + chunk) * a.h + hd) * (1 + nrel);
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int k = 0; k < AT_WARPS; k++) s += red[k];
    part[0] = s;
  }
  for (int r = threadIdx.x; r < nrel; r += AT_THREADS) {
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < AT_WARPS; k++) s += Rw[k * nrel + r];
    part[1 + r] = s;
  }
}

// Backward, column phase (attn.rs:270-274, 322-327): one CTA per (head,
// image, chunk of AT_KC keys); warp w owns keys w, w+4, ... of the chunk and
// lane d the head-dim columns d, d+32: dV[j][d] += sum_i P[i][j] dO[i][d],
// dK[j][d] += sum_i (tau dS)[i][j] Q[i][d], with the chunk's P / dS columns
// and all Q / dO rows staged in shared memory.
template <int DH>
__global__ void __launch_bounds__(AT_THREADS) attn_bwd_cols_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) float sm[];
  constexpr int KPW = AT_KC / AT_WARPS;       // keys per warp
  constexpr int DPL = (DH + 31) / 32;         // columns per lane
  const int hd = blockIdx.x, img = blockIdx.y, k0 = blockIdx.z * AT_KC;
  const int nk = min(AT_KC, a.tk - k0), tq = a.tq, tk = a.tk, c = a.h * DH;
  float* Qs = sm;                  // [tq][DH]
  float* Os = Qs + tq * DH;        // [tq][DH]  dO
  float* Ps = Os + tq * DH;        // [tq][AT_KC]
  float* Ss = Ps + tq * AT_KC;     // [tq][AT_KC]  tau * dS
  for (int e = threadIdx.x; e < tq * DH; e += AT_THREADS) {
    const int r = e / DH, d = e - r * DH;
    Qs[e] = a.q[((size_t)img * tq + r) * a.qstride + a.qoff + hd * DH + d];
    Os[e] = a.dout[((size_t)img * tq + r) * c + hd * DH + d];
  }
  const size_t pb = (((size_t)img * a.h + hd) * tq) * tk + k0;
  for (int e = threadIdx.x; e < tq * AT_KC; e += AT_THREADS) {
    const int r = e / AT_KC, j = e - r * AT_KC;
    const bool ok = j < nk;
    Ps[e] = ok ? a.pin[pb + (size_t)r * tk + j] : 0.0f;
    Ss[e] = ok ? a.ds[pb + (size_t)r * tk + j] : 0.0f;
  }
  __syncthreads();
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  float dv[KPW][DPL], dk[KPW][DPL];
#pragma unroll
  for (int u = 0; u < KPW; u++)
#pragma unroll
    for (int v = 0; v < DPL; v++) dv[u][v] = dk[u][v] = 0.0f;
  for (int i = 0; i < tq; i++) {
    float qv[DPL], ov[DPL];
#pragma unroll
    for (int v = 0; v < DPL; v++) {
      const int d = l + 32 * v;
      qv[v] = d < DH ? Qs[i * DH + d] : 0.0f;
      ov[v] = d < DH ? Os[i * DH + d] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < KPW; u++) {
      const float p = Ps[i * AT_KC + w + AT_WARPS * u];
      const float g = Ss[i * AT_KC + w + AT_WARPS * u];
#pragma unroll
      for (int v = 0; v < DPL; v++) {
        dv[u][v] = fmaf(p, ov[v], dv[u][v]);
        dk[u][v] = fmaf(g, qv[v], dk[u][v]);
      }
    }
  }
#pragma unroll
  for (int u = 0; u < KPW; u++) {
    const int j = w + AT_WARPS * u;
    if (j >= nk) continue;
    float* row = a.dkv + ((size_t)img * tk + k0 + j) * a.kvstride + hd * DH;
#pragma unroll
    for (int v = 0; v < DPL; v++) {
      const int d = l + 32 * v;
      if (d < DH) {
        row[a.voff + d] += dv[u][v];
        row[a.koff + d] += dk[u][v];
      }
    }
  }
}

// dtau[hd] += sum over (image, chunk) of part[..][0]; drel[hd*nrel+r] +=
// sum of part[..][1+r].  One warp per output: lane l adds items l, l+32, ...
// in order, then a fixed shuffle tree; deterministic.
__global__ void attn_reduce_kernel(const float* __restrict__ part, int items, int h, int nrel,
                                   float* __restrict__ dtau, float* __restrict__ drel) {
  const int total = h * (1 + nrel);
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, l = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int e = warp; e < total; e += nwarps) {
    const int hd = e / (1 + nrel), r = e - hd * (1 + nrel);
    float s = 0.0f;
    for (int it = l; it < items; it += 32) s += part[((size_t)it * h + hd) * (1 + nrel) + r];
    s = warp_sum(s);
    if (l == 0) {
      if (r == 0) dtau[hd] += s;
      else drel[(size_t)hd * nrel + r - 1] += s;
    }
  }
}

// ---------------------------------------------------------------- host

constexpr size_t ATT_SMEM_CAP = 200 * 1024;

static size_t fwd_smem(int dh, int tk) {
  return sizeof(float) * (2 * (size_t)tk * attn_ld(dh) + (size_t)AT_WARPS * tk);
}
static size_t rows_smem(int dh, int tk, int nrel) {
  return sizeof(float) * (2 * (size_t)tk * attn_bwd_ld(dh) + (size_t)AT_WARPS * tk + (size_t)AT_WARPS * nrel);
}
static size_t cols_smem(int dh, int tq) {
  return sizeof(float) * (2 * (size_t)tq * dh + 2 * (size_t)tq * AT_KC);
}

template <int DH>
static int launch_fwd(rnn_ctx* ctx, AttnArgs a) {
  RNN_REQUIRE(a.tk <= 32 * AT_MAXK, "attention: %d keys unsupported (at most %d)", a.tk, 32 * AT_MAXK);
  const size_t smem = fwd_smem(DH, a.tk);
  RNN_REQUIRE(smem <= ATT_SMEM_CAP, "attention: %d keys of head dim %d do not fit in shared memory", a.tk, DH);
  a.qc = AT_QC;
  RNN_CUDA(cudaFuncSetAttribute(attn_fwd_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid(a.h, a.n, (a.tq + a.qc - 1) / a.qc);
  attn_fwd_kernel<DH><<<grid, AT_THREADS, smem, ctx->stream>>>(a);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

template <int DH>
static int launch_bwd(rnn_ctx* ctx, AttnArgs a, float* dtau, float* drel) {
  RNN_REQUIRE(a.tk <= 32 * AT_MAXK, "attention backward: %d keys unsupported (at most %d)", a.tk, 32 * AT_MAXK);
  const size_t rsm = rows_smem(DH, a.tk, a.nrel), csm = cols_smem(DH, a.tq);
  RNN_REQUIRE(rsm <= ATT_SMEM_CAP && csm <= ATT_SMEM_CAP,
              "attention backward: %d queries x %d keys of head dim %d do not fit in shared memory", a.tq, a.tk,
              DH);
  a.qc = AT_QC;
  a.nchunk = (a.tq + a.qc - 1) / a.qc;
  const size_t ds_floats = (size_t)a.n * a.h * a.tq * a.tk;
  const size_t part_floats = (size_t)a.n * a.nchunk * a.h * (1 + a.nrel);
  const size_t ds_bytes = (ds_floats * sizeof(float) + 255) & ~(size_t)255;
  RNN_TRY(ensure_ws(ctx, ds_bytes + part_floats * sizeof(float)));
  a.ds = static_cast<float*>(ctx->ws);
  a.part = reinterpret_cast<float*>(static_cast<char*>(ctx->ws) + ds_bytes);
  RNN_RANGE(a.ds, ds_floats * sizeof(float));
  RNN_RANGE(a.part, part_floats * sizeof(float));
  RNN_CUDA(cudaFuncSetAttribute(attn_bwd_rows_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsm));
  RNN_CUDA(cudaFuncSetAttribute(attn_bwd_cols_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csm));
  attn_bwd_rows_kernel<DH><<<dim3(a.h, a.n, a.nchunk), AT_THREADS, rsm, ctx->stream>>>(a);
  RNN_CHECK_LAUNCH();
  attn_bwd_cols_kernel<DH><<<dim3(a.h, a.n, (a.tk + AT_KC - 1) / AT_KC), AT_THREADS, csm, ctx->stream>>>(a);
  RNN_CHECK_LAUNCH();
  const int total = a.h * (1 + a.nrel);
  const int blocks = std::min((total + 7) / 8, ctx->num_sms * 16);
  attn_reduce_kernel<<<blocks, 256, 0, ctx->stream>>>(a.part, a.n * a.nchunk, a.h, a.nrel, dtau, drel);
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

// RNN_ATTN_SIMT=1 keeps every call on the SIMT kernels above (A/B runs);
// by default calls the tensor-core path covers go there (attn_tc.cu).
static bool attn_simt_forced() {
  const char* v = getenv("RNN_ATTN_SIMT");
  return v && v[0] && v[0] != '0';
}

static AttnTC tc_args(const AttnArgs& a, int dh) {
  AttnTC t{};
  t.n = a.n; t.h = a.h; t.dh = dh; t.tq = a.tq; t.tk = a.tk; t.nrel = a.nrel; t.mask = a.mask; t.hp = a.h / 2;
  t.relidx = a.relidx;
  t.q = a.q; t.qstride = a.qstride; t.qoff = a.qoff;
  t.kv = a.kv; t.kvstride = a.kvstride; t.koff = a.koff; t.voff = a.voff;
  t.tau = a.tau; t.rel = a.rel; t.p = a.p; t.o = a.o;
  t.pin = a.pin; t.dout = a.dout; t.dq = a.dq; t.dkv = a.dkv;
  return t;
}

static size_t al256(size_t bytes) { return (bytes + 255) & ~(size_t)255; }

static int tc_fwd(rnn_ctx* ctx, AttnTC t) {
  const size_t bias_floats = (size_t)t.h * t.tq * t.tk;
  RNN_TRY(ensure_ws(ctx, bias_floats * sizeof(float)));
  float* bias = static_cast<float*>(ctx->ws);
  RNN_RANGE(bias, bias_floats * sizeof(float));
  RNN_TRY(tc::attn_bias_build(ctx, t, bias));
  t.bias = bias;
  return tc::attn_tc_fwd(ctx, t);
}

static int tc_bwd(rnn_ctx* ctx, AttnTC t, int th, int tw, int mh, int mw, float* dtau, float* drel) {
  const int* inv = nullptr;
  RNN_TRY(rel_inv_table(ctx, th, tw, mh, mw, &inv));
  const size_t ds_floats = (size_t)t.n * t.h * t.tq * t.tk;
  const size_t part_floats = (size_t)t.n * 2 * t.h;
  const size_t sum_floats = (size_t)t.h * t.tq * t.tk;
  const size_t ds_bytes = al256(ds_floats * sizeof(float)), part_bytes = al256(part_floats * sizeof(float));
  RNN_TRY(ensure_ws(ctx, ds_bytes + part_bytes + sum_floats * sizeof(float)));
  char* ws = static_cast<char*>(ctx->ws);
  t.ds = reinterpret_cast<float*>(ws);
  t.part = reinterpret_cast<float*>(ws + ds_bytes);
  float* dssum = reinterpret_cast<float*>(ws + ds_bytes + part_bytes);
  RNN_RANGE(t.ds, ds_floats * sizeof(float));
  RNN_RANGE(t.part, part_floats * sizeof(float));
  RNN_RANGE(dssum, sum_floats * sizeof(float));
  RNN_TRY(tc::attn_tc_bwd(ctx, t));
  attn_reduce_kernel<<<1, 256, 0, ctx->stream>>>(t.part, t.n * 2, t.h, 0, dtau, drel);
  RNN_CHECK_LAUNCH();
  return tc::attn_drel(ctx, t, inv, dssum, drel);
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
  const AttnTC t = tc_args(a, dh);
  if (!attn_simt_forced() && tc::attn_tc_ok(t, false)) return tc_fwd(ctx, t);
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
  const AttnTC t = tc_args(a, dh);
  if (!attn_simt_forced() && tc::attn_tc_ok(t, true)) return tc_bwd(ctx, t, th, tw, mh, mw, dtau, drel);
  ATTN_DISPATCH(launch_bwd, dh, ctx, a, dtau, drel)
}
