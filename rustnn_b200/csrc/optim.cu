// Optimisers of the rustvit path (optim.rs): Muon with its Newton-Schulz
// orthogonalisation, AdamW, the global-norm clip and the weight EMA.
//
// Newton-Schulz (optim.rs:70-145) runs on the wide orientation (m <= n, the
// tall case transposed in and out), normalises by the Frobenius norm + 1e-7,
// then iterates X <- a X + (b A + c A A) X with A = X X^T.  The three
// products per iteration are tcgen05 3xTF32 GEMMs; the b A + c AA and
// a X + T combinations and the reductions are small fused kernels.  The
// sum-of-squares reductions (Frobenius norm, clip) are fixed-order two-pass
// reductions (f32 for NS like the reference's f32 sum, f64 for clip like
// optim.rs:238-241).
#include <algorithm>
#include <cmath>
#include <utility>
#include <vector>

#include "ew.cuh"

namespace rnn {

constexpr float NS_A = 3.4445f, NS_B = -4.7750f, NS_C = 2.0315f;  // optim.rs:24-26

__global__ void transpose_kernel(const float* __restrict__ in, int rows, int cols, float* __restrict__ out) {
  __shared__ float tile[32][33];
  const int bx = blockIdx.x * 32, by = blockIdx.y * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int r = by + k, c = bx + threadIdx.x;
    if (r < rows && c < cols) tile[k][threadIdx.x] = in[(size_t)r * cols + c];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int c = bx + k, r = by + threadIdx.x;
    if (r < rows && c < cols) out[(size_t)c * rows + r] = tile[threadIdx.x][k];
  }
}

static int transpose(rnn_ctx* ctx, const float* in, int rows, int cols, float* out) {
  dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
  transpose_kernel<<<grid, block, 0, ctx->stream>>>(in, rows, cols, out);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

// part[b] = sum over block b's grid-stride slice of x^2 (double when D)
template <bool D>
__global__ void sumsq_partial_kernel(const float* __restrict__ x, size_t n, double* __restrict__ part) {
  __shared__ double sh[256];
  double s = 0.0;
  float sf = 0.0f;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    if (D) s += (double)x[i] * (double)x[i];
    else sf += x[i] * x[i];
  }
  sh[threadIdx.x] = D ? s : (double)sf;
  __syncthreads();
  for (int k = 128; k > 0; k >>= 1) {
    if (threadIdx.x < k) sh[threadIdx.x] += sh[threadIdx.x + k];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = sh[0];
}

// NS normalise: x *= 1 / (sqrt(sum) + 1e-7) (optim.rs:133-135)
__global__ void ns_scale_kernel(float* __restrict__ x, size_t n, const double* __restrict__ part, int nb) {
  __shared__ float inv;
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int b = 0; b < nb; b++) s += part[b];
    inv = 1.0f / (sqrtf((float)s) + 1e-7f);
  }
  __syncthreads();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    x[i] *= inv;
}

// a = b*a + c*aa (optim.rs:101-103)
__global__ void ns_poly_kernel(float* __restrict__ a, const float* __restrict__ aa, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    a[i] = NS_B * a[i] + NS_C * aa[i];
}
// x = a*x + t (optim.rs:117-119)
__global__ void ns_axpy_kernel(float* __restrict__ x, const float* __restrict__ t, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    x[i] = NS_A * x[i] + t[i];
}

static unsigned egrid(size_t n, int sms) {
  return (unsigned)std::max<size_t>(1, std::min<size_t>((n + 255) / 256, (size_t)sms * 8));
}

constexpr int RED_BLOCKS = 256;

static size_t ns_scratch_floats(int rows, int cols) {
  const size_t m = std::min(rows, cols), n = std::max(rows, cols);
  return 2 * m * n + 2 * m * m + 2 * RED_BLOCKS + 64;  // x, t, a, aa, partials (as doubles)
}

// In place on g [rows x cols]; scratch holds ns_scratch_floats floats.
int newton_schulz(rnn_ctx* ctx, float* g, int rows, int cols, int steps, float* scratch) {
  const bool tr = rows > cols;
  const int m = tr ? cols : rows, n = tr ? rows : cols;
  const size_t mn = (size_t)m * n, mm = (size_t)m * m;
  float* x = scratch;
  float* t = x + mn;
  float* a = t + mn;
  float* aa = a + mm;
  double* part = reinterpret_cast<double*>(aa + mm);  // byte offset 8*(mn+mm): 8-aligned
  if (tr) RNN_TRY(transpose(ctx, g, rows, cols, x));
  else RNN_CUDA(cudaMemcpyAsync(x, g, mn * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  sumsq_partial_kernel<false><<<RED_BLOCKS, 256, 0, ctx->stream>>>(x, mn, part);
  RNN_CHECK_LAUNCH();
  ns_scale_kernel<<<egrid(mn, ctx->num_sms), 256, 0, ctx->stream>>>(x, mn, part, RED_BLOCKS);
  RNN_CHECK_LAUNCH();
  for (int s = 0; s < steps; s++) {
    RNN_TRY(tc::gemm_dev(ctx, m, m, n, x, false, x, true, a, false, false));   // A = X X^T
    RNN_TRY(tc::gemm_dev(ctx, m, m, m, a, false, a, false, aa, false, false)); // AA = A A
    ns_poly_kernel<<<egrid(mm, ctx->num_sms), 256, 0, ctx->stream>>>(a, aa, mm);
    RNN_CHECK_LAUNCH();
    RNN_TRY(tc::gemm_dev(ctx, m, n, m, a, false, x, false, t, false, false));  // T = B X
    ns_axpy_kernel<<<egrid(mn, ctx->num_sms), 256, 0, ctx->stream>>>(x, t, mn);
    RNN_CHECK_LAUNCH();
  }
  if (tr) return transpose(ctx, x, m, n, g);  // x is [cols x rows]
  RNN_CUDA(cudaMemcpyAsync(g, x, mn * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  return RNN_OK;
}

// ---- Newton-Schulz over many matrices at once
//
// Per item the arithmetic is that of newton_schulz (the same f32
// sum-of-squares slices, RED_BLOCKS per item, whose f64 sums are combined by
// a warp instead of one thread) and the same products.

// Padded classes.  Every matrix's working shape (m, n) is rounded up to
// (mc, nc), multiples of 128, and matrices of one class are batched; an
// item's slot holds its X in the top-left m x n corner and zeros elsewhere.
// The zeros are exact under every step (they add 0 to each real sum: the
// real K blocks come first and the padding only appends zero blocks; A, AA
// and T inherit zero rows and columns), so the real block is the same
// Newton-Schulz iterate.  The gather into the slots, the normalisation and
// the scatter back are one launch each over all matrices, the two
// combinations one launch per iteration over all classes; only the GEMMs run
// per class.  The sum of squares of item i walks its real elements in the
// same slices as the unpadded form.
struct NsItem {
  float* g;           // the matrix (rows x cols), read and written in place
  int rows, cols;     // as given; tall ones (rows > cols) are transposed
  int m, n, mc, nc;   // working and padded shapes
  size_t x;           // float offset of the item's slot in the X / T regions
};

__global__ void ns_gather_kernel(const NsItem* __restrict__ items, float* __restrict__ xall) {
  const NsItem it = items[blockIdx.y];
  const size_t slot = (size_t)it.mc * it.nc;
  float* x = xall + it.x;
  const bool tr = it.rows > it.cols;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < slot; e += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(e / it.nc), c = (int)(e - (size_t)r * it.nc);
    float v = 0.0f;
    if (r < it.m && c < it.n) v = tr ? it.g[(size_t)c * it.cols + r] : it.g[(size_t)r * it.n + c];
    x[e] = v;
  }
}
__global__ void ns_scatter_kernel(const NsItem* __restrict__ items, const float* __restrict__ xall) {
  const NsItem it = items[blockIdx.y];
  const size_t real = (size_t)it.m * it.n;
  const float* x = xall + it.x;
  const bool tr = it.rows > it.cols;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < real; e += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(e / it.n), c = (int)(e - (size_t)r * it.n);
    const float v = x[(size_t)r * it.nc + c];
    if (tr) it.g[(size_t)c * it.cols + r] = v;
    else it.g[e] = v;
  }
}
// part[item][b] = f32 sum of squares over block b's slice of the item's
// real elements (row-major order of the m x n working matrix)
__global__ void ns_sumsq_slots_kernel(const NsItem* __restrict__ items, const float* __restrict__ xall,
                                      double* __restrict__ part) {
  __shared__ double sh[256];
  const NsItem it = items[blockIdx.y];
  const size_t real = (size_t)it.m * it.n;
  const float* x = xall + it.x;
  float sf = 0.0f;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < real; e += (size_t)gridDim.x * blockDim.x) {
    const size_t r = e / it.n;
    const float v = x[r * it.nc + (e - r * it.n)];
    sf += v * v;
  }
  sh[threadIdx.x] = (double)sf;
  __syncthreads();
  for (int k = 128; k > 0; k >>= 1) {
    if (threadIdx.x < k) sh[threadIdx.x] += sh[threadIdx.x + k];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[(size_t)blockIdx.y * gridDim.x + blockIdx.x] = sh[0];
}
__global__ void ns_scale_slots_kernel(const NsItem* __restrict__ items, float* __restrict__ xall,
                                      const double* __restrict__ part, int nb) {
  __shared__ float inv;
  const NsItem it = items[blockIdx.y];
  if (threadIdx.x < 32) {  // lane l sums partials l, l+32, ..., then a fixed shuffle tree
    double s = 0.0;
    for (int b = threadIdx.x; b < nb; b += 32) s += part[(size_t)blockIdx.y * nb + b];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) inv = 1.0f / (sqrtf((float)s) + 1e-7f);
  }
  __syncthreads();
  float* x = xall + it.x;
  const size_t slot = (size_t)it.mc * it.nc;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < slot; e += (size_t)gridDim.x * blockDim.x)
    x[e] *= inv;
}

int newton_schulz_grouped(rnn_ctx* ctx, int count, float* const* g, const int* rows, const int* cols, int steps) {
  if (count <= 0) return RNN_OK;
  // classes by padded working shape, in first-appearance order
  struct Cls {
    int mc, nc;
    std::vector<int> members;
    size_t x, a;  // float offsets of the class's first slot in the X / A regions
  };
  std::vector<Cls> cls;
  auto up = [](int v) { return (v + 127) / 128 * 128; };
  for (int i = 0; i < count; i++) {
    const int mc = up(std::min(rows[i], cols[i])), nc = up(std::max(rows[i], cols[i]));
    size_t ci = 0;
    while (ci < cls.size() && !(cls[ci].mc == mc && cls[ci].nc == nc)) ci++;
    if (ci == cls.size()) cls.push_back({mc, nc, {}, 0, 0});
    cls[ci].members.push_back(i);
  }
  std::vector<NsItem> items;
  size_t xf = 0, af = 0, slot_max = 0;
  for (Cls& c : cls) {
    c.x = xf;
    c.a = af;
    for (int i : c.members) {
      NsItem it;
      it.g = g[i];
      it.rows = rows[i];
      it.cols = cols[i];
      it.m = std::min(rows[i], cols[i]);
      it.n = std::max(rows[i], cols[i]);
      it.mc = c.mc;
      it.nc = c.nc;
      it.x = xf;
      items.push_back(it);
      xf += (size_t)c.mc * c.nc;
      af += (size_t)c.mc * c.mc;
      slot_max = std::max(slot_max, (size_t)c.mc * c.nc);
      RNN_RANGE(g[i], sizeof(float) * (size_t)rows[i] * cols[i]);
    }
  }
  const int ni = (int)items.size();
  // aux: X, T [xf], A, AA [af], partials [ni][RED_BLOCKS] (doubles), items
  const size_t part_off = ((2 * xf + 2 * af) * 4 + 255) / 256 * 256;
  const size_t items_off = part_off + (size_t)ni * RED_BLOCKS * 8;
  RNN_TRY(ensure_aux(ctx, items_off + sizeof(NsItem) * ni + 64));
  char* base = static_cast<char*>(ctx->aux);
  float* xall = reinterpret_cast<float*>(base);
  float* tall = xall + xf;
  float* aall = tall + xf;
  float* aaall = aall + af;
  double* part = reinterpret_cast<double*>(base + part_off);
  NsItem* ditems = reinterpret_cast<NsItem*>(base + items_off);
  // (staged before cudaMemcpyAsync returns: `items` may go out of scope)
  RNN_CUDA(cudaMemcpyAsync(ditems, items.data(), sizeof(NsItem) * ni, cudaMemcpyHostToDevice, ctx->stream));
  const unsigned gx = std::max(1u, egrid(slot_max, ctx->num_sms) / 4);
  ns_gather_kernel<<<dim3(gx, ni), 256, 0, ctx->stream>>>(ditems, xall);
  RNN_CHECK_LAUNCH();
  ns_sumsq_slots_kernel<<<dim3(RED_BLOCKS, ni), 256, 0, ctx->stream>>>(ditems, xall, part);
  RNN_CHECK_LAUNCH();
  ns_scale_slots_kernel<<<dim3(gx, ni), 256, 0, ctx->stream>>>(ditems, xall, part, RED_BLOCKS);
  RNN_CHECK_LAUNCH();
  for (int st = 0; st < steps; st++) {
    for (const Cls& c : cls) {  // A = X X^T
      const size_t mn = (size_t)c.mc * c.nc, mm = (size_t)c.mc * c.mc;
      RNN_TRY(tc::gemm_batched_dev(ctx, (int)c.members.size(), c.mc, c.mc, c.nc, xall + c.x, mn, false, xall + c.x,
                                   mn, true, aall + c.a, mm, false));
    }
    for (const Cls& c : cls) {  // AA = A A
      const size_t mm = (size_t)c.mc * c.mc;
      RNN_TRY(tc::gemm_batched_dev(ctx, (int)c.members.size(), c.mc, c.mc, c.mc, aall + c.a, mm, false, aall + c.a,
                                   mm, false, aaall + c.a, mm, false));
    }
    ns_poly_kernel<<<egrid(af, ctx->num_sms), 256, 0, ctx->stream>>>(aall, aaall, af);
    RNN_CHECK_LAUNCH();
    for (const Cls& c : cls) {  // T = B X
      const size_t mn = (size_t)c.mc * c.nc, mm = (size_t)c.mc * c.mc;
      RNN_TRY(tc::gemm_batched_dev(ctx, (int)c.members.size(), c.mc, c.nc, c.mc, aall + c.a, mm, false, xall + c.x,
                                   mn, false, tall + c.x, mn, false));
    }
    ns_axpy_kernel<<<egrid(xf, ctx->num_sms), 256, 0, ctx->stream>>>(xall, tall, xf);
    RNN_CHECK_LAUNCH();
  }
  ns_scatter_kernel<<<dim3(gx, ni), 256, 0, ctx->stream>>>(ditems, xall);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

// Muon momentum (optim.rs:186-190): m = mom m + g; g += mom m
__global__ void muon_mom_kernel(float* __restrict__ g, float* __restrict__ m, size_t n, float mom) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float mm = mom * m[i] + g[i];
    m[i] = mm;
    g[i] += mom * mm;
  }
}
// v -= lr (scale g + wd v); g = 0 (optim.rs:192-196)
__global__ void muon_update_kernel(float* __restrict__ v, float* __restrict__ g, size_t n, float lr, float scale,
                                   float wd) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    v[i] -= lr * (scale * g[i] + wd * v[i]);
    g[i] = 0.0f;
  }
}

// step_adam (optim.rs:205-233)
__global__ void adamw_kernel(float* __restrict__ v, float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v2, size_t n, float lr, float wd, float b1, float b2, float eps,
                             float c1, float c2) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float gg = g[i];
    const float mm = b1 * m[i] + (1.0f - b1) * gg;
    const float vv = b2 * v2[i] + (1.0f - b2) * gg * gg;
    m[i] = mm;
    v2[i] = vv;
    v[i] -= lr * ((mm / c1) / (sqrtf(vv / c2) + eps) + wd * v[i]);
    g[i] = 0.0f;
  }
}

// clip_ (optim.rs:237-250): norm = sqrt(sum g^2) in f64; rescale if above max
__global__ void clip_scale_kernel(float* __restrict__ g, size_t n, const double* __restrict__ part, int nb, float max,
                                  float* __restrict__ norm_out) {
  __shared__ float s;
  if (threadIdx.x == 0) {
    double q = 0.0;
    for (int b = 0; b < nb; b++) q += part[b];
    const float norm = (float)sqrt(q);
    s = (norm > max && norm > 0.0f) ? max / norm : 1.0f;
    if (blockIdx.x == 0 && norm_out) *norm_out = norm;
  }
  __syncthreads();
  if (s == 1.0f) return;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    g[i] *= s;
}

// Ema::update (optim.rs:281-286)
__global__ void ema_kernel(float* __restrict__ e, const float* __restrict__ v, size_t n, float d) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    e[i] = d * e[i] + (1.0f - d) * v[i];
}

}  // namespace rnn

using namespace rnn;

extern "C" int rnn_newton_schulz_dev(rnn_ctx* ctx, float* g, int rows, int cols, int steps) {
  RNN_REQUIRE(ctx && g && rows > 0 && cols > 0 && steps >= 0, "newton_schulz: bad arguments");
  RNN_RANGE(g, (size_t)rows * cols * 4);
  RNN_TRY(ensure_aux(ctx, ns_scratch_floats(rows, cols) * 4));
  return newton_schulz(ctx, g, rows, cols, steps, static_cast<float*>(ctx->aux));
}

namespace rnn {

int muon_momentum(rnn_ctx* ctx, float* g, float* m, size_t n, float mom) {
  RNN_RANGE(g, n * 4);
  RNN_RANGE(m, n * 4);
  muon_mom_kernel<<<egrid(n, ctx->num_sms), 256, 0, ctx->stream>>>(g, m, n, mom);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

float muon_scale(int rows, int cols) { return 0.2f * sqrtf((float)std::max(rows, cols)); }

// Segmented forms: blockIdx.y selects the segment, the x grid strides over it.
__global__ void muon_mom_seg_kernel(float* __restrict__ g, float* __restrict__ m, const OptSeg* __restrict__ segs,
                                    float mom) {
  const OptSeg sg = segs[blockIdx.y];
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < sg.n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t e = sg.off + i;
    const float mm = mom * m[e] + g[e];
    m[e] = mm;
    g[e] += mom * mm;
  }
}
__global__ void muon_update_seg_kernel(float* __restrict__ v, float* __restrict__ g, const OptSeg* __restrict__ segs,
                                       float lr, float wd) {
  const OptSeg sg = segs[blockIdx.y];
  const float w = sg.decay ? wd : 0.0f;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < sg.n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t e = sg.off + i;
    v[e] -= lr * (sg.scale * g[e] + w * v[e]);
    g[e] = 0.0f;
  }
}
__global__ void adamw_seg_kernel(float* __restrict__ v, float* __restrict__ g, float* __restrict__ m,
                                 float* __restrict__ v2, const OptSeg* __restrict__ segs, float lr, float wd, float b1,
                                 float b2, float eps, float c1, float c2) {
  const OptSeg sg = segs[blockIdx.y];
  const float w = sg.decay ? wd : 0.0f;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < sg.n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t e = sg.off + i;
    const float gg = g[e];
    const float mm = b1 * m[e] + (1.0f - b1) * gg;
    const float vv = b2 * v2[e] + (1.0f - b2) * gg * gg;
    m[e] = mm;
    v2[e] = vv;
    v[e] -= lr * ((mm / c1) / (sqrtf(vv / c2) + eps) + w * v[e]);
    g[e] = 0.0f;
  }
}

static dim3 seg_grid(size_t max_n, int nseg, int sms) {
  const size_t gx = std::max<size_t>(1, std::min<size_t>((max_n + 255) / 256, (size_t)sms * 4));
  return dim3((unsigned)gx, (unsigned)nseg);
}

int muon_momentum_segs(rnn_ctx* ctx, float* g, float* m, const OptSeg* segs, int nseg, size_t max_n, float mom) {
  if (nseg <= 0) return RNN_OK;
  muon_mom_seg_kernel<<<seg_grid(max_n, nseg, ctx->num_sms), 256, 0, ctx->stream>>>(g, m, segs, mom);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int muon_update_segs(rnn_ctx* ctx, float* v, float* g, const OptSeg* segs, int nseg, size_t max_n, float lr,
                     float wd) {
  if (nseg <= 0) return RNN_OK;
  muon_update_seg_kernel<<<seg_grid(max_n, nseg, ctx->num_sms), 256, 0, ctx->stream>>>(v, g, segs, lr, wd);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int adamw_segs(rnn_ctx* ctx, float* v, float* g, float* m, float* v2, const OptSeg* segs, int nseg, size_t max_n,
               float lr, float wd, float b1, float b2, float eps, int t) {
  if (nseg <= 0) return RNN_OK;
  const float c1 = 1.0f - powf(b1, (float)(t + 1)), c2 = 1.0f - powf(b2, (float)(t + 1));
  adamw_seg_kernel<<<seg_grid(max_n, nseg, ctx->num_sms), 256, 0, ctx->stream>>>(v, g, m, v2, segs, lr, wd, b1, b2,
                                                                                 eps, c1, c2);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int muon_update(rnn_ctx* ctx, float* v, float* g, int rows, int cols, float lr, float wd, int decay) {
  const size_t n = (size_t)rows * cols;
  RNN_RANGE(v, n * 4);
  RNN_RANGE(g, n * 4);
  const float scale = muon_scale(rows, cols);
  muon_update_kernel<<<egrid(n, ctx->num_sms), 256, 0, ctx->stream>>>(v, g, n, lr, scale, decay ? wd : 0.0f);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

}  // namespace rnn

extern "C" int rnn_muon_step_dev(rnn_ctx* ctx, float* v, float* g, float* m, int rows, int cols, int steps, float lr,
                                 float mom, float wd, int decay) {
  RNN_REQUIRE(ctx && v && g && m && rows > 0 && cols > 0, "muon_step: bad arguments");
  RNN_TRY(rnn::muon_momentum(ctx, g, m, (size_t)rows * cols, mom));
  RNN_TRY(rnn_newton_schulz_dev(ctx, g, rows, cols, steps));
  return rnn::muon_update(ctx, v, g, rows, cols, lr, wd, decay);
}

extern "C" int rnn_adamw_step_dev(rnn_ctx* ctx, float* v, float* g, float* m, float* v2, size_t n, float lr, float wd,
                                  int decay, float b1, float b2, float eps, int t) {
  RNN_REQUIRE(ctx && v && g && m && v2 && t >= 0, "adamw_step: bad arguments");
  if (n == 0) return RNN_OK;
  RNN_RANGE(v, n * 4);
  RNN_RANGE(g, n * 4);
  RNN_RANGE(m, n * 4);
  RNN_RANGE(v2, n * 4);
  const float c1 = 1.0f - powf(b1, (float)(t + 1)), c2 = 1.0f - powf(b2, (float)(t + 1));
  adamw_kernel<<<egrid(n, ctx->num_sms), 256, 0, ctx->stream>>>(v, g, m, v2, n, lr, decay ? wd : 0.0f, b1, b2, eps,
                                                                 c1, c2);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

extern "C" int rnn_clip_dev(rnn_ctx* ctx, float* g, size_t n, float max, float* norm_out) {
  RNN_REQUIRE(ctx && g, "clip: null argument");
  if (n == 0) return RNN_OK;
  RNN_RANGE(g, n * 4);
  if (norm_out) RNN_RANGE(norm_out, 4);
  RNN_TRY(ensure_aux(ctx, RED_BLOCKS * sizeof(double)));
  double* part = static_cast<double*>(ctx->aux);
  sumsq_partial_kernel<true><<<RED_BLOCKS, 256, 0, ctx->stream>>>(g, n, part);
  RNN_CHECK_LAUNCH();
  clip_scale_kernel<<<egrid(n, ctx->num_sms), 256, 0, ctx->stream>>>(g, n, part, RED_BLOCKS, max, norm_out);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

extern "C" int rnn_ema_update_dev(rnn_ctx* ctx, float* e, const float* v, size_t n, float decay, int t) {
  RNN_REQUIRE(ctx && e && v && t >= 1, "ema_update: bad arguments");
  if (n == 0) return RNN_OK;
  RNN_RANGE(e, n * 4);
  RNN_RANGE(v, n * 4);
  const float cap = (1.0f + (float)t) / (10.0f + (float)t);
  ema_kernel<<<egrid(n, ctx->num_sms), 256, 0, ctx->stream>>>(e, v, n, std::min(decay, cap));
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}
