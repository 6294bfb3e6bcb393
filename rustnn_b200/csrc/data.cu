// Training-batch construction on the device: data::make_batch_train
// (data.rs:384-412: RandAugment on the bytes, crop offset, flip, normalise,
// random erasing) and data::mix_batch (data.rs:467-491: mixup / cutmix of
// the batch with a permutation of itself).
//
// make_batch_train runs one CTA per image with the image's bytes in shared
// memory.  Thread 0 replays the image's generator (Rng::new(seed ^ b *
// 0x9E3779B97F4A7C15), data.rs:400) and draws every random value the
// reference draws, in its order; the ops then run over the CTA.  The f32
// arithmetic uses the round-to-nearest intrinsics operation by operation, as
// the reference's unfused expressions round.
//
// The reference's f32 logf / cosf / sinf are the C library's, and those are
// not correctly rounded for every argument, so the device takes their results
// from the C library itself instead of evaluating its own:
//   * Rng::normal (rng.rs:55-59) is sqrt(-2 ln u1) * cos(TAU u2) with u1, u2
//     24-bit uniforms k * 2^-24, so ln u1 and cos(TAU u2) each take at most
//     2^24 values.  Two 64-MB tables, ln_tab[k] = logf(max(k 2^-24, 1e-7)) and
//     cos_tab[k] = cosf(TAU * k 2^-24) (the f32 product), are computed once
//     per process and device with the host's logf / cosf and indexed by the
//     drawn integers.  The sqrt and the products are IEEE-rounded.
//   * The rotation's cos t / sin t (data.rs:264-266) take an arbitrary f32 t:
//     the host replays each image's RandAugment draws (a handful of
//     generator steps per image; the normals with the same C library calls)
//     and passes cosf(t), sinf(t) of every rotation to the kernel.
// Both are therefore bit-exact against the reference's libm on this host.
//
// mix_batch draws its permutation and lambda on the host from the caller's
// generator state (a handful of draws per batch) and mixes on the device.
#include <math.h>

#include <algorithm>
#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"
#include "rng.h"

namespace rnn {

namespace {

constexpr int IMG = 32, PLANE = IMG * IMG, PIX = 3 * PLANE, NOPS = 13, MAX_RA = 8;
constexpr int THREADS = 128;
constexpr uint64_t GOLDEN = 0x9E3779B97F4A7C15ULL;

struct Aug {  // data.rs:281-293
  int pad;
  float ra_mag;
  int ra_n;
  float erase;
  int erase_side;
};

__device__ __forceinline__ float mean_of(int c) { return c == 0 ? 0.5071f : (c == 1 ? 0.4865f : 0.4409f); }
__device__ __forceinline__ float std_of(int c) { return c == 0 ? 0.2673f : (c == 1 ? 0.2564f : 0.2762f); }

// `v.clamp(0.0, 255.0) as u8`
__device__ __forceinline__ uint8_t clamp_u8(float v) { return (uint8_t)fminf(fmaxf(v, 0.0f), 255.0f); }

constexpr int NORMAL_TAB = 1 << 24;  // one entry per 24-bit uniform
constexpr float TAU = 6.28318530717958647692f;

struct NormalTabs {
  const float* ln;  // [2^24] logf(max(k 2^-24, 1e-7))
  const float* cs;  // [2^24] cosf(TAU * k 2^-24)
};

// Rng::normal (rng.rs:55-59) from the two drawn 24-bit integers:
// sqrt(-2 ln u1) * cos(TAU u2), each step in f32
__device__ __forceinline__ float normal_of(const NormalTabs& t, uint32_t k1, uint32_t k2) {
  return __fmul_rn(__fsqrt_rn(__fmul_rn(-2.0f, __ldg(t.ln + k1))), __ldg(t.cs + k2));
}

__device__ __forceinline__ float normal_dev(Rng& r, const NormalTabs& t) {
  const uint32_t k1 = (uint32_t)(r.next_u64() >> 40);
  const uint32_t k2 = (uint32_t)(r.next_u64() >> 40);
  return normal_of(t, k1, k2);
}

// data.rs:105-111
__device__ __forceinline__ float px(const uint8_t* im, int c, int y, int x) {
  if (y < 0 || x < 0 || y >= IMG || x >= IMG) return 128.0f;
  return (float)im[c * PLANE + y * IMG + x];
}

// blend (data.rs:137-142) of one byte
__device__ __forceinline__ uint8_t blend1(uint8_t im, uint8_t other, float f) {
  const float o = (float)other;
  return clamp_u8(__fadd_rn(o, __fmul_rn(f, __fsub_rn((float)im, o))));
}

// grayscale (data.rs:144-156) of pixel p
__device__ __forceinline__ uint8_t gray1(const uint8_t* im, int p) {
  const float v = __fadd_rn(__fadd_rn(__fmul_rn(0.299f, (float)im[p]), __fmul_rn(0.587f, (float)im[PLANE + p])),
                            __fmul_rn(0.114f, (float)im[2 * PLANE + p]));
  return clamp_u8(v);
}

struct Draws {
  int op[MAX_RA];
  float v[MAX_RA];
  float sign[MAX_RA];
  float ct[MAX_RA], st[MAX_RA];  // cos t, sin t of a rotation (from the host)
  int dy, dx, flip;
  int erase, y0, y1, x0, x1;
  int nnoise;
};

__global__ void __launch_bounds__(THREADS) make_batch_train_kernel(
    const uint8_t* __restrict__ images, const uint8_t* __restrict__ labels, const uint8_t* __restrict__ coarse,
    size_t len, const uint32_t* __restrict__ idx, Aug aug, uint64_t seed, NormalTabs tabs,
    const float2* __restrict__ rot, float* __restrict__ out, uint32_t* __restrict__ labels_out,
    uint32_t* __restrict__ coarse_out, int* __restrict__ dev_error) {
  __shared__ uint8_t work[PIX], src[PIX], tmp[PIX];
  __shared__ uint32_t red[3][256];
  __shared__ uint32_t eq_lo[3];
  __shared__ Draws d;
  extern __shared__ uint32_t noise[];  // [2][nnoise_cap]: the 24-bit u1 then u2 of each normal
  const int tid = threadIdx.x;
  const int b = blockIdx.x;
  const size_t img = idx[b];
  if (img >= len) {  // the reference panics on the slice index; flag it and leave zeros
    if (tid == 0) {
      atomicOr(dev_error, DEV_ERR_INDEX);
      labels_out[b] = 0;
      if (coarse_out) coarse_out[b] = 0;
    }
    for (int i = tid; i < PIX; i += THREADS) out[(size_t)b * PIX + i] = 0.0f;
    return;
  }

  if (tid == 0) {
    labels_out[b] = labels[img];
    if (coarse && coarse_out) coarse_out[b] = coarse[img];
    Rng rng(seed ^ ((uint64_t)b * GOLDEN));
    // randaugment (data.rs:297-306) with apply_op's sign (data.rs:262)
    const int nra = aug.ra_mag > 0.0f ? aug.ra_n : 0;
    for (int i = 0; i < nra; i++) {
      d.op[i] = (int)(rng.next_u64() % NOPS);
      const float n = normal_dev(rng, tabs);
      d.v[i] = fminf(fmaxf(__fmul_rn(aug.ra_mag, __fadd_rn(1.0f, __fmul_rn(0.5f, n))), 0.0f), 1.0f);
      d.sign[i] = ((rng.next_u64() >> 32) & 1u) ? 1.0f : -1.0f;
      const float2 cs = rot[(size_t)b * MAX_RA + i];
      d.ct[i] = cs.x;
      d.st[i] = cs.y;
    }
    // crop_offset (data.rs:309-318), flip (data.rs:407)
    d.dy = d.dx = 0;
    if (aug.pad > 0) {
      d.dy = (int)(rng.next_u64() % (uint64_t)(2 * aug.pad + 1)) - aug.pad;
      d.dx = (int)(rng.next_u64() % (uint64_t)(2 * aug.pad + 1)) - aug.pad;
    }
    d.flip = (int)((rng.next_u64() >> 32) & 1u);
    // random_erase (data.rs:364-377): the rectangle, then the uniforms of its
    // normals in (c, y, x) order
    d.erase = 0;
    d.nnoise = 0;
    d.y0 = d.y1 = d.x0 = d.x1 = 0;
    if (aug.erase > 0.0f && !(rng.uniform() >= aug.erase)) {
      const int cy = (int)(rng.next_u64() % IMG), cx = (int)(rng.next_u64() % IMG);
      const int h = aug.erase_side / 2;
      d.y0 = max(cy - h, 0);
      d.y1 = min(cy + h, IMG);
      d.x0 = max(cx - h, 0);
      d.x1 = min(cx + h, IMG);
      const int cnt = d.y1 > d.y0 && d.x1 > d.x0 ? 3 * (d.y1 - d.y0) * (d.x1 - d.x0) : 0;
      d.erase = cnt > 0;
      d.nnoise = cnt;
      for (int k = 0; k < cnt; k++) {
        noise[k] = (uint32_t)(rng.next_u64() >> 40);
        noise[cnt + k] = (uint32_t)(rng.next_u64() >> 40);
      }
    }
  }
  for (int i = tid; i < PIX; i += THREADS) work[i] = images[img * PIX + i];
  __syncthreads();

  const int nra = aug.ra_mag > 0.0f ? aug.ra_n : 0;
  for (int r = 0; r < nra; r++) {
    const int op = d.op[r];
    const float v = d.v[r], sign = d.sign[r];
    const float f = __fadd_rn(1.0f, __fmul_rn(__fmul_rn(sign, 0.9f), v));
    if (op <= 4) {
      // affine (data.rs:114-135) with the parameters of data.rs:265-272
      float a = 1.0f, bb = 0.0f, tx = 0.0f, c_ = 0.0f, dd = 1.0f, ty = 0.0f;
      if (op == 0) bb = __fmul_rn(__fmul_rn(sign, 0.3f), v);
      if (op == 1) c_ = __fmul_rn(__fmul_rn(sign, 0.3f), v);
      if (op == 2) tx = __fmul_rn(__fmul_rn(sign, 10.0f), v);
      if (op == 3) ty = __fmul_rn(__fmul_rn(sign, 10.0f), v);
      if (op == 4) {  // t = sign 30 v pi / 180; cos t and sin t from the host
        a = d.ct[r];
        bb = -d.st[r];
        c_ = d.st[r];
        dd = d.ct[r];
      }
      for (int i = tid; i < PIX; i += THREADS) src[i] = work[i];
      __syncthreads();
      const float cy = 15.5f, cx = 15.5f;
      for (int i = tid; i < PIX; i += THREADS) {
        const int ch = i / PLANE, y = (i / IMG) % IMG, x = i % IMG;
        const float fy = __fsub_rn((float)y, cy), fx = __fsub_rn((float)x, cx);
        const float sx = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(a, fx), __fmul_rn(bb, fy)), tx), cx);
        const float sy = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(c_, fx), __fmul_rn(dd, fy)), ty), cy);
        const float x0f = floorf(sx), y0f = floorf(sy);
        const float wx = __fsub_rn(sx, x0f), wy = __fsub_rn(sy, y0f);
        const int x0 = (int)x0f, y0 = (int)y0f;
        const float ux = __fsub_rn(1.0f, wx), uy = __fsub_rn(1.0f, wy);
        float s = __fmul_rn(__fmul_rn(px(src, ch, y0, x0), ux), uy);
        s = __fadd_rn(s, __fmul_rn(__fmul_rn(px(src, ch, y0, x0 + 1), wx), uy));
        s = __fadd_rn(s, __fmul_rn(__fmul_rn(px(src, ch, y0 + 1, x0), ux), wy));
        s = __fadd_rn(s, __fmul_rn(__fmul_rn(px(src, ch, y0 + 1, x0 + 1), wx), wy));
        work[i] = clamp_u8(s);
      }
    } else if (op == 5) {  // posterize (data.rs:160-164)
      const uint32_t bits = 8u - (uint32_t)__fmul_rn(4.0f, v);
      const uint8_t mask = (uint8_t)~((1u << (8u - bits)) - 1u);
      for (int i = tid; i < PIX; i += THREADS) work[i] &= mask;
    } else if (op == 6) {  // solarize (data.rs:166-173)
      const uint8_t th = clamp_u8(__fmul_rn(255.0f, __fsub_rn(1.0f, v)));
      for (int i = tid; i < PIX; i += THREADS)
        if (work[i] >= th) work[i] = (uint8_t)(255 - work[i]);
    } else if (op == 7) {  // autocontrast (data.rs:176-187)
      if (tid < 3) {
        red[tid][0] = 255;
        red[tid][1] = 0;
      }
      __syncthreads();
      for (int i = tid; i < PIX; i += THREADS) {
        atomicMin(&red[i / PLANE][0], (uint32_t)work[i]);
        atomicMax(&red[i / PLANE][1], (uint32_t)work[i]);
      }
      __syncthreads();
      for (int i = tid; i < PIX; i += THREADS) {
        const uint32_t lo = red[i / PLANE][0], hi = red[i / PLANE][1];
        if (hi > lo) {
          const float k = __fdiv_rn(255.0f, (float)(hi - lo));
          work[i] = clamp_u8(__fmul_rn((float)(work[i] - lo), k));
        }
      }
    } else if (op == 8) {  // equalize (data.rs:190-207)
      for (int i = tid; i < 3 * 256; i += THREADS) red[i / 256][i % 256] = 0;
      __syncthreads();
      for (int i = tid; i < PIX; i += THREADS) atomicAdd(&red[i / PLANE][work[i]], 1u);
      __syncthreads();
      if (tid < 3) {  // inclusive prefix sum = cdf; lo = its first non-zero entry
        uint32_t acc = 0, lo = 0;
        for (int j = 0; j < 256; j++) {
          acc += red[tid][j];
          red[tid][j] = acc;
          if (lo == 0 && acc > 0) lo = acc;
        }
        eq_lo[tid] = lo;
      }
      __syncthreads();
      for (int i = tid; i < PIX; i += THREADS) {
        const uint32_t* cdf = red[i / PLANE];
        const uint32_t lo = eq_lo[i / PLANE];
        const uint32_t den = max((uint32_t)PLANE > lo ? (uint32_t)PLANE - lo : 0u, 1u);
        work[i] = (uint8_t)(((cdf[work[i]] - lo) * 255u) / den);
      }
    } else if (op == 9) {  // brightness (data.rs:209-212)
      for (int i = tid; i < PIX; i += THREADS) work[i] = blend1(work[i], 0, f);
    } else if (op == 10) {  // saturation (data.rs:214-217)
      for (int p = tid; p < PLANE; p += THREADS) tmp[p] = gray1(work, p);
      __syncthreads();
      for (int i = tid; i < PIX; i += THREADS) work[i] = blend1(work[i], tmp[i % PLANE], f);
    } else if (op == 11) {  // contrast (data.rs:219-224)
      if (tid == 0) red[0][0] = 0;
      __syncthreads();
      uint32_t part = 0;
      for (int p = tid; p < PLANE; p += THREADS) part += gray1(work, p);
      atomicAdd(&red[0][0], part);
      __syncthreads();
      const uint8_t mean = (uint8_t)(red[0][0] / PLANE);
      for (int i = tid; i < PIX; i += THREADS) work[i] = blend1(work[i], mean, f);
    } else {  // sharpness (data.rs:227-253)
      for (int i = tid; i < PIX; i += THREADS) src[i] = work[i];
      __syncthreads();
      for (int i = tid; i < PIX; i += THREADS) {
        const int ch = i / PLANE, y = (i / IMG) % IMG, x = i % IMG;
        uint8_t bl = src[i];
        if (y >= 1 && y < IMG - 1 && x >= 1 && x < IMG - 1) {
          float s = 0.0f;
          for (int dy = 0; dy < 3; dy++)
            for (int dx = 0; dx < 3; dx++) {
              const float w = (dy == 1 && dx == 1) ? 5.0f : 0.375f;
              s = __fadd_rn(s, __fmul_rn(w, px(src, ch, y + dy - 1, x + dx - 1)));
            }
          bl = clamp_u8(__fdiv_rn(s, 8.0f));
        }
        tmp[i] = bl;
      }
      __syncthreads();
      for (int i = tid; i < PIX; i += THREADS) work[i] = blend1(src[i], tmp[i], f);
    }
    __syncthreads();
  }

  // crop_flip_normalize (data.rs:331-360) and the erased rectangle
  float* dst = out + (size_t)b * PIX;
  const int ny = d.y1 - d.y0, nx = d.x1 - d.x0;
  for (int i = tid; i < PIX; i += THREADS) {
    const int c = i / PLANE, y = (i / IMG) % IMG, x = i % IMG;
    float val;
    if (d.erase && y >= d.y0 && y < d.y1 && x >= d.x0 && x < d.x1) {
      const int k = (c * ny + (y - d.y0)) * nx + (x - d.x0);
      val = normal_of(tabs, noise[k], noise[d.nnoise + k]);
    } else {
      const int sy = y + d.dy;
      const int sx = (d.flip ? IMG - 1 - x : x) + d.dx;
      if (sy >= 0 && sy < IMG && sx >= 0 && sx < IMG)
        val = __fdiv_rn(__fsub_rn(__fdiv_rn((float)work[c * PLANE + sy * IMG + sx], 255.0f), mean_of(c)), std_of(c));
      else
        val = __fdiv_rn(-mean_of(c), std_of(c));
    }
    dst[i] = val;
  }
}

// mixup (data.rs:459-469): x[b] = l * src[b] + (1 - l) * src[perm[b]]
__global__ void mixup_kernel(float* __restrict__ x, const float* __restrict__ src, const uint32_t* __restrict__ perm,
                             int bs, float l) {
  const size_t n4 = (size_t)bs * (PIX / 4);
  const float m = __fsub_rn(1.0f, l);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const size_t b = i / (PIX / 4), o = i % (PIX / 4);
    const float4 a = reinterpret_cast<const float4*>(src)[i];
    const float4 p = reinterpret_cast<const float4*>(src)[(size_t)perm[b] * (PIX / 4) + o];
    float4 r;
    r.x = __fadd_rn(__fmul_rn(l, a.x), __fmul_rn(m, p.x));
    r.y = __fadd_rn(__fmul_rn(l, a.y), __fmul_rn(m, p.y));
    r.z = __fadd_rn(__fmul_rn(l, a.z), __fmul_rn(m, p.z));
    r.w = __fadd_rn(__fmul_rn(l, a.w), __fmul_rn(m, p.w));
    reinterpret_cast<float4*>(x)[i] = r;
  }
}

// cutmix (data.rs:436-456): the rectangle of image perm[b] pasted into b
__global__ void cutmix_kernel(float* __restrict__ x, const float* __restrict__ src, const uint32_t* __restrict__ perm,
                              int bs, int y0, int y1, int x0, int x1) {
  const int ny = y1 - y0, nx = x1 - x0;
  const size_t n = (size_t)bs * 3 * ny * nx;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t b = i / (3 * ny * nx);
    const int r = (int)(i % (3 * ny * nx));
    const int c = r / (ny * nx), y = y0 + (r / nx) % ny, xx = x0 + r % nx;
    const int o = c * PLANE + y * IMG + xx;
    x[b * PIX + o] = src[(size_t)perm[b] * PIX + o];
  }
}

// beta_like (data.rs:417-431) on the host
float beta_like(float a, Rng& rng) {
  const float u = rng.uniform();
  if (a >= 1.0f) return u;
  if (u < 0.5f) return powf(2.0f * u, 1.0f / a) * 0.5f;
  return 1.0f - powf(2.0f * (1.0f - u), 1.0f / a) * 0.5f;
}

// The Box-Muller tables of one device, computed on first use with the C
// library's logf / cosf (the functions the reference calls) over every 24-bit
// uniform, and kept until exit.
std::mutex g_tab_mu;
NormalTabs g_tabs[64];

int normal_tables(int device, NormalTabs* out) {
  RNN_REQUIRE(device >= 0 && device < 64, "make_batch_train: device ordinal %d >= 64", device);
  std::lock_guard<std::mutex> lock(g_tab_mu);
  if (!g_tabs[device].ln) {
    std::vector<float> host(2 * (size_t)NORMAL_TAB);
    const unsigned nth = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    std::vector<std::thread> pool;
    for (unsigned t = 0; t < nth; t++)
      pool.emplace_back([&host, t, nth] {
        const size_t lo = (size_t)NORMAL_TAB * t / nth, hi = (size_t)NORMAL_TAB * (t + 1) / nth;
        for (size_t k = lo; k < hi; k++) {
          const float u = (float)k * (1.0f / (float)NORMAL_TAB);  // Rng::uniform, exact
          const float u1 = u < 1e-7f ? 1e-7f : u;
          const float arg = TAU * u;  // one f32 rounding, as the reference's product
          host[k] = logf(u1);
          host[NORMAL_TAB + k] = cosf(arg);
        }
      });
    for (auto& th : pool) th.join();
    int prev = 0;
    RNN_CUDA(cudaGetDevice(&prev));
    RNN_CUDA(cudaSetDevice(device));
    float* dev = nullptr;
    cudaError_t e = cudaMalloc(&dev, sizeof(float) * host.size());
    if (e == cudaSuccess) {
      e = cudaMemcpy(dev, host.data(), sizeof(float) * host.size(), cudaMemcpyHostToDevice);
      if (e != cudaSuccess) cudaFree(dev);
    }
    cudaSetDevice(prev);
    RNN_CUDA(e);
    g_tabs[device].ln = dev;
    g_tabs[device].cs = dev + NORMAL_TAB;
  }
  *out = g_tabs[device];
  return RNN_OK;
}

}  // namespace

int make_batch_train(rnn_ctx* ctx, const uint8_t* images, const uint8_t* labels, const uint8_t* coarse,
                     size_t len, const uint32_t* idx, int bs, int pad, float ra_mag, int ra_n, float erase, int erase_side,
                     uint64_t seed, float* out, uint32_t* labels_out, uint32_t* coarse_out) {
  RNN_REQUIRE(bs >= 0 && pad >= 0 && ra_n >= 0 && erase_side >= 0, "make_batch_train: negative argument");
  RNN_REQUIRE(ra_mag <= 0.0f || ra_n <= MAX_RA, "make_batch_train: at most %d RandAugment ops (ra_n %d)", MAX_RA,
              ra_n);
  if (bs == 0) return RNN_OK;
  RNN_RANGE(images, (size_t)PIX * len);
  RNN_RANGE(labels, len);
  if (coarse) RNN_RANGE(coarse, len);
  RNN_RANGE(idx, sizeof(uint32_t) * (size_t)bs);
  RNN_RANGE(out, sizeof(float) * (size_t)bs * PIX);
  RNN_RANGE(labels_out, sizeof(uint32_t) * (size_t)bs);
  if (coarse_out) RNN_RANGE(coarse_out, sizeof(uint32_t) * (size_t)bs);
  const int span = erase > 0.0f ? std::min(2 * (erase_side / 2), IMG) : 0;
  const size_t smem = sizeof(uint32_t) * 2 * 3 * (size_t)span * span;
  Aug aug{pad, ra_mag, ra_n, erase, erase_side};
  const int nra = ra_mag > 0.0f ? ra_n : 0;
  NormalTabs tabs{nullptr, nullptr};
  if (nra > 0 || erase > 0.0f) RNN_TRY(normal_tables(ctx->device, &tabs));
  // cos t / sin t of every rotation: replay each image's RandAugment draws
  // (data.rs:297-306, 262-266) with the host's C library, in the order the
  // kernel draws them
  std::vector<float2> rot((size_t)bs * MAX_RA, make_float2(1.0f, 0.0f));
  bool any_rot = false;
  for (int b = 0; b < bs && nra > 0; b++) {
    Rng rng(seed ^ ((uint64_t)b * GOLDEN));
    for (int i = 0; i < nra; i++) {
      const int op = (int)(rng.next_u64() % NOPS);
      const float n = rng.normal();
      float v = ra_mag * (1.0f + 0.5f * n);
      v = std::min(std::max(v, 0.0f), 1.0f);
      const float sign = ((rng.next_u64() >> 32) & 1u) ? 1.0f : -1.0f;
      if (op == 4) {
        const float t = sign * 30.0f * v * 3.14159265358979323846f / 180.0f;
        rot[(size_t)b * MAX_RA + i] = make_float2(cosf(t), sinf(t));
        any_rot = true;
      }
    }
  }
  const float2* drot = nullptr;
  if (any_rot) {
    RNN_TRY(ensure_ws(ctx, sizeof(float2) * rot.size()));
    RNN_CUDA(cudaMemcpyAsync(ctx->ws, rot.data(), sizeof(float2) * rot.size(), cudaMemcpyHostToDevice,
                             ctx->stream));
    drot = static_cast<const float2*>(ctx->ws);
  } else if (nra > 0) {
    // no image rotates: the kernel still reads its (unused) slots
    RNN_TRY(ensure_ws(ctx, sizeof(float2) * rot.size()));
    RNN_CUDA(cudaMemsetAsync(ctx->ws, 0, sizeof(float2) * rot.size(), ctx->stream));
    drot = static_cast<const float2*>(ctx->ws);
  }
  make_batch_train_kernel<<<bs, THREADS, smem, ctx->stream>>>(images, labels, coarse, len, idx, aug, seed, tabs,
                                                              drot, out, labels_out, coarse_out, ctx->dev_error);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int mix_batch(rnn_ctx* ctx, float* x, int bs, float alpha_mix, float alpha_cut, float sw, uint64_t* state,
              uint32_t* perm_out, float* lam_out) {
  RNN_REQUIRE(bs >= 0, "mix_batch: negative batch");
  Rng rng(0);
  for (int i = 0; i < 4; i++) rng.s[i] = state[i];
  std::vector<uint32_t> perm(bs);
  for (int i = 0; i < bs; i++) perm[i] = (uint32_t)i;
  for (int i = bs - 1; i >= 1; i--) {  // Rng::shuffle (rng.rs:61-65)
    const uint32_t j = (uint32_t)(rng.next_u64() % (uint64_t)(i + 1));
    std::swap(perm[i], perm[j]);
  }
  std::vector<float> lam(bs, 1.0f);
  if (!(alpha_mix <= 0.0f && alpha_cut <= 0.0f) && bs > 0) {
    const bool cut = alpha_cut > 0.0f && (alpha_mix <= 0.0f || rng.uniform() < sw);
    const float l = beta_like(cut ? alpha_cut : alpha_mix, rng);
    RNN_RANGE(x, sizeof(float) * (size_t)bs * PIX);
    RNN_REQUIRE(((uintptr_t)x & 15) == 0, "mix_batch: x must be 16-byte aligned");
    const size_t xbytes = sizeof(float) * (size_t)bs * PIX;
    RNN_TRY(ensure_ws(ctx, xbytes + sizeof(uint32_t) * (size_t)bs));
    float* src = static_cast<float*>(ctx->ws);
    uint32_t* dperm = reinterpret_cast<uint32_t*>(static_cast<char*>(ctx->ws) + xbytes);
    RNN_CUDA(cudaMemcpyAsync(src, x, xbytes, cudaMemcpyDeviceToDevice, ctx->stream));
    RNN_CUDA(cudaMemcpyAsync(dperm, perm.data(), sizeof(uint32_t) * (size_t)bs, cudaMemcpyHostToDevice,
                             ctx->stream));
    if (cut) {
      const float r = sqrtf(1.0f - l);
      const int side = std::min((int)((float)IMG * r), IMG);
      const int cy = (int)(rng.next_u64() % IMG), cx = (int)(rng.next_u64() % IMG);
      const int y0 = std::max(cy - side / 2, 0), y1 = std::min(cy + side / 2, IMG);
      const int x0 = std::max(cx - side / 2, 0), x1 = std::min(cx + side / 2, IMG);
      const float area = (float)((y1 - y0) * (x1 - x0)) / (float)(IMG * IMG);
      for (int b = 0; b < bs; b++) lam[b] = 1.0f - area;
      const size_t n = (size_t)bs * 3 * (y1 - y0) * (x1 - x0);
      if (n > 0) {
        cutmix_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 4096), 256, 0, ctx->stream>>>(
            x, src, dperm, bs, y0, y1, x0, x1);
        RNN_CHECK_LAUNCH();
      }
    } else {
      for (int b = 0; b < bs; b++) lam[b] = l;
      const size_t n4 = (size_t)bs * (PIX / 4);
      mixup_kernel<<<(unsigned)std::min<size_t>((n4 + 255) / 256, 4096), 256, 0, ctx->stream>>>(x, src, dperm, bs,
                                                                                              l);
      RNN_CHECK_LAUNCH();
    }
    // (a copy from pageable memory is staged before cudaMemcpyAsync returns,
    // so `perm` may leave scope while the kernel runs)
  }
  for (int i = 0; i < 4; i++) state[i] = rng.s[i];
  if (perm_out) std::copy(perm.begin(), perm.end(), perm_out);
  if (lam_out) std::copy(lam.begin(), lam.end(), lam_out);
  return RNN_OK;
}

}  // namespace rnn

extern "C" int rnn_make_batch_train_dev(rnn_ctx* ctx, const uint8_t* images, const uint8_t* labels,
                                        const uint8_t* coarse, size_t len, const uint32_t* idx, int bs, int pad,
                                        float ra_mag, int ra_n, float erase, int erase_side, uint64_t seed, float* out,
                                        uint32_t* labels_out, uint32_t* coarse_out) {
  RNN_REQUIRE(ctx && images && labels && idx && out && labels_out, "make_batch_train: null argument");
  return rnn::make_batch_train(ctx, images, labels, coarse, len, idx, bs, pad, ra_mag, ra_n, erase, erase_side, seed, out,
                               labels_out, coarse_out);
}

extern "C" int rnn_mix_batch_dev(rnn_ctx* ctx, float* x, int bs, float alpha_mix, float alpha_cut, float sw,
                                 uint64_t* rng_state, uint32_t* perm, float* lam) {
  RNN_REQUIRE(ctx && rng_state && (bs == 0 || x), "mix_batch: null argument");
  return rnn::mix_batch(ctx, x, bs, alpha_mix, alpha_cut, sw, rng_state, perm, lam);
}
