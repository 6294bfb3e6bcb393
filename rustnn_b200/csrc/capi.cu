// Context, error reporting and the host-pointer tier of the C ABI.
#include <cuda.h>
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "ew.cuh"

namespace rnn {

static thread_local char g_err[1024] = "";
unsigned long long g_launches = 0;

static int env_flag(const char* name) {
  const char* v = getenv(name);
  return v && v[0] && v[0] != '0';
}

bool range_checks_enabled() {
  static const int on = env_flag("RNN_CHECK_RANGES");
  return on != 0;
}

bool debug_sync_enabled() {
  static const int on = env_flag("RNN_DEBUG_SYNC");
  return on != 0;
}

typedef CUresult (*GetRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

static GetRangeFn get_range_fn() {
  static GetRangeFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetRangeFn>(p);
  }
  return fn;
}

int check_range(const void* p, size_t bytes, const char* what, const char* file, int line) {
  if (bytes == 0) return RNN_OK;
  if (p == nullptr) return set_error(RNN_ERR_ARG, "%s:%d: %s is null but %zu bytes are accessed", file, line, what, bytes);
  GetRangeFn fn = get_range_fn();
  if (!fn) return set_error(RNN_ERR_CUDA, "range check: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = fn(&base, &size, reinterpret_cast<CUdeviceptr>(p));
  if (r != CUDA_SUCCESS)
    return set_error(RNN_ERR_ARG, "%s:%d: %s = %p is not in a device allocation (CUresult %d)", file, line, what, p,
                     (int)r);
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  if (a + bytes > (uintptr_t)base + size)
    return set_error(RNN_ERR_ARG, "%s:%d: %s = %p + %zu bytes overruns its allocation [%p, +%zu)", file, line, what,
                     p, bytes, (void*)base, size);
  return RNN_OK;
}

int debug_sync_check(const char* file, int line) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_error(RNN_ERR_CUDA, "%s:%d: kernel failed: %s", file, line, cudaGetErrorString(e));
  return RNN_OK;
}

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int ensure_ws(rnn_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->ws_bytes) return RNN_OK;
  size_t want = std::max(bytes, ctx->ws_bytes * 2);
  want = (want + (1 << 20) - 1) & ~(size_t)((1 << 20) - 1);
  if (ctx->ws) {
    RNN_CUDA(cudaStreamSynchronize(ctx->stream));
    RNN_CUDA(cudaFree(ctx->ws));
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
  }
  RNN_CUDA(cudaMalloc(&ctx->ws, want));
  ctx->ws_bytes = want;
  ctx->mem_epoch++;
  return RNN_OK;
}

int ensure_stage(rnn_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->stage_bytes) return RNN_OK;
  size_t want = std::max(bytes, ctx->stage_bytes * 2);
  want = (want + (1 << 20) - 1) & ~(size_t)((1 << 20) - 1);
  if (ctx->stage) {
    RNN_CUDA(cudaStreamSynchronize(ctx->stream));
    RNN_CUDA(cudaFree(ctx->stage));
    ctx->stage = nullptr;
    ctx->stage_bytes = 0;
  }
  RNN_CUDA(cudaMalloc(&ctx->stage, want));
  ctx->stage_bytes = want;
  ctx->mem_epoch++;
  return RNN_OK;
}

int ensure_aux(rnn_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->aux_bytes) return RNN_OK;
  size_t want = std::max(bytes, ctx->aux_bytes * 2);
  want = (want + (1 << 20) - 1) & ~(size_t)((1 << 20) - 1);
  if (ctx->aux) {
    RNN_CUDA(cudaStreamSynchronize(ctx->stream));
    RNN_CUDA(cudaFree(ctx->aux));
    ctx->aux = nullptr;
    ctx->aux_bytes = 0;
  }
  RNN_CUDA(cudaMalloc(&ctx->aux, want));
  ctx->aux_bytes = want;
  ctx->mem_epoch++;
  return RNN_OK;
}

int ensure_statp(rnn_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->statp_bytes) return RNN_OK;
  size_t want = std::max(bytes, (size_t)1 << 20);
  if (ctx->statp) {
    RNN_CUDA(cudaStreamSynchronize(ctx->stream));
    RNN_CUDA(cudaFree(ctx->statp));
    ctx->statp = nullptr;
    ctx->statp_bytes = 0;
  }
  RNN_CUDA(cudaMalloc(&ctx->statp, want));
  ctx->statp_bytes = want;
  ctx->mem_epoch++;
  return RNN_OK;
}

int ensure_pack(rnn_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->pack_bytes) return RNN_OK;
  size_t want = std::max(bytes, ctx->pack_bytes * 2);
  want = (want + (1 << 20) - 1) & ~(size_t)((1 << 20) - 1);
  if (ctx->pack) {
    RNN_CUDA(cudaStreamSynchronize(ctx->stream));
    RNN_CUDA(cudaFree(ctx->pack));
    ctx->pack = nullptr;
    ctx->pack_bytes = 0;
  }
  RNN_CUDA(cudaMalloc(&ctx->pack, want));
  ctx->pack_bytes = want;
  ctx->mem_epoch++;
  return RNN_OK;
}

}  // namespace rnn

using namespace rnn;

extern "C" const char* rnn_last_error(void) { return g_err; }

extern "C" unsigned long long rnn_launch_count(void) { return __atomic_load_n(&g_launches, __ATOMIC_RELAXED); }

extern "C" int rnn_device_ok(int device) {
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, device) != cudaSuccess) return 0;
  return p.major == 10 && p.minor == 0 ? 1 : 0;
}

extern "C" int rnn_ctx_create(rnn_ctx** out, int device) {
  RNN_REQUIRE(out != nullptr, "ctx_create: null out");
  *out = nullptr;
  RNN_CUDA(cudaSetDevice(device));
  cudaDeviceProp p;
  RNN_CUDA(cudaGetDeviceProperties(&p, device));
  if (!(p.major == 10 && p.minor == 0))
    return set_error(RNN_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200)",
                     device, p.major, p.minor);
  rnn_ctx* ctx = new rnn_ctx();
  ctx->device = device;
  ctx->num_sms = p.multiProcessorCount;
  cudaError_t e = cudaStreamCreateWithFlags(&ctx->own, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete ctx;
    return set_error(RNN_ERR_CUDA, "stream create: %s", cudaGetErrorString(e));
  }
  ctx->stream = ctx->own;
  e = cudaMalloc(&ctx->dev_error, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(ctx->dev_error, 0, sizeof(int));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->counters, 16 * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(ctx->counters, 0, 16 * sizeof(unsigned));
  if (e != cudaSuccess) {
    cudaStreamDestroy(ctx->own);
    delete ctx;
    return set_error(RNN_ERR_CUDA, "ctx alloc: %s", cudaGetErrorString(e));
  }
  *out = ctx;
  return RNN_OK;
}

extern "C" int rnn_ctx_destroy(rnn_ctx* ctx) {
  if (!ctx) return RNN_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->ws) cudaFree(ctx->ws);
  if (ctx->stage) cudaFree(ctx->stage);
  if (ctx->pack) cudaFree(ctx->pack);
  if (ctx->aux) cudaFree(ctx->aux);
  if (ctx->dev_error) cudaFree(ctx->dev_error);
  if (ctx->counters) cudaFree(ctx->counters);
  if (ctx->statp) cudaFree(ctx->statp);
  if (ctx->own) cudaStreamDestroy(ctx->own);
  delete ctx;
  return RNN_OK;
}

extern "C" int rnn_ctx_set_stream(rnn_ctx* ctx, void* stream) {
  RNN_REQUIRE(ctx != nullptr, "null context");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (s == ctx->stream) return RNN_OK;
  // work already queued on the old stream finishes before the switch
  RNN_CUDA(cudaStreamSynchronize(ctx->stream));
  ctx->stream = s;
  return RNN_OK;
}

extern "C" int rnn_ctx_use_own_stream(rnn_ctx* ctx) {
  RNN_REQUIRE(ctx != nullptr, "null context");
  return rnn_ctx_set_stream(ctx, ctx->own);
}

extern "C" void* rnn_ctx_stream(rnn_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

extern "C" int rnn_ctx_synchronize(rnn_ctx* ctx) {
  RNN_REQUIRE(ctx != nullptr, "null context");
  RNN_CUDA(cudaStreamSynchronize(ctx->stream));
  int err = 0;
  RNN_CUDA(cudaMemcpy(&err, ctx->dev_error, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) {
    RNN_CUDA(cudaMemset(ctx->dev_error, 0, sizeof(int)));
    return set_error(RNN_ERR_DEVICE, "device error 0x%x (%s%s%s%s)", err,
                     (err & 1) ? "a kernel gave up waiting on a pipeline barrier " : "",
                     (err & 2) ? "a label is >= nclass " : "",
                     (err & 4) ? "a peer GPU did not publish its statistics in time " : "",
                     (err & 8) ? "a batch index is outside the dataset" : "");
  }
  return RNN_OK;
}

// ---------------------------------------------------------------- host tier
// Each call stages its operands in the context's staging buffer, runs the
// device entry point and copies the result back.

namespace {
struct Staged {
  char* base;
  size_t off = 0;
  float* take(size_t n) {
    float* p = reinterpret_cast<float*>(base + off);
    off += (n * sizeof(float) + 255) & ~(size_t)255;
    return p;
  }
};
size_t padded(size_t n) { return (n * sizeof(float) + 255) & ~(size_t)255; }
}  // namespace

#define H2D(dst, src, n) RNN_CUDA(cudaMemcpyAsync(dst, src, (n) * sizeof(float), cudaMemcpyHostToDevice, ctx->stream))
#define D2H(dst, src, n) RNN_CUDA(cudaMemcpyAsync(dst, src, (n) * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream))

extern "C" int rnn_gemm(rnn_ctx* ctx, int m, int n, int k, const float* a, int at, const float* b, int bt,
                        float* c, int acc) {
  RNN_REQUIRE(ctx != nullptr, "null context");
  size_t na = (size_t)m * k, nb = (size_t)k * n, nc = (size_t)m * n;
  RNN_TRY(ensure_stage(ctx, padded(na) + padded(nb) + padded(nc)));
  Staged s{static_cast<char*>(ctx->stage)};
  float *da = s.take(na), *db = s.take(nb), *dc = s.take(nc);
  H2D(da, a, na);
  H2D(db, b, nb);
  if (acc) H2D(dc, c, nc);
  RNN_TRY(rnn_gemm_dev(ctx, m, n, k, da, at, db, bt, dc, acc));
  D2H(c, dc, nc);
  return rnn_ctx_synchronize(ctx);
}

extern "C" int rnn_gemm_dw(rnn_ctx* ctx, int m, int n, int k, const float* a, const float* b, float* c) {
  RNN_REQUIRE(ctx != nullptr, "null context");
  size_t na = (size_t)k * m, nb = (size_t)k * n, nc = (size_t)m * n;
  RNN_TRY(ensure_stage(ctx, padded(na) + padded(nb) + padded(nc)));
  Staged s{static_cast<char*>(ctx->stage)};
  float *da = s.take(na), *db = s.take(nb), *dc = s.take(nc);
  H2D(da, a, na);
  H2D(db, b, nb);
  H2D(dc, c, nc);
  RNN_TRY(rnn_gemm_dw_dev(ctx, m, n, k, da, db, dc));
  D2H(c, dc, nc);
  return rnn_ctx_synchronize(ctx);
}

static int out_dim(int h, int k, int stride, int pad) { return (h + 2 * pad - k) / stride + 1; }

extern "C" int rnn_conv2d_fwd(rnn_ctx* ctx, const float* x, int n, int cin, int h, int w, const float* wt, int cout,
                              int k, int stride, int pad, float* y) {
  RNN_REQUIRE(ctx != nullptr, "null context");
  const int oh = out_dim(h, k, stride, pad), ow = out_dim(w, k, stride, pad);
  RNN_REQUIRE(oh > 0 && ow > 0, "conv2d_fwd: empty output");
  size_t nx = (size_t)n * cin * h * w, nw = (size_t)cout * cin * k * k, ny = (size_t)n * cout * oh * ow;
  RNN_TRY(ensure_stage(ctx, padded(nx) + padded(nw) + padded(ny)));
  Staged s{static_cast<char*>(ctx->stage)};
  float *dx = s.take(nx), *dw = s.take(nw), *dy = s.take(ny);
  H2D(dx, x, nx);
  H2D(dw, wt, nw);
  RNN_TRY(rnn_conv2d_fwd_dev(ctx, dx, n, cin, h, w, dw, cout, k, stride, pad, dy, 0));
  D2H(y, dy, ny);
  return rnn_ctx_synchronize(ctx);
}

extern "C" int rnn_conv2d_dgrad(rnn_ctx* ctx, const float* dy, int n, int cin, int h, int w, const float* wt,
                                int cout, int k, int stride, int pad, float* dx) {
  RNN_REQUIRE(ctx != nullptr, "null context");
  const int oh = out_dim(h, k, stride, pad), ow = out_dim(w, k, stride, pad);
  RNN_REQUIRE(oh > 0 && ow > 0, "conv2d_dgrad: empty output");
  size_t nx = (size_t)n * cin * h * w, nw = (size_t)cout * cin * k * k, ny = (size_t)n * cout * oh * ow;
  RNN_TRY(ensure_stage(ctx, padded(nx) + padded(nw) + padded(ny)));
  Staged s{static_cast<char*>(ctx->stage)};
  float *ddx = s.take(nx), *dw = s.take(nw), *ddy = s.take(ny);
  H2D(ddy, dy, ny);
  H2D(dw, wt, nw);
  RNN_TRY(rnn_conv2d_dgrad_dev(ctx, ddy, n, cin, h, w, dw, cout, k, stride, pad, ddx, 0));
  D2H(dx, ddx, nx);
  return rnn_ctx_synchronize(ctx);
}

extern "C" int rnn_conv2d_wgrad(rnn_ctx* ctx, const float* x, const float* dy, int n, int cin, int h, int w,
                                int cout, int k, int stride, int pad, float* dw) {
  RNN_REQUIRE(ctx != nullptr, "null context");
  const int oh = out_dim(h, k, stride, pad), ow = out_dim(w, k, stride, pad);
  RNN_REQUIRE(oh > 0 && ow > 0, "conv2d_wgrad: empty output");
  size_t nx = (size_t)n * cin * h * w, nw = (size_t)cout * cin * k * k, ny = (size_t)n * cout * oh * ow;
  RNN_TRY(ensure_stage(ctx, padded(nx) + padded(nw) + padded(ny)));
  Staged s{static_cast<char*>(ctx->stage)};
  float *ddx = s.take(nx), *ddw = s.take(nw), *ddy = s.take(ny);
  H2D(ddx, x, nx);
  H2D(ddy, dy, ny);
  H2D(ddw, dw, nw);
  RNN_TRY(rnn_conv2d_wgrad_dev(ctx, ddx, ddy, n, cin, h, w, cout, k, stride, pad, ddw));
  D2H(dw, ddw, nw);
  return rnn_ctx_synchronize(ctx);
}
