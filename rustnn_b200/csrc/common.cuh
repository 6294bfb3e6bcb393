// Shared host/device plumbing for librnn_b200: status codes, the per-thread
// error string, the context (stream + device workspace + device error word).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <string>

#include "../../include/rnn_b200.h"

namespace rnn {

// Sets the thread-local message returned by rnn_last_error() and returns code.
int set_error(int code, const char* fmt, ...);

#define RNN_CUDA(call)                                                              \
  do {                                                                              \
    cudaError_t e__ = (call);                                                       \
    if (e__ != cudaSuccess)                                                         \
      return ::rnn::set_error(RNN_ERR_CUDA, "%s:%d %s: %s", __FILE__, __LINE__,     \
                              #call, cudaGetErrorString(e__));                      \
  } while (0)

// Every kernel launch of the library is followed by RNN_CHECK_LAUNCH(), which
// also counts it (rnn_launch_count()).
extern unsigned long long g_launches;
#define RNN_CHECK_LAUNCH()                                   \
  do {                                                       \
    __atomic_add_fetch(&::rnn::g_launches, 1ull, __ATOMIC_RELAXED); \
    RNN_CUDA(cudaGetLastError());                            \
  } while (0)

#define RNN_REQUIRE(cond, ...)                                  \
  do {                                                          \
    if (!(cond)) return ::rnn::set_error(RNN_ERR_ARG, __VA_ARGS__); \
  } while (0)

#define RNN_TRY(expr)          \
  do {                         \
    int s__ = (expr);          \
    if (s__ != RNN_OK) return s__; \
  } while (0)

// Device-side error word.  Kernels with bounded waits OR in a code instead of
// hanging; the host reads it at rnn_ctx_synchronize().
enum DeviceError : int {
  DEV_ERR_TIMEOUT = 1,
};

}  // namespace rnn

struct rnn_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  // growable device workspace (split-K partials, BN partial sums, host-API
  // staging).  Reused across calls: all users run in stream order.
  void* ws = nullptr;
  size_t ws_bytes = 0;
  int* dev_error = nullptr;  // one int in device memory
  // host-API staging buffer
  void* stage = nullptr;
  size_t stage_bytes = 0;
};

namespace rnn {
// Ensures ctx->ws holds at least `bytes`.  Synchronises the stream before
// growing so no in-flight kernel still reads the old buffer.
int ensure_ws(rnn_ctx* ctx, size_t bytes);
int ensure_stage(rnn_ctx* ctx, size_t bytes);
}  // namespace rnn
