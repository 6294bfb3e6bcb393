// Shared host/device plumbing for librnn_b200: status codes, the per-thread
// error string, the context (stream + device workspace + device error word).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <string>
#include <vector>

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
// With RNN_DEBUG_SYNC=1 it also waits for the kernel and names the launch
// site of a failing kernel.
extern unsigned long long g_launches;
bool debug_sync_enabled();
int debug_sync_check(const char* file, int line);
#define RNN_CHECK_LAUNCH()                                                \
  do {                                                                    \
    __atomic_add_fetch(&::rnn::g_launches, 1ull, __ATOMIC_RELAXED);       \
    RNN_CUDA(cudaGetLastError());                                         \
    if (::rnn::debug_sync_enabled()) {                                    \
      int d__ = ::rnn::debug_sync_check(__FILE__, __LINE__);             \
      if (d__ != RNN_OK) return d__;                                      \
    }                                                                     \
  } while (0)

#define RNN_REQUIRE(cond, ...)                                  \
  do {                                                          \
    if (!(cond)) return ::rnn::set_error(RNN_ERR_ARG, __VA_ARGS__); \
  } while (0)

// Launch-argument validation (enabled with RNN_CHECK_RANGES=1): every device
// range a launch will touch must lie inside one live device allocation; a
// violation is reported as RNN_ERR_ARG and the launch is not made.
bool range_checks_enabled();
int check_range(const void* p, size_t bytes, const char* what, const char* file, int line);
#define RNN_RANGE(p, bytes)                                                          \
  do {                                                                               \
    if (::rnn::range_checks_enabled()) {                                             \
      int r__ = ::rnn::check_range((const void*)(p), (size_t)(bytes), #p, __FILE__, __LINE__); \
      if (r__ != RNN_OK) return r__;                                                 \
    }                                                                                \
  } while (0)

#define RNN_TRY(expr)          \
  do {                         \
    int s__ = (expr);          \
    if (s__ != RNN_OK) return s__; \
  } while (0)

// Device-side error word.  Kernels with bounded waits OR in a code instead of
// hanging; the host reads it at rnn_ctx_synchronize().
enum DeviceError : int {
  DEV_ERR_TIMEOUT = 1,  // a pipeline wait gave up
  DEV_ERR_LABEL = 2,    // softmax_ce saw a label >= nclass
  DEV_ERR_PEER = 4,     // a peer GPU did not publish its SyncBN sums in time
  DEV_ERR_INDEX = 8,    // a batch index is outside its dataset
};

}  // namespace rnn

struct rnn_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;  // stream every call enqueues on
  cudaStream_t own = nullptr;     // the context's own stream
  // growable device workspace (split-K partials, BN partial sums, host-API
  // staging).  Reused across calls: all users run in stream order.
  void* ws = nullptr;
  size_t ws_bytes = 0;
  int* dev_error = nullptr;  // one int in device memory
  // host-API staging buffer
  void* stage = nullptr;
  size_t stage_bytes = 0;
  // packed B-operand images (weights in the MMA's shared-memory layout)
  void* pack = nullptr;
  size_t pack_bytes = 0;
  // optimiser scratch (Newton-Schulz iterates), separate from ws because the
  // GEMMs it issues use ws for their split-K partials
  void* aux = nullptr;
  size_t aux_bytes = 0;
  // per-CTA partial sums of the convolution epilogues' BN statistics
  void* statp = nullptr;
  size_t statp_bytes = 0;
  // device counters for kernels whose last CTA finishes a reduction
  // (zeroed at creation; each such kernel leaves its slot at zero again)
  unsigned* counters = nullptr;
  // bumped whenever a workspace above is reallocated, so that a captured
  // CUDA graph holding the old pointers is recaptured instead of replayed
  unsigned long long mem_epoch = 0;
};

namespace rnn {
// Ensures ctx->ws holds at least `bytes`.  Synchronises the stream before
// growing so no in-flight kernel still reads the old buffer.
int ensure_ws(rnn_ctx* ctx, size_t bytes);
int ensure_stage(rnn_ctx* ctx, size_t bytes);
int ensure_pack(rnn_ctx* ctx, size_t bytes);
int ensure_aux(rnn_ctx* ctx, size_t bytes);
int ensure_statp(rnn_ctx* ctx, size_t bytes);
// ctx->counters slots: 0 BatchNorm partial-sum kernels, 1 convolution
// epilogue statistics, 2 .. 15 the one-launch column sums (colsum.cuh)
constexpr int COUNTER_BN = 0, COUNTER_CONV_STATS = 1;

// ---- CUDA-graph replay of a whole training step
//
// run_step_graph(ctx, g, key, body) performs one step per call.  `body`
// enqueues the step's work (kernels, memsets, device copies, NCCL calls) on
// ctx->stream and must not synchronise.  The first call with a given key
// runs body eagerly (which sizes every lazily grown workspace); the second
// captures it on a private stream into a graph and launches the graph; later
// calls with the same key replay the graph.  The key must hold every value
// the body bakes into launches (pointers, sizes, scalars) and the epochs of
// the allocations it uses; a changed key drops the graph.
struct StepGraph {
  cudaGraphExec_t exec = nullptr;
  cudaStream_t cap = nullptr;
  cudaEvent_t ev = nullptr;
  std::vector<unsigned long long> key, last_key;
  unsigned long long kernels = 0;  // launches per replay, for rnn_launch_count
  void release() {
    if (exec) cudaGraphExecDestroy(exec);
    exec = nullptr;
    key.clear();
  }
  void destroy() {
    release();
    if (cap) cudaStreamDestroy(cap);
    if (ev) cudaEventDestroy(ev);
    cap = nullptr;
    ev = nullptr;
  }
};

template <class F>
int run_step_graph(rnn_ctx* ctx, StepGraph& g, std::vector<unsigned long long> key, F&& body) {
  key.push_back(ctx->mem_epoch);
  if (g.exec && key == g.key) {
    RNN_CUDA(cudaGraphLaunch(g.exec, ctx->stream));
    __atomic_add_fetch(&g_launches, g.kernels, __ATOMIC_RELAXED);
    return RNN_OK;
  }
  g.release();
  if (key != g.last_key) {  // eager step; capture on the next call if nothing moves
    RNN_TRY(body());
    key.back() = ctx->mem_epoch;
    g.last_key = key;
    return RNN_OK;
  }
  if (!g.cap) RNN_CUDA(cudaStreamCreateWithFlags(&g.cap, cudaStreamNonBlocking));
  if (!g.ev) RNN_CUDA(cudaEventCreateWithFlags(&g.ev, cudaEventDisableTiming));
  cudaStream_t user = ctx->stream;
  RNN_CUDA(cudaEventRecord(g.ev, user));
  RNN_CUDA(cudaStreamWaitEvent(g.cap, g.ev, 0));
  const unsigned long long l0 = __atomic_load_n(&g_launches, __ATOMIC_RELAXED);
  ctx->stream = g.cap;
  cudaError_t e = cudaStreamBeginCapture(g.cap, cudaStreamCaptureModeRelaxed);
  int rc = e == cudaSuccess ? body() : set_error(RNN_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
  cudaGraph_t graph = nullptr;
  cudaError_t e2 = cudaSuccess;
  if (e == cudaSuccess) e2 = cudaStreamEndCapture(g.cap, &graph);
  ctx->stream = user;
  cudaGetLastError();
  if (rc == RNN_OK && e2 == cudaSuccess && graph && ctx->mem_epoch == key.back()) {
    cudaGraphExec_t exec = nullptr;
    if (cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess) {
      g.exec = exec;
      g.key = key;
      g.kernels = __atomic_load_n(&g_launches, __ATOMIC_RELAXED) - l0;
    }
  }
  if (graph) cudaGraphDestroy(graph);
  __atomic_sub_fetch(&g_launches, __atomic_load_n(&g_launches, __ATOMIC_RELAXED) - l0, __ATOMIC_RELAXED);
  if (g.exec) {
    RNN_CUDA(cudaGraphLaunch(g.exec, ctx->stream));
    __atomic_add_fetch(&g_launches, g.kernels, __ATOMIC_RELAXED);
    return RNN_OK;
  }
  // capture was not possible (nothing of it ran): do the step eagerly
  cudaGetLastError();
  g.last_key.clear();
  return body();
}
}  // namespace rnn
