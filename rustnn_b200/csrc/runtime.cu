// Tier-2 runtime entry points of the C ABI: device memory and copies on a
// context's stream, and a standalone communicator for the data-parallel
// gradient sum with failure detection.
//
// The reference is one process with host memory only (pool.rs is its
// allocator, there is no collective), so none of these has a counterpart in
// it; they are what a Rust host needs to keep the step's tensors resident on
// the device and to run the batch-sharded step of train.rs:684-699 on several
// GPUs without linking CUDA or NCCL itself.
//
// Failure detection.  An NCCL collective whose peer never arrives spins on
// the GPU; nothing in the stream returns.  rnn_comm_wait is the host-side
// watchdog: it polls the stream's completion and the communicator's
// asynchronous error (ncclCommGetAsyncError) every millisecond, and when the
// communicator reports an error or the wait outlives its limit it aborts the
// communicator (ncclCommAbort, which makes NCCL's kernels return) and reports
// RNN_ERR_NCCL.  The communicator is unusable afterwards; the caller destroys
// it and builds a new one with the ranks that remain.
#include <nccl.h>
#include <string.h>
#include <time.h>

#include <chrono>
#include <thread>

#include "comm.cuh"
#include "common.cuh"

using namespace rnn;

extern "C" int rnn_alloc(rnn_ctx* ctx, size_t bytes, void** out) {
  RNN_REQUIRE(ctx && out, "alloc: null argument");
  *out = nullptr;
  if (bytes == 0) return RNN_OK;
  RNN_CUDA(cudaSetDevice(ctx->device));
  RNN_CUDA(cudaMalloc(out, bytes));
  return RNN_OK;
}

extern "C" int rnn_free(rnn_ctx* ctx, void* p) {
  RNN_REQUIRE(ctx, "free: null context");
  if (!p) return RNN_OK;
  RNN_CUDA(cudaSetDevice(ctx->device));
  // work already queued on the context's stream may still read p
  RNN_CUDA(cudaStreamSynchronize(ctx->stream));
  RNN_CUDA(cudaFree(p));
  return RNN_OK;
}

extern "C" int rnn_memcpy_h2d(rnn_ctx* ctx, void* dst, const void* src, size_t bytes) {
  RNN_REQUIRE(ctx && (bytes == 0 || (dst && src)), "memcpy_h2d: null argument");
  if (bytes == 0) return RNN_OK;
  RNN_RANGE(dst, bytes);
  RNN_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  return RNN_OK;
}

extern "C" int rnn_memcpy_d2h(rnn_ctx* ctx, void* dst, const void* src, size_t bytes) {
  RNN_REQUIRE(ctx && (bytes == 0 || (dst && src)), "memcpy_d2h: null argument");
  if (bytes == 0) return RNN_OK;
  RNN_RANGE(src, bytes);
  RNN_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  return RNN_OK;
}

// ------------------------------------------------------------------ comm

extern "C" int rnn_comm_init(rnn_comm** out, int device, int rank, int world, const unsigned char* uid) {
  RNN_REQUIRE(out && uid, "comm_init: null argument");
  RNN_REQUIRE(world >= 1 && rank >= 0 && rank < world, "comm_init: rank %d of world %d", rank, world);
  *out = nullptr;
  RNN_CUDA(cudaSetDevice(device));
  ncclUniqueId id;
  memcpy(&id, uid, sizeof(id));
  rnn_comm* c = new rnn_comm();
  c->device = device;
  c->rank = rank;
  c->world = world;
  ncclResult_t r = ncclCommInitRank(&c->comm, world, id, rank);
  if (r != ncclSuccess) {
    delete c;
    return set_error(RNN_ERR_NCCL, "ncclCommInitRank: %s", ncclGetErrorString(r));
  }
  *out = c;
  return RNN_OK;
}

extern "C" int rnn_comm_destroy(rnn_comm* c) {
  if (!c) return RNN_OK;
  RNN_REQUIRE(c->owned, "comm_destroy: this communicator belongs to a network; destroy the network");
  cudaSetDevice(c->device);
  if (c->comm && !c->aborted) ncclCommDestroy(c->comm);  // an abort already released it
  delete c;
  return RNN_OK;
}

// sum (average != 0: mean) of a flat f32 gradient buffer over every rank, in
// place, enqueued on the context's stream
extern "C" int rnn_allreduce_grads(rnn_ctx* ctx, rnn_comm* c, float* grads, size_t n, int average) {
  RNN_REQUIRE(ctx && c && (n == 0 || grads), "allreduce_grads: null argument");
  RNN_REQUIRE(!c->aborted, "allreduce_grads: the communicator was aborted");
  RNN_REQUIRE(c->device == ctx->device, "allreduce_grads: context on device %d, communicator on %d", ctx->device,
              c->device);
  if (n == 0) return RNN_OK;
  RNN_RANGE(grads, n * sizeof(float));
  ncclResult_t r = ncclAllReduce(grads, grads, n, ncclFloat, average ? ncclAvg : ncclSum, c->comm, ctx->stream);
  if (r != ncclSuccess) return set_error(RNN_ERR_NCCL, "gradient allreduce: %s", ncclGetErrorString(r));
  return RNN_OK;
}

extern "C" int rnn_comm_check(rnn_comm* c) {
  RNN_REQUIRE(c, "comm_check: null communicator");
  if (c->aborted) return set_error(RNN_ERR_NCCL, "communicator aborted");
  ncclResult_t async = ncclSuccess;
  ncclResult_t r = ncclCommGetAsyncError(c->comm, &async);
  if (r != ncclSuccess) return set_error(RNN_ERR_NCCL, "ncclCommGetAsyncError: %s", ncclGetErrorString(r));
  if (async != ncclSuccess && async != ncclInProgress)
    return set_error(RNN_ERR_NCCL, "communicator error: %s", ncclGetErrorString(async));
  return RNN_OK;
}

extern "C" int rnn_comm_abort(rnn_comm* c) {
  RNN_REQUIRE(c, "comm_abort: null communicator");
  if (c->aborted) return RNN_OK;
  cudaSetDevice(c->device);
  ncclResult_t r = ncclCommAbort(c->comm);
  c->aborted = true;
  if (r != ncclSuccess) return set_error(RNN_ERR_NCCL, "ncclCommAbort: %s", ncclGetErrorString(r));
  return RNN_OK;
}

extern "C" int rnn_comm_wait(rnn_ctx* ctx, rnn_comm* c, int timeout_ms) {
  RNN_REQUIRE(ctx && c, "comm_wait: null argument");
  RNN_REQUIRE(timeout_ms > 0, "comm_wait: timeout %d ms", timeout_ms);
  RNN_CUDA(cudaSetDevice(ctx->device));
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    const cudaError_t q = cudaStreamQuery(ctx->stream);
    if (q == cudaSuccess) return rnn_comm_check(c);
    if (q != cudaErrorNotReady) return set_error(RNN_ERR_CUDA, "comm_wait: %s", cudaGetErrorString(q));
    if (rnn_comm_check(c) != RNN_OK) {
      const std::string why = rnn_last_error();
      rnn_comm_abort(c);
      return set_error(RNN_ERR_NCCL, "comm_wait: %s; communicator aborted", why.c_str());
    }
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
    if (ms.count() > timeout_ms) {
      rnn_comm_abort(c);
      // the aborted collective returns; let the stream drain (bounded)
      const auto t1 = std::chrono::steady_clock::now();
      while (cudaStreamQuery(ctx->stream) == cudaErrorNotReady &&
             std::chrono::steady_clock::now() - t1 < std::chrono::seconds(10))
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
      cudaGetLastError();
      return set_error(RNN_ERR_NCCL,
                       "comm_wait: no completion within %d ms (a peer did not join the collective); "
                       "communicator aborted",
                       timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
}
