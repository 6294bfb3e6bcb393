// Evaluation: the eval batch builder (data.rs:494-512) and the batching loop
// of eval.rs:15-39 on the device.  The loop keeps the loss sum and the hit
// count on the device and reads them back once at the end of the pass.
#include <math.h>

#include "eval.cuh"
#include "ew.cuh"

namespace rnn {

namespace {

constexpr int IMG = 32, PLANE = IMG * IMG, PIX = 3 * PLANE;

// norm (data.rs:95-98): (v / 255 - mean[c]) / std[c] in f32, each operation
// rounded to nearest as in the reference (no contraction).
__device__ __forceinline__ float eval_norm(uint32_t v, int c) {
  // data.rs:13-14
  const float mean = c == 0 ? 0.5071f : (c == 1 ? 0.4865f : 0.4409f);
  const float sd = c == 0 ? 0.2673f : (c == 1 ? 0.2564f : 0.2762f);
  return __fdiv_rn(__fsub_rn(__fdiv_rn((float)v, 255.0f), mean), sd);
}

// One thread per 4 consecutive output pixels of a row: with no shift every
// source pixel lies inside the image, so crop_flip_normalize (data.rs:331-360)
// reduces to norm() of column x, or of column 31 - x when mirrored.
template <bool VEC>
__global__ void make_batch_eval_kernel(const uint8_t* __restrict__ images, const uint8_t* __restrict__ labels,
                                       size_t start, int bs, int flip, float* __restrict__ out,
                                       uint32_t* __restrict__ labels_out) {
  const size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (g < (size_t)bs) labels_out[g] = labels[start + g];
  if (g >= (size_t)bs * (PIX / 4)) return;
  const int b = (int)(g / (PIX / 4));
  const int r = (int)(g % (PIX / 4));
  const int c = r / (PLANE / 4);
  const int y = (r / (IMG / 4)) % IMG;
  const int x0 = (r % (IMG / 4)) * 4;
  const uint8_t* src = images + (start + b) * (size_t)PIX + c * PLANE + y * IMG;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; i++) v[i] = eval_norm(src[flip ? IMG - 1 - (x0 + i) : x0 + i], c);
  float* dst = out + (size_t)b * PIX + c * PLANE + y * IMG + x0;
  if constexpr (VEC) {
    *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
#pragma unroll
    for (int i = 0; i < 4; i++) dst[i] = v[i];
  }
}

// eval.rs:33-34: sum += l * bs (a rounded product, then the add); correct += c
__global__ void eval_accum_kernel(const float* __restrict__ batch_loss, const int* __restrict__ batch_hit, int bs,
                                  float* __restrict__ sum, unsigned long long* __restrict__ correct) {
  *sum = __fadd_rn(*sum, __fmul_rn(*batch_loss, (float)bs));
  *correct += (unsigned long long)*batch_hit;
}

// eval.rs:58-60: a = 0.5 * (a + b)
__global__ void tta_mean_kernel(float* __restrict__ a, const float* __restrict__ b, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    a[i] = __fmul_rn(0.5f, __fadd_rn(a[i], b[i]));
}

size_t round256(size_t b) { return (b + 255) & ~(size_t)255; }

}  // namespace

int eval_ws_ensure(EvalWs& ws, int n, int nclass) {
  if (n <= ws.cap_n && nclass <= ws.cap_nc) return RNN_OK;
  n = n > ws.cap_n ? n : ws.cap_n;
  nclass = nclass > ws.cap_nc ? nclass : ws.cap_nc;
  const size_t lg = round256(sizeof(float) * (size_t)n * nclass);
  const size_t sizes[] = {round256(sizeof(float) * (size_t)n * PIX), round256(sizeof(uint32_t) * n), lg, lg,
                          round256(sizeof(float) * n), round256(sizeof(int) * n), 256, 256, 256, 256};
  size_t total = 0;
  for (size_t s : sizes) total += s;
  if (ws.block) RNN_CUDA(cudaFree(ws.block));
  ws.block = nullptr;
  ws.cap_n = ws.cap_nc = 0;
  RNN_CUDA(cudaMalloc(&ws.block, total));
  char* p = static_cast<char*>(ws.block);
  void** slots[] = {(void**)&ws.x,   (void**)&ws.lab,        (void**)&ws.lg,        (void**)&ws.dl,
                    (void**)&ws.row_loss, (void**)&ws.hit,   (void**)&ws.batch_loss, (void**)&ws.batch_hit,
                    (void**)&ws.sum, (void**)&ws.correct};
  for (int i = 0; i < 10; i++) {
    *slots[i] = p;
    p += sizes[i];
  }
  ws.cap_n = n;
  ws.cap_nc = nclass;
  return RNN_OK;
}

int eval_ws_stage(EvalWs& ws, rnn_ctx* ctx, const uint8_t* h_images, const uint8_t* h_labels, int len,
                  const uint8_t** images, const uint8_t** labels) {
  const size_t need = (size_t)len * PIX + (size_t)len;
  if (need > ws.data_cap) {
    RNN_CUDA(cudaStreamSynchronize(ctx->stream));
    if (ws.data) RNN_CUDA(cudaFree(ws.data));
    ws.data = nullptr;
    ws.data_cap = 0;
    RNN_CUDA(cudaMalloc(&ws.data, need));
    ws.data_cap = need;
  }
  RNN_CUDA(cudaMemcpyAsync(ws.data, h_images, (size_t)len * PIX, cudaMemcpyHostToDevice, ctx->stream));
  RNN_CUDA(cudaMemcpyAsync(ws.data + (size_t)len * PIX, h_labels, (size_t)len, cudaMemcpyHostToDevice,
                           ctx->stream));
  *images = ws.data;
  *labels = ws.data + (size_t)len * PIX;
  return RNN_OK;
}

void eval_ws_free(EvalWs& ws) {
  if (ws.block) cudaFree(ws.block);
  if (ws.data) cudaFree(ws.data);
  ws = EvalWs{};
}

int make_batch_eval(rnn_ctx* ctx, const uint8_t* images, const uint8_t* labels, size_t start, int bs, bool flip,
                    float* out, uint32_t* labels_out) {
  if (bs == 0) return RNN_OK;
  RNN_RANGE(images + start * PIX, (size_t)bs * PIX);
  RNN_RANGE(labels + start, (size_t)bs);
  RNN_RANGE(out, sizeof(float) * (size_t)bs * PIX);
  RNN_RANGE(labels_out, sizeof(uint32_t) * (size_t)bs);
  const size_t threads = (size_t)bs * (PIX / 4);
  const unsigned grid = (unsigned)((threads + 255) / 256);
  if (((uintptr_t)out & 15) == 0)
    make_batch_eval_kernel<true><<<grid, 256, 0, ctx->stream>>>(images, labels, start, bs, flip, out, labels_out);
  else
    make_batch_eval_kernel<false><<<grid, 256, 0, ctx->stream>>>(images, labels, start, bs, flip, out, labels_out);
  RNN_CHECK_LAUNCH();
  return RNN_OK;
}

int eval_loop(rnn_ctx* ctx, EvalWs& ws, const uint8_t* images, const uint8_t* labels, int len, int batch,
              int nclass, bool tta, const EvalLogits& logits, float* out2) {
  RNN_REQUIRE(len >= 0 && batch > 0 && nclass > 0, "eval: bad sizes (len %d, batch %d)", len, batch);
  if (len == 0) {  // eval.rs:38 divides by seen = 0
    out2[0] = out2[1] = NAN;
    return RNN_OK;
  }
  const int nb = batch < len ? batch : len;
  RNN_TRY(eval_ws_ensure(ws, nb, nclass));
  RNN_CUDA(cudaMemsetAsync(ws.sum, 0, sizeof(float), ctx->stream));
  RNN_CUDA(cudaMemsetAsync(ws.correct, 0, sizeof(unsigned long long), ctx->stream));
  for (int s = 0; s < len;) {
    const int bs = batch < len - s ? batch : len - s;
    RNN_TRY(make_batch_eval(ctx, images, labels, (size_t)s, bs, false, ws.x, ws.lab));
    const float* lg = nullptr;
    RNN_TRY(logits(ws.x, bs, &lg));
    if (tta) {
      // eval.rs:52-61: keep these logits, run the mirrored batch, average
      const size_t nl = (size_t)bs * nclass;
      RNN_CUDA(cudaMemcpyAsync(ws.lg, lg, sizeof(float) * nl, cudaMemcpyDeviceToDevice, ctx->stream));
      RNN_TRY(make_batch_eval(ctx, images, labels, (size_t)s, bs, true, ws.x, ws.lab));
      const float* mirrored = nullptr;
      RNN_TRY(logits(ws.x, bs, &mirrored));
      RNN_RANGE(mirrored, sizeof(float) * nl);
      tta_mean_kernel<<<(unsigned)((nl + 255) / 256), 256, 0, ctx->stream>>>(ws.lg, mirrored, nl);
      RNN_CHECK_LAUNCH();
      lg = ws.lg;
    }
    RNN_TRY(softmax_ce(ctx, lg, ws.lab, bs, nclass, 0.0f, ws.dl, ws.row_loss, ws.hit, ws.batch_loss,
                       ws.batch_hit));
    eval_accum_kernel<<<1, 1, 0, ctx->stream>>>(ws.batch_loss, ws.batch_hit, bs, ws.sum, ws.correct);
    RNN_CHECK_LAUNCH();
    s += bs;
  }
  float sum = 0.0f;
  unsigned long long correct = 0;
  RNN_CUDA(cudaMemcpyAsync(&sum, ws.sum, sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
  RNN_CUDA(cudaMemcpyAsync(&correct, ws.correct, sizeof(correct), cudaMemcpyDeviceToHost, ctx->stream));
  RNN_TRY(rnn_ctx_synchronize(ctx));
  // eval.rs:38
  out2[0] = sum / (float)len;
  out2[1] = (float)correct / (float)len;
  return RNN_OK;
}

}  // namespace rnn

extern "C" int rnn_make_batch_eval_dev(rnn_ctx* ctx, const uint8_t* images, const uint8_t* labels, size_t len,
                                       size_t start, int bs, int flip, float* out, uint32_t* labels_out) {
  RNN_REQUIRE(ctx && images && labels && out && labels_out, "make_batch_eval: null argument");
  RNN_REQUIRE(bs >= 0, "make_batch_eval: negative batch");
  RNN_REQUIRE(start <= len && (size_t)bs <= len - start,
              "make_batch_eval: images [%zu, %zu) are outside a dataset of %zu", start, start + (size_t)bs, len);
  return rnn::make_batch_eval(ctx, images, labels, start, bs, flip != 0, out, labels_out);
}
