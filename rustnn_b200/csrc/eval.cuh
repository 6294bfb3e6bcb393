// Evaluation over a u8 dataset: the batch builder of data.rs:494-512 on the
// device and the batching loop of eval.rs:15-39, shared by the ResNet and
// rustvit entry points (resnet.cu, vit.cu).
#pragma once

#include <functional>

#include "common.cuh"

namespace rnn {

// Device buffers of one evaluation pass, grown on demand and owned by the
// model that evaluates.
struct EvalWs {
  uint8_t* data = nullptr;  // a host dataset staged on the device (images, then labels)
  size_t data_cap = 0;
  void* block = nullptr;  // per-batch buffers, carved below
  int cap_n = 0, cap_nc = 0;
  float* x = nullptr;          // [n, 3, 32, 32]
  uint32_t* lab = nullptr;     // [n]
  float* lg = nullptr;         // [n, nclass] averaged test-time-augmentation logits
  float* dl = nullptr;         // [n, nclass] softmax_ce gradient (unused, as in eval.rs:22)
  float* row_loss = nullptr;   // [n]
  int* hit = nullptr;          // [n]
  float* batch_loss = nullptr;  // 1
  int* batch_hit = nullptr;     // 1
  float* sum = nullptr;         // running sum of l * bs (f32, eval.rs:33)
  unsigned long long* correct = nullptr;
};

int eval_ws_ensure(EvalWs& ws, int n, int nclass);
// Copies a host dataset (len images of 3 x 32 x 32 bytes, len labels) into
// ws.data; *images / *labels point at the device copies.
int eval_ws_stage(EvalWs& ws, rnn_ctx* ctx, const uint8_t* h_images, const uint8_t* h_labels, int len,
                  const uint8_t** images, const uint8_t** labels);
void eval_ws_free(EvalWs& ws);

// data::make_batch_eval (data.rs:494-512) on the device.
int make_batch_eval(rnn_ctx* ctx, const uint8_t* images, const uint8_t* labels, size_t start, int bs, bool flip,
                    float* out, uint32_t* labels_out);

// Runs the model on the batch x [bs, 3, 32, 32] (device) and points *logits
// at its [bs, nclass] logits (device, valid until the next call).
using EvalLogits = std::function<int(const float* x, int bs, const float** logits)>;

// eval.rs:15-39 (with the test-time augmentation of eval.rs:50-61 when tta):
// images / labels are the device dataset; out2 (host) = {mean loss, accuracy}.
int eval_loop(rnn_ctx* ctx, EvalWs& ws, const uint8_t* images, const uint8_t* labels, int len, int batch,
              int nclass, bool tta, const EvalLogits& logits, float* out2);

}  // namespace rnn
