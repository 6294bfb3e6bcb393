// Device-resident CIFAR ResNet training step (model.rs, nn.rs, train.rs).
//
// Parameters, gradients and momenta live in three flat device buffers in the
// reference's for_each_param order (model.rs:159-168), so the SGD update is
// one launch and the data-parallel gradient allreduce is one NCCL call.
// Activations are preallocated for the batch capacity and reused each step:
// per block x_in (the previous block's output), y1 = conv1(x), h1 =
// relu(bn1(y1)), y2 = conv2(h1), yd = convd(x) (down-sampling blocks) and
// out = relu(bn2(y2) + shortcut), which is exactly what model.rs:39-55 keeps
// alive for its backward.  BatchNorm keeps its input y and recomputes xhat.
#include <nccl.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "bn.cuh"
#include "ckpt.cuh"
#include "comm.cuh"
#include "eval.cuh"
#include "ew.cuh"
#include "rng.h"

namespace rnn {

struct ConvL {
  int cin, cout, k, stride, pad;
  size_t w_off;  // offset into the flat parameter buffer
};

struct BNL {
  int c;
  size_t g_off, b_off;  // gamma, beta offsets in the flat buffer
  size_t rm_off;        // running mean offset in the buffer array; rv follows
  float* mean = nullptr;
  float* invstd = nullptr;
  // the statistics of the next forward pass were summed by the producing
  // convolution's epilogue (over all ranks when pre_reduced)
  bool pre = false, pre_reduced = false;
};

struct Block {
  ConvL c1, c2, cd;
  BNL b1, b2, bd;
  bool down = false;
  int cin, cout, stride;
  float *y1 = nullptr, *h1 = nullptr, *y2 = nullptr, *yd = nullptr, *out = nullptr;
  // ReLU outcomes of h1 and of the join as bits (valid when *_ok)
  uint32_t *m1 = nullptr, *mout = nullptr;
  bool m1_ok = false, mout_ok = false;
  const float* x_in = nullptr;
  int n = 0, h = 0, w = 0, oh = 0, ow = 0;
};

}  // namespace rnn

using namespace rnn;

struct rnn_resnet {
  rnn_ctx* ctx = nullptr;
  int depth_n = 0, width = 0, nclass = 0;
  ConvL stem{};
  BNL stem_bn{};
  std::vector<Block> blocks;
  size_t fcw_off = 0, fcb_off = 0;
  int fin = 0, fout = 0;
  // flat parameter state
  size_t nparams = 0;
  float *v = nullptr, *g = nullptr, *m = nullptr;
  uint8_t* decay = nullptr;
  std::vector<uint8_t> decay_host;
  // BN running statistics (for_each_buffer order: [rm, rv] per BN)
  size_t nbuf = 0;
  float* bnbuf = nullptr;
  // tensor counts of for_each_param / for_each_buffer (checkpoint header)
  int n_param_tensors = 0, n_buf_tensors = 0;
  float* bnstat = nullptr;  // mean/invstd arrays of every BN
  // activations
  int cap_n = 0, cap_h = 0, cap_w = 0;
  uint32_t* stem_m = nullptr;  // ReLU outcome of stem_out as bits (valid when stem_m_ok)
  bool stem_m_ok = false;
  float *stem_y = nullptr, *stem_out = nullptr, *pooled = nullptr, *logits = nullptr, *dlogits = nullptr,
        *dpool = nullptr;
  float* gbuf[4] = {nullptr, nullptr, nullptr, nullptr};
  size_t gbuf_elems = 0;
  void* scratch = nullptr;  // BN partials/sums, CE row buffers
  size_t scratch_bytes = 0;
  float* x_stage = nullptr;
  uint32_t* lab_stage = nullptr;
  float* loss_dev = nullptr;
  int* correct_dev = nullptr;
  std::vector<void*> act_allocs;
  // last forward
  int n = 0, h = 0, w = 0, fh = 0, fw = 0;
  const float* x_in = nullptr;
  // data parallel
  ncclComm_t comm = nullptr;
  rnn_comm handle;  // the communicator as a C ABI handle (rnn_resnet_comm), borrowed
  // gradient buckets: all-reduced on comm_stream while the backward goes on
  cudaStream_t comm_stream = nullptr;
  cudaEvent_t bucket_ev = nullptr, comm_done = nullptr;
  size_t bucket_floats = 0;  // 0: one all-reduce after the backward
  bool in_step = false;      // buckets only inside train_step, which joins them
  int rank = 0, world = 1;
  bool sync_bn = false;
  // SyncBN over peer memory (bn.cuh PeerSums); world 1 = NCCL path
  rnn::PeerSums peer;
  char* mail = nullptr;                 // this rank's mailbox
  std::vector<char*> peer_mail;         // mapped peer mailboxes (IPC)
  char** mail_dev = nullptr;            // device array of every rank's mailbox
  unsigned long long* peer_seq = nullptr;
  // CUDA-graph replay of the training step (rnn_resnet_set_graph)
  bool use_graph = false;
  rnn::StepGraph graph;
  // evaluation buffers (rnn_resnet_eval)
  rnn::EvalWs eval;
  unsigned long long act_epoch = 0;  // bumped when the activations are reallocated
};

namespace rnn {

static size_t bn_scratch_need(rnn_resnet* net, int n) {
  size_t a = 0;
  for (int c : {net->width, net->width * 2, net->width * 4})
    a = std::max(a, bn_scratch_bytes(n, c, net->ctx->num_sms));
  size_t ce = (((size_t)n * 4 + 255) & ~(size_t)255) * 2;
  return a + ce + 4096;
}

static void free_acts(rnn_resnet* net) {
  for (void* p : net->act_allocs) cudaFree(p);
  net->act_allocs.clear();
  for (auto& b : net->blocks) {
    b.y1 = b.h1 = b.y2 = b.yd = b.out = nullptr;
    b.m1 = b.mout = nullptr;
    b.m1_ok = b.mout_ok = false;
  }
  net->stem_m = nullptr;
  net->stem_m_ok = false;
  net->stem_y = net->stem_out = net->pooled = net->logits = net->dlogits = net->dpool = nullptr;
  for (auto& p : net->gbuf) p = nullptr;
  net->scratch = nullptr;
  net->x_stage = nullptr;
  net->lab_stage = nullptr;
  net->cap_n = net->cap_h = net->cap_w = 0;
}

static int alloc_f(rnn_resnet* net, float** p, size_t n) {
  void* q = nullptr;
  RNN_CUDA(cudaMalloc(&q, std::max<size_t>(n, 1) * sizeof(float)));
  net->act_allocs.push_back(q);
  *p = static_cast<float*>(q);
  return RNN_OK;
}

// (Re)allocates every activation for batch n at h x w input.
// one bit per element, whole 32-bit words
static int alloc_mask(rnn_resnet* net, uint32_t** p, size_t elems) {
  float* f = nullptr;
  RNN_TRY(alloc_f(net, &f, (elems + 31) / 32));
  *p = reinterpret_cast<uint32_t*>(f);
  return RNN_OK;
}

static int ensure_acts(rnn_resnet* net, int n, int h, int w) {
  if (n <= net->cap_n && h == net->cap_h && w == net->cap_w) return RNN_OK;
  RNN_CUDA(cudaStreamSynchronize(net->ctx->stream));
  free_acts(net);
  net->act_epoch++;
  const int W = net->width;
  size_t stem = (size_t)n * W * h * w;
  RNN_TRY(alloc_f(net, &net->stem_y, stem));
  RNN_TRY(alloc_f(net, &net->stem_out, stem));
  RNN_TRY(alloc_mask(net, &net->stem_m, stem));
  size_t gmax = stem;
  int ch = h, cw = w;
  for (auto& b : net->blocks) {
    const int oh = (ch + 2 - 3) / b.stride + 1, ow = (cw + 2 - 3) / b.stride + 1;
    const size_t no = (size_t)n * b.cout * oh * ow;
    RNN_TRY(alloc_f(net, &b.y1, no));
    RNN_TRY(alloc_f(net, &b.h1, no));
    RNN_TRY(alloc_f(net, &b.y2, no));
    RNN_TRY(alloc_f(net, &b.out, no));
    RNN_TRY(alloc_mask(net, &b.m1, no));
    RNN_TRY(alloc_mask(net, &b.mout, no));
    if (b.down) RNN_TRY(alloc_f(net, &b.yd, no));
    gmax = std::max(gmax, no);
    gmax = std::max(gmax, (size_t)n * b.cin * ch * cw);
    ch = oh;
    cw = ow;
  }
  for (auto& p : net->gbuf) RNN_TRY(alloc_f(net, &p, gmax));
  net->gbuf_elems = gmax;
  RNN_TRY(alloc_f(net, &net->pooled, (size_t)n * net->fin));
  RNN_TRY(alloc_f(net, &net->dpool, (size_t)n * net->fin));
  RNN_TRY(alloc_f(net, &net->logits, (size_t)n * net->fout));
  RNN_TRY(alloc_f(net, &net->dlogits, (size_t)n * net->fout));
  RNN_TRY(alloc_f(net, &net->x_stage, (size_t)n * 3 * h * w));
  float* lab = nullptr;
  RNN_TRY(alloc_f(net, &lab, (size_t)n));
  net->lab_stage = reinterpret_cast<uint32_t*>(lab);
  net->scratch_bytes = bn_scratch_need(net, n);
  float* scr = nullptr;
  RNN_TRY(alloc_f(net, &scr, net->scratch_bytes / sizeof(float) + 1));
  net->scratch = scr;
  net->cap_n = n;
  net->cap_h = h;
  net->cap_w = w;
  return RNN_OK;
}

// BN scratch layout inside net->scratch
struct BnScratch {
  double* part;
  double* sums;
  float* dgb;
  float* row_loss;
  int* hit;
};

static BnScratch bn_scratch(rnn_resnet* net, int n, int C) {
  BnScratch s;
  char* base = static_cast<char*>(net->scratch);
  const int P = bn_parts(n, C, net->ctx->num_sms);
  size_t a = ((size_t)C * P * 2 * sizeof(double) + 255) & ~(size_t)255;
  size_t b = ((size_t)C * 2 * sizeof(double) + 255) & ~(size_t)255;
  s.part = reinterpret_cast<double*>(base);
  s.sums = reinterpret_cast<double*>(base + a);
  s.dgb = reinterpret_cast<float*>(base + a + b);
  // CE buffers live at the end of the scratch block
  size_t ce = ((size_t)n * 4 + 255) & ~(size_t)255;
  char* tail = base + net->scratch_bytes - 2 * ce - 1024;
  s.row_loss = reinterpret_cast<float*>(tail);
  s.hit = reinterpret_cast<int*>(tail + ce);
  return s;
}

static int allreduce_sums(rnn_resnet* net, double* sums, int C) {
  if (!net->comm || !net->sync_bn) return RNN_OK;
  ncclResult_t r = ncclAllReduce(sums, sums, (size_t)C * 2, ncclDouble, ncclSum, net->comm, net->ctx->stream);
  if (r != ncclSuccess) return set_error(RNN_ERR_NCCL, "SyncBN allreduce: %s", ncclGetErrorString(r));
  return RNN_OK;
}

// out = [relu](bn(y) [+ res]): with res the block's residual join
// (model.rs:52-54, add_relu_) is fused into the normalisation pass.
static int bn_forward(rnn_resnet* net, BNL& bn, const float* y, int n, int hw, bool train, bool relu,
                      float* out, const float* res = nullptr, uint32_t* mask = nullptr, bool* masked = nullptr) {
  if (masked) *masked = false;
  rnn_ctx* ctx = net->ctx;
  float* gamma = net->v + bn.g_off;
  float* beta = net->v + bn.b_off;
  float* rm = net->bnbuf + bn.rm_off;
  float* rv = rm + bn.c;
  if (!train) {
    if (!res) return rnn_batchnorm_eval_dev(ctx, y, n, bn.c, hw, gamma, beta, rm, rv, 1e-5f, relu, out);
    const size_t len = (size_t)n * bn.c * hw;
    if (res == out) {  // out already holds the other branch: out = relu(out + bn(y))
      float* tmp = net->gbuf[0];
      RNN_TRY(rnn_batchnorm_eval_dev(ctx, y, n, bn.c, hw, gamma, beta, rm, rv, 1e-5f, 0, tmp));
      return add(ctx, out, tmp, len, relu);
    }
    RNN_TRY(rnn_batchnorm_eval_dev(ctx, y, n, bn.c, hw, gamma, beta, rm, rv, 1e-5f, 0, out));
    return add(ctx, out, res, len, relu);
  }
  BnScratch s = bn_scratch(net, n, bn.c);
  bool reduced = false;
  if (bn.pre) {
    reduced = bn.pre_reduced;
    bn.pre = false;
  } else {
    RNN_TRY(bn_fwd_sums(ctx, y, n, bn.c, hw, s.part, s.sums, net->sync_bn ? &net->peer : nullptr, &reduced));
  }
  if (!reduced) RNN_TRY(allreduce_sums(net, s.sums, bn.c));
  const double count = (double)n * hw * (net->sync_bn ? net->world : 1);
  return bn_fwd_finish(ctx, y, n, bn.c, hw, count, s.sums, gamma, beta, rm, rv, 0.1f, 1e-5f, relu ? 1 : 0,
                       bn.mean, bn.invstd, out, res, mask, masked);
}

// With `consumer` (the 3x3 convolution whose wgrad reads dx next, whose
// output rows are `ow` wide), dx is also written as that wgrad's packed B
// image in ctx->pack when the shapes allow; *dx_packed returns it or null.
static int bn_backward(rnn_resnet* net, BNL& bn, const float* dy, const float* y, const float* relu_out, int n,
                       int hw, float* dx, const ConvL* consumer = nullptr, int ow = 0,
                       const float** dx_packed = nullptr, const uint32_t* relu_mask = nullptr) {
  rnn_ctx* ctx = net->ctx;
  float* pack = nullptr;
  int pbn = 0;
  if (consumer && dx_packed) {
    *dx_packed = nullptr;
    pbn = tc::wgrad_dy_pack_bn(n, consumer->cout, consumer->k, hw / ow, ow, dx);
    if (pbn) {
      RNN_TRY(ensure_pack(ctx, (size_t)n * bn.c * hw * 2 * sizeof(float)));
      pack = static_cast<float*>(ctx->pack);
    }
  }
  BnScratch s = bn_scratch(net, n, bn.c);
  bool reduced = false;
  RNN_TRY(bn_bwd_sums(ctx, dy, y, relu_out, n, bn.c, hw, bn.mean, bn.invstd, s.part, s.sums,
                      net->sync_bn ? &net->peer : nullptr, &reduced, relu_mask));
  if (!reduced) RNN_TRY(allreduce_sums(net, s.sums, bn.c));
  const bool sb = net->sync_bn && net->comm;
  const double count = (double)n * hw * (sb ? net->world : 1);
  const float pscale = sb ? 1.0f / (float)net->world : 1.0f;
  bool packed = false;
  RNN_TRY(bn_bwd_finish(ctx, dy, y, relu_out, n, bn.c, hw, count, s.sums, net->v + bn.g_off, bn.mean, bn.invstd,
                        s.dgb, dx, net->g + bn.g_off, net->g + bn.b_off, pscale, pack, pbn, &packed, relu_mask));
  if (dx_packed) *dx_packed = packed ? pack : nullptr;
  return RNN_OK;
}

// With `bn` (training), the convolution's epilogue also sums the BN
// statistics of y where its kernel can (bn->pre says it did).
static int conv_forward(rnn_resnet* net, const ConvL& c, const float* x, int n, int h, int w, float* y,
                        BNL* bn = nullptr) {
  if (!bn) return tc::conv_fwd(net->ctx, x, n, c.cin, h, w, net->v + c.w_off, c.cout, c.k, c.stride, c.pad, y, false);
  tc::ConvStats st;
  st.sums = bn_scratch(net, n, bn->c).sums;
  st.ps = net->sync_bn ? &net->peer : nullptr;
  RNN_TRY(tc::conv_fwd(net->ctx, x, n, c.cin, h, w, net->v + c.w_off, c.cout, c.k, c.stride, c.pad, y, false, &st));
  bn->pre = st.fused;
  bn->pre_reduced = st.reduced;
  return RNN_OK;
}

// nn.rs:230-250: backward_w then dX
static int conv_backward(rnn_resnet* net, const ConvL& c, const float* x, const float* dy, int n, int h, int w,
                         float* dx, bool dx_acc, const float* dy_packed = nullptr) {
  RNN_TRY(tc::conv_wgrad(net->ctx, x, dy, n, c.cin, h, w, c.cout, c.k, c.stride, c.pad, net->g + c.w_off, 0,
                         dy_packed));
  if (dx)
    RNN_TRY(tc::conv_dgrad(net->ctx, dy, n, c.cin, h, w, net->v + c.w_off, c.cout, c.k, c.stride, c.pad, dx,
                           dx_acc));
  return RNN_OK;
}

static int resnet_forward(rnn_resnet* net, const float* x, int n, int h, int w, bool train, float* logits) {
  RNN_TRY(ensure_acts(net, n, h, w));
  // stem conv + BN + ReLU (model.rs:136)
  RNN_TRY(conv_forward(net, net->stem, x, n, h, w, net->stem_y, train ? &net->stem_bn : nullptr));
  RNN_TRY(bn_forward(net, net->stem_bn, net->stem_y, n, h * w, train, true, net->stem_out, nullptr, net->stem_m,
                     &net->stem_m_ok));
  const float* cur = net->stem_out;
  int ch = h, cw = w;
  for (auto& b : net->blocks) {
    // model.rs:39-55
    const int oh = (ch + 2 - 3) / b.stride + 1, ow = (cw + 2 - 3) / b.stride + 1;
    const int ohw = oh * ow;
    b.x_in = cur;
    b.n = n; b.h = ch; b.w = cw; b.oh = oh; b.ow = ow;
    RNN_TRY(conv_forward(net, b.c1, cur, n, ch, cw, b.y1, train ? &b.b1 : nullptr));
    RNN_TRY(bn_forward(net, b.b1, b.y1, n, ohw, train, true, b.h1, nullptr, b.m1, &b.m1_ok));
    RNN_TRY(conv_forward(net, b.c2, b.h1, n, oh, ow, b.y2, train ? &b.b2 : nullptr));
    if (b.down) {
      // out = relu(bn2(y2) + bnd(yd)): bn2 first, then bnd joins it in place
      RNN_TRY(bn_forward(net, b.b2, b.y2, n, ohw, train, false, b.out));
      RNN_TRY(conv_forward(net, b.cd, cur, n, ch, cw, b.yd, train ? &b.bd : nullptr));
      RNN_TRY(bn_forward(net, b.bd, b.yd, n, ohw, train, true, b.out, b.out, b.mout, &b.mout_ok));
    } else {
      RNN_TRY(bn_forward(net, b.b2, b.y2, n, ohw, train, true, b.out, cur, b.mout, &b.mout_ok));
    }
    cur = b.out;
    ch = oh;
    cw = ow;
  }
  net->n = n; net->h = h; net->w = w; net->fh = ch; net->fw = cw;
  net->x_in = x;
  RNN_TRY(gap_fwd(net->ctx, cur, n * net->fin, ch * cw, net->pooled));
  RNN_TRY(fc_fwd(net->ctx, net->pooled, n, net->fin, net->fout, net->v + net->fcw_off, net->v + net->fcb_off,
                 logits));
  return RNN_OK;
}

// Sum of grads [lo, hi) over the ranks on comm_stream, after everything the
// compute stream has queued so far (the backward that finished them).
static int grad_bucket(rnn_resnet* net, size_t lo, size_t hi) {
  RNN_CUDA(cudaEventRecord(net->bucket_ev, net->ctx->stream));
  RNN_CUDA(cudaStreamWaitEvent(net->comm_stream, net->bucket_ev, 0));
  ncclResult_t r = ncclAllReduce(net->g + lo, net->g + lo, hi - lo, ncclFloat, ncclSum, net->comm, net->comm_stream);
  if (r != ncclSuccess) return set_error(RNN_ERR_NCCL, "gradient bucket all-reduce: %s", ncclGetErrorString(r));
  return RNN_OK;
}

static int resnet_backward(rnn_resnet* net, const float* dlogits) {
  rnn_ctx* ctx = net->ctx;
  const int n = net->n;
  // model.rs:148-157
  RNN_TRY(fc_bwd(ctx, net->pooled, dlogits, n, net->fin, net->fout, net->v + net->fcw_off, net->g + net->fcw_off,
                 net->g + net->fcb_off, net->dpool));
  // The parameters are laid out stem, blocks, classifier and the backward
  // finishes them from the end: [lo, pending_hi) is final and not yet summed.
  size_t pending_hi = net->nparams;
  auto flush = [&](size_t lo, bool last) -> int {
    if (!net->in_step || !net->bucket_floats || pending_hi == lo) return RNN_OK;
    if (!last && pending_hi - lo < net->bucket_floats) return RNN_OK;
    RNN_TRY(grad_bucket(net, lo, pending_hi));
    pending_hi = lo;
    return RNN_OK;
  };
  int id = 0, it = 1, idm = 2, idx = 3;
  float** G = net->gbuf;
  RNN_TRY(gap_bwd(ctx, net->dpool, n * net->fin, net->fh * net->fw, G[id]));
  for (int bi = (int)net->blocks.size() - 1; bi >= 0; bi--) {
    Block& b = net->blocks[bi];
    const int ohw = b.oh * b.ow;
    float *d = G[id], *t = G[it], *dmain = G[idm], *dx = G[idx];
    // model.rs:57-72
    // relu_back_ of the join (model.rs:59) is applied on the fly: every
    // consumer of d masks it with out > 0
    // the BN backward passes also write dY as the next wgrad's B image
    const float* tp = nullptr;
    // the ReLU masks come as bits from the forward when it could store them
    const uint32_t* mo = b.mout_ok ? b.mout : nullptr;
    RNN_TRY(bn_backward(net, b.b2, d, b.y2, b.out, n, ohw, t, &b.c2, b.ow, &tp, mo));
    RNN_TRY(conv_backward(net, b.c2, b.h1, t, n, b.oh, b.ow, dmain, false, tp));
    RNN_TRY(bn_backward(net, b.b1, dmain, b.y1, b.h1, n, ohw, t, &b.c1, b.ow, &tp, b.m1_ok ? b.m1 : nullptr));
    RNN_TRY(conv_backward(net, b.c1, b.x_in, t, n, b.h, b.w, dx, false, tp));
    if (b.down) {
      RNN_TRY(bn_backward(net, b.bd, d, b.yd, b.out, n, ohw, t, nullptr, 0, nullptr, mo));
      RNN_TRY(conv_backward(net, b.cd, b.x_in, t, n, b.h, b.w, dx, true));
    } else {
      // identity shortcut: a separate streaming pass; joined in the dgrad
      // epilogue the loads of d and out stall the epilogue warps (measured
      // 2-3x the dgrad's own time)
      RNN_TRY(add_masked(ctx, dx, d, b.out, (size_t)n * b.cin * b.h * b.w, mo));
    }
    std::swap(id, idx);
    RNN_TRY(flush(b.c1.w_off, false));  // the block's parameters start at its first conv
  }
  // stem: relu_back, BN backward, dW only (model.rs:154-156)
  const int hw = net->h * net->w;
  float *d = G[id], *t = G[it];
  const float* tp = nullptr;
  RNN_TRY(bn_backward(net, net->stem_bn, d, net->stem_y, net->stem_out, n, hw, t, &net->stem, net->w, &tp,
                      net->stem_m_ok ? net->stem_m : nullptr));
  RNN_TRY(conv_backward(net, net->stem, net->x_in, t, n, net->h, net->w, nullptr, false, tp));
  return flush(0, true);
}

static int resnet_step(rnn_resnet* net, float lr, float mom, float wd) {
  const float gscale = net->comm ? 1.0f / (float)net->world : 1.0f;
  return sgd_nesterov(net->ctx, net->v, net->g, net->m, net->decay, 0, net->nparams, lr, mom, wd, gscale);
}

// Unmaps the peers' mailboxes and frees this rank's (after the device is idle).
static void peer_release(rnn_resnet* net) {
  for (char* p : net->peer_mail)
    if (p) cudaIpcCloseMemHandle(p);
  net->peer_mail.clear();
  if (net->mail) cudaFree(net->mail);
  if (net->mail_dev) cudaFree(net->mail_dev);
  if (net->peer_seq) cudaFree(net->peer_seq);
  net->mail = nullptr;
  net->mail_dev = nullptr;
  net->peer_seq = nullptr;
  net->peer = PeerSums{};
}

// Maps every rank's SyncBN mailbox into this process (CUDA IPC handles
// exchanged with one NCCL all-gather).  Returns RNN_OK without enabling the
// peer path when the GPUs cannot reach each other; SyncBN then uses NCCL.
static int peer_setup(rnn_resnet* net) {
  const int world = net->world, rank = net->rank;
  const int cmax = 4 * net->width;  // widest BatchNorm of the network
  RNN_CUDA(cudaMalloc(&net->mail, peer_mail_bytes(cmax)));
  RNN_CUDA(cudaMemset(net->mail, 0, peer_mail_bytes(cmax)));
  RNN_CUDA(cudaMalloc(&net->peer_seq, sizeof(unsigned long long)));
  RNN_CUDA(cudaMemset(net->peer_seq, 0, sizeof(unsigned long long)));
  cudaIpcMemHandle_t h;
  RNN_CUDA(cudaIpcGetMemHandle(&h, net->mail));
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  char* dh = nullptr;
  RNN_CUDA(cudaMalloc(&dh, hb * world));
  RNN_CUDA(cudaMemcpy(dh + hb * rank, &h, hb, cudaMemcpyHostToDevice));
  ncclResult_t r = ncclAllGather(dh + hb * rank, dh, hb, ncclChar, net->comm, net->ctx->stream);
  std::vector<cudaIpcMemHandle_t> all(world);
  cudaError_t e = cudaStreamSynchronize(net->ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpy(all.data(), dh, hb * world, cudaMemcpyDeviceToHost);
  cudaFree(dh);
  if (r != ncclSuccess) return set_error(RNN_ERR_NCCL, "mailbox handle exchange: %s", ncclGetErrorString(r));
  RNN_CUDA(e);
  std::vector<char*> ptrs(world, nullptr);
  ptrs[rank] = net->mail;
  bool ok = true;
  for (int q = 0; q < world && ok; q++) {
    if (q == rank) continue;
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, all[q], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = false;
      break;
    }
    ptrs[q] = static_cast<char*>(p);
    net->peer_mail.push_back(ptrs[q]);
  }
  // every rank must agree on the path: any failure anywhere -> NCCL for all
  int flag = ok ? 1 : 0, *dflag = nullptr;
  RNN_CUDA(cudaMalloc(&dflag, sizeof(int)));
  RNN_CUDA(cudaMemcpy(dflag, &flag, sizeof(int), cudaMemcpyHostToDevice));
  r = ncclAllReduce(dflag, dflag, 1, ncclInt, ncclMin, net->comm, net->ctx->stream);
  e = cudaStreamSynchronize(net->ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpy(&flag, dflag, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(dflag);
  if (r != ncclSuccess) return set_error(RNN_ERR_NCCL, "mailbox agreement: %s", ncclGetErrorString(r));
  RNN_CUDA(e);
  if (!flag) {
    peer_release(net);
    return RNN_OK;
  }
  RNN_CUDA(cudaMalloc(&net->mail_dev, world * sizeof(char*)));
  RNN_CUDA(cudaMemcpy(net->mail_dev, ptrs.data(), world * sizeof(char*), cudaMemcpyHostToDevice));
  net->peer.rank = rank;
  net->peer.world = world;
  net->peer.cmax = cmax;
  net->peer.mail = net->mail_dev;
  net->peer.seq = net->peer_seq;
  net->peer.dev_error = net->ctx->dev_error;
  return RNN_OK;
}

static int allreduce_grads(rnn_resnet* net) {
  if (!net->comm || net->world <= 1) return RNN_OK;
  if (net->bucket_floats) {  // the buckets ran during train_step's backward: join them
    RNN_CUDA(cudaEventRecord(net->comm_done, net->comm_stream));
    RNN_CUDA(cudaStreamWaitEvent(net->ctx->stream, net->comm_done, 0));
    return RNN_OK;
  }
  ncclResult_t r = ncclAllReduce(net->g, net->g, net->nparams, ncclFloat, ncclSum, net->comm, net->ctx->stream);
  if (r != ncclSuccess) return set_error(RNN_ERR_NCCL, "gradient allreduce: %s", ncclGetErrorString(r));
  return RNN_OK;
}

static int train_step(rnn_resnet* net, const float* x, const uint32_t* labels, int n, float smooth, float lr,
                      float mom, float wd, float* loss, int* correct) {
  // allocate first: net->logits / dlogits / scratch exist only after this
  RNN_TRY(ensure_acts(net, n, 32, 32));
  RNN_TRY(resnet_forward(net, x, n, 32, 32, true, net->logits));
  BnScratch s = bn_scratch(net, n, 1);
  RNN_TRY(softmax_ce(net->ctx, net->logits, labels, n, net->fout, smooth, net->dlogits, s.row_loss, s.hit, loss,
                     correct));
  net->in_step = net->comm && net->world > 1;
  const int rc = resnet_backward(net, net->dlogits);
  net->in_step = false;
  RNN_TRY(rc);
  RNN_TRY(allreduce_grads(net));
  return resnet_step(net, lr, mom, wd);
}

static unsigned long long fbits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

// train_step, replayed from a CUDA graph when enabled (one launch per step
// instead of ~900; the NCCL calls of the data-parallel step are captured too)
static int train_step_any(rnn_resnet* net, const float* x, const uint32_t* labels, int n, float smooth, float lr,
                          float mom, float wd, float* loss, int* correct) {
  if (!net->use_graph) return train_step(net, x, labels, n, smooth, lr, mom, wd, loss, correct);
  RNN_TRY(ensure_acts(net, n, 32, 32));
  std::vector<unsigned long long> key = {(uintptr_t)x, (uintptr_t)labels, (unsigned long long)n, fbits(smooth),
                                         fbits(lr), fbits(mom), fbits(wd), (uintptr_t)loss, (uintptr_t)correct,
                                         net->act_epoch};
  return run_step_graph(net->ctx, net->graph, key,
                        [&]() { return train_step(net, x, labels, n, smooth, lr, mom, wd, loss, correct); });
}

}  // namespace rnn

// ==================================================================== C ABI

extern "C" int rnn_resnet_create(rnn_ctx* ctx, int depth_n, int width, int nclass, uint64_t seed,
                                 rnn_resnet** out) {
  RNN_REQUIRE(ctx && out, "resnet_create: null argument");
  RNN_REQUIRE(depth_n >= 1 && width >= 1 && nclass >= 1, "resnet_create: bad config");
  *out = nullptr;
  rnn_resnet* net = new rnn_resnet();
  net->ctx = ctx;
  net->depth_n = depth_n;
  net->width = width;
  net->nclass = nclass;

  // ---- layout in for_each_param order (model.rs:159-168, :74-86)
  size_t off = 0, boff = 0;
  std::vector<size_t> sizes;
  std::vector<uint8_t> dec;
  auto take = [&](size_t n, bool decay) {
    size_t o = off;
    off += n;
    sizes.push_back(n);
    dec.push_back(decay ? 1 : 0);
    return o;
  };
  auto mk_conv = [&](ConvL& c, int cin, int cout, int k, int stride, int pad) {
    c.cin = cin; c.cout = cout; c.k = k; c.stride = stride; c.pad = pad;
    c.w_off = take((size_t)cout * cin * k * k, true);  // Param::kaiming: decay
  };
  auto mk_bn = [&](BNL& b, int c) {
    b.c = c;
    net->n_buf_tensors += 2;  // running mean, running variance
    b.g_off = take(c, false);
    b.b_off = take(c, false);
    b.rm_off = boff;
    boff += 2 * (size_t)c;
  };
  mk_conv(net->stem, 3, width, 3, 1, 1);
  mk_bn(net->stem_bn, width);
  const int widths[3] = {width, width * 2, width * 4};
  int cin = width;
  for (int s = 0; s < 3; s++)
    for (int bb = 0; bb < depth_n; bb++) {
      Block b;
      b.stride = (s > 0 && bb == 0) ? 2 : 1;
      b.cin = cin;
      b.cout = widths[s];
      b.down = b.stride != 1 || cin != b.cout;
      mk_conv(b.c1, cin, b.cout, 3, b.stride, 1);
      mk_bn(b.b1, b.cout);
      mk_conv(b.c2, b.cout, b.cout, 3, 1, 1);
      mk_bn(b.b2, b.cout);
      if (b.down) {
        mk_conv(b.cd, cin, b.cout, 1, b.stride, 0);
        mk_bn(b.bd, b.cout);
      }
      net->blocks.push_back(b);
      cin = b.cout;
    }
  net->fin = width * 4;
  net->fout = nclass;
  net->fcw_off = take((size_t)net->fin * nclass, true);
  net->fcb_off = take(nclass, false);
  net->nparams = off;
  net->nbuf = boff;
  net->n_param_tensors = (int)sizes.size();

  // ---- initial values, drawn in ResNet::new order (model.rs:112-133):
  // every block (c1, c2, shortcut conv) first, then the stem, then the
  // classifier (nn.rs:487-498, halved); BN gamma 1 (0 for each block's bn2,
  // model.rs:22-23), beta 0.
  std::vector<float> hv(net->nparams, 0.0f);
  Rng rng(seed);
  auto kaiming = [&](const ConvL& c) {
    const float s = sqrtf(2.0f / (float)(c.cin * c.k * c.k));
    const size_t n = (size_t)c.cout * c.cin * c.k * c.k;
    for (size_t i = 0; i < n; i++) hv[c.w_off + i] = rng.normal() * s;
  };
  auto bn_init = [&](const BNL& b, float gamma) {
    for (int i = 0; i < b.c; i++) hv[b.g_off + i] = gamma;
  };
  for (auto& b : net->blocks) {
    kaiming(b.c1);
    kaiming(b.c2);
    if (b.down) kaiming(b.cd);
    bn_init(b.b1, 1.0f);
    bn_init(b.b2, 0.0f);
    if (b.down) bn_init(b.bd, 1.0f);
  }
  kaiming(net->stem);
  bn_init(net->stem_bn, 1.0f);
  {
    const float s = sqrtf(2.0f / (float)net->fin);
    for (size_t i = 0; i < (size_t)net->fin * nclass; i++) hv[net->fcw_off + i] = rng.normal() * s * 0.5f;
  }

  // ---- device state
  net->decay_host.resize(net->nparams);
  {
    size_t o = 0;
    for (size_t i = 0; i < sizes.size(); i++) {
      memset(net->decay_host.data() + o, dec[i], sizes[i]);
      o += sizes[i];
    }
  }
  auto fail = [&](int code) {
    rnn_resnet_destroy(net);
    return code;
  };
  if (cudaMalloc(&net->v, net->nparams * 4) != cudaSuccess || cudaMalloc(&net->g, net->nparams * 4) != cudaSuccess ||
      cudaMalloc(&net->m, net->nparams * 4) != cudaSuccess || cudaMalloc(&net->decay, net->nparams) != cudaSuccess ||
      cudaMalloc(&net->bnbuf, net->nbuf * 4) != cudaSuccess)
    return fail(set_error(RNN_ERR_CUDA, "resnet_create: out of device memory"));
  // mean/invstd of every BN
  size_t nstat = 0;
  nstat += 2 * (size_t)net->stem_bn.c;
  for (auto& b : net->blocks) nstat += 2 * (size_t)(b.b1.c + b.b2.c + (b.down ? b.bd.c : 0));
  if (cudaMalloc(&net->bnstat, nstat * 4) != cudaSuccess)
    return fail(set_error(RNN_ERR_CUDA, "resnet_create: out of device memory"));
  {
    float* p = net->bnstat;
    auto assign = [&](BNL& b) {
      b.mean = p;
      b.invstd = p + b.c;
      p += 2 * b.c;
    };
    assign(net->stem_bn);
    for (auto& b : net->blocks) {
      assign(b.b1);
      assign(b.b2);
      if (b.down) assign(b.bd);
    }
  }
  std::vector<float> hb(net->nbuf);
  {
    // running mean 0, running var 1 (nn.rs:271-272)
    auto fillb = [&](const BNL& b) {
      for (int i = 0; i < b.c; i++) {
        hb[b.rm_off + i] = 0.0f;
        hb[b.rm_off + b.c + i] = 1.0f;
      }
    };
    fillb(net->stem_bn);
    for (auto& b : net->blocks) {
      fillb(b.b1);
      fillb(b.b2);
      if (b.down) fillb(b.bd);
    }
  }
  if (cudaMemcpy(net->v, hv.data(), net->nparams * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemset(net->g, 0, net->nparams * 4) != cudaSuccess || cudaMemset(net->m, 0, net->nparams * 4) != cudaSuccess ||
      cudaMemcpy(net->decay, net->decay_host.data(), net->nparams, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(net->bnbuf, hb.data(), net->nbuf * 4, cudaMemcpyHostToDevice) != cudaSuccess)
    return fail(set_error(RNN_ERR_CUDA, "resnet_create: upload failed"));
  if (cudaMalloc(&net->loss_dev, 4) != cudaSuccess || cudaMalloc(&net->correct_dev, 4) != cudaSuccess)
    return fail(set_error(RNN_ERR_CUDA, "resnet_create: out of device memory"));
  *out = net;
  return RNN_OK;
}

extern "C" int rnn_resnet_destroy(rnn_resnet* net) {
  if (!net) return RNN_OK;
  // the context may already be gone (interpreter teardown releases objects
  // in any order): wait on the device, not on the context's stream
  cudaDeviceSynchronize();
  net->graph.destroy();  // before the NCCL communicator its graph may hold
  peer_release(net);
  free_acts(net);
  rnn::eval_ws_free(net->eval);
  cudaFree(net->v);
  cudaFree(net->g);
  cudaFree(net->m);
  cudaFree(net->decay);
  cudaFree(net->bnbuf);
  cudaFree(net->bnstat);
  cudaFree(net->loss_dev);
  cudaFree(net->correct_dev);
  if (net->comm && !net->handle.aborted) ncclCommDestroy(net->comm);  // an abort already released it
  if (net->comm_stream) cudaStreamDestroy(net->comm_stream);
  if (net->bucket_ev) cudaEventDestroy(net->bucket_ev);
  if (net->comm_done) cudaEventDestroy(net->comm_done);
  delete net;
  return RNN_OK;
}

extern "C" int rnn_resnet_num_params(rnn_resnet* net, size_t* out) {
  RNN_REQUIRE(net && out, "null argument");
  *out = net->nparams;
  return RNN_OK;
}

extern "C" int rnn_resnet_num_buffers(rnn_resnet* net, size_t* out) {
  RNN_REQUIRE(net && out, "null argument");
  *out = net->nbuf;
  return RNN_OK;
}

static int copy_out(rnn_resnet* net, float* dst, const float* src, size_t n) {
  RNN_CUDA(cudaStreamSynchronize(net->ctx->stream));
  RNN_CUDA(cudaMemcpy(dst, src, n * 4, cudaMemcpyDeviceToHost));
  return RNN_OK;
}

extern "C" int rnn_resnet_get_params(rnn_resnet* net, float* out) {
  RNN_REQUIRE(net && out, "null argument");
  return copy_out(net, out, net->v, net->nparams);
}
extern "C" int rnn_resnet_get_grads(rnn_resnet* net, float* out) {
  RNN_REQUIRE(net && out, "null argument");
  return copy_out(net, out, net->g, net->nparams);
}
extern "C" int rnn_resnet_get_moments(rnn_resnet* net, float* out) {
  RNN_REQUIRE(net && out, "null argument");
  return copy_out(net, out, net->m, net->nparams);
}
extern "C" int rnn_resnet_get_buffers(rnn_resnet* net, float* out) {
  RNN_REQUIRE(net && out, "null argument");
  return copy_out(net, out, net->bnbuf, net->nbuf);
}
extern "C" int rnn_resnet_set_params(rnn_resnet* net, const float* in) {
  RNN_REQUIRE(net && in, "null argument");
  RNN_CUDA(cudaStreamSynchronize(net->ctx->stream));
  RNN_CUDA(cudaMemcpy(net->v, in, net->nparams * 4, cudaMemcpyHostToDevice));
  return RNN_OK;
}
extern "C" int rnn_resnet_grad_buffer(rnn_resnet* net, float** out, size_t* len) {
  RNN_REQUIRE(net && out && len, "null argument");
  *out = net->g;
  *len = net->nparams;
  return RNN_OK;
}

extern "C" int rnn_resnet_forward_dev(rnn_resnet* net, const float* x, int n, int h, int w, int train,
                                      float* logits) {
  RNN_REQUIRE(net && x && logits, "resnet_forward: null argument");
  RNN_REQUIRE(n > 0 && h > 0 && w > 0, "resnet_forward: bad shape");
  return resnet_forward(net, x, n, h, w, train != 0, logits);
}

extern "C" int rnn_resnet_backward_dev(rnn_resnet* net, const float* dlogits) {
  RNN_REQUIRE(net && dlogits, "resnet_backward: null argument");
  RNN_REQUIRE(net->n > 0, "resnet_backward: no forward pass recorded");
  return resnet_backward(net, dlogits);
}

extern "C" int rnn_resnet_set_graph(rnn_resnet* net, int enable) {
  RNN_REQUIRE(net, "set_graph: null argument");
  net->use_graph = enable != 0;
  if (!net->use_graph) net->graph.release();
  return RNN_OK;
}

extern "C" int rnn_resnet_step(rnn_resnet* net, float lr, float mom, float wd) {
  RNN_REQUIRE(net, "null argument");
  return resnet_step(net, lr, mom, wd);
}

extern "C" int rnn_resnet_train_step_dev(rnn_resnet* net, const float* x, const uint32_t* labels, int n,
                                         float smooth, float lr, float mom, float wd, float* loss, int* correct) {
  RNN_REQUIRE(net && x && labels, "train_step: null argument");
  RNN_REQUIRE(n > 0, "train_step: empty batch");
  return train_step_any(net, x, labels, n, smooth, lr, mom, wd, loss ? loss : net->loss_dev,
                        correct ? correct : net->correct_dev);
}

extern "C" int rnn_resnet_train_step(rnn_resnet* net, const float* x, const uint32_t* labels, int n, float smooth,
                                     float lr, float mom, float wd, float* loss, int* correct) {
  RNN_REQUIRE(net && x && labels, "train_step: null argument");
  RNN_REQUIRE(n > 0, "train_step: empty batch");
  rnn_ctx* ctx = net->ctx;
  RNN_TRY(ensure_acts(net, n, 32, 32));
  RNN_CUDA(cudaMemcpyAsync(net->x_stage, x, (size_t)n * 3 * 32 * 32 * 4, cudaMemcpyHostToDevice, ctx->stream));
  RNN_CUDA(cudaMemcpyAsync(net->lab_stage, labels, (size_t)n * 4, cudaMemcpyHostToDevice, ctx->stream));
  RNN_TRY(train_step_any(net, net->x_stage, net->lab_stage, n, smooth, lr, mom, wd, net->loss_dev,
                         net->correct_dev));
  float l = 0.0f;
  int c = 0;
  RNN_CUDA(cudaMemcpyAsync(&l, net->loss_dev, 4, cudaMemcpyDeviceToHost, ctx->stream));
  RNN_CUDA(cudaMemcpyAsync(&c, net->correct_dev, 4, cudaMemcpyDeviceToHost, ctx->stream));
  RNN_TRY(rnn_ctx_synchronize(ctx));
  if (loss) *loss = l;
  if (correct) *correct = c;
  return RNN_OK;
}

// ---------------------------------------------------------------- eval

// eval::resnet (eval.rs:41-43): forward with train false over the dataset
static int resnet_eval(rnn_resnet* net, const uint8_t* images, const uint8_t* labels, int len, int batch,
                       float* loss, float* acc) {
  float out2[2];
  RNN_TRY(rnn::eval_loop(net->ctx, net->eval, images, labels, len, batch, net->fout, false,
                         [net](const float* x, int bs, const float** lg) {
                           RNN_TRY(ensure_acts(net, bs, 32, 32));
                           RNN_TRY(resnet_forward(net, x, bs, 32, 32, false, net->logits));
                           *lg = net->logits;
                           return (int)RNN_OK;
                         },
                         out2));
  if (loss) *loss = out2[0];
  if (acc) *acc = out2[1];
  return RNN_OK;
}

extern "C" int rnn_resnet_eval_dev(rnn_resnet* net, const uint8_t* images, const uint8_t* labels, int len,
                                   int batch, float* loss, float* acc) {
  RNN_REQUIRE(net && (len == 0 || (images && labels)), "resnet_eval: null argument");
  return resnet_eval(net, images, labels, len, batch, loss, acc);
}

extern "C" int rnn_resnet_eval(rnn_resnet* net, const uint8_t* images, const uint8_t* labels, int len, int batch,
                               float* loss, float* acc) {
  RNN_REQUIRE(net && (len == 0 || (images && labels)), "resnet_eval: null argument");
  RNN_REQUIRE(len >= 0 && batch > 0, "resnet_eval: bad sizes");
  const uint8_t *di = nullptr, *dl = nullptr;
  if (len > 0) RNN_TRY(rnn::eval_ws_stage(net->eval, net->ctx, images, labels, len, &di, &dl));
  return resnet_eval(net, di, dl, len, batch, loss, acc);
}

// ---------------------------------------------------------------- checkpoints

// ResNet::config_hash (model.rs:220-229): blocks / 3 = depth_n, the stem's
// cout = width, the classifier's fout = nclass
static uint64_t resnet_hash(const rnn_resnet* net, const char* kind) {
  const uint64_t v[3] = {(uint64_t)net->depth_n, (uint64_t)net->width, (uint64_t)net->nclass};
  return rnn::ckpt_hash(kind, strlen(kind), v, 3);
}

static int to_host(rnn_resnet* net, std::vector<float>& h, const float* d, size_t n) {
  h.resize(n);
  if (n) RNN_CUDA(cudaMemcpyAsync(h.data(), d, n * sizeof(float), cudaMemcpyDeviceToHost, net->ctx->stream));
  return RNN_OK;
}

extern "C" int rnn_resnet_save(rnn_resnet* net, const char* path) {
  RNN_REQUIRE(net && path, "resnet_save: null argument");
  std::vector<float> v, b;
  RNN_TRY(to_host(net, v, net->v, net->nparams));
  RNN_TRY(to_host(net, b, net->bnbuf, net->nbuf));
  RNN_TRY(rnn_ctx_synchronize(net->ctx));
  return rnn::ckpt_write(path, (uint32_t)(net->n_param_tensors + net->n_buf_tensors), resnet_hash(net, "resnet"),
                         {{v.data(), v.size()}, {b.data(), b.size()}});
}

extern "C" int rnn_resnet_load(rnn_resnet* net, const char* path) {
  RNN_REQUIRE(net && path, "resnet_load: null argument");
  std::vector<float> p;
  RNN_TRY(rnn::ckpt_read(path, (uint32_t)(net->n_param_tensors + net->n_buf_tensors), resnet_hash(net, "resnet"),
                         net->nparams + net->nbuf, p));
  RNN_CUDA(cudaMemcpyAsync(net->v, p.data(), net->nparams * sizeof(float), cudaMemcpyHostToDevice,
                           net->ctx->stream));
  RNN_CUDA(cudaMemcpyAsync(net->bnbuf, p.data() + net->nparams, net->nbuf * sizeof(float), cudaMemcpyHostToDevice,
                           net->ctx->stream));
  return rnn_ctx_synchronize(net->ctx);
}

extern "C" int rnn_resnet_save_optim(rnn_resnet* net, const char* path) {
  RNN_REQUIRE(net && path, "resnet_save_optim: null argument");
  std::vector<float> m;
  RNN_TRY(to_host(net, m, net->m, net->nparams));
  RNN_TRY(rnn_ctx_synchronize(net->ctx));
  return rnn::ckpt_write(path, (uint32_t)net->n_param_tensors, resnet_hash(net, "resnet-optim"),
                         {{m.data(), m.size()}});
}

extern "C" int rnn_resnet_load_optim(rnn_resnet* net, const char* path) {
  RNN_REQUIRE(net && path, "resnet_load_optim: null argument");
  std::vector<float> m;
  RNN_TRY(rnn::ckpt_read(path, (uint32_t)net->n_param_tensors, resnet_hash(net, "resnet-optim"), net->nparams, m));
  RNN_CUDA(cudaMemcpyAsync(net->m, m.data(), net->nparams * sizeof(float), cudaMemcpyHostToDevice,
                           net->ctx->stream));
  return rnn_ctx_synchronize(net->ctx);
}

// ---------------------------------------------------------------- DP

extern "C" int rnn_dp_unique_id(unsigned char* uid_out) {
  RNN_REQUIRE(uid_out, "null argument");
  static_assert(sizeof(ncclUniqueId) == RNN_UID_BYTES, "uid size");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return set_error(RNN_ERR_NCCL, "ncclGetUniqueId: %s", ncclGetErrorString(r));
  memcpy(uid_out, &id, sizeof(id));
  return RNN_OK;
}

// RNN_SYNCBN_NCCL=1 keeps SyncBN on NCCL all-reduces (for comparison).
static bool peer_sync_disabled() {
  const char* v = getenv("RNN_SYNCBN_NCCL");
  return v && v[0] == '1';
}

extern "C" int rnn_resnet_dp_init(rnn_resnet* net, int rank, int world, const unsigned char* uid, int sync_bn) {
  RNN_REQUIRE(net && uid, "null argument");
  RNN_REQUIRE(world >= 1 && rank >= 0 && rank < world, "dp_init: bad rank/world");
  cudaDeviceSynchronize();
  net->graph.release();
  peer_release(net);
  if (net->comm) {
    if (!net->handle.aborted) ncclCommDestroy(net->comm);
    net->comm = nullptr;
  }
  ncclUniqueId id;
  memcpy(&id, uid, sizeof(id));
  RNN_CUDA(cudaSetDevice(net->ctx->device));
  ncclResult_t r = ncclCommInitRank(&net->comm, world, id, rank);
  if (r != ncclSuccess) return set_error(RNN_ERR_NCCL, "ncclCommInitRank: %s", ncclGetErrorString(r));
  net->handle = rnn_comm{};
  net->handle.comm = net->comm;
  net->handle.device = net->ctx->device;
  net->handle.rank = rank;
  net->handle.world = world;
  net->handle.owned = false;
  net->rank = rank;
  net->world = world;
  net->sync_bn = sync_bn != 0;
  // gradient buckets of ~8 MB (RNN_GRAD_BUCKET_MB, 0 = one all-reduce after
  // the backward), summed on their own stream while the backward goes on
  net->bucket_floats = 0;
  if (world > 1) {
    const char* e = getenv("RNN_GRAD_BUCKET_MB");
    const double mb = e && e[0] ? atof(e) : 8.0;
    if (mb > 0) {
      net->bucket_floats = (size_t)(mb * (1 << 20) / sizeof(float));
      if (!net->comm_stream) RNN_CUDA(cudaStreamCreateWithFlags(&net->comm_stream, cudaStreamNonBlocking));
      if (!net->bucket_ev) RNN_CUDA(cudaEventCreateWithFlags(&net->bucket_ev, cudaEventDisableTiming));
      if (!net->comm_done) RNN_CUDA(cudaEventCreateWithFlags(&net->comm_done, cudaEventDisableTiming));
    }
  }
  if (world > 1 && net->sync_bn && !peer_sync_disabled()) RNN_TRY(peer_setup(net));
  return RNN_OK;
}

extern "C" int rnn_resnet_comm(rnn_resnet* net, rnn_comm** out) {
  RNN_REQUIRE(net && out, "resnet_comm: null argument");
  *out = nullptr;
  RNN_REQUIRE(net->comm, "resnet_comm: the network is not data-parallel (rnn_resnet_dp_init)");
  *out = &net->handle;
  return RNN_OK;
}
