// Device-resident rustvit training step (vit.rs, attn.rs:347-560, norm.rs,
// linear.rs, loss.rs, optim.rs, train.rs:70-118 and 346-387).
//
// The network is composed on the host from the library's own device entry
// points (every arithmetic step runs in a kernel of this library; nothing is
// computed on the CPU).  Parameters, gradients and the two optimiser moments
// live in four flat device buffers in the reference's for_each_param order
// (vit.rs:687-719), so clip_ is one call over the whole gradient and whole-
// model vectors compare elementwise with the CPU oracle.  Initial values are
// drawn on the host with the restated Rng in the reference's construction
// order (blocks first, then the struct-literal fields, vit.rs:441-509), so
// the device starts from the reference's exact parameters.
//
// Activations are preallocated for the batch capacity; each layer keeps what
// its reference counterpart keeps for the backward (LayerNorm xhat/invstd,
// Linear inputs, attention P, SwiGLU pre-activation, LayerScale inputs, the
// depthwise branch output for the gamma gradient, BatchNorm inputs).
#include <string.h>

#include <algorithm>
#include <vector>

#include "../../include/rnn_b200.h"
#include "ckpt.cuh"
#include "common.cuh"
#include "eval.cuh"
#include "ew.cuh"
#include "rng.h"

namespace rnn {
namespace vit {

// ---------------------------------------------------------------- host init

// Param::trunc_normal, nn.rs:77-89
static void trunc_normal(Rng& r, std::vector<float>& out, size_t n, float std_) {
  out.resize(n);
  for (size_t i = 0; i < n; i++) {
    float z = r.normal();
    int tries = 0;
    while (fabsf(z) > 2.0f && tries < 8) {
      z = r.normal();
      tries++;
    }
    z = z < -2.0f ? -2.0f : (z > 2.0f ? 2.0f : z);
    out[i] = z * std_;
  }
}

// Param::kaiming, nn.rs:95-100
static void kaiming(Rng& r, std::vector<float>& out, size_t n, int fan_in) {
  out.resize(n);
  const float s = sqrtf(2.0f / (float)fan_in);
  for (size_t i = 0; i < n; i++) out[i] = r.normal() * s;
}

struct HostParam {
  std::vector<float> v;
  bool decay;
  int rows, cols;  // > 0 for Linear weights (Muon-eligible when both > 1)
};

struct Registry {
  std::vector<HostParam> ps;
  int add(std::vector<float>&& v, bool decay, int rows = 0, int cols = 0) {
    ps.push_back(HostParam{std::move(v), decay, rows, cols});
    return (int)ps.size() - 1;
  }
  int zeros(size_t n, bool decay) { return add(std::vector<float>(n, 0.0f), decay); }
  int filled(size_t n, float val, bool decay) { return add(std::vector<float>(n, val), decay); }
};

// ---------------------------------------------------------------- layers

struct ConvL {
  int w = -1, cin = 0, cout = 0, k = 0, stride = 1, pad = 0;
  void init(Registry& R, Rng& r, int ci, int co, int ks, int st, int pd) {
    cin = ci; cout = co; k = ks; stride = st; pad = pd;
    std::vector<float> v;
    kaiming(r, v, (size_t)co * ci * ks * ks, ci * ks * ks);
    w = R.add(std::move(v), true);
  }
  int out(int h) const { return (h + 2 * pad - k) / stride + 1; }
};

struct BNL {
  int g = -1, b = -1, c = 0;
  size_t rm = 0, rv = 0;  // offsets into the running-statistics buffer
  float *mean = nullptr, *invstd = nullptr;
  void init(Registry& R, int ch) {
    c = ch;
    g = R.filled(ch, 1.0f, false);
    b = R.zeros(ch, false);
  }
};

struct LinL {
  int w = -1, b = -1, fin = 0, fout = 0;
  const float* x = nullptr;  // saved input
  int rows = 0;
  void init(Registry& R, Rng& r, int fi, int fo, bool bias, float std_) {
    fin = fi; fout = fo;
    std::vector<float> v;
    trunc_normal(r, v, (size_t)fi * fo, std_);
    w = R.add(std::move(v), true, fo, fi);
    if (bias) b = R.zeros(fo, false);
  }
  void scaled(Registry& R, Rng& r, int fi, int fo, bool bias, int depth) {
    init(R, r, fi, fo, bias, 0.02f / sqrtf(2.0f * (float)depth));
  }
};

struct LNL {
  int g = -1, b = -1, c = 0;
  float *xhat = nullptr, *invstd = nullptr;
  int rows = 0;
  void init(Registry& R, int ch) {
    c = ch;
    g = R.filled(ch, 1.0f, false);
    b = R.zeros(ch, false);
  }
};

struct LSL {  // LayerScale
  int l = -1, c = 0;
  const float* x = nullptr;  // saved input
  void init(Registry& R, int ch, float v0) {
    c = ch;
    l = R.filled(ch, v0, false);
  }
};

struct DPL {  // DropPath
  float p = 0.0f;
  float* mask = nullptr;
  bool active = false;
};

struct SelfAttnL {
  LinL qkv, proj;
  int tau = -1, rel = -1, h = 0, dh = 0, c = 0, th = 0;
  float *ab = nullptr, *p = nullptr, *o = nullptr;
  void init(Registry& R, Rng& r, int ch, int heads, int t_h, int depth) {
    c = ch; h = heads; dh = ch / heads; th = t_h;
    int nrel = 0;
    rnn_rel_index(th, th, th, th, nullptr, &nrel);
    qkv.init(R, r, c, 3 * c, true, 0.02f);
    proj.scaled(R, r, c, c, true, depth);
    tau = R.filled(h, 1.0f / sqrtf((float)dh), false);
    rel = R.zeros((size_t)h * nrel, false);
  }
};

struct CrossAttnL {
  LinL wq, proj;
  int tau = -1, rel = -1, h = 0, dh = 0, c = 0, th = 0, mh = 0;
  float *q = nullptr, *p = nullptr, *o = nullptr;
  void init(Registry& R, Rng& r, int ch, int heads, int t_h, int m_h, int depth) {
    c = ch; h = heads; dh = ch / heads; th = t_h; mh = m_h;
    int nrel = 0;
    rnn_rel_index(th, th, mh, mh, nullptr, &nrel);
    wq.init(R, r, c, c, true, 0.02f);
    proj.scaled(R, r, c, c, true, depth);
    tau = R.filled(h, 1.0f / sqrtf((float)dh), false);
    rel = R.zeros((size_t)h * nrel, false);
  }
};

struct SwiL {
  LinL wg, wd;
  int h = 0;
  float *ab = nullptr, *u = nullptr;
  void init(Registry& R, Rng& r, int c, int hid, int depth) {
    h = hid;
    wg.init(R, r, c, 2 * hid, true, 0.02f);
    wd.scaled(R, r, hid, c, true, depth);
  }
};

struct DwL {
  int w = -1, b = -1, c = 0, th = 0;
  const float* x = nullptr;
  void init(Registry& R, Rng& r, int ch, int t_h) {
    c = ch; th = t_h;
    std::vector<float> v;
    trunc_normal(r, v, (size_t)9 * ch, 0.1f);
    w = R.add(std::move(v), false);
    b = R.zeros(ch, false);
  }
};

struct Block {
  LNL n1, n2;
  SelfAttnL attn;
  DwL dw;
  int gamma = -1;
  LSL ls1, lsm, ls2;
  bool has_cross = false;
  CrossAttnL cross;
  SwiL mlp;
  DPL dp1, dp2, dp3;
  int c = 0, th = 0;
  uint64_t idx = 0;
  // activations
  float *hb = nullptr, *a = nullptr, *dwo = nullptr, *tmp = nullptr, *s1 = nullptr, *y = nullptr;
  float *cm = nullptr, *s2 = nullptr, *h2 = nullptr, *m = nullptr, *s3 = nullptr;
  void init(Registry& R, Rng& r, int ch, int heads, int t_h, int m_h, int depth, float drop, uint64_t id,
            float ls_init) {
    c = ch; th = t_h; idx = id;
    const int hidden = ((4 * ch / 3) + 15) / 16 * 16;  // (4c/3).div_ceil(16)*16
    n1.init(R, ch);
    attn.init(R, r, ch, heads, t_h, depth);
    dw.init(R, r, ch, t_h);
    gamma = R.filled(ch, 0.5f, false);
    ls1.init(R, ch, ls_init);
    if (m_h > 0) {
      has_cross = true;
      cross.init(R, r, ch, heads, t_h, m_h, depth);
      lsm.init(R, ch, ls_init);
    }
    n2.init(R, ch);
    mlp.init(R, r, ch, hidden, depth);
    ls2.init(R, ch, ls_init);
    dp1.p = dp2.p = dp3.p = drop;
  }
};

struct BasicBlockL {  // model.rs:10-98
  ConvL c1, c2, cd;
  BNL b1, b2, bd;
  bool down = false;
  int hin = 0, hout = 0;
  const float* x = nullptr;
  float *y1 = nullptr, *h1 = nullptr, *y2 = nullptr, *yd = nullptr, *out = nullptr;
  void init(Registry& R, Rng& r, int cin, int cout, int stride, int h) {
    // b2 is built first and zero_gamma'd (model.rs:21-23); BatchNorm draws
    // nothing from the rng, so only the convolutions order the stream
    b2.init(R, cout);
    std::fill(R.ps[b2.g].v.begin(), R.ps[b2.g].v.end(), 0.0f);
    c1.init(R, r, cin, cout, 3, stride, 1);
    b1.init(R, cout);
    c2.init(R, r, cout, cout, 3, 1, 1);
    down = stride != 1 || cin != cout;
    if (down) {
      cd.init(R, r, cin, cout, 1, stride, 0);
      bd.init(R, cout);
    }
    hin = h;
    hout = c1.out(h);
  }
};

struct SeqPoolL {
  int p = -1, c = 0, t = 0;
  const float* x = nullptr;
  float* w = nullptr;
  void init(Registry& R, Rng& r, int ch) {
    c = ch;
    std::vector<float> v;
    trunc_normal(r, v, ch, 0.02f);
    p = R.add(std::move(v), true);
  }
};

struct Cfg {
  int width, cmid, dim, heads, depth3, dim4, heads4, depth4, img;
  std::vector<int> mem_at;
  float droppath;
};

}  // namespace vit
}  // namespace rnn

using namespace rnn;
using namespace rnn::vit;

struct rnn_rustvit {
  rnn_ctx* ctx = nullptr;
  Cfg cfg;
  int nf = 0, nc = 0, th = 0, mh = 0;
  uint32_t* parent = nullptr;  // device [nf]
  std::vector<uint32_t> parent_host;  // for the checkpoint hash
  int n_buf_tensors = 0;
  // parameters
  Registry R;
  std::vector<size_t> off;  // per registry id
  std::vector<int> order;   // registry ids in for_each_param order
  size_t np = 0;
  float *V = nullptr, *G = nullptr, *M = nullptr, *V2 = nullptr, *E = nullptr;
  // running statistics (stem_bn, c1, c2, tok_bn: for_each_buffer order)
  float* B = nullptr;
  size_t nb = 0;
  // data-parallel step (rnn_rustvit_dp_attach): borrowed communicator or null
  rnn_comm* comm = nullptr;
  // layers
  ConvL stem, memconv, tokconv;
  BNL stem_bn, tok_bn;
  BasicBlockL c1, c2;
  LNL memln, mergeln, headln;
  LinL merge;
  std::vector<Block> blocks3, blocks4;
  SeqPoolL pool, pool2;
  LinL head_coarse, head_resid, e1_fc, e1_hint, e2_fc, e2_hint;
  bool use_exits = true;
  rnn::EvalWs eval;  // evaluation buffers (rnn_rustvit_eval)
  // optimiser state
  int opt_t = 0, ema_t = 0;
  bool ema_ready = false;
  // step_all's segment tables (device): the Muon matrices, then the AdamW runs
  rnn::OptSeg* opt_segs = nullptr;
  int n_mu = 0, n_ad = 0;
  size_t mu_max = 0, ad_max = 0;
  // activations
  std::vector<void*> allocs;
  int cap = 0;
  int n = 0;
  float *y0 = nullptr, *stem_out = nullptr, *mcv = nullptr, *memt = nullptr, *mem = nullptr;
  float *tcv = nullptr, *tbn = nullptr, *z0 = nullptr;
  float *f2 = nullptr, *e2l = nullptr, *h2v = nullptr, *zm = nullptr, *zn = nullptr, *z4 = nullptr;
  float *zf = nullptr, *feat = nullptr, *zc = nullptr, *zl = nullptr, *gp = nullptr, *e1l = nullptr,
        *h1v = nullptr;
  // backward scratch
  float *g_logits = nullptr, *g_coarse = nullptr, *g_e1 = nullptr, *g_e2 = nullptr, *g_h1 = nullptr,
        *g_h2 = nullptr;
  float *b_small1 = nullptr, *b_small2 = nullptr, *b_small3 = nullptr, *b_small4 = nullptr;
  float *b_rows4 = nullptr, *b_rows4b = nullptr, *b_merge = nullptr, *b_merge2 = nullptr;
  float *b_rows3 = nullptr, *dmem = nullptr, *dmem2 = nullptr;
  float *bs1 = nullptr, *bs2 = nullptr, *bs3 = nullptr, *bs4 = nullptr, *bs_wide = nullptr, *bs_wide2 = nullptr,
        *bs_qkv = nullptr;
  float *b_img_a = nullptr, *b_img_b = nullptr, *b_img_c = nullptr, *b_img_d = nullptr, *b_c2 = nullptr,
        *b_c2b = nullptr;
  // packed A image of the last LayerNorm output that feeds a GEMM
  float* aimg = nullptr;
  const float* x_in = nullptr;  // the batch of the last forward
  float* xkeep = nullptr;
  float* losses = nullptr;  // device [8]
  int* correct = nullptr;   // device [4]
  float* clip_norm = nullptr;
  // host-tier staging
  float *st_x = nullptr, *st_tf = nullptr, *st_tc = nullptr;
  uint32_t* st_hard = nullptr;
  int st_cap = 0;
};

namespace rnn {
namespace vit {

static float* P(rnn_rustvit* net, int id) { return net->V + net->off[id]; }
static float* Gd(rnn_rustvit* net, int id) { return net->G + net->off[id]; }
static float* Popt(rnn_rustvit* net, int id) { return id < 0 ? nullptr : P(net, id); }
static float* Gopt(rnn_rustvit* net, int id) { return id < 0 ? nullptr : Gd(net, id); }

// ---- parameter order (vit.rs:687-719 and the layers' for_each_param)

static void ord_lin(std::vector<int>& o, const LinL& l) {
  o.push_back(l.w);
  if (l.b >= 0) o.push_back(l.b);
}
static void ord_ln(std::vector<int>& o, const LNL& l) {
  o.push_back(l.g);
  o.push_back(l.b);
}
static void ord_bb(std::vector<int>& o, const BasicBlockL& b) {
  o.push_back(b.c1.w); o.push_back(b.b1.g); o.push_back(b.b1.b);
  o.push_back(b.c2.w); o.push_back(b.b2.g); o.push_back(b.b2.b);
  if (b.down) { o.push_back(b.cd.w); o.push_back(b.bd.g); o.push_back(b.bd.b); }
}
static void ord_block(std::vector<int>& o, const Block& b) {
  ord_ln(o, b.n1);
  ord_lin(o, b.attn.qkv); ord_lin(o, b.attn.proj); o.push_back(b.attn.tau); o.push_back(b.attn.rel);
  o.push_back(b.dw.w); o.push_back(b.dw.b);
  o.push_back(b.gamma);
  o.push_back(b.ls1.l);
  if (b.has_cross) {
    ord_lin(o, b.cross.wq); ord_lin(o, b.cross.proj); o.push_back(b.cross.tau); o.push_back(b.cross.rel);
    o.push_back(b.lsm.l);
  }
  ord_ln(o, b.n2);
  ord_lin(o, b.mlp.wg); ord_lin(o, b.mlp.wd);
  o.push_back(b.ls2.l);
}
static std::vector<int> param_order(const rnn_rustvit* n) {
  std::vector<int> o;
  o.push_back(n->stem.w); o.push_back(n->stem_bn.g); o.push_back(n->stem_bn.b);
  ord_bb(o, n->c1);
  ord_bb(o, n->c2);
  o.push_back(n->memconv.w);
  ord_ln(o, n->memln);
  o.push_back(n->tokconv.w); o.push_back(n->tok_bn.g); o.push_back(n->tok_bn.b);
  for (auto& b : n->blocks3) ord_block(o, b);
  ord_ln(o, n->mergeln);
  ord_lin(o, n->merge);
  for (auto& b : n->blocks4) ord_block(o, b);
  ord_ln(o, n->headln);
  o.push_back(n->pool.p);
  ord_lin(o, n->head_coarse); ord_lin(o, n->head_resid);
  if (n->use_exits) {
    ord_lin(o, n->e1_fc); ord_lin(o, n->e1_hint);
    o.push_back(n->pool2.p);
    ord_lin(o, n->e2_fc); ord_lin(o, n->e2_hint);
  }
  return o;
}

// ---- activation arena

static int dalloc(rnn_rustvit* net, float** p, size_t nfl) {
  void* q = nullptr;
  RNN_CUDA(cudaMalloc(&q, std::max<size_t>(nfl, 1) * sizeof(float)));
  net->allocs.push_back(q);
  *p = static_cast<float*>(q);
  return RNN_OK;
}

static void free_acts(rnn_rustvit* net) {
  for (void* p : net->allocs) cudaFree(p);
  net->allocs.clear();
  net->cap = 0;
}

static int alloc_block(rnn_rustvit* net, Block& b, int n, bool first_of_stage) {
  const size_t rows = (size_t)n * b.th * b.th, c = b.c;
  const int t = b.th * b.th;
  (void)first_of_stage;
  RNN_TRY(dalloc(net, &b.hb, rows * c));
  RNN_TRY(dalloc(net, &b.n1.xhat, rows * c));
  RNN_TRY(dalloc(net, &b.n1.invstd, rows));
  RNN_TRY(dalloc(net, &b.attn.ab, rows * 3 * c));
  RNN_TRY(dalloc(net, &b.attn.p, (size_t)n * b.attn.h * t * t));
  RNN_TRY(dalloc(net, &b.attn.o, rows * c));
  RNN_TRY(dalloc(net, &b.a, rows * c));
  RNN_TRY(dalloc(net, &b.dwo, rows * c));
  RNN_TRY(dalloc(net, &b.tmp, rows * c));
  RNN_TRY(dalloc(net, &b.s1, rows * c));
  RNN_TRY(dalloc(net, &b.y, rows * c));
  if (b.has_cross) {
    const int tk = b.cross.mh * b.cross.mh;
    RNN_TRY(dalloc(net, &b.cross.q, rows * c));
    RNN_TRY(dalloc(net, &b.cross.p, (size_t)n * b.cross.h * t * tk));
    RNN_TRY(dalloc(net, &b.cross.o, rows * c));
    RNN_TRY(dalloc(net, &b.cm, rows * c));
    RNN_TRY(dalloc(net, &b.s2, rows * c));
  }
  RNN_TRY(dalloc(net, &b.h2, rows * c));
  RNN_TRY(dalloc(net, &b.n2.xhat, rows * c));
  RNN_TRY(dalloc(net, &b.n2.invstd, rows));
  RNN_TRY(dalloc(net, &b.mlp.ab, rows * 2 * b.mlp.h));
  RNN_TRY(dalloc(net, &b.mlp.u, rows * b.mlp.h));
  RNN_TRY(dalloc(net, &b.m, rows * c));
  RNN_TRY(dalloc(net, &b.s3, rows * c));
  RNN_TRY(dalloc(net, &b.dp1.mask, n));
  RNN_TRY(dalloc(net, &b.dp2.mask, n));
  RNN_TRY(dalloc(net, &b.dp3.mask, n));
  return RNN_OK;
}

static int alloc_bn(rnn_rustvit* net, BNL& b) {
  RNN_TRY(dalloc(net, &b.mean, b.c));
  RNN_TRY(dalloc(net, &b.invstd, b.c));
  return RNN_OK;
}

static int ensure_acts(rnn_rustvit* net, int n) {
  if (n <= net->cap) return RNN_OK;
  free_acts(net);
  const Cfg& c = net->cfg;
  const size_t img = (size_t)c.img * c.img, r2 = (size_t)net->mh * net->mh, t3 = (size_t)net->th * net->th;
  const size_t t4 = t3 / 4;
  const int w = c.width, cm = c.cmid, d = c.dim, d4 = c.dim4;
  RNN_TRY(dalloc(net, &net->xkeep, (size_t)n * 3 * img));
  RNN_TRY(dalloc(net, &net->y0, n * w * img));
  RNN_TRY(dalloc(net, &net->stem_out, n * w * img));
  RNN_TRY(alloc_bn(net, net->stem_bn));
  for (BasicBlockL* b : {&net->c1, &net->c2}) {
    const size_t ho = (size_t)b->hout * b->hout, co = b->c2.cout;
    RNN_TRY(dalloc(net, &b->y1, n * co * ho));
    RNN_TRY(dalloc(net, &b->h1, n * co * ho));
    RNN_TRY(dalloc(net, &b->y2, n * co * ho));
    RNN_TRY(dalloc(net, &b->out, n * co * ho));
    if (b->down) RNN_TRY(dalloc(net, &b->yd, n * co * ho));
    RNN_TRY(alloc_bn(net, b->b1));
    RNN_TRY(alloc_bn(net, b->b2));
    if (b->down) RNN_TRY(alloc_bn(net, b->bd));
  }
  RNN_TRY(dalloc(net, &net->mcv, n * 2 * d * r2));
  RNN_TRY(dalloc(net, &net->memt, n * 2 * d * r2));
  RNN_TRY(dalloc(net, &net->mem, n * 2 * d * r2));
  RNN_TRY(dalloc(net, &net->memln.xhat, n * 2 * d * r2));
  RNN_TRY(dalloc(net, &net->memln.invstd, n * r2));
  RNN_TRY(dalloc(net, &net->tcv, n * d * t3));
  RNN_TRY(dalloc(net, &net->tbn, n * d * t3));
  RNN_TRY(alloc_bn(net, net->tok_bn));
  RNN_TRY(dalloc(net, &net->z0, n * d * t3));
  for (size_t i = 0; i < net->blocks3.size(); i++) RNN_TRY(alloc_block(net, net->blocks3[i], n, i == 0));
  for (size_t i = 0; i < net->blocks4.size(); i++) RNN_TRY(alloc_block(net, net->blocks4[i], n, i == 0));
  RNN_TRY(dalloc(net, &net->f2, (size_t)n * d));
  RNN_TRY(dalloc(net, &net->pool2.w, n * t3));
  RNN_TRY(dalloc(net, &net->e2l, (size_t)n * net->nf));
  RNN_TRY(dalloc(net, &net->h2v, (size_t)n * d4));
  RNN_TRY(dalloc(net, &net->zm, n * t3 * d));
  RNN_TRY(dalloc(net, &net->zn, n * t3 * d));
  RNN_TRY(dalloc(net, &net->mergeln.xhat, n * t3 * d));
  RNN_TRY(dalloc(net, &net->mergeln.invstd, n * t4));
  RNN_TRY(dalloc(net, &net->z4, n * t4 * d4));
  RNN_TRY(dalloc(net, &net->zf, n * t4 * d4));
  RNN_TRY(dalloc(net, &net->headln.xhat, n * t4 * d4));
  RNN_TRY(dalloc(net, &net->headln.invstd, n * t4));
  RNN_TRY(dalloc(net, &net->feat, (size_t)n * d4));
  RNN_TRY(dalloc(net, &net->pool.w, n * t4));
  RNN_TRY(dalloc(net, &net->zc, (size_t)n * net->nc));
  RNN_TRY(dalloc(net, &net->zl, (size_t)n * net->nf));
  RNN_TRY(dalloc(net, &net->gp, (size_t)n * cm));
  RNN_TRY(dalloc(net, &net->e1l, (size_t)n * net->nf));
  RNN_TRY(dalloc(net, &net->h1v, (size_t)n * d4));
  // backward
  const size_t nfmax = std::max(net->nf, net->nc);
  RNN_TRY(dalloc(net, &net->g_logits, (size_t)n * net->nf));
  RNN_TRY(dalloc(net, &net->g_coarse, (size_t)n * net->nc));
  RNN_TRY(dalloc(net, &net->g_e1, (size_t)n * net->nf));
  RNN_TRY(dalloc(net, &net->g_e2, (size_t)n * net->nf));
  RNN_TRY(dalloc(net, &net->g_h1, (size_t)n * d4));
  RNN_TRY(dalloc(net, &net->g_h2, (size_t)n * d4));
  const size_t small = (size_t)n * std::max<size_t>({(size_t)d4, (size_t)d, (size_t)cm, nfmax});
  RNN_TRY(dalloc(net, &net->b_small1, small));
  RNN_TRY(dalloc(net, &net->b_small2, small));
  RNN_TRY(dalloc(net, &net->b_small3, small));
  RNN_TRY(dalloc(net, &net->b_small4, small));
  RNN_TRY(dalloc(net, &net->b_rows4, n * t4 * d4));
  RNN_TRY(dalloc(net, &net->b_rows4b, n * t4 * d4));
  RNN_TRY(dalloc(net, &net->b_merge, n * t3 * d));
  RNN_TRY(dalloc(net, &net->b_merge2, n * t3 * d));
  RNN_TRY(dalloc(net, &net->b_rows3, n * t3 * d));
  RNN_TRY(dalloc(net, &net->dmem, n * 2 * d * r2));
  RNN_TRY(dalloc(net, &net->dmem2, n * 2 * d * r2));
  // per-block backward scratch, sized for the widest stage
  size_t rc = std::max(n * t3 * d, n * t4 * d4);
  size_t hmax = 0;
  for (auto* v : {&net->blocks3, &net->blocks4})
    for (auto& b : *v) hmax = std::max(hmax, (size_t)n * b.th * b.th * 2 * b.mlp.h);
  RNN_TRY(dalloc(net, &net->bs1, rc));
  RNN_TRY(dalloc(net, &net->bs2, rc));
  RNN_TRY(dalloc(net, &net->bs3, rc));
  RNN_TRY(dalloc(net, &net->bs4, rc));
  RNN_TRY(dalloc(net, &net->bs_wide, hmax));
  RNN_TRY(dalloc(net, &net->bs_wide2, hmax));
  RNN_TRY(dalloc(net, &net->bs_qkv, 3 * rc));
  {
    size_t amax = 0;  // ceil(rows / 128) * 128 rows of c columns, hi and lo
    for (auto* v : {&net->blocks3, &net->blocks4})
      for (auto& b : *v) amax = std::max(amax, ((size_t)n * b.th * b.th + 127) / 128 * 128 * b.c * 2);
    RNN_TRY(dalloc(net, &net->aimg, amax));
  }
  const size_t imgmax = std::max((size_t)n * w * img, (size_t)n * cm * r2);
  RNN_TRY(dalloc(net, &net->b_img_a, imgmax));
  RNN_TRY(dalloc(net, &net->b_img_b, imgmax));
  RNN_TRY(dalloc(net, &net->b_img_c, imgmax));
  RNN_TRY(dalloc(net, &net->b_img_d, imgmax));
  RNN_TRY(dalloc(net, &net->b_c2, (size_t)n * cm * r2));
  RNN_TRY(dalloc(net, &net->b_c2b, (size_t)n * cm * r2));
  RNN_TRY(dalloc(net, &net->losses, 8));
  float* ci = nullptr;
  RNN_TRY(dalloc(net, &ci, 4));
  net->correct = reinterpret_cast<int*>(ci);
  RNN_TRY(dalloc(net, &net->clip_norm, 1));
  net->cap = n;
  return RNN_OK;
}

// ---- layer steps

static int lin_fwd(rnn_rustvit* net, LinL& l, const float* x, int rows, float* y) {
  l.x = x;
  l.rows = rows;
  return rnn_linear_fwd_dev(net->ctx, x, rows, l.fin, l.fout, P(net, l.w), Popt(net, l.b), y);
}
static int lin_bwd(rnn_rustvit* net, LinL& l, const float* dy, float* dx) {
  return rnn_linear_bwd_dev(net->ctx, l.x, dy, l.rows, l.fin, l.fout, P(net, l.w), Gd(net, l.w), Gopt(net, l.b),
                            dx);
}
// dx += the Linear input gradient (the GEMM epilogue adds it)
static int lin_bwd_acc(rnn_rustvit* net, LinL& l, const float* dy, float* dx) {
  return linear_bwd(net->ctx, l.x, dy, l.rows, l.fin, l.fout, P(net, l.w), Gd(net, l.w), Gopt(net, l.b), dx, true);
}
static int ln_fwd(rnn_rustvit* net, LNL& l, const float* x, int rows, float* y) {
  l.rows = rows;
  return rnn_layernorm_fwd_dev(net->ctx, x, rows, l.c, P(net, l.g), P(net, l.b), 1e-5f, y, l.xhat, l.invstd);
}
// The fused forms (csrc/fused.cu) where the shapes allow them: LayerNorm of
// x (+ r1) (+ r2) writing the packed A image, and the GEMMs reading it.
static bool ln_fusable(int c) { return c % 128 == 0 && c <= 512; }
static int ln_res_fwd(rnn_rustvit* net, LNL& l, const float* x, const float* r1, const float* r2, int rows,
                      float* sum_out, float* y, float* img) {
  l.rows = rows;
  return rnn_layernorm_res_fwd_dev(net->ctx, x, r1, r2, rows, l.c, P(net, l.g), P(net, l.b), 1e-5f, sum_out, y,
                                   l.xhat, l.invstd, img);
}
static int lin_fwd_img(rnn_rustvit* net, LinL& l, const float* img, const float* x, int rows, float* y) {
  l.x = x;  // the backward's dW reads the row-major input
  l.rows = rows;
  return rnn_linear_fwd_packed_dev(net->ctx, img, rows, l.fin, l.fout, P(net, l.w), Popt(net, l.b), y);
}
static int ln_bwd(rnn_rustvit* net, LNL& l, const float* dy, float* dx) {
  return rnn_layernorm_bwd_dev(net->ctx, dy, l.xhat, l.invstd, l.rows, l.c, P(net, l.g), dx, Gd(net, l.g),
                               Gd(net, l.b));
}
// dx += the LayerNorm input gradient (a residual join)
static int ln_bwd_acc(rnn_rustvit* net, LNL& l, const float* dy, float* dx) {
  return layernorm_bwd(net->ctx, dy, l.xhat, l.invstd, l.rows, l.c, P(net, l.g), dx, Gd(net, l.g), Gd(net, l.b),
                       true);
}
static int ls_fwd(rnn_rustvit* net, LSL& l, const float* x, int rows, float* y) {
  l.x = x;
  return rnn_layerscale_fwd_dev(net->ctx, x, rows, l.c, P(net, l.l), y);
}
static int ls_bwd(rnn_rustvit* net, LSL& l, const float* dy, int rows, float* dx) {
  return rnn_layerscale_bwd_dev(net->ctx, dy, l.x, rows, l.c, P(net, l.l), Gd(net, l.l), dx);
}
static int dp_fwd(rnn_rustvit* net, DPL& d, float* x, int n, size_t per, bool train, uint64_t seed) {
  d.active = train && d.p > 0.0f;
  if (!d.active) return RNN_OK;
  return rnn_droppath_fwd_dev(net->ctx, x, n, per, d.p, seed, d.mask);
}
static int dp_bwd(rnn_rustvit* net, DPL& d, float* dy, int n, size_t per) {
  if (!d.active) return RNN_OK;
  return rnn_droppath_bwd_dev(net->ctx, dy, n, per, d.mask);
}
static int copy(rnn_rustvit* net, float* dst, const float* src, size_t nfl) {
  RNN_CUDA(cudaMemcpyAsync(dst, src, nfl * sizeof(float), cudaMemcpyDeviceToDevice, net->ctx->stream));
  return RNN_OK;
}
static int zero(rnn_rustvit* net, float* dst, size_t nfl) {
  RNN_CUDA(cudaMemsetAsync(dst, 0, nfl * sizeof(float), net->ctx->stream));
  return RNN_OK;
}

static int bn_fwd(rnn_rustvit* net, BNL& b, const float* y, int n, int hw, bool train, bool relu, float* out) {
  if (train)
    return rnn_batchnorm_fwd_dev(net->ctx, y, n, b.c, hw, P(net, b.g), P(net, b.b), net->B + b.rm, net->B + b.rv,
                                 0.1f, 1e-5f, relu ? 1 : 0, b.mean, b.invstd, out);
  return rnn_batchnorm_eval_dev(net->ctx, y, n, b.c, hw, P(net, b.g), P(net, b.b), net->B + b.rm, net->B + b.rv,
                                1e-5f, relu ? 1 : 0, out);
}
static int bn_bwd(rnn_rustvit* net, BNL& b, const float* dy, const float* y, int n, int hw, const float* relu_out,
                  float* dx) {
  return rnn_batchnorm_bwd_dev(net->ctx, dy, y, n, b.c, hw, P(net, b.g), b.mean, b.invstd, relu_out, dx,
                               Gd(net, b.g), Gd(net, b.b));
}
static int conv_fwd(rnn_rustvit* net, ConvL& c, const float* x, int n, int h, float* y) {
  return rnn_conv2d_fwd_dev(net->ctx, x, n, c.cin, h, h, P(net, c.w), c.cout, c.k, c.stride, c.pad, y, 0);
}
// dW += ; dx written (acc=0) or accumulated (acc=1); dx may be null
static int conv_bwd(rnn_rustvit* net, ConvL& c, const float* x, const float* dy, int n, int h, float* dx,
                    bool acc) {
  RNN_TRY(rnn_conv2d_wgrad_dev(net->ctx, x, dy, n, c.cin, h, h, c.cout, c.k, c.stride, c.pad, Gd(net, c.w)));
  if (!dx) return RNN_OK;
  return rnn_conv2d_dgrad_dev(net->ctx, dy, n, c.cin, h, h, P(net, c.w), c.cout, c.k, c.stride, c.pad, dx,
                              acc ? 1 : 0);
}

// BasicBlock (model.rs:39-72)
static int bb_fwd(rnn_rustvit* net, BasicBlockL& b, const float* x, int n, bool train) {
  const int ho = b.hout;
  b.x = x;
  RNN_TRY(conv_fwd(net, b.c1, x, n, b.hin, b.y1));
  RNN_TRY(bn_fwd(net, b.b1, b.y1, n, ho * ho, train, true, b.h1));
  RNN_TRY(conv_fwd(net, b.c2, b.h1, n, ho, b.y2));
  RNN_TRY(bn_fwd(net, b.b2, b.y2, n, ho * ho, train, false, b.out));
  const size_t len = (size_t)n * b.c2.cout * ho * ho;
  if (b.down) {
    float* s = net->b_img_c;
    RNN_TRY(conv_fwd(net, b.cd, x, n, b.hin, b.yd));
    RNN_TRY(bn_fwd(net, b.bd, b.yd, n, ho * ho, train, false, s));
    return rnn_add_relu_dev(net->ctx, b.out, s, len);
  }
  return rnn_add_relu_dev(net->ctx, b.out, x, len);
}

// d: gradient wrt the block output (overwritten); writes dx [n, cin, hin, hin]
static int bb_bwd(rnn_rustvit* net, BasicBlockL& b, float* d, int n, float* dx) {
  const int ho = b.hout;
  const size_t len = (size_t)n * b.c2.cout * ho * ho;
  RNN_TRY(rnn_relu_back_dev(net->ctx, d, b.out, len));
  float* t = net->b_img_a;
  float* t2 = net->b_img_b;
  RNN_TRY(bn_bwd(net, b.b2, d, b.y2, n, ho * ho, nullptr, t));   // dy2
  RNN_TRY(conv_bwd(net, b.c2, b.h1, t, n, ho, t2, false));       // dh1
  RNN_TRY(bn_bwd(net, b.b1, t2, b.y1, n, ho * ho, b.h1, t));     // relu_back fused, dy1
  RNN_TRY(conv_bwd(net, b.c1, b.x, t, n, b.hin, dx, false));
  if (b.down) {
    RNN_TRY(bn_bwd(net, b.bd, d, b.yd, n, ho * ho, nullptr, t));
    RNN_TRY(conv_bwd(net, b.cd, b.x, t, n, b.hin, dx, true));
    return RNN_OK;
  }
  return rnn_add_dev(net->ctx, dx, d, len);
}

// ---- transformer block (vit.rs:141-232)

static int block_fwd(rnn_rustvit* net, Block& b, const float* x, const float* mem, int n, bool train,
                     uint64_t seed) {
  const int c = b.c, t = b.th * b.th, rows = n * t;
  const size_t rc = (size_t)rows * c, per = (size_t)t * c;
  const bool fuse = ln_fusable(c);
  if (fuse) RNN_TRY(ln_res_fwd(net, b.n1, x, nullptr, nullptr, rows, nullptr, b.hb, net->aimg));
  else RNN_TRY(ln_fwd(net, b.n1, x, rows, b.hb));
  // self-attention (attn.rs:387-413)
  SelfAttnL& A = b.attn;
  if (fuse) RNN_TRY(lin_fwd_img(net, A.qkv, net->aimg, b.hb, rows, A.ab));
  else RNN_TRY(lin_fwd(net, A.qkv, b.hb, rows, A.ab));
  RNN_TRY(rnn_attn_fwd_dev(net->ctx, n, A.h, A.dh, A.th, A.th, A.th, A.th, 1, A.ab, 3 * c, 0, A.ab, 3 * c, c,
                           2 * c, P(net, A.tau), P(net, A.rel), A.p, A.o));
  RNN_TRY(lin_fwd(net, A.proj, A.o, rows, b.a));
  // depthwise branch, a += gamma * d
  b.dw.x = b.hb;
  RNN_TRY(rnn_dwconv3_fwd_dev(net->ctx, b.hb, n, b.th, b.th, c, P(net, b.dw.w), P(net, b.dw.b), b.dwo));
  RNN_TRY(rnn_layerscale_fwd_dev(net->ctx, b.dwo, rows, c, P(net, b.gamma), b.tmp));
  RNN_TRY(rnn_add_dev(net->ctx, b.a, b.tmp, rc));
  RNN_TRY(ls_fwd(net, b.ls1, b.a, rows, b.s1));
  RNN_TRY(dp_fwd(net, b.dp1, b.s1, n, per, train, seed ^ b.idx));
  if (!fuse) {
    RNN_TRY(copy(net, b.y, x, rc));
    RNN_TRY(rnn_add_dev(net->ctx, b.y, b.s1, rc));
  }
  if (b.has_cross) {
    CrossAttnL& X = b.cross;
    // the image still holds LN1's output (no LayerNorm ran since)
    if (fuse) RNN_TRY(lin_fwd_img(net, X.wq, net->aimg, b.hb, rows, X.q));
    else RNN_TRY(lin_fwd(net, X.wq, b.hb, rows, X.q));
    RNN_TRY(rnn_attn_fwd_dev(net->ctx, n, X.h, X.dh, X.th, X.th, X.mh, X.mh, 0, X.q, c, 0, mem, 2 * c, 0, c,
                             P(net, X.tau), P(net, X.rel), X.p, X.o));
    RNN_TRY(lin_fwd(net, X.proj, X.o, rows, b.cm));
    RNN_TRY(ls_fwd(net, b.lsm, b.cm, rows, b.s2));
    RNN_TRY(dp_fwd(net, b.dp2, b.s2, n, per, train, seed ^ b.idx ^ 0x5151ULL));
    if (!fuse) RNN_TRY(rnn_add_dev(net->ctx, b.y, b.s2, rc));
  }
  // y = x + s1 (+ s2) joined into the LayerNorm that reads it
  if (fuse) RNN_TRY(ln_res_fwd(net, b.n2, x, b.s1, b.has_cross ? b.s2 : nullptr, rows, b.y, b.h2, net->aimg));
  else RNN_TRY(ln_fwd(net, b.n2, b.y, rows, b.h2));
  // SwiGLU (norm.rs:250-268); fused: the gate in the first GEMM's epilogue
  if (fuse && b.mlp.h % 16 == 0) {
    LinL& g = b.mlp.wg;
    g.x = b.h2;
    g.rows = rows;
    RNN_TRY(rnn_swiglu_fwd_dev(net->ctx, b.h2, net->aimg, rows, c, b.mlp.h, P(net, g.w), P(net, g.b), b.mlp.ab,
                               b.mlp.u));
  } else {
    RNN_TRY(lin_fwd(net, b.mlp.wg, b.h2, rows, b.mlp.ab));
    RNN_TRY(rnn_swiglu_act_fwd_dev(net->ctx, b.mlp.ab, rows, b.mlp.h, b.mlp.u));
  }
  RNN_TRY(lin_fwd(net, b.mlp.wd, b.mlp.u, rows, b.m));
  RNN_TRY(ls_fwd(net, b.ls2, b.m, rows, b.s3));
  RNN_TRY(dp_fwd(net, b.dp3, b.s3, n, per, train, seed ^ b.idx ^ 0xA2A2ULL));
  return rnn_add_dev(net->ctx, b.y, b.s3, rc);  // block output lives in b.y
}

// dz: gradient wrt the block output; on return holds the gradient wrt the
// block input.  dmem (nullable) accumulates the memory gradient.
static int block_bwd(rnn_rustvit* net, Block& b, float* dz, const float* mem, float* dmem, int n) {
  const int c = b.c, t = b.th * b.th, rows = n * t;
  const size_t rc = (size_t)rows * c, per = (size_t)t * c;
  float *t1 = net->bs1, *t2 = net->bs2, *dh = net->bs3, *t4 = net->bs4;
  // MLP branch: dm = ls2.backward(dp3.backward(dz))
  RNN_TRY(copy(net, t1, dz, rc));
  RNN_TRY(dp_bwd(net, b.dp3, t1, n, per));
  RNN_TRY(ls_bwd(net, b.ls2, t1, rows, t2));  // t2 = dm
  RNN_TRY(lin_bwd(net, b.mlp.wd, t2, net->bs_wide2));  // du [rows, h]
  RNN_TRY(rnn_swiglu_act_bwd_dev(net->ctx, net->bs_wide2, b.mlp.ab, rows, b.mlp.h, net->bs_wide));  // dab
  RNN_TRY(lin_bwd(net, b.mlp.wg, net->bs_wide, t1));  // t1 = dh2
  RNN_TRY(ln_bwd_acc(net, b.n2, t1, dz));  // dz now dy
  // dh accumulates the three branches that read LN1's output
  bool dh_set = false;
  if (b.has_cross) {
    CrossAttnL& X = b.cross;
    RNN_TRY(copy(net, t1, dz, rc));
    RNN_TRY(dp_bwd(net, b.dp2, t1, n, per));
    RNN_TRY(ls_bwd(net, b.lsm, t1, rows, t2));       // dc
    RNN_TRY(lin_bwd(net, X.proj, t2, t1));           // dobuf
    RNN_TRY(zero(net, t4, rc));                      // dq
    RNN_TRY(rnn_attn_bwd_dev(net->ctx, n, X.h, X.dh, X.th, X.th, X.mh, X.mh, X.q, c, 0, mem, 2 * c, 0, c,
                             P(net, X.tau), X.p, t1, t4, dmem, Gd(net, X.tau), Gd(net, X.rel)));
    RNN_TRY(lin_bwd(net, X.wq, t4, dh));
    dh_set = true;
  }
  RNN_TRY(copy(net, t1, dz, rc));
  RNN_TRY(dp_bwd(net, b.dp1, t1, n, per));
  RNN_TRY(ls_bwd(net, b.ls1, t1, rows, t2));  // t2 = da
  // dgamma += sum(da * dwo); t4 = ddw = gamma * da
  RNN_TRY(rnn_layerscale_bwd_dev(net->ctx, t2, b.dwo, rows, c, P(net, b.gamma), Gd(net, b.gamma), t4));
  // self-attention backward (attn.rs:415-440)
  SelfAttnL& A = b.attn;
  RNN_TRY(lin_bwd(net, A.proj, t2, t1));  // dobuf
  // dq lands in columns [0, c) of the qkv gradient, dk / dv in [c, 3c):
  // disjoint, so one zeroed buffer takes both
  RNN_TRY(zero(net, net->bs_qkv, rc * 3));
  RNN_TRY(rnn_attn_bwd_dev(net->ctx, n, A.h, A.dh, A.th, A.th, A.th, A.th, A.ab, 3 * c, 0, A.ab, 3 * c, c, 2 * c,
                           P(net, A.tau), A.p, t1, net->bs_qkv, net->bs_qkv, Gd(net, A.tau), Gd(net, A.rel)));
  if (dh_set) {
    RNN_TRY(lin_bwd_acc(net, A.qkv, net->bs_qkv, dh));
  } else {
    RNN_TRY(lin_bwd(net, A.qkv, net->bs_qkv, dh));
  }
  // depthwise branch
  RNN_TRY(dwconv3_bwd(net->ctx, t4, b.dw.x, n, b.th, b.th, c, P(net, b.dw.w), Gd(net, b.dw.w), Gd(net, b.dw.b),
                      dh, true));
  return ln_bwd_acc(net, b.n1, dh, dz);
}

// ---- whole network (vit.rs:511-685)

struct Outs {
  float *logits, *coarse, *e1, *e2, *h1, *h2, *feat;
};

static int forward(rnn_rustvit* net, const float* x, int n, bool train, uint64_t seed) {
  RNN_TRY(ensure_acts(net, n));
  net->n = n;
  const Cfg& c = net->cfg;
  const int img = c.img, th = net->th, mh = net->mh, d = c.dim, d4 = c.dim4;
  const int th4 = th / 2;
  // the stem's weight gradient needs the batch in the backward (Conv2d keeps
  // its input, nn.rs:171): keep a copy so the caller may release x
  RNN_TRY(copy(net, net->xkeep, x, (size_t)n * 3 * img * img));
  net->x_in = net->xkeep;
  RNN_TRY(conv_fwd(net, net->stem, net->x_in, n, img, net->y0));
  RNN_TRY(bn_fwd(net, net->stem_bn, net->y0, n, img * img, train, true, net->stem_out));
  RNN_TRY(bb_fwd(net, net->c1, net->stem_out, n, train));
  RNN_TRY(bb_fwd(net, net->c2, net->c1.out, n, train));
  const float* c2o = net->c2.out;
  // memory: 1x1 conv -> tokens -> LayerNorm (K | V for the reader blocks)
  RNN_TRY(conv_fwd(net, net->memconv, c2o, n, mh, net->mcv));
  RNN_TRY(rnn_tok_layout_dev(net->ctx, net->mcv, n, 2 * d, mh * mh, net->memt, 0));
  RNN_TRY(ln_fwd(net, net->memln, net->memt, n * mh * mh, net->mem));
  // 8x8 tokens
  RNN_TRY(conv_fwd(net, net->tokconv, c2o, n, mh, net->tcv));
  RNN_TRY(bn_fwd(net, net->tok_bn, net->tcv, n, th * th, train, false, net->tbn));
  RNN_TRY(rnn_tok_layout_dev(net->ctx, net->tbn, n, d, th * th, net->z0, 0));
  const float* z = net->z0;
  for (auto& b : net->blocks3) {
    RNN_TRY(block_fwd(net, b, z, net->mem, n, train, seed));
    z = b.y;
  }
  const bool exits = net->use_exits && train;
  if (exits) {
    net->pool2.x = z;
    net->pool2.t = th * th;
    RNN_TRY(rnn_seqpool_fwd_dev(net->ctx, z, n, th * th, d, P(net, net->pool2.p), net->f2, net->pool2.w));
    RNN_TRY(lin_fwd(net, net->e2_fc, net->f2, n, net->e2l));
    RNN_TRY(lin_fwd(net, net->e2_hint, net->f2, n, net->h2v));
  }
  RNN_TRY(rnn_token_merge_dev(net->ctx, z, n, th, d, net->zm, 0));
  RNN_TRY(ln_fwd(net, net->mergeln, net->zm, n * th4 * th4, net->zn));
  RNN_TRY(lin_fwd(net, net->merge, net->zn, n * th4 * th4, net->z4));
  const float* z4 = net->z4;
  for (auto& b : net->blocks4) {
    RNN_TRY(block_fwd(net, b, z4, nullptr, n, train, seed));
    z4 = b.y;
  }
  RNN_TRY(ln_fwd(net, net->headln, z4, n * th4 * th4, net->zf));
  net->pool.x = net->zf;
  net->pool.t = th4 * th4;
  RNN_TRY(rnn_seqpool_fwd_dev(net->ctx, net->zf, n, th4 * th4, d4, P(net, net->pool.p), net->feat, net->pool.w));
  // TaxoHead (vit.rs:263-295)
  RNN_TRY(lin_fwd(net, net->head_coarse, net->feat, n, net->zc));
  RNN_TRY(lin_fwd(net, net->head_resid, net->feat, n, net->zl));
  RNN_TRY(rnn_taxo_combine_fwd_dev(net->ctx, net->zl, net->zc, n, net->nf, net->nc, net->parent));
  if (exits) {
    RNN_TRY(rnn_gap_fwd_dev(net->ctx, c2o, n * c.cmid, mh * mh, net->gp));
    RNN_TRY(lin_fwd(net, net->e1_fc, net->gp, n, net->e1l));
    RNN_TRY(lin_fwd(net, net->e1_hint, net->gp, n, net->h1v));
  }
  return RNN_OK;
}

// grads: logits/coarse required; e1/e2/h1/h2 when exits ran; hfinal nullable
static int backward(rnn_rustvit* net, const float* dlogits, const float* dcoarse, const float* de1,
                    const float* de2, const float* dh1, const float* dh2, const float* dhfinal) {
  const int n = net->n;
  const Cfg& c = net->cfg;
  const int th = net->th, mh = net->mh, d = c.dim, d4 = c.dim4, cm = c.cmid, th4 = th / 2;
  const size_t r3 = (size_t)n * th * th;
  // TaxoHead backward (vit.rs:297-310)
  float *dc = net->b_small1, *df = net->b_small2, *dfc = net->b_small3;
  RNN_TRY(rnn_taxo_combine_bwd_dev(net->ctx, dlogits, dcoarse, n, net->nf, net->nc, net->parent, dc));
  RNN_TRY(lin_bwd(net, net->head_resid, dlogits, df));
  RNN_TRY(lin_bwd(net, net->head_coarse, dc, dfc));
  RNN_TRY(rnn_add_dev(net->ctx, df, dfc, (size_t)n * d4));
  if (dhfinal) RNN_TRY(rnn_add_dev(net->ctx, df, dhfinal, (size_t)n * d4));
  float *dz4 = net->b_rows4, *tmp4 = net->b_rows4b;
  RNN_TRY(rnn_seqpool_bwd_dev(net->ctx, df, net->pool.x, net->pool.w, n, th4 * th4, d4, P(net, net->pool.p),
                              Gd(net, net->pool.p), tmp4));
  RNN_TRY(ln_bwd(net, net->headln, tmp4, dz4));
  for (int i = (int)net->blocks4.size() - 1; i >= 0; i--) RNN_TRY(block_bwd(net, net->blocks4[i], dz4, nullptr,
                                                                           nullptr, n));
  RNN_TRY(lin_bwd(net, net->merge, dz4, net->b_merge));
  RNN_TRY(ln_bwd(net, net->mergeln, net->b_merge, net->b_merge2));
  float* dz = net->b_rows3;
  RNN_TRY(rnn_token_merge_dev(net->ctx, net->b_merge2, n, th, d, dz, 1));
  const bool exits = net->use_exits && de2;
  if (exits) {
    float *df2 = net->b_small1, *dfh = net->b_small3;
    RNN_TRY(lin_bwd(net, net->e2_fc, de2, df2));
    RNN_TRY(lin_bwd(net, net->e2_hint, dh2, dfh));
    RNN_TRY(rnn_add_dev(net->ctx, df2, dfh, (size_t)n * d));
    RNN_TRY(rnn_seqpool_bwd_dev(net->ctx, df2, net->pool2.x, net->pool2.w, n, th * th, d, P(net, net->pool2.p),
                                Gd(net, net->pool2.p), net->b_merge));
    RNN_TRY(rnn_add_dev(net->ctx, dz, net->b_merge, r3 * d));
  }
  const size_t memn = (size_t)n * mh * mh * 2 * d;
  RNN_TRY(zero(net, net->dmem, memn));
  for (int i = (int)net->blocks3.size() - 1; i >= 0; i--)
    RNN_TRY(block_bwd(net, net->blocks3[i], dz, net->mem, net->dmem, n));
  // token path: to NCHW -> tok_bn -> tokconv (dx into dc2)
  float* dc2 = net->b_c2;
  RNN_TRY(rnn_tok_layout_dev(net->ctx, dz, n, d, th * th, net->b_merge, 1));
  RNN_TRY(bn_bwd(net, net->tok_bn, net->b_merge, net->tcv, n, th * th, nullptr, net->b_merge2));
  RNN_TRY(conv_bwd(net, net->tokconv, net->c2.out, net->b_merge2, n, mh, dc2, false));
  // memory path: LayerNorm -> to NCHW -> memconv (dx accumulated into dc2)
  RNN_TRY(ln_bwd(net, net->memln, net->dmem, net->dmem2));
  RNN_TRY(rnn_tok_layout_dev(net->ctx, net->dmem2, n, 2 * d, mh * mh, net->dmem, 1));
  RNN_TRY(conv_bwd(net, net->memconv, net->c2.out, net->dmem, n, mh, dc2, true));
  if (net->use_exits && de1) {
    float *dg = net->b_small1, *dgh = net->b_small3;
    RNN_TRY(lin_bwd(net, net->e1_fc, de1, dg));
    RNN_TRY(lin_bwd(net, net->e1_hint, dh1, dgh));
    RNN_TRY(rnn_add_dev(net->ctx, dg, dgh, (size_t)n * cm));
    RNN_TRY(rnn_gap_bwd_dev(net->ctx, dg, n * cm, mh * mh, net->b_c2b));
    RNN_TRY(rnn_add_dev(net->ctx, dc2, net->b_c2b, (size_t)n * cm * mh * mh));
  }
  // convolutional stem: C2, C1 (model.rs:57-72), ReLU mask, stem BN, stem dW
  float *d_c1out = net->b_img_c, *d_stem = net->b_img_d;
  RNN_TRY(bb_bwd(net, net->c2, dc2, n, d_c1out));
  RNN_TRY(bb_bwd(net, net->c1, d_c1out, n, d_stem));
  const int img = c.img;
  RNN_TRY(bn_bwd(net, net->stem_bn, d_stem, net->y0, n, img * img, net->stem_out, net->b_img_a));
  RNN_TRY(conv_bwd(net, net->stem, net->x_in, net->b_img_a, n, img, nullptr, false));
  return RNN_OK;
}

}  // namespace vit
}  // namespace rnn

namespace rnn {
namespace vit {

// ---- construction (vit.rs:389-509: blocks first, then the struct literal)

static int build(rnn_rustvit* net, uint64_t seed) {
  Rng r(seed);
  Registry& R = net->R;
  const Cfg& c = net->cfg;
  const int w = c.width, cm = c.cmid, d = c.dim, d4 = c.dim4;
  net->mh = c.img / 2;
  net->th = c.img / 4;
  const int th4 = net->th / 2;
  const int depth = c.depth3 + c.depth4;
  const float den = (float)(std::max(depth, 2) - 1);
  net->blocks3.resize(c.depth3);
  for (int i = 0; i < c.depth3; i++) {
    const float dp = c.droppath * (float)i / den;
    const bool reader = std::find(c.mem_at.begin(), c.mem_at.end(), i) != c.mem_at.end();
    net->blocks3[i].init(R, r, d, c.heads, net->th, reader ? net->mh : 0, depth, dp, (uint64_t)i + 1, 1e-4f);
  }
  net->blocks4.resize(c.depth4);
  for (int i = 0; i < c.depth4; i++) {
    const float dp = c.droppath * (float)(c.depth3 + i) / den;
    net->blocks4[i].init(R, r, d4, c.heads4, th4, 0, depth, dp, (uint64_t)(c.depth3 + i) + 1, 1e-4f);
  }
  net->stem.init(R, r, 3, w, 3, 1, 1);
  net->stem_bn.init(R, w);
  net->c1.init(R, r, w, w, 1, c.img);
  net->c2.init(R, r, w, cm, 2, c.img);
  net->memconv.init(R, r, cm, 2 * d, 1, 1, 0);
  net->memln.init(R, 2 * d);
  net->tokconv.init(R, r, cm, d, 3, 2, 1);
  net->tok_bn.init(R, d);
  net->mergeln.init(R, 4 * d);
  net->merge.init(R, r, 4 * d, d4, true, 0.02f);
  net->headln.init(R, d4);
  net->pool.init(R, r, d4);
  net->head_coarse.init(R, r, d4, net->nc, true, 0.02f);
  net->head_resid.init(R, r, d4, net->nf, true, 0.02f);
  net->e1_fc.init(R, r, cm, net->nf, true, 0.02f);
  net->e1_hint.init(R, r, cm, d4, false, 0.02f);
  net->pool2.init(R, r, d);
  net->e2_fc.init(R, r, d, net->nf, true, 0.02f);
  net->e2_hint.init(R, r, d, d4, false, 0.02f);

  // flat parameter layout in for_each_param order
  net->order = param_order(net);
  net->off.assign(R.ps.size(), (size_t)-1);
  size_t off = 0;
  for (int id : net->order) {
    RNN_REQUIRE(net->off[id] == (size_t)-1, "rustvit: parameter %d listed twice", id);
    net->off[id] = off;
    off += R.ps[id].v.size();
  }
  for (size_t id = 0; id < R.ps.size(); id++)
    RNN_REQUIRE(net->off[id] != (size_t)-1, "rustvit: parameter %zu not in the parameter order", id);
  net->np = off;
  std::vector<float> hv(off);
  for (int id : net->order) std::copy(R.ps[id].v.begin(), R.ps[id].v.end(), hv.begin() + net->off[id]);
  for (float** p : {&net->V, &net->G, &net->M, &net->V2}) RNN_CUDA(cudaMalloc(p, off * sizeof(float)));
  RNN_CUDA(cudaMemcpy(net->V, hv.data(), off * sizeof(float), cudaMemcpyHostToDevice));
  for (float* p : {net->G, net->M, net->V2}) RNN_CUDA(cudaMemset(p, 0, off * sizeof(float)));

  // running statistics in for_each_buffer order (vit.rs:721-728)
  std::vector<BNL*> bns = {&net->stem_bn, &net->c1.b1, &net->c1.b2};
  if (net->c1.down) bns.push_back(&net->c1.bd);
  bns.push_back(&net->c2.b1);
  bns.push_back(&net->c2.b2);
  if (net->c2.down) bns.push_back(&net->c2.bd);
  bns.push_back(&net->tok_bn);
  std::vector<float> hb;
  for (BNL* b : bns) {
    b->rm = hb.size();
    hb.insert(hb.end(), b->c, 0.0f);
    b->rv = hb.size();
    hb.insert(hb.end(), b->c, 1.0f);
  }
  net->nb = hb.size();
  net->n_buf_tensors = 2 * (int)bns.size();
  RNN_CUDA(cudaMalloc(&net->B, hb.size() * sizeof(float)));
  RNN_CUDA(cudaMemcpy(net->B, hb.data(), hb.size() * sizeof(float), cudaMemcpyHostToDevice));
  return RNN_OK;
}

// ---- loss, optimiser, step (train.rs:70-118, optim.rs:177-287, train.rs:346-387)

struct LossCfg {
  float coarse_w = 0.4f, w1 = 0.3f, w2 = 0.6f, alpha = 1.0f, temp = 3.0f, beta = 0.03f;  // cli.rs:98-112
};

static int build_loss(rnn_rustvit* net, const float* tf, const float* tc, const uint32_t* hard,
                      const uint32_t* hardc, int n) {
  const LossCfg L;
  rnn_ctx* ctx = net->ctx;
  const int nf = net->nf, nc = net->nc, d4 = net->cfg.dim4;
  RNN_TRY(rnn_ce_soft_dev(ctx, net->zl, tf, hard, n, nf, 1.0f, net->g_logits, net->losses + 0, net->correct + 0));
  RNN_TRY(rnn_ce_soft_dev(ctx, net->zc, tc, hardc, n, nc, L.coarse_w, net->g_coarse, net->losses + 1,
                          net->correct + 1));
  RNN_TRY(rnn_ce_soft_dev(ctx, net->e1l, tf, hard, n, nf, L.w1, net->g_e1, net->losses + 2, net->correct + 2));
  RNN_TRY(rnn_ce_soft_dev(ctx, net->e2l, tf, hard, n, nf, L.w2, net->g_e2, net->losses + 3, net->correct + 3));
  // the teacher (the final logits) is detached: nothing flows back into it
  RNN_TRY(rnn_kl_distill_dev(ctx, net->e1l, net->zl, n, nf, L.temp, L.alpha, net->g_e1, net->losses + 4));
  RNN_TRY(rnn_kl_distill_dev(ctx, net->e2l, net->zl, n, nf, L.temp, L.alpha, net->g_e2, net->losses + 5));
  RNN_TRY(zero(net, net->g_h1, (size_t)n * d4));
  RNN_TRY(zero(net, net->g_h2, (size_t)n * d4));
  RNN_TRY(rnn_hint_mse_dev(ctx, net->h1v, net->feat, n, d4, L.beta, net->g_h1, net->losses + 6));
  RNN_TRY(rnn_hint_mse_dev(ctx, net->h2v, net->feat, n, d4, L.beta, net->g_h2, net->losses + 7));
  return RNN_OK;
}

static bool is_muon(const HostParam& p) { return p.rows > 0 && std::min(p.rows, p.cols) > 1; }

// Optim::step_all (optim.rs:177-203): Muon per 2-D Linear weight, AdamW for
// the rest (consecutive parameters with the same decay flag in one call).
static int step_all(rnn_rustvit* net, float lr, float wd) {
  rnn_ctx* ctx = net->ctx;
  if (!net->opt_segs) {
    // The segments depend only on the network's layout: built on the first
    // step.  Muon matrices in for_each_param order; AdamW over runs of
    // consecutive non-Muon parameters with the same decay flag.
    std::vector<rnn::OptSeg> mu, ad;
    size_t run0 = 0, runlen = 0;
    int rundecay = -1;
    auto flush = [&]() {
      if (runlen) {
        ad.push_back({run0, runlen, 0.0f, rundecay});
        net->ad_max = std::max(net->ad_max, runlen);
      }
      runlen = 0;
    };
    for (int id : net->order) {
      const HostParam& p = net->R.ps[id];
      const size_t o = net->off[id], len = p.v.size();
      if (is_muon(p)) {
        flush();
        const size_t n = (size_t)p.rows * p.cols;
        mu.push_back({o, n, rnn::muon_scale(p.rows, p.cols), p.decay ? 1 : 0});
        net->mu_max = std::max(net->mu_max, n);
        continue;
      }
      const int dec = p.decay ? 1 : 0;
      if (runlen && (dec != rundecay || run0 + runlen != o)) flush();
      if (!runlen) {
        run0 = o;
        rundecay = dec;
      }
      runlen += len;
    }
    flush();
    std::vector<rnn::OptSeg> all(mu);
    all.insert(all.end(), ad.begin(), ad.end());
    if (!all.empty()) {
      RNN_CUDA(cudaMalloc(&net->opt_segs, all.size() * sizeof(rnn::OptSeg)));
      RNN_CUDA(cudaMemcpy(net->opt_segs, all.data(), all.size() * sizeof(rnn::OptSeg), cudaMemcpyHostToDevice));
    }
    net->n_mu = (int)mu.size();
    net->n_ad = (int)ad.size();
  }
  // Muon (optim.rs:183-196) per matrix: momentum, Newton-Schulz, update.
  // The matrices are independent, so the momentum of all of them runs
  // first (one launch), then one grouped Newton-Schulz over every gradient,
  // then the updates (one launch); AdamW (optim.rs:205-233) over its runs in
  // one launch.
  RNN_TRY(rnn::muon_momentum_segs(ctx, net->G, net->M, net->opt_segs, net->n_mu, net->mu_max, 0.95f));
  std::vector<float*> mg;
  std::vector<int> mr, mc;
  for (int id : net->order) {
    const HostParam& p = net->R.ps[id];
    if (!is_muon(p)) continue;
    mg.push_back(net->G + net->off[id]);
    mr.push_back(p.rows);
    mc.push_back(p.cols);
  }
  RNN_TRY(rnn::newton_schulz_grouped(ctx, (int)mg.size(), mg.data(), mr.data(), mc.data(), 3));
  RNN_TRY(rnn::muon_update_segs(ctx, net->V, net->G, net->opt_segs, net->n_mu, net->mu_max, lr, wd));
  RNN_TRY(rnn::adamw_segs(ctx, net->V, net->G, net->M, net->V2, net->opt_segs + net->n_mu, net->n_ad, net->ad_max, lr,
                          wd, 0.9f, 0.999f, 1e-8f, net->opt_t));
  net->opt_t++;
  return RNN_OK;
}

// Ema::update (optim.rs:270-287)
static int ema_update(rnn_rustvit* net, float decay) {
  net->ema_t++;
  if (!net->E) RNN_CUDA(cudaMalloc(&net->E, net->np * sizeof(float)));
  if (!net->ema_ready) {
    net->ema_ready = true;
    return copy(net, net->E, net->V, net->np);
  }
  return rnn_ema_update_dev(net->ctx, net->E, net->V, net->np, decay, net->ema_t);
}

static int train_step(rnn_rustvit* net, const float* x, const float* tf, const float* tc, const uint32_t* hard,
                      const uint32_t* hardc, int n, float lr, float wd, float clip, float ema, uint64_t seed,
                      float* stats) {
  RNN_TRY(forward(net, x, n, true, seed));
  // data-parallel: every rank leaves the forward with the mean of the
  // ranks' updated running statistics, so the buffers stay identical
  if (net->comm) RNN_TRY(rnn_allreduce_grads(net->ctx, net->comm, net->B, net->nb, 1));
  RNN_TRY(build_loss(net, tf, tc, hard, hardc, n));
  RNN_TRY(backward(net, net->g_logits, net->g_coarse, net->g_e1, net->g_e2, net->g_h1, net->g_h2, nullptr));
  // data-parallel: the mean of the ranks' shard gradients (equal shards: the
  // gradient of the mean loss over the whole batch) before clip_ and the
  // optimiser, which then run identically on every rank
  if (net->comm) RNN_TRY(rnn_allreduce_grads(net->ctx, net->comm, net->G, net->np, 1));
  if (clip > 0.0f) RNN_TRY(rnn_clip_dev(net->ctx, net->G, net->np, clip, net->clip_norm));
  RNN_TRY(step_all(net, lr, wd));
  if (ema > 0.0f) RNN_TRY(ema_update(net, ema));
  if (stats) {
    float l[8];
    int cor = 0;
    RNN_CUDA(cudaMemcpyAsync(l, net->losses, sizeof(l), cudaMemcpyDeviceToHost, net->ctx->stream));
    RNN_CUDA(cudaMemcpyAsync(&cor, net->correct, sizeof(int), cudaMemcpyDeviceToHost, net->ctx->stream));
    RNN_CUDA(cudaStreamSynchronize(net->ctx->stream));
    const LossCfg L;
    float total = l[0];  // train.rs:93-115, same association
    total += L.coarse_w * l[1];
    total += L.w1 * l[2] + L.w2 * l[3];
    total += L.alpha * (l[4] + l[5]);
    total += l[6] + l[7];
    stats[0] = total;
    stats[1] = l[0];
    stats[2] = (float)cor;
  }
  return RNN_OK;
}

static int copy_out(rnn_rustvit* net, float* dst, const float* src, size_t nfl) {
  RNN_CUDA(cudaMemcpyAsync(dst, src, nfl * sizeof(float), cudaMemcpyDefault, net->ctx->stream));
  RNN_CUDA(cudaStreamSynchronize(net->ctx->stream));
  return RNN_OK;
}

}  // namespace vit
}  // namespace rnn

// ---------------------------------------------------------------- C ABI

extern "C" int rnn_rustvit_create(rnn_ctx* ctx, const int* cfg9, const int* mem_at, int n_mem, float droppath,
                                  const uint32_t* parent, int nf, int ncoarse, uint64_t seed, rnn_rustvit** out) {
  RNN_REQUIRE(ctx && cfg9 && parent && out && nf > 0 && ncoarse > 0 && n_mem >= 0 && (n_mem == 0 || mem_at),
              "rustvit_create: bad arguments");
  *out = nullptr;
  Cfg c;
  c.width = cfg9[0]; c.cmid = cfg9[1]; c.dim = cfg9[2]; c.heads = cfg9[3]; c.depth3 = cfg9[4];
  c.dim4 = cfg9[5]; c.heads4 = cfg9[6]; c.depth4 = cfg9[7]; c.img = cfg9[8];
  c.mem_at.assign(mem_at, mem_at + n_mem);
  c.droppath = droppath;
  RNN_REQUIRE(c.width > 0 && c.cmid > 0 && c.dim > 0 && c.dim4 > 0 && c.depth3 >= 0 && c.depth4 >= 0,
              "rustvit_create: bad configuration");
  RNN_REQUIRE(c.heads > 0 && c.dim % c.heads == 0 && c.heads4 > 0 && c.dim4 % c.heads4 == 0,
              "rustvit_create: heads must divide the width");
  RNN_REQUIRE(c.img % 8 == 0, "rustvit_create: image side must be a multiple of 8 (got %d)", c.img);
  RNN_REQUIRE(droppath >= 0.0f && droppath < 1.0f, "rustvit_create: droppath in [0, 1)");
  for (int i = 0; i < nf; i++) RNN_REQUIRE((int)parent[i] < ncoarse, "rustvit_create: parent[%d] out of range", i);
  rnn_rustvit* net = new rnn_rustvit();
  net->ctx = ctx;
  net->cfg = c;
  net->nf = nf;
  net->nc = ncoarse;
  net->parent_host.assign(parent, parent + nf);
  int rc = cudaMalloc(&net->parent, nf * sizeof(uint32_t)) == cudaSuccess
               ? RNN_OK
               : set_error(RNN_ERR_CUDA, "rustvit_create: cudaMalloc failed");
  if (rc == RNN_OK && cudaMemcpy(net->parent, parent, nf * sizeof(uint32_t), cudaMemcpyHostToDevice) != cudaSuccess)
    rc = set_error(RNN_ERR_CUDA, "rustvit_create: copy of parent failed");
  if (rc == RNN_OK) rc = build(net, seed);
  if (rc != RNN_OK) {
    rnn_rustvit_destroy(net);
    return rc;
  }
  *out = net;
  return RNN_OK;
}

extern "C" int rnn_rustvit_destroy(rnn_rustvit* net) {
  if (!net) return RNN_OK;
  // the context may already be gone (interpreter teardown releases objects
  // in any order): wait on the device, not on the context's stream
  cudaDeviceSynchronize();
  free_acts(net);
  rnn::eval_ws_free(net->eval);
  for (void* p : {(void*)net->V, (void*)net->G, (void*)net->M, (void*)net->V2, (void*)net->E, (void*)net->B,
                  (void*)net->parent, (void*)net->st_x, (void*)net->st_tf, (void*)net->st_tc, (void*)net->st_hard,
                  (void*)net->opt_segs})
    if (p) cudaFree(p);
  delete net;
  return RNN_OK;
}

extern "C" int rnn_rustvit_dp_attach(rnn_rustvit* net, rnn_comm* comm) {
  RNN_REQUIRE(net, "rustvit_dp_attach: null network");
  net->comm = comm;
  return RNN_OK;
}

extern "C" int rnn_rustvit_num_params(rnn_rustvit* net, size_t* out) {
  RNN_REQUIRE(net && out, "rustvit_num_params: null argument");
  *out = net->np;
  return RNN_OK;
}

extern "C" int rnn_rustvit_num_buffers(rnn_rustvit* net, size_t* out) {
  RNN_REQUIRE(net && out, "rustvit_num_buffers: null argument");
  *out = net->nb;
  return RNN_OK;
}

extern "C" int rnn_rustvit_get_params(rnn_rustvit* net, float* out) {
  RNN_REQUIRE(net && out, "rustvit_get_params: null argument");
  return copy_out(net, out, net->V, net->np);
}
extern "C" int rnn_rustvit_set_params(rnn_rustvit* net, const float* in) {
  RNN_REQUIRE(net && in, "rustvit_set_params: null argument");
  return copy_out(net, net->V, in, net->np);
}
extern "C" int rnn_rustvit_get_grads(rnn_rustvit* net, float* out) {
  RNN_REQUIRE(net && out, "rustvit_get_grads: null argument");
  return copy_out(net, out, net->G, net->np);
}
extern "C" int rnn_rustvit_get_moments(rnn_rustvit* net, float* m, float* v2) {
  RNN_REQUIRE(net && m && v2, "rustvit_get_moments: null argument");
  RNN_TRY(copy_out(net, m, net->M, net->np));
  return copy_out(net, v2, net->V2, net->np);
}
extern "C" int rnn_rustvit_get_ema(rnn_rustvit* net, float* out) {
  RNN_REQUIRE(net && out, "rustvit_get_ema: null argument");
  RNN_REQUIRE(net->ema_ready, "rustvit_get_ema: no EMA update has run");
  return copy_out(net, out, net->E, net->np);
}
extern "C" int rnn_rustvit_get_buffers(rnn_rustvit* net, float* out) {
  RNN_REQUIRE(net && out, "rustvit_get_buffers: null argument");
  return copy_out(net, out, net->B, net->nb);
}
extern "C" int rnn_rustvit_zero_grads(rnn_rustvit* net) {
  RNN_REQUIRE(net, "rustvit_zero_grads: null argument");
  return zero(net, net->G, net->np);
}

extern "C" int rnn_rustvit_forward_dev(rnn_rustvit* net, const float* x, int n, int train, uint64_t drop_seed,
                                       float* logits, float* coarse, float* e1, float* e2, float* h1, float* h2,
                                       float* feat) {
  RNN_REQUIRE(net && x && n > 0, "rustvit_forward: bad arguments");
  RNN_RANGE(x, (size_t)n * 3 * net->cfg.img * net->cfg.img * sizeof(float));
  RNN_TRY(forward(net, x, n, train != 0, drop_seed));
  const size_t nf = (size_t)n * net->nf, d4 = (size_t)n * net->cfg.dim4;
  const bool ex = train && net->use_exits;
  const struct {
    float* dst;
    const float* src;
    size_t len;
    bool ok;
  } outs[] = {{logits, net->zl, nf, true},   {coarse, net->zc, (size_t)n * net->nc, true},
              {e1, net->e1l, nf, ex},         {e2, net->e2l, nf, ex},
              {h1, net->h1v, d4, ex},         {h2, net->h2v, d4, ex},
              {feat, net->feat, d4, true}};
  for (const auto& o : outs) {
    if (!o.dst) continue;
    RNN_REQUIRE(o.ok, "rustvit_forward: the exits exist only in training mode");
    RNN_RANGE(o.dst, o.len * sizeof(float));
    RNN_TRY(copy(net, o.dst, o.src, o.len));
  }
  return RNN_OK;
}

extern "C" int rnn_rustvit_backward_dev(rnn_rustvit* net, const float* dlogits, const float* dcoarse,
                                        const float* de1, const float* de2, const float* dh1, const float* dh2,
                                        const float* dhfinal) {
  RNN_REQUIRE(net && dlogits && dcoarse && net->n > 0, "rustvit_backward: bad arguments (forward first)");
  RNN_REQUIRE((de1 && de2 && dh1 && dh2) || (!de1 && !de2 && !dh1 && !dh2),
              "rustvit_backward: exit gradients come as a set");
  return backward(net, dlogits, dcoarse, de1, de2, dh1, dh2, dhfinal);
}

extern "C" int rnn_rustvit_train_step_dev(rnn_rustvit* net, const float* x, const float* tf, const float* tc,
                                          const uint32_t* hard, const uint32_t* hardc, int n, float lr, float wd,
                                          float clip, float ema, uint64_t drop_seed, float* stats) {
  RNN_REQUIRE(net && x && tf && tc && hard && hardc && n > 0, "rustvit_train_step: bad arguments");
  RNN_RANGE(x, (size_t)n * 3 * net->cfg.img * net->cfg.img * sizeof(float));
  RNN_RANGE(tf, (size_t)n * net->nf * sizeof(float));
  RNN_RANGE(tc, (size_t)n * net->nc * sizeof(float));
  RNN_RANGE(hard, (size_t)n * sizeof(uint32_t));
  RNN_RANGE(hardc, (size_t)n * sizeof(uint32_t));
  return train_step(net, x, tf, tc, hard, hardc, n, lr, wd, clip, ema, drop_seed, stats);
}

// Host tier: copies the batch (images, soft targets, hard labels) into
// device staging, runs the step and returns (total, ce, correct).
extern "C" int rnn_rustvit_train_step(rnn_rustvit* net, const float* x, const float* tf, const float* tc,
                                      const uint32_t* hard, const uint32_t* hardc, int n, float lr, float wd,
                                      float clip, float ema, uint64_t drop_seed, float* stats) {
  RNN_REQUIRE(net && x && tf && tc && hard && hardc && n > 0 && stats, "rustvit_train_step: bad arguments");
  const size_t xs = (size_t)n * 3 * net->cfg.img * net->cfg.img, fs = (size_t)n * net->nf,
               cs = (size_t)n * net->nc;
  if (n > net->st_cap) {
    for (void* p : {(void*)net->st_x, (void*)net->st_tf, (void*)net->st_tc, (void*)net->st_hard})
      if (p) cudaFree(p);
    net->st_x = net->st_tf = net->st_tc = nullptr;
    net->st_hard = nullptr;
    RNN_CUDA(cudaMalloc(&net->st_x, xs * sizeof(float)));
    RNN_CUDA(cudaMalloc(&net->st_tf, fs * sizeof(float)));
    RNN_CUDA(cudaMalloc(&net->st_tc, cs * sizeof(float)));
    RNN_CUDA(cudaMalloc(&net->st_hard, 2 * (size_t)n * sizeof(uint32_t)));
    net->st_cap = n;
  }
  cudaStream_t s = net->ctx->stream;
  RNN_CUDA(cudaMemcpyAsync(net->st_x, x, xs * sizeof(float), cudaMemcpyHostToDevice, s));
  RNN_CUDA(cudaMemcpyAsync(net->st_tf, tf, fs * sizeof(float), cudaMemcpyHostToDevice, s));
  RNN_CUDA(cudaMemcpyAsync(net->st_tc, tc, cs * sizeof(float), cudaMemcpyHostToDevice, s));
  RNN_CUDA(cudaMemcpyAsync(net->st_hard, hard, n * sizeof(uint32_t), cudaMemcpyHostToDevice, s));
  RNN_CUDA(cudaMemcpyAsync(net->st_hard + n, hardc, n * sizeof(uint32_t), cudaMemcpyHostToDevice, s));
  return train_step(net, net->st_x, net->st_tf, net->st_tc, net->st_hard, net->st_hard + n, n, lr, wd, clip, ema,
                    drop_seed, stats);
}

// ---------------------------------------------------------------- eval

namespace {

// Trainer::eval_ema (train.rs:390-402) swaps the EMA weights in around the
// evaluation; the flat parameter and EMA buffers have one layout and every
// layer reads its weights through net->V, so the swap is an exchange of the
// two pointers, undone when the guard leaves scope.
struct EmaSwap {
  rnn_rustvit* net;
  bool on;
  EmaSwap(rnn_rustvit* n, bool use) : net(n), on(use) {
    if (on) std::swap(net->V, net->E);
  }
  ~EmaSwap() {
    if (on) std::swap(net->V, net->E);
  }
};

// eval::vit (eval.rs:47-66): exits off (they run only in training, vit.rs:539
// and :565), forward with train false, test-time augmentation when tta
int vit_eval(rnn_rustvit* net, const uint8_t* images, const uint8_t* labels, int len, int batch, bool tta,
             bool use_ema, float* loss, float* acc) {
  RNN_REQUIRE(net->cfg.img == 32, "rustvit_eval: the dataset images are 32x32, the model takes %d", net->cfg.img);
  RNN_REQUIRE(!use_ema || net->ema_ready, "rustvit_eval: no EMA update has run");
  float out2[2];
  {
    EmaSwap swap(net, use_ema);
    RNN_TRY(rnn::eval_loop(net->ctx, net->eval, images, labels, len, batch, net->nf, tta,
                           [net](const float* x, int bs, const float** lg) {
                             RNN_TRY(forward(net, x, bs, false, 0));
                             *lg = net->zl;
                             return (int)RNN_OK;
                           },
                           out2));
  }
  if (loss) *loss = out2[0];
  if (acc) *acc = out2[1];
  return RNN_OK;
}

}  // namespace

extern "C" int rnn_rustvit_eval_dev(rnn_rustvit* net, const uint8_t* images, const uint8_t* labels, int len,
                                    int batch, int tta, int use_ema, float* loss, float* acc) {
  RNN_REQUIRE(net && (len == 0 || (images && labels)), "rustvit_eval: null argument");
  return vit_eval(net, images, labels, len, batch, tta != 0, use_ema != 0, loss, acc);
}

extern "C" int rnn_rustvit_eval(rnn_rustvit* net, const uint8_t* images, const uint8_t* labels, int len,
                                int batch, int tta, int use_ema, float* loss, float* acc) {
  RNN_REQUIRE(net && (len == 0 || (images && labels)), "rustvit_eval: null argument");
  RNN_REQUIRE(len >= 0 && batch > 0, "rustvit_eval: bad sizes");
  const uint8_t *di = nullptr, *dl = nullptr;
  if (len > 0) RNN_TRY(rnn::eval_ws_stage(net->eval, net->ctx, images, labels, len, &di, &dl));
  return vit_eval(net, di, dl, len, batch, tta != 0, use_ema != 0, loss, acc);
}

// ---------------------------------------------------------------- checkpoints

namespace {

// RustViT::config_hash (vit.rs:780-801)
uint64_t vit_hash(const rnn_rustvit* net, const char* kind) {
  const Cfg& c = net->cfg;
  uint32_t dp_bits;
  memcpy(&dp_bits, &c.droppath, 4);
  std::vector<uint64_t> f = {(uint64_t)c.width, (uint64_t)c.cmid,   (uint64_t)c.dim,    (uint64_t)c.heads,
                             (uint64_t)c.depth3, (uint64_t)c.dim4,  (uint64_t)c.heads4, (uint64_t)c.depth4,
                             (uint64_t)dp_bits,  (uint64_t)c.img,   (uint64_t)net->nf,  (uint64_t)net->nc,
                             (uint64_t)net->use_exits, (uint64_t)c.mem_at.size()};
  for (int m : c.mem_at) f.push_back((uint64_t)m);
  f.push_back(net->parent_host.size());
  for (uint32_t p : net->parent_host) f.push_back(p);
  return rnn::ckpt_hash(kind, strlen(kind), f.data(), f.size());
}

int vit_to_host(rnn_rustvit* net, std::vector<float>& h, const float* d, size_t n) {
  h.assign(n, 0.0f);
  if (n && d) RNN_CUDA(cudaMemcpyAsync(h.data(), d, n * sizeof(float), cudaMemcpyDeviceToHost, net->ctx->stream));
  return RNN_OK;
}

}  // namespace

extern "C" int rnn_rustvit_save(rnn_rustvit* net, const char* path) {
  RNN_REQUIRE(net && path, "rustvit_save: null argument");
  std::vector<float> v, b;
  RNN_TRY(vit_to_host(net, v, net->V, net->np));
  RNN_TRY(vit_to_host(net, b, net->B, net->nb));
  RNN_TRY(rnn_ctx_synchronize(net->ctx));
  return rnn::ckpt_write(path, (uint32_t)(net->order.size() + net->n_buf_tensors), vit_hash(net, "rustvit"),
                         {{v.data(), v.size()}, {b.data(), b.size()}});
}

extern "C" int rnn_rustvit_load(rnn_rustvit* net, const char* path) {
  RNN_REQUIRE(net && path, "rustvit_load: null argument");
  std::vector<float> p;
  RNN_TRY(rnn::ckpt_read(path, (uint32_t)(net->order.size() + net->n_buf_tensors), vit_hash(net, "rustvit"),
                         net->np + net->nb, p));
  RNN_CUDA(cudaMemcpyAsync(net->V, p.data(), net->np * sizeof(float), cudaMemcpyHostToDevice, net->ctx->stream));
  RNN_CUDA(cudaMemcpyAsync(net->B, p.data() + net->np, net->nb * sizeof(float), cudaMemcpyHostToDevice,
                           net->ctx->stream));
  return rnn_ctx_synchronize(net->ctx);
}

// payload: M, V2, E (zeros until the first EMA update), then the u32 words
// opt_t, ema_t, ema_ready
extern "C" int rnn_rustvit_save_optim(rnn_rustvit* net, const char* path) {
  RNN_REQUIRE(net && path, "rustvit_save_optim: null argument");
  std::vector<float> m, v2, e;
  RNN_TRY(vit_to_host(net, m, net->M, net->np));
  RNN_TRY(vit_to_host(net, v2, net->V2, net->np));
  RNN_TRY(vit_to_host(net, e, net->ema_ready ? net->E : nullptr, net->np));
  RNN_TRY(rnn_ctx_synchronize(net->ctx));
  const uint32_t words[3] = {(uint32_t)net->opt_t, (uint32_t)net->ema_t, (uint32_t)net->ema_ready};
  float tail[3];
  memcpy(tail, words, sizeof(words));
  return rnn::ckpt_write(path, (uint32_t)(3 * net->order.size() + 1), vit_hash(net, "rustvit-optim"),
                         {{m.data(), m.size()}, {v2.data(), v2.size()}, {e.data(), e.size()}, {tail, 3}});
}

extern "C" int rnn_rustvit_load_optim(rnn_rustvit* net, const char* path) {
  RNN_REQUIRE(net && path, "rustvit_load_optim: null argument");
  std::vector<float> p;
  const size_t np = net->np;
  RNN_TRY(rnn::ckpt_read(path, (uint32_t)(3 * net->order.size() + 1), vit_hash(net, "rustvit-optim"), 3 * np + 3, p));
  uint32_t words[3];
  memcpy(words, p.data() + 3 * np, sizeof(words));
  if (words[2] && !net->E) RNN_CUDA(cudaMalloc(&net->E, np * sizeof(float)));
  RNN_CUDA(cudaMemcpyAsync(net->M, p.data(), np * sizeof(float), cudaMemcpyHostToDevice, net->ctx->stream));
  RNN_CUDA(cudaMemcpyAsync(net->V2, p.data() + np, np * sizeof(float), cudaMemcpyHostToDevice, net->ctx->stream));
  if (words[2])
    RNN_CUDA(cudaMemcpyAsync(net->E, p.data() + 2 * np, np * sizeof(float), cudaMemcpyHostToDevice,
                             net->ctx->stream));
  RNN_TRY(rnn_ctx_synchronize(net->ctx));
  net->opt_t = (int)words[0];
  net->ema_t = (int)words[1];
  net->ema_ready = words[2] != 0;
  return RNN_OK;
}
