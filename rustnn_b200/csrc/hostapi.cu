// Host-pointer tier of the C ABI for the attention, normalisation and
// optimiser entry points: each call stages its operands in the context's
// staging buffer, runs the device entry point on the context's stream, copies
// the results back and synchronises.  Arguments keep the meaning of the
// matching _dev entry (and of the reference function it replaces, cited in
// include/rnn_b200.h); gradient outputs accumulate exactly where the device
// entry accumulates, so they are staged in both directions.
#include <string.h>

#include <vector>

#include "common.cuh"
#include "ew.cuh"

using namespace rnn;

namespace {

struct Plan {
  size_t bytes = 0;
  size_t add(size_t b) {
    const size_t o = bytes;
    bytes += (b + 255) & ~(size_t)255;
    return o;
  }
};

struct Stager {
  rnn_ctx* ctx;
  char* base;
  template <class T>
  T* at(size_t off) const {
    return reinterpret_cast<T*>(base + off);
  }
  int in(void* dst, const void* src, size_t b) const {
    if (b) RNN_CUDA(cudaMemcpyAsync(dst, src, b, cudaMemcpyHostToDevice, ctx->stream));
    return RNN_OK;
  }
  int out(void* dst, const void* src, size_t b) const {
    if (b) RNN_CUDA(cudaMemcpyAsync(dst, src, b, cudaMemcpyDeviceToHost, ctx->stream));
    return RNN_OK;
  }
};

int begin(rnn_ctx* ctx, const Plan& p, Stager* s) {
  RNN_REQUIRE(ctx != nullptr, "null context");
  RNN_TRY(ensure_stage(ctx, p.bytes ? p.bytes : 256));
  s->ctx = ctx;
  s->base = static_cast<char*>(ctx->stage);
  return RNN_OK;
}

const size_t F = sizeof(float);

}  // namespace

// ---------------------------------------------------------------- attention

extern "C" int rnn_attn_fwd(rnn_ctx* ctx, int n, int h, int dh, int th, int tw, int mh, int mw, int mask_diag,
                            const float* q, int qstride, int qoff, const float* kv, int kvstride, int koff, int voff,
                            const float* tau, const float* rel, float* p, float* o) {
  RNN_REQUIRE(q && kv && tau && rel && p && o && n > 0 && h > 0 && dh > 0, "attn_fwd: bad arguments");
  int nrel = 0;
  RNN_TRY(rnn_rel_index(th, tw, mh, mw, nullptr, &nrel));
  const size_t tq = (size_t)th * tw, tk = (size_t)mh * mw;
  const size_t nq = n * tq * qstride, nkv = n * tk * kvstride, np = (size_t)n * h * tq * tk, no = n * tq * h * dh;
  const bool shared = kv == q && kvstride == qstride;  // fused qkv buffer (attn.rs:393-405)
  Plan pl;
  const size_t oq = pl.add(nq * F), okv = shared ? oq : pl.add(nkv * F), ot = pl.add(h * F),
               orl = pl.add(h * nrel * F), op = pl.add(np * F), oo = pl.add(no * F);
  Stager s;
  RNN_TRY(begin(ctx, pl, &s));
  RNN_TRY(s.in(s.at<float>(oq), q, nq * F));
  if (!shared) RNN_TRY(s.in(s.at<float>(okv), kv, nkv * F));
  RNN_TRY(s.in(s.at<float>(ot), tau, h * F));
  RNN_TRY(s.in(s.at<float>(orl), rel, h * nrel * F));
  RNN_TRY(rnn_attn_fwd_dev(ctx, n, h, dh, th, tw, mh, mw, mask_diag, s.at<float>(oq), qstride, qoff,
                           s.at<float>(okv), kvstride, koff, voff, s.at<float>(ot), s.at<float>(orl),
                           s.at<float>(op), s.at<float>(oo)));
  RNN_TRY(s.out(p, s.at<float>(op), np * F));
  RNN_TRY(s.out(o, s.at<float>(oo), no * F));
  return rnn_ctx_synchronize(ctx);
}

extern "C" int rnn_attn_bwd(rnn_ctx* ctx, int n, int h, int dh, int th, int tw, int mh, int mw, const float* q,
                            int qstride, int qoff, const float* kv, int kvstride, int koff, int voff,
                            const float* tau, const float* p, const float* dout, float* dq, float* dkv,
                            float* dtau, float* drel) {
  RNN_REQUIRE(q && kv && tau && p && dout && dq && dkv && dtau && drel && n > 0 && h > 0 && dh > 0,
              "attn_bwd: bad arguments");
  int nrel = 0;
  RNN_TRY(rnn_rel_index(th, tw, mh, mw, nullptr, &nrel));
  const size_t tq = (size_t)th * tw, tk = (size_t)mh * mw;
  const size_t nq = n * tq * qstride, nkv = n * tk * kvstride, np = (size_t)n * h * tq * tk, no = n * tq * h * dh;
  const bool shared = kv == q && kvstride == qstride;
  const bool dshared = dkv == dq && kvstride == qstride;
  Plan pl;
  const size_t oq = pl.add(nq * F), okv = shared ? oq : pl.add(nkv * F), ot = pl.add(h * F),
               op = pl.add(np * F), odo = pl.add(no * F), odq = pl.add(nq * F),
               odkv = dshared ? odq : pl.add(nkv * F), odt = pl.add(h * F), odr = pl.add(h * nrel * F);
  Stager s;
  RNN_TRY(begin(ctx, pl, &s));
  RNN_TRY(s.in(s.at<float>(oq), q, nq * F));
  if (!shared) RNN_TRY(s.in(s.at<float>(okv), kv, nkv * F));
  RNN_TRY(s.in(s.at<float>(ot), tau, h * F));
  RNN_TRY(s.in(s.at<float>(op), p, np * F));
  RNN_TRY(s.in(s.at<float>(odo), dout, no * F));
  RNN_TRY(s.in(s.at<float>(odq), dq, nq * F));
  if (!dshared) RNN_TRY(s.in(s.at<float>(odkv), dkv, nkv * F));
  RNN_TRY(s.in(s.at<float>(odt), dtau, h * F));
  RNN_TRY(s.in(s.at<float>(odr), drel, h * nrel * F));
  RNN_TRY(rnn_attn_bwd_dev(ctx, n, h, dh, th, tw, mh, mw, s.at<float>(oq), qstride, qoff, s.at<float>(okv),
                           kvstride, koff, voff, s.at<float>(ot), s.at<float>(op), s.at<float>(odo),
                           s.at<float>(odq), s.at<float>(odkv), s.at<float>(odt), s.at<float>(odr)));
  RNN_TRY(s.out(dq, s.at<float>(odq), nq * F));
  if (!dshared) RNN_TRY(s.out(dkv, s.at<float>(odkv), nkv * F));
  RNN_TRY(s.out(dtau, s.at<float>(odt), h * F));
  RNN_TRY(s.out(drel, s.at<float>(odr), h * nrel * F));
  return rnn_ctx_synchronize(ctx);
}

// ---------------------------------------------------------------- LayerNorm, Linear

extern "C" int rnn_layernorm_fwd(rnn_ctx* ctx, const float* x, int rows, int c, const float* gamma,
                                 const float* beta, float eps, float* y, float* xhat, float* invstd) {
  RNN_REQUIRE(x && gamma && beta && y && xhat && invstd && rows > 0 && c > 0, "layernorm_fwd: bad arguments");
  const size_t nx = (size_t)rows * c;
  Plan pl;
  const size_t ox = pl.add(nx * F), og = pl.add(c * F), ob = pl.add(c * F), oy = pl.add(nx * F),
               oh = pl.add(nx * F), oi = pl.add(rows * F);
  Stager s;
  RNN_TRY(begin(ctx, pl, &s));
  RNN_TRY(s.in(s.at<float>(ox), x, nx * F));
  RNN_TRY(s.in(s.at<float>(og), gamma, c * F));
  RNN_TRY(s.in(s.at<float>(ob), beta, c * F));
  RNN_TRY(rnn_layernorm_fwd_dev(ctx, s.at<float>(ox), rows, c, s.at<float>(og), s.at<float>(ob), eps,
                                s.at<float>(oy), s.at<float>(oh), s.at<float>(oi)));
  RNN_TRY(s.out(y, s.at<float>(oy), nx * F));
  RNN_TRY(s.out(xhat, s.at<float>(oh), nx * F));
  RNN_TRY(s.out(invstd, s.at<float>(oi), rows * F));
  return rnn_ctx_synchronize(ctx);
}

extern "C" int rnn_layernorm_bwd(rnn_ctx* ctx, const float* dy, const float* xhat, const float* invstd, int rows,
                                 int c, const float* gamma, float* dx, float* dgamma, float* dbeta) {
  RNN_REQUIRE(dy && xhat && invstd && gamma && dx && dgamma && dbeta && rows > 0 && c > 0,
              "layernorm_bwd: bad arguments");
  const size_t nx = (size_t)rows * c;
  Plan pl;
  const size_t ody = pl.add(nx * F), oh = pl.add(nx * F), oi = pl.add(rows * F), og = pl.add(c * F),
               odx = pl.add(nx * F), odg = pl.add(c * F), odb = pl.add(c * F);
  Stager s;
  RNN_TRY(begin(ctx, pl, &s));
  RNN_TRY(s.in(s.at<float>(ody), dy, nx * F));
  RNN_TRY(s.in(s.at<float>(oh), xhat, nx * F));
  RNN_TRY(s.in(s.at<float>(oi), invstd, rows * F));
  RNN_TRY(s.in(s.at<float>(og), gamma, c * F));
  RNN_TRY(s.in(s.at<float>(odg), dgamma, c * F));
  RNN_TRY(s.in(s.at<float>(odb), dbeta, c * F));
  RNN_TRY(rnn_layernorm_bwd_dev(ctx, s.at<float>(ody), s.at<float>(oh), s.at<float>(oi), rows, c, s.at<float>(og),
                                s.at<float>(odx), s.at<float>(odg), s.at<float>(odb)));
  RNN_TRY(s.out(dx, s.at<float>(odx), nx * F));
  RNN_TRY(s.out(dgamma, s.at<float>(odg), c * F));
  RNN_TRY(s.out(dbeta, s.at<float>(odb), c * F));
  return rnn_ctx_synchronize(ctx);
}

extern "C" int rnn_linear_fwd(rnn_ctx* ctx, const float* x, int rows, int fin, int fout, const float* w,
                              const float* b, float* y) {
  RNN_REQUIRE(x && w && y && rows > 0 && fin > 0 && fout > 0, "linear_fwd: bad arguments");
  const size_t nx = (size_t)rows * fin, nw = (size_t)fout * fin, ny = (size_t)rows * fout;
  Plan pl;
  const size_t ox = pl.add(nx * F), ow = pl.add(nw * F), ob = pl.add(fout * F), oy = pl.add(ny * F);
  Stager s;
  RNN_TRY(begin(ctx, pl, &s));
  RNN_TRY(s.in(s.at<float>(ox), x, nx * F));
  RNN_TRY(s.in(s.at<float>(ow), w, nw * F));
  if (b) RNN_TRY(s.in(s.at<float>(ob), b, fout * F));
  RNN_TRY(rnn_linear_fwd_dev(ctx, s.at<float>(ox), rows, fin, fout, s.at<float>(ow), b ? s.at<float>(ob) : nullptr,
                             s.at<float>(oy)));
  RNN_TRY(s.out(y, s.at<float>(oy), ny * F));
  return rnn_ctx_synchronize(ctx);
}

extern "C" int rnn_linear_bwd(rnn_ctx* ctx, const float* x, const float* dy, int rows, int fin, int fout,
                              const float* w, float* dw, float* db, float* dx) {
  RNN_REQUIRE(x && dy && w && dw && dx && rows > 0 && fin > 0 && fout > 0, "linear_bwd: bad arguments");
  const size_t nx = (size_t)rows * fin, nw = (size_t)fout * fin, ny = (size_t)rows * fout;
  Plan pl;
  const size_t ox = pl.add(nx * F), ody = pl.add(ny * F), ow = pl.add(nw * F), odw = pl.add(nw * F),
               odb = pl.add(fout * F), odx = pl.add(nx * F);
  Stager s;
  RNN_TRY(begin(ctx, pl, &s));
  RNN_TRY(s.in(s.at<float>(ox), x, nx * F));
  RNN_TRY(s.in(s.at<float>(ody), dy, ny * F));
  RNN_TRY(s.in(s.at<float>(ow), w, nw * F));
  RNN_TRY(s.in(s.at<float>(odw), dw, nw * F));
  if (db) RNN_TRY(s.in(s.at<float>(odb), db, fout * F));
  RNN_TRY(rnn_linear_bwd_dev(ctx, s.at<float>(ox), s.at<float>(ody), rows, fin, fout, s.at<float>(ow),
                             s.at<float>(odw), db ? s.at<float>(odb) : nullptr, s.at<float>(odx)));
  RNN_TRY(s.out(dw, s.at<float>(odw), nw * F));
  if (db) RNN_TRY(s.out(db, s.at<float>(odb), fout * F));
  RNN_TRY(s.out(dx, s.at<float>(odx), nx * F));
  return rnn_ctx_synchronize(ctx);
}

// ---------------------------------------------------------------- BatchNorm2d

extern "C" int rnn_batchnorm_fwd(rnn_ctx* ctx, const float* y, int n, int c, int hw, const float* gamma,
                                 const float* beta, float* rmean, float* rvar, float mom, float eps, int relu,
                                 float* mean, float* invstd, float* out) {
  RNN_REQUIRE(y && gamma && beta && mean && invstd && out && n > 0 && c > 0 && hw > 0,
              "batchnorm_fwd: bad arguments");
  const size_t ny = (size_t)n * c * hw;
  Plan pl;
  const size_t oy = pl.add(ny * F), og = pl.add(c * F), ob = pl.add(c * F), orm = pl.add(c * F),
               orv = pl.add(c * F), om = pl.add(c * F), oi = pl.add(c * F), oo = pl.add(ny * F);
  Stager s;
  RNN_TRY(begin(ctx, pl, &s));
  RNN_TRY(s.in(s.at<float>(oy), y, ny * F));
  RNN_TRY(s.in(s.at<float>(og), gamma, c * F));
  RNN_TRY(s.in(s.at<float>(ob), beta, c * F));
  if (rmean) RNN_TRY(s.in(s.at<float>(orm), rmean, c * F));
  if (rvar) RNN_TRY(s.in(s.at<float>(orv), rvar, c * F));
  RNN_TRY(rnn_batchnorm_fwd_dev(ctx, s.at<float>(oy), n, c, hw, s.at<float>(og), s.at<float>(ob),
                                rmean ? s.at<float>(orm) : nullptr, rvar ? s.at<float>(orv) : nullptr, mom, eps,
                                relu, s.at<float>(om), s.at<float>(oi), s.at<float>(oo)));
  if (rmean) RNN_TRY(s.out(rmean, s.at<float>(orm), c * F));
  if (rvar) RNN_TRY(s.out(rvar, s.at<float>(orv), c * F));
  RNN_TRY(s.out(mean, s.at<float>(om), c * F));
  RNN_TRY(s.out(invstd, s.at<float>(oi), c * F));
  RNN_TRY(s.out(out, s.at<float>(oo), ny * F));
  return rnn_ctx_synchronize(ctx);
}

extern "C" int rnn_batchnorm_bwd(rnn_ctx* ctx, const float* dy, const float* y, int n, int c, int hw,
                                 const float* gamma, const float* mean, const float* invstd, const float* relu_out,
                                 float* dx, float* dgamma, float* dbeta) {
  RNN_REQUIRE(dy && y && gamma && mean && invstd && dx && n > 0 && c > 0 && hw > 0, "batchnorm_bwd: bad arguments");
  const size_t ny = (size_t)n * c * hw;
  Plan pl;
  const size_t ody = pl.add(ny * F), oy = pl.add(ny * F), og = pl.add(c * F), om = pl.add(c * F),
               oi = pl.add(c * F), orl = pl.add(ny * F), odx = pl.add(ny * F), odg = pl.add(c * F),
               odb = pl.add(c * F);
  Stager s;
  RNN_TRY(begin(ctx, pl, &s));
  RNN_TRY(s.in(s.at<float>(ody), dy, ny * F));
  RNN_TRY(s.in(s.at<float>(oy), y, ny * F));
  RNN_TRY(s.in(s.at<float>(og), gamma, c * F));
  RNN_TRY(s.in(s.at<float>(om), mean, c * F));
  RNN_TRY(s.in(s.at<float>(oi), invstd, c * F));
  if (relu_out) RNN_TRY(s.in(s.at<float>(orl), relu_out, ny * F));
  if (dgamma) RNN_TRY(s.in(s.at<float>(odg), dgamma, c * F));
  if (dbeta) RNN_TRY(s.in(s.at<float>(odb), dbeta, c * F));
  RNN_TRY(rnn_batchnorm_bwd_dev(ctx, s.at<float>(ody), s.at<float>(oy), n, c, hw, s.at<float>(og), s.at<float>(om),
                                s.at<float>(oi), relu_out ? s.at<float>(orl) : nullptr, s.at<float>(odx),
                                dgamma ? s.at<float>(odg) : nullptr, dbeta ? s.at<float>(odb) : nullptr));
  RNN_TRY(s.out(dx, s.at<float>(odx), ny * F));
  if (dgamma) RNN_TRY(s.out(dgamma, s.at<float>(odg), c * F));
  if (dbeta) RNN_TRY(s.out(dbeta, s.at<float>(odb), c * F));
  return rnn_ctx_synchronize(ctx);
}

// ---------------------------------------------------------------- optimisers

extern "C" int rnn_newton_schulz_batched_dev(rnn_ctx* ctx, int count, float* const* g, const int* rows,
                                             const int* cols, int steps) {
  RNN_REQUIRE(ctx && count >= 0 && (count == 0 || (g && rows && cols)), "newton_schulz_batched: bad arguments");
  for (int i = 0; i < count; i++) {
    RNN_REQUIRE(g[i] && rows[i] > 0 && cols[i] > 0, "newton_schulz_batched: matrix %d is empty", i);
    RNN_RANGE(g[i], (size_t)rows[i] * cols[i] * 4);
  }
  RNN_REQUIRE(steps >= 0, "newton_schulz_batched: negative steps");
  return rnn::newton_schulz_grouped(ctx, count, g, rows, cols, steps);
}

extern "C" int rnn_newton_schulz_batched(rnn_ctx* ctx, int count, float* const* g, const int* rows,
                                         const int* cols, int steps) {
  RNN_REQUIRE(ctx && count >= 0 && (count == 0 || (g && rows && cols)), "newton_schulz_batched: bad arguments");
  Plan pl;
  std::vector<size_t> off(count);
  for (int i = 0; i < count; i++) {
    RNN_REQUIRE(g[i] && rows[i] > 0 && cols[i] > 0, "newton_schulz_batched: matrix %d is empty", i);
    off[i] = pl.add((size_t)rows[i] * cols[i] * F);
  }
  Stager s;
  RNN_TRY(begin(ctx, pl, &s));
  std::vector<float*> dg(count);
  for (int i = 0; i < count; i++) {
    dg[i] = s.at<float>(off[i]);
    RNN_TRY(s.in(dg[i], g[i], (size_t)rows[i] * cols[i] * F));
  }
  RNN_TRY(rnn_newton_schulz_batched_dev(ctx, count, dg.data(), rows, cols, steps));
  for (int i = 0; i < count; i++) RNN_TRY(s.out(g[i], dg[i], (size_t)rows[i] * cols[i] * F));
  return rnn_ctx_synchronize(ctx);
}

extern "C" int rnn_muon_step(rnn_ctx* ctx, float* v, float* g, float* m, int rows, int cols, int steps, float lr,
                             float mom, float wd, int decay) {
  RNN_REQUIRE(v && g && m && rows > 0 && cols > 0, "muon_step: bad arguments");
  const size_t nn = (size_t)rows * cols;
  Plan pl;
  const size_t ov = pl.add(nn * F), og = pl.add(nn * F), om = pl.add(nn * F);
  Stager s;
  RNN_TRY(begin(ctx, pl, &s));
  for (auto [o, p] : {std::pair<size_t, float*>{ov, v}, {og, g}, {om, m}}) RNN_TRY(s.in(s.at<float>(o), p, nn * F));
  RNN_TRY(rnn_muon_step_dev(ctx, s.at<float>(ov), s.at<float>(og), s.at<float>(om), rows, cols, steps, lr, mom, wd,
                            decay));
  for (auto [o, p] : {std::pair<size_t, float*>{ov, v}, {og, g}, {om, m}}) RNN_TRY(s.out(p, s.at<float>(o), nn * F));
  return rnn_ctx_synchronize(ctx);
}

extern "C" int rnn_adamw_step(rnn_ctx* ctx, float* v, float* g, float* m, float* v2, size_t n, float lr, float wd,
                              int decay, float b1, float b2, float eps, int t) {
  RNN_REQUIRE(v && g && m && v2, "adamw_step: bad arguments");
  Plan pl;
  const size_t ov = pl.add(n * F), og = pl.add(n * F), om = pl.add(n * F), o2 = pl.add(n * F);
  Stager s;
  RNN_TRY(begin(ctx, pl, &s));
  const std::pair<size_t, float*> io[] = {{ov, v}, {og, g}, {om, m}, {o2, v2}};
  for (auto [o, p] : io) RNN_TRY(s.in(s.at<float>(o), p, n * F));
  RNN_TRY(rnn_adamw_step_dev(ctx, s.at<float>(ov), s.at<float>(og), s.at<float>(om), s.at<float>(o2), n, lr, wd,
                             decay, b1, b2, eps, t));
  for (auto [o, p] : io) RNN_TRY(s.out(p, s.at<float>(o), n * F));
  return rnn_ctx_synchronize(ctx);
}

extern "C" int rnn_sgd_nesterov(rnn_ctx* ctx, float* v, float* g, float* m, size_t len, float lr, float mom,
                                float wd, int decay) {
  RNN_REQUIRE(v && g && m, "sgd_nesterov: bad arguments");
  Plan pl;
  const size_t ov = pl.add(len * F), og = pl.add(len * F), om = pl.add(len * F);
  Stager s;
  RNN_TRY(begin(ctx, pl, &s));
  const std::pair<size_t, float*> io[] = {{ov, v}, {og, g}, {om, m}};
  for (auto [o, p] : io) RNN_TRY(s.in(s.at<float>(o), p, len * F));
  RNN_TRY(rnn_sgd_nesterov_dev(ctx, s.at<float>(ov), s.at<float>(og), s.at<float>(om), len, lr, mom, wd, decay));
  for (auto [o, p] : io) RNN_TRY(s.out(p, s.at<float>(o), len * F));
  return rnn_ctx_synchronize(ctx);
}

extern "C" int rnn_clip(rnn_ctx* ctx, float* g, size_t n, float max, float* norm_out) {
  RNN_REQUIRE(g, "clip: bad arguments");
  Plan pl;
  const size_t og = pl.add(n * F), on = pl.add(F);
  Stager s;
  RNN_TRY(begin(ctx, pl, &s));
  RNN_TRY(s.in(s.at<float>(og), g, n * F));
  RNN_TRY(rnn_clip_dev(ctx, s.at<float>(og), n, max, s.at<float>(on)));
  RNN_TRY(s.out(g, s.at<float>(og), n * F));
  if (norm_out) RNN_TRY(s.out(norm_out, s.at<float>(on), F));
  return rnn_ctx_synchronize(ctx);
}

extern "C" int rnn_ema_update(rnn_ctx* ctx, float* e, const float* v, size_t n, float decay, int t) {
  RNN_REQUIRE(e && v, "ema_update: bad arguments");
  Plan pl;
  const size_t oe = pl.add(n * F), ov = pl.add(n * F);
  Stager s;
  RNN_TRY(begin(ctx, pl, &s));
  RNN_TRY(s.in(s.at<float>(oe), e, n * F));
  RNN_TRY(s.in(s.at<float>(ov), v, n * F));
  RNN_TRY(rnn_ema_update_dev(ctx, s.at<float>(oe), s.at<float>(ov), n, decay, t));
  RNN_TRY(s.out(e, s.at<float>(oe), n * F));
  return rnn_ctx_synchronize(ctx);
}
