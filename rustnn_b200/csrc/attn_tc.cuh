// Tensor-core attention: the (image, head) products of attn.rs Core::forward
// (:148-223) and Core::backward (:226-343) as problems of the tcgen05 3xTF32
// engine (tc_gemm.cuh).  See attn_tc.cu.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace rnn {

// Arguments of one Core call (attn.rs:148-161, 226-242), as the C ABI takes
// them, plus the backward's workspace.
struct AttnTC {
  int n, h, dh, tq, tk, nrel, mask;
  int hp;  // head pairs, h / 2
  const uint32_t* relidx;  // [tq][tk] relative-position index (attn.rs:53-72)
  const float* q;
  int qstride, qoff;
  const float* kv;
  int kvstride, koff, voff;
  const float* tau;  // [h]
  const float* rel;  // [h][nrel]
  float* p;          // forward: P [n][h][tq][tk]
  float* o;          // forward: O [n*tq][h*dh]
  const float* pin;  // backward: P
  const float* dout; // backward: dO [n*tq][h*dh]
  float* dq;         // += , strided like q
  float* dkv;        // += , strided like kv
  const float* bias; // forward: rel[h][relidx[i][j]], -inf on a masked diagonal, [h][tq][tk]
  float* ds;         // backward workspace: dS [n][h][tq][tk] (before the tau scale)
  float* part;       // backward: dtau partials [n*2][h]
};

namespace tc {
// True when the tensor-core path covers the call: 64 query tokens (the 8x8
// grid), an even head count, head dim 32 or 64, a key count that is a
// multiple of 32 up to 256, and 16-byte aligned rows.
bool attn_tc_ok(const AttnTC& a, bool backward);
// a.bias must hold the table (attn_bias_build).
int attn_tc_fwd(rnn_ctx* ctx, const AttnTC& a);
// Writes ds and the dtau partials; the caller reduces them (attn_reduce) and
// forms drel from ds (attn_drel).
int attn_tc_bwd(rnn_ctx* ctx, const AttnTC& a);
// bias[h][i][j] = rel[h][relidx[i][j]], -inf at j == i under the mask.
int attn_bias_build(rnn_ctx* ctx, const AttnTC& a, float* bias);
// drel[h][r] += sum over images n and queries i of ds[n][h][i][inv[i][r]]
// (inv[i][r] = the key of query i at relative index r, or -1), in a fixed
// order: first the image sum of ds into dssum [h][tq][tk], then the gather.
int attn_drel(rnn_ctx* ctx, const AttnTC& a, const int* inv, float* dssum, float* drel);
}  // namespace tc
}  // namespace rnn
