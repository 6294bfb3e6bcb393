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
  float* ds;         // backward workspace: dS [n][h][tq][tk] (before the tau scale)
  float* part;       // backward partials [n*2][h][1 + nrel]: dtau, then drel
};

namespace tc {
// True when the tensor-core path covers the call: 64 query tokens (the 8x8
// grid), an even head count, head dim 32 or 64, a key count that is a
// multiple of 32 up to 256, and 16-byte aligned rows.
bool attn_tc_ok(const AttnTC& a, bool backward);
int attn_tc_fwd(rnn_ctx* ctx, const AttnTC& a);
// Writes ds and part; the caller reduces part into dtau / drel.
int attn_tc_bwd(rnn_ctx* ctx, const AttnTC& a);
// Largest relative-position table the backward's per-warp buffers hold.
constexpr int ATTN_TC_MAX_NREL = 1024;
}  // namespace tc
}  // namespace rnn
