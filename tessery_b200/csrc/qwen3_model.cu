// The Qwen3 embedding forward as one native call (tx_qwen3_forward): the layer loop of
// the reference's Qwen3Backend.forward (src/metal_inference/qwen3.py:112-296), which its
// Python host issues as one Metal command buffer of per-layer dispatches
// (qwen3.py:191-280), queued here from C++ through this library's own entry points, so a
// forward costs one foreign call and the calling thread holds no interpreter lock while
// the ~250 launches are queued (several host threads can then drive several GPUs).
//
// Per layer (fast mode): rms_norm -> q, k, v projections (bf16 out) -> attention with
// the q/k RMSNorm + RoPE prologue -> o projection added to the fp32 residual stream ->
// rms_norm -> fused gate/up projection with the SiLU-gated epilogue -> down projection
// added to the residual stream; then the final RMSNorm of each sequence's last token,
// pooled and L2-normalised (qwen3.py:281-290).  Precise mode carries every projection
// operand as a bf16 pair and runs q/k/v and the attention in fp32.
#include <cmath>
#include <cstdint>

#include "../../include/tessattn.h"
#include "kernels.h"

namespace {

struct Layout {
  uint64_t x, xn, q, k, v, att, att2, gated, total;
};

uint64_t round256(uint64_t bytes) { return (bytes + 255) & ~uint64_t(255); }

bool supported(const TxQwen3Model &m) {
  return m.head_dim == 128 && m.kv_heads && m.heads % m.kv_heads == 0 && m.hidden &&
         m.hidden % 256 == 0 && (m.heads * m.head_dim) % 256 == 0 &&
         (m.kv_heads * m.head_dim) % 256 == 0 && m.intermediate && m.intermediate % 128 == 0 &&
         m.layers && m.vocab && m.layer && m.embed_packed && m.embed_scales && m.embed_biases &&
         m.final_norm && m.eps >= 0.f && m.theta > 0.f;
}

// Workspace regions (byte offsets), each 256-byte aligned.  A bf16 pair [rows, cols] is
// the hi part followed by the lo part.
Layout layout(const TxQwen3Model &m, uint64_t tokens) {
  const uint64_t hid = m.hidden, qd = uint64_t(m.heads) * m.head_dim,
                 kd = uint64_t(m.kv_heads) * m.head_dim, inter = m.intermediate;
  const uint64_t pair = m.precise ? 2 : 1;   // bf16 operands: one part or a pair
  const uint64_t qkv = m.precise ? 4 : 2;    // q/k/v/attention element bytes
  Layout L{};
  uint64_t off = 0;
  auto take = [&](uint64_t bytes) {
    const uint64_t at = off;
    off += round256(bytes);
    return at;
  };
  L.x = take(tokens * hid * 4);
  L.xn = take(pair * tokens * hid * 2);
  L.q = take(tokens * qd * qkv);
  L.k = take(tokens * kd * qkv);
  L.v = take(tokens * kd * qkv);
  L.att = take(tokens * qd * qkv);
  L.att2 = m.precise ? take(2 * tokens * qd * 2) : 0;
  L.gated = take(pair * tokens * inter * 2);
  L.total = off;
  return L;
}

}  // namespace

extern "C" {

uint64_t tx_qwen3_workspace_bytes(const TxQwen3Model *model, uint32_t tokens) {
  if (!model || !supported(*model)) return 0;
  return layout(*model, tokens).total;
}

int tx_qwen3_forward(void *ctx, const TxQwen3Model *model, const uint32_t *ids,
                     const int32_t *cu_seqlens, const int32_t *cu_host, uint32_t nseq,
                     float *pooled, uint32_t dimensions, void *workspace,
                     uint64_t workspace_bytes, void *stream) {
  if (!ctx) return TX_EINVAL;
  if (!model || !supported(*model))
    return tx::ctx_fail(ctx, TX_EINVAL, "qwen3_forward: unsupported model description");
  const TxQwen3Model &m = *model;
  if (!ids || !cu_seqlens || !cu_host || !pooled || !workspace || !nseq)
    return tx::ctx_fail(ctx, TX_EINVAL, "qwen3_forward: null pointer or empty batch");
  if (!dimensions || dimensions > m.hidden)
    return tx::ctx_fail(ctx, TX_EINVAL, "qwen3_forward: need 0 < dimensions <= hidden");
  if (cu_host[0] != 0) return tx::ctx_fail(ctx, TX_EINVAL, "qwen3_forward: cu_seqlens[0] != 0");
  uint32_t max_len = 0;
  for (uint32_t b = 0; b < nseq; ++b) {
    if (cu_host[b + 1] <= cu_host[b])
      return tx::ctx_fail(ctx, TX_EINVAL, "qwen3_forward: every sequence needs a token");
    const uint32_t n = uint32_t(cu_host[b + 1] - cu_host[b]);
    max_len = n > max_len ? n : max_len;
  }
  const uint32_t T = uint32_t(cu_host[nseq]);
  const Layout L = layout(m, T);
  if (workspace_bytes < L.total || (uintptr_t)workspace % 256)
    return tx::ctx_fail(ctx, TX_EINVAL, "qwen3_forward: workspace too small or misaligned");

  char *ws = (char *)workspace;
  float *x = (float *)(ws + L.x);
  uint16_t *xn = (uint16_t *)(ws + L.xn);
  void *q = ws + L.q, *k = ws + L.k, *v = ws + L.v, *att = ws + L.att;
  uint16_t *att2 = (uint16_t *)(ws + L.att2);
  uint16_t *gated = (uint16_t *)(ws + L.gated);
  const uint32_t hid = m.hidden, H = m.heads, KV = m.kv_heads, D = m.head_dim;
  const uint32_t qd = H * D, kd = KV * D, inter = m.intermediate;
  const float scale = float(std::pow(double(D), -0.5));
  const int io = m.precise ? TX_F32 : TX_BF16;
  const int proj_out = m.precise ? TX_LINEAR_STORE_F32 : TX_LINEAR_STORE_BF16;

  // One projection: a [T, kdim] (a bf16 pair in precise mode) times w [n, kdim]^T.
  auto linear = [&](const uint16_t *a, uint32_t kdim, const uint16_t *w, void *out, uint32_t n,
                    int mode) {
    const uint16_t *a_lo = m.precise ? a + uint64_t(T) * kdim : nullptr;
    const uint16_t *w_lo = m.precise ? w + uint64_t(n) * kdim : nullptr;
    return tx_linear(ctx, a, a_lo, w, w_lo, nullptr, out, T, n, kdim, mode, TX_BF16, n, stream);
  };
  const int norm_out = m.precise ? TX_BF16X2 : TX_BF16;

#define TX_TRY(call)            \
  do {                          \
    const int rc_ = (call);     \
    if (rc_ != TX_OK) return rc_; \
  } while (0)

  TX_TRY(tx_embedding4(ctx, ids, T, m.embed_packed, m.embed_scales, m.embed_biases, x, hid,
                       m.vocab, stream));
  for (uint32_t l = 0; l < m.layers; ++l) {
    const TxQwen3Layer &w = m.layer[l];
    if (!w.input_norm || !w.post_norm || !w.q_norm || !w.k_norm || !w.q_proj || !w.k_proj ||
        !w.v_proj || !w.o_proj || !w.gate_up || !w.down)
      return tx::ctx_fail(ctx, TX_EINVAL, "qwen3_forward: null weight pointer");
    TX_TRY(tx_rms_norm_rows(ctx, x, w.input_norm, xn, norm_out, T, hid, m.eps, stream));
    TX_TRY(linear(xn, hid, w.q_proj, q, qd, proj_out));
    TX_TRY(linear(xn, hid, w.k_proj, k, kd, proj_out));
    TX_TRY(linear(xn, hid, w.v_proj, v, kd, proj_out));
    TX_TRY(tx_attention_varlen(ctx, q, k, v, cu_seqlens, cu_host, nseq, T, max_len, att, H, KV,
                               D, io, io, /*causal=*/1, scale, w.q_norm, w.k_norm, m.eps,
                               m.theta, stream));
    const uint16_t *att_in = (const uint16_t *)att;
    if (m.precise) {
      TX_TRY(tx_split_bf16(ctx, (const float *)att, att2, uint64_t(T) * qd, stream));
      att_in = att2;
    }
    TX_TRY(linear(att_in, qd, w.o_proj, x, hid, TX_LINEAR_ADD_F32));
    TX_TRY(tx_rms_norm_rows(ctx, x, w.post_norm, xn, norm_out, T, hid, m.eps, stream));
    TX_TRY(linear(xn, hid, w.gate_up, gated, 2 * inter, TX_LINEAR_GATED_BF16));
    TX_TRY(linear(gated, inter, w.down, x, hid, TX_LINEAR_ADD_F32));
  }
  TX_TRY(tx_pool_project(ctx, x, TX_F32, nullptr, cu_seqlens, pooled, nseq, 0, hid, dimensions,
                         /*first_token=*/0, m.final_norm, m.eps, stream));
#undef TX_TRY
  return TX_OK;
}

}  // extern "C"
