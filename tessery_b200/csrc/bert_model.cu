// The BERT (BGE-small) fp32 embedding forward as one native call (tx_bert_forward): the
// layer loop of the reference's BertBackend.forward (src/metal_inference/bert.py:104-235),
// which its host issues as one Metal command of per-layer dispatches (bert.py:174-231),
// queued here from C++ through this library's own entry points.
//
// Sequences are packed by cu_seqlens (no padded rows: with the key-padding mask of the
// bidirectional attention, kernels.metal:86-99, a padded row never reaches a valid row).
// Per layer: the fused q/k/v projection (TF32 tensor cores, bias in the epilogue, q, k and
// v written to three matrices) -> head_dim-32 bidirectional attention (fp32) -> its output
// split into a TF32 operand pair -> output projection + bias added to the residual stream
// -> LayerNorm (writing the fp32 row and the next operand pair) -> intermediate projection
// + bias with the GELU epilogue (writing an operand pair) -> output projection + bias
// added to the residual stream -> LayerNorm.  Then the CLS row of each sequence,
// L2-normalised (bert.py:232-241, pool_project with first_token).
#include <cmath>
#include <cstdint>

#include "../../include/tessattn.h"
#include "kernels.h"

namespace {

struct Layout {
  uint64_t x, xs, qkv, att, atts, act, total;
};

uint64_t round256(uint64_t bytes) { return (bytes + 255) & ~uint64_t(255); }

bool supported(const TxBertModel &m) {
  return m.hidden && m.hidden % 128 == 0 && tx::bert_cols_ok(m.hidden) && m.heads &&
         m.hidden % m.heads == 0 && m.intermediate && m.intermediate % 128 == 0 && m.layers &&
         m.vocab && m.max_pos && m.layer && m.words && m.positions && m.types && m.ln_w &&
         m.ln_b && m.eps >= 0.f;
}

// Workspace regions (byte offsets), each 256-byte aligned.  An operand pair [rows, cols]
// is the hi part followed by the lo part, fp32 each.
Layout layout(const TxBertModel &m, uint64_t tokens) {
  const uint64_t hid = m.hidden, inter = m.intermediate, row = tokens * hid * 4;
  Layout L{};
  uint64_t off = 0;
  auto take = [&](uint64_t bytes) {
    const uint64_t at = off;
    off += round256(bytes);
    return at;
  };
  L.x = take(row);
  L.xs = take(2 * row);
  L.qkv = take(3 * row);
  L.att = take(row);
  L.atts = take(2 * row);
  L.act = take(2 * tokens * inter * 4);
  L.total = off;
  return L;
}

}  // namespace

extern "C" {

uint64_t tx_bert_workspace_bytes(const TxBertModel *model, uint32_t tokens) {
  if (!model || !supported(*model)) return 0;
  return layout(*model, tokens).total;
}

int tx_bert_forward(void *ctx, const TxBertModel *model, const uint32_t *ids,
                    const int32_t *cu_seqlens, const int32_t *cu_host, uint32_t nseq,
                    float *pooled, void *workspace, uint64_t workspace_bytes, void *stream) {
  if (!ctx) return TX_EINVAL;
  if (!model || !supported(*model))
    return tx::ctx_fail(ctx, TX_EINVAL, "bert_forward: unsupported model description");
  const TxBertModel &m = *model;
  if (!ids || !cu_seqlens || !cu_host || !pooled || !workspace || !nseq)
    return tx::ctx_fail(ctx, TX_EINVAL, "bert_forward: null pointer or empty batch");
  if (cu_host[0] != 0) return tx::ctx_fail(ctx, TX_EINVAL, "bert_forward: cu_seqlens[0] != 0");
  uint32_t max_len = 0;
  for (uint32_t b = 0; b < nseq; ++b) {
    if (cu_host[b + 1] <= cu_host[b])
      return tx::ctx_fail(ctx, TX_EINVAL, "bert_forward: every sequence needs a token");
    const uint32_t n = uint32_t(cu_host[b + 1] - cu_host[b]);
    max_len = n > max_len ? n : max_len;
  }
  if (max_len > m.max_pos)
    return tx::ctx_fail(ctx, TX_EINVAL, "bert_forward: a sequence longer than max_pos");
  const uint32_t T = uint32_t(cu_host[nseq]);
  const Layout L = layout(m, T);
  if (workspace_bytes < L.total || (uintptr_t)workspace % 256)
    return tx::ctx_fail(ctx, TX_EINVAL, "bert_forward: workspace too small or misaligned");

  char *ws = (char *)workspace;
  float *x = (float *)(ws + L.x), *xs = (float *)(ws + L.xs), *qkv = (float *)(ws + L.qkv);
  float *att = (float *)(ws + L.att), *atts = (float *)(ws + L.atts);
  float *act = (float *)(ws + L.act);
  const uint32_t hid = m.hidden, inter = m.intermediate, H = m.heads, D = hid / H;
  const uint64_t plane = uint64_t(T) * hid;
  const float scale = float(std::pow(double(D), -0.5));

  // One projection: a [T, kdim] operand pair times w [2][n, kdim] (+ bias).
  auto linear = [&](const float *a, uint32_t kdim, const float *w, const float *bias,
                    void *out, uint32_t n, int mode, uint32_t part) {
    const float *a_lo = m.precise ? a + uint64_t(T) * kdim : nullptr;
    const float *w_lo = m.precise ? w + uint64_t(n) * kdim : nullptr;
    return tx_linear(ctx, a, a_lo, w, w_lo, bias, out, T, n, kdim, mode, TX_F32, part, stream);
  };

#define TX_TRY(call)              \
  do {                            \
    const int rc_ = (call);       \
    if (rc_ != TX_OK) return rc_; \
  } while (0)

  TX_TRY(tx_bert_embed(ctx, ids, cu_seqlens, nseq, 0, T, m.words, m.positions, m.types, m.vocab,
                       m.max_pos, m.ln_w, m.ln_b, m.eps, x, xs, TX_F32, hid, stream));
  for (uint32_t l = 0; l < m.layers; ++l) {
    const TxBertLayer &w = m.layer[l];
    if (!w.qkv_w || !w.qkv_b || !w.o_w || !w.o_b || !w.ln1_w || !w.ln1_b || !w.i_w || !w.i_b ||
        !w.out_w || !w.out_b || !w.ln2_w || !w.ln2_b)
      return tx::ctx_fail(ctx, TX_EINVAL, "bert_forward: null weight pointer");
    // q, k, v: three [T, hidden] matrices, one after the other.
    TX_TRY(linear(xs, hid, w.qkv_w, w.qkv_b, qkv, 3 * hid, TX_LINEAR_STORE_F32, hid));
    TX_TRY(tx_attention_varlen(ctx, qkv, qkv + plane, qkv + 2 * plane, cu_seqlens, cu_host, nseq,
                               T, max_len, att, H, H, D, TX_F32, TX_F32, /*causal=*/0, scale,
                               nullptr, nullptr, 0.f, 0.f, stream));
    TX_TRY(tx_split_tf32(ctx, att, atts, plane, stream));
    TX_TRY(linear(atts, hid, w.o_w, w.o_b, x, hid, TX_LINEAR_ADD_F32, hid));
    TX_TRY(tx_layer_norm_rows(ctx, x, w.ln1_w, w.ln1_b, x, xs, TX_F32, T, hid, m.eps, stream));
    TX_TRY(linear(xs, hid, w.i_w, w.i_b, act, inter, TX_LINEAR_GELU_SPLIT, inter));
    TX_TRY(linear(act, inter, w.out_w, w.out_b, x, hid, TX_LINEAR_ADD_F32, hid));
    TX_TRY(tx_layer_norm_rows(ctx, x, w.ln2_w, w.ln2_b, x, xs, TX_F32, T, hid, m.eps, stream));
  }
  TX_TRY(tx_pool_project(ctx, x, TX_F32, nullptr, cu_seqlens, pooled, nseq, 0, hid, hid,
                         /*first_token=*/1, nullptr, 0.f, stream));
#undef TX_TRY
  return TX_OK;
}

}  // extern "C"
