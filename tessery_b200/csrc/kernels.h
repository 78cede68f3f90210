// Host-side launch interface between the C ABI (runtime.cu) and the kernel files.
// All launchers enqueue on `stream` and return cudaGetLastError() of the launch.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace tx {

// One attention problem, in element units.  Pointers are device addresses.
struct AttnProblem {
  const void *q, *k, *v;
  void *out;
  const uint32_t *lengths;   // padded layout: [batch] valid lengths (device)
  const int32_t *cu_seqlens; // varlen layout: [nseq+1] offsets (device); NULL = padded
  uint32_t batch;            // padded: batch; varlen: nseq
  uint32_t seq;              // padded: L; varlen: max sequence length
  uint32_t total;            // varlen: total rows; padded: batch*seq
  uint32_t heads, kv_heads, dim;
  int in_dtype, out_dtype;   // TX_F32 / TX_BF16
  int causal;
  float scale;
};

// Reference-semantics kernels (kernels.metal:53-103 restated for CUDA).
cudaError_t launch_rms_norm(const float *x, const uint16_t *w, float *out, uint32_t rows,
                            uint32_t cols, float eps, cudaStream_t stream);
cudaError_t launch_rope(float *x, uint32_t n, uint32_t heads, uint32_t seq, uint32_t dim,
                        float theta, cudaStream_t stream);
// General attention: any dim <= 256, f32/bf16 in, f32/bf16 out, padded or varlen.
cudaError_t launch_attention_simt(const AttnProblem &p, cudaStream_t stream);
// head_dim 32, fp32 in and out: Q.K^T and P.V on tensor cores (TF32 split operands), the
// softmax on the FP32 pipe (attn_d32_tc.cu); 64-key tiles while the grid fits one wave
// at two CTAs per SM, 32-key tiles at three CTAs per SM beyond.  `status`: the device
// status word.
bool d32_tc_supported(const AttnProblem &p);
cudaError_t launch_attention_d32_tc(const AttnProblem &p, int *status, cudaStream_t stream,
                                    int num_sms);
// head_dim 128, fp32 in and out: scores on tensor cores (TF32 split operands), the softmax
// and P.V on the FP32 pipe (attn_f32_tc.cu).
bool f32_tc_supported(const AttnProblem &p);
cudaError_t launch_attention_f32_tc(const AttnProblem &p, int *status, cudaStream_t stream);

// Fused q/k RMSNorm + RoPE prologue.  Rows: tokens*heads (q) and tokens*kv_heads (k).
// q or k may be NULL to transform only the other one.  With `lengths` (padded layout),
// tokens at positions >= their sequence's length are skipped (their rows are left
// untouched): used for k, whose padded rows no attention reads.
struct PrologueProblem {
  const void *q, *k;
  void *q_out, *k_out;
  uint32_t tokens, seq;       // padded: position = token % seq
  const int32_t *cu_seqlens;  // varlen: position = token - cu_seqlens[seq_of(token)]
  uint32_t nseq;
  uint32_t heads, kv_heads, dim;
  int in_dtype, out_dtype;
  const uint16_t *q_w, *k_w;
  float eps, theta;
  const uint32_t *lengths;    // optional, padded layout only
  float inv_freq[128];        // theta^(-2c/dim) per column c < dim/2 (set by the launcher)
};
cudaError_t launch_qk_norm_rope(const PrologueProblem &p, cudaStream_t stream);

// Embedding pooling: one row per sequence (last valid or first token), optional
// RMSNorm with a bf16 weight over all cols, L2 normalisation of the first dim columns.
struct PoolProblem {
  const void *x;                // padded [batch, seq, cols] or packed [total, cols]
  int in_dtype;                 // 0 f32, 1 bf16
  const uint32_t *lengths;      // padded layout
  const int32_t *cu_seqlens;    // packed layout (exactly one of lengths / cu_seqlens)
  float *out;                   // [batch, dim]
  uint32_t batch, seq, cols, dim;
  int first_token;
  const uint16_t *norm_w;       // bf16 [cols] or nullptr
  float eps;
  bool vector_ok;               // set by the launcher
};
cudaError_t launch_pool_project(const PoolProblem &p, cudaStream_t stream);

// Short sequences (at most 32 tokens each), head_dim 128, bf16 q/k/v, up to 4 query heads
// per kv head: one CTA per (sequence, kv head) with the q/k RMSNorm + RoPE fused (q_w,
// k_w optional).  A sequence longer than 32 in a device cu_seqlens is reported in
// `status` as a bad argument.
bool short_attention_supported(const AttnProblem &p);
cudaError_t launch_attention_short(const AttnProblem &p, const uint16_t *q_w, const uint16_t *k_w,
                                   float eps, float theta, int *status, cudaStream_t stream);


// Bandwidth-oriented fp32 kernel for head_dim 32 (BERT/BGE shapes).
cudaError_t launch_attention_d32(const AttnProblem &p, cudaStream_t stream);

// tcgen05/TMEM/TMA attention for head_dim 128 with bf16 q/k/v.
// `units` is a device work list (see attn_tc.cu for the encoding), `status` the
// context's device status word.
bool tc_attention_supported(const AttnProblem &p);
// q_norm_w: bf16 q RMSNorm weight [128] applied with RoPE to each Q tile in the kernel
// (NULL: q is used as given).
// after_prologue: the kernel launched just before on `stream` is this library's k
// prologue (the launch may then overlap its tail, programmatic dependent launch).
// wait_cycles: limit of each bounded wait in SM cycles (<= 0: about a second).
// exact_units: the work list was built with host lengths (tc_units_exact).
// k_norm_w: the weights of the k RMSNorm the prologue applied to k in this call (NULL when
// k was not normalised here); with q_norm_w they bound every score, and the kernel then
// takes one pass over each score tile (no row maximum).
cudaError_t launch_attention_tc(const AttnProblem &p, const uint32_t *units, uint32_t n_units,
                                int num_sms, int *status, const uint16_t *q_norm_w, float eps,
                                float theta, cudaStream_t stream, bool after_prologue,
                                long long wait_cycles, bool exact_units,
                                const uint16_t *k_norm_w = nullptr);
// Whether tc_build_units writes units with their lengths (host lengths or cu_seqlens of
// the problem's layout given).
inline bool tc_units_exact(const AttnProblem &p, const uint32_t *lengths_host,
                           const int32_t *cu_host) {
  return p.cu_seqlens ? cu_host != nullptr : lengths_host != nullptr;
}
// Loads the tensor-core kernel's module on the current device (no launch).
cudaError_t tc_preload();
// Host-side work-list construction for launch_attention_tc (same num_sms for both).
// `sorted` is host scratch of tc_max_units words; `work` (tc_work_words words) receives
// the n units grouped by CTA (two words each) followed by grid+1 offsets; returns n.
// The launcher takes `work` (on the device, 8-byte aligned) and n.
uint32_t tc_max_units(const AttnProblem &p);
uint32_t tc_work_words(const AttnProblem &p, int num_sms);
uint32_t tc_grid(uint32_t n_units, int num_sms);
uint32_t tc_build_units(const AttnProblem &p, const uint32_t *lengths_host,
                        const int32_t *cu_host, int num_sms, uint32_t *sorted, uint32_t *work);

// Qwen3 forward pieces (qwen_ops.cu, linear.cu).
cudaError_t launch_dequant4(const uint32_t *packed, const uint16_t *scales,
                            const uint16_t *biases, uint16_t *out, uint16_t *out_lo, uint32_t rows,
                            uint32_t cols, cudaStream_t stream);
cudaError_t launch_embedding4(const uint32_t *ids, uint32_t tokens, const uint32_t *packed,
                              const uint16_t *scales, const uint16_t *biases, float *out,
                              uint32_t cols, uint32_t vocab, int *status, cudaStream_t stream);
// out_kind: 0 fp32, 1 bf16, 2 bf16 pair (hi then lo).
cudaError_t launch_rms_norm_rows(const float *x, const uint16_t *w, void *out, int out_kind,
                                 uint32_t rows, uint32_t cols, float eps, cudaStream_t stream);
cudaError_t launch_split_bf16(const float *x, uint16_t *out, uint64_t n, cudaStream_t stream);
// fp32 kernels behind the reference's Params-block dispatch names (linear4, silu_gate, add).
cudaError_t launch_linear4_f32(const float *x, const uint32_t *packed, const uint16_t *scales,
                               const uint16_t *biases, float *out, uint32_t t0, uint32_t t1,
                               uint32_t cols, uint32_t k, cudaStream_t stream);
cudaError_t launch_silu_gate(float *gate, const float *up, uint64_t n, cudaStream_t stream);
cudaError_t launch_add(const float *a, const float *b, float *out, uint64_t n,
                       cudaStream_t stream);
// Output tile width of the GEMM for these shapes (0: unsupported).
uint32_t linear_tile_n(uint32_t n, uint32_t part, int mode);
// fmt: TX_BF16 (bf16 operands) or TX_F32 (fp32 operands read as TF32); part: output
// column-block width (see linear.cu).
bool linear_supported(uint32_t m, uint32_t n, uint32_t k, int mode, int fmt, uint32_t part,
                      const void *x, const void *w, const void *out);
// x_lo / w_lo (both or neither): the lo parts of split operands; bias fp32 [n] or NULL.
cudaError_t launch_linear(const void *x, const void *x_lo, const void *w, const void *w_lo,
                          const float *bias, void *out, uint32_t m, uint32_t n, uint32_t k,
                          int mode, int fmt, uint32_t part, int *status, long long wait_cycles,
                          cudaStream_t stream);

// ---- BERT fp32 forward (bert_ops.cu) ----
// Word + token-type-0 + absolute-position embeddings of `tokens` tokens, LayerNorm'd; the
// position of a token is its index inside its packed sequence (cu, nseq) or t % seq.
struct BertEmbedProblem {
  const uint32_t *ids;
  const int32_t *cu;  // NULL: padded layout with `seq` rows per sequence
  uint32_t nseq, seq, tokens, cols, vocab, max_pos;
  const float *words, *positions, *types, *ln_w, *ln_b;
  float eps;
  float *out;   // fp32 [tokens, cols]
  void *pair;   // split operand of the next GEMM (or NULL), format `split`
  int split;    // TX_F32: TF32 pair in fp32 containers; TX_BF16X2: bf16 pair
  int *status;
};
bool bert_cols_ok(uint32_t cols);
cudaError_t launch_bert_embed(const BertEmbedProblem &p, cudaStream_t stream);
cudaError_t launch_layer_norm_rows(const float *x, const float *w, const float *b, float *out,
                                   void *pair, int split, uint32_t rows, uint32_t cols, float eps,
                                   cudaStream_t stream);
cudaError_t launch_split_tf32(const float *x, float *out, uint64_t n, cudaStream_t stream);
cudaError_t launch_gelu(float *x, uint32_t n, cudaStream_t stream);
cudaError_t launch_add_bias(float *x, const float *bias, uint32_t n, uint32_t cols,
                            cudaStream_t stream);
cudaError_t launch_silu(const float *x, float *out, uint32_t n, cudaStream_t stream);
cudaError_t launch_transpose(const float *x, float *out, uint32_t rows, uint32_t cols,
                             cudaStream_t stream);
cudaError_t launch_embedding_position(const uint32_t *ids, const float *words,
                                      const float *positions, const float *types, float *out,
                                      uint32_t n, uint32_t cols, uint32_t seq,
                                      cudaStream_t stream);
cudaError_t launch_matmul_f32(const float *a, const float *bt, const float *bias, float *out,
                              uint32_t row0, uint32_t rows, uint32_t cols, uint32_t k,
                              cudaStream_t stream);

// Records `msg` as the context's last error (tx_last_error) and returns `code`: for entry
// points built outside runtime.cu on top of the public ones.
int ctx_fail(void *ctx, int code, const char *msg);

}  // namespace tx
