/* tessattn.h -- C ABI of libtessattn.so, the B200 (sm_100a) encoder-attention library.
 *
 * This library replaces the attention hot path of Tessery's native Metal runtime
 * (src/metal_inference/native/runtime.mm, bound over ctypes in
 * src/metal_inference/metal.py:27-91).  Every entry point below names the reference
 * interface it stands in for.  Conventions shared by all entry points:
 *
 *   - Plain C types only: opaque handles, raw pointers, sizes.  No C++ or framework
 *     types cross the boundary.
 *   - Status codes (int): TX_OK (0), TX_EINVAL (1, rejected before any GPU work, or by
 *     a kernel's own argument check, reported at the next tx_sync / tx_finish),
 *     TX_ECUDA (2, CUDA runtime error), TX_ETIMEOUT (3, a bounded device-side wait gave
 *     up; the kernel returned and the context stays usable).  tx_last_error() gives a
 *     one-line, payload-free description for the calling context.
 *     The reference returns 0/1 from every mi_* call (runtime.mm:81-297); 0 keeps the
 *     same meaning and every failure is non-zero.
 *   - The library never aborts the process and never frees caller memory.
 *   - One context per device; calls on one context are serialised by a mutex, as the
 *     reference serialises commands per runtime (metal.py:191, 375-414).
 */
#ifndef TESSATTN_H
#define TESSATTN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  TX_OK = 0,
  TX_EINVAL = 1,
  TX_ECUDA = 2,
  TX_ETIMEOUT = 3
};

/* Element types of attention inputs/outputs.  TX_BF16X2 (tx_rms_norm_rows output only): a
 * bf16 pair -- hi = bf16(v) in the output array, lo = bf16(v - hi) in a second array of the
 * same shape right after it -- which keeps about 16 significant bits of v. */
enum { TX_F32 = 0, TX_BF16 = 1, TX_BF16X2 = 2 };

/* ABI version; bumped on any signature change.  The Python loader refuses a library
 * whose version differs, as metal.py:84-90 refuses a stale native build. */
uint32_t tx_abi_version(void);

/* ---- lifecycle -------------------------------------------------------------------- */

/* Replaces mi_create (runtime.mm:43-58).  Opens a context on CUDA device `device`
 * (stream, events, status word).  Returns NULL when no usable sm_100 device exists;
 * the reason is available from tx_last_error(NULL). */
void *tx_create(int device);

/* Replaces mi_destroy (runtime.mm:60-62).  Waits for queued work, frees every buffer
 * and scratch allocation the context owns. */
void tx_destroy(void *ctx);

/* Payload-free description of the last failure on `ctx` (or of the last failed
 * tx_create when ctx is NULL).  The string stays valid until the next call on ctx. */
const char *tx_last_error(void *ctx);

/* Number of streaming multiprocessors of the context's device. */
int tx_device_sms(void *ctx);

/* Limit, in SM clock cycles, of each bounded wait inside the tensor-core attention
 * kernel launched by this context (0 restores the default, about one second).  A wait
 * that runs out makes the kernel drain what it has in flight and return, and the next
 * tx_sync / tx_finish reports TX_ETIMEOUT; the context stays usable.  Counterpart of the
 * status check of mi_finish (runtime.mm:217-253): lets a test make that error path run
 * without any fault.  Returns TX_EINVAL for a negative limit. */
int tx_set_wait_limit(void *ctx, int64_t cycles);

/* Name of the last attention kernel this context launched ("tc_bf16_d128",
 * "simt", "d32_f32") or "" -- the route a call took, as the reference's tests read
 * kernel names from MetalRuntime.diagnostics()["dispatches"] (metal.py:208-234). */
const char *tx_last_kernel(void *ctx);

/* Number of kernels this context has launched since it was created (every entry
 * point counts its own launches), so callers can report launches per step. */
uint64_t tx_launch_count(void *ctx);

/* ---- device buffers --------------------------------------------------------------- */

/* Replaces mi_buffer (runtime.mm:65-76).  Allocates `size` bytes of device memory,
 * copying `host` into it when non-NULL, zero-filled otherwise.  NULL on failure
 * (size 0 included, as in the reference). */
void *tx_buffer(void *ctx, const void *host, uint64_t size);

/* Replaces mi_free (runtime.mm:78-80). */
void tx_free(void *buffer);

/* Memory accounting of the context's buffers (the counters metal.py:94-119 keeps per
 * Buffer and diagnostics() reports, metal.py:208-234): out[0] bytes live now, out[1] the
 * most bytes ever live at once, out[2] allocations made, out[3] bytes allocated in all.
 * Scratch the context owns for its kernels is not counted. */
int tx_memory_stats(void *ctx, uint64_t *out);

/* Replaces mi_read (runtime.mm:81-86): synchronous device-to-host copy of the first
 * `bytes` bytes.  Returns 1 when bytes exceeds the buffer size. */
int tx_read(void *buffer, void *out, uint64_t bytes);

/* Host-to-device copy into an existing buffer (the reference writes shared memory
 * directly; CUDA needs an explicit copy).  Returns 1 when bytes exceeds the size. */
int tx_write(void *buffer, const void *src, uint64_t bytes);

/* Device address and size of a buffer, for the typed entry points below. */
void *tx_buffer_device_ptr(void *buffer);
uint64_t tx_buffer_size(void *buffer);

/* Page-locked host memory for asynchronous copies (e2e measurement, staging). */
void *tx_host_alloc(uint64_t size);
void tx_host_free(void *ptr);

/* ---- commands (one stream-ordered batch of dispatches) ---------------------------- */

/* Replaces mi_begin (runtime.mm:88-107).  Returns 1 when a command is already open. */
int tx_begin(void *ctx);

/* Replaces mi_dispatch (runtime.mm:109-146).  `name` selects a kernel by the
 * reference's kernel names ("rms_norm", "rope", "attention", "attention_tiled",
 * "attention_tail_32", "attention_tail_128", "pool_project", "embedding4", "linear4",
 * "linear4_tiled", "linear4_tail", "linear4_16x32_k64", "linear4_32x32_k64",
 * "linear4_small3", "silu_gate", "add"; fp32 like the reference) plus this library's
 * additions ("attention_d32", "qk_norm_rope").  `buffers` are tx_buffer handles in the
 * reference's slot order, `params` is the reference's 64-byte Params block
 * (kernels.metal:5-8, packed "<12I4f" by metal.py:596-614), and `threads`/`group`
 * are the reference's Metal grid, from which the row/batch counts are derived exactly
 * as the reference kernels derive them.  The CUDA grid is chosen by the library. */
int tx_dispatch(void *ctx, const char *name, void **buffers, uint32_t count,
                const void *params, uint32_t size, uint64_t threads, uint32_t group);

/* Replaces mi_finish (runtime.mm:217-253): waits for the command, checks CUDA errors
 * and the device status word, records the command's GPU time. */
int tx_finish(void *ctx);

/* Replaces mi_abort (runtime.mm:289-297).  CUDA cannot discard launched work, so
 * abort waits for it, then drops the open command and its timing. */
void tx_abort(void *ctx);

/* Replaces mi_gpu_seconds (runtime.mm:285-287): device time of the last finished
 * command (CUDA events), or -1 when unavailable. */
double tx_gpu_seconds(void *ctx);

/* Replace mi_profile_enable / mi_profile_read (runtime.mm:256-283): per-dispatch
 * device timings (one CUDA event pair per dispatch) for the next commands. */
int tx_profile_enable(void *ctx, int enabled);
int tx_profile_read(void *ctx, double *seconds, uint32_t count);

/* Per-kernel device times of the typed attention entry points (no reference
 * counterpart; the typed calls have no command to profile).  While enabled, every
 * kernel launch of a tx_attention_* call is bracketed by a CUDA event pair on the
 * call's stream (which also keeps the attention kernel from overlapping the prologue
 * launch before it); tx_kernel_times waits for the last call's launches (the last chunk
 * of a host-buffer call) and writes their durations in launch order: the q/k prologue
 * when the call ran one, then the attention kernel.  *count = number of launches;
 * TX_EINVAL when cap is smaller. */
int tx_kernel_timing(void *ctx, int enabled);
int tx_kernel_times(void *ctx, double *seconds, uint32_t cap, uint32_t *count);

/* ---- typed attention entry points -------------------------------------------------

 * These replace the Params-block route for callers that hold device pointers.  They
 * implement the operator reached through MetalRuntime._attention (metal.py:532-569)
 * and, when `q_norm_w`/`k_norm_w` are non-NULL, the q/k RMSNorm + RoPE calls that
 * precede it in Qwen3Backend.forward (qwen3.py:216-237).
 *
 * Layouts (row-major, d contiguous):
 *   padded: q/out [batch, seq, heads, dim], k/v [batch, seq, kv_heads, dim]
 *   varlen: q/out [total, heads, dim],      k/v [total, kv_heads, dim],
 *           sequence s spans rows cu_seqlens[s] .. cu_seqlens[s+1]-1.
 * Semantics (kernels.metal:78-103): query row at position p of a sequence of length n
 * attends to keys [0, causal ? min(p+1, n) : n); padded query rows (p >= n) are
 * computed too and attend to [0, n); kv head = head / (heads / kv_heads).  Padded k/v
 * rows (positions >= n) are never attended and may hold any value, NaN and Inf included
 * (the reference never reads them, kernels.metal:89-99).
 * `scale` multiplies q.k (the reference passes dim^-0.5).
 * in_dtype: TX_F32 or TX_BF16 for q, k, v.  out_dtype: TX_F32 or TX_BF16.
 * q_norm_w / k_norm_w: bf16 bit patterns [dim] (kernels.metal:53-63 reads its weight
 * as bf16); a non-NULL weight applies RMSNorm + RoPE to that input first (NULL: the
 * input is used as given, e.g. k already normalised by tx_qk_norm_rope).  eps/theta as
 * in the reference Params.
 * Positions for RoPE: the padded index (kernels.metal:68) or the index within the
 * sequence (varlen).
 * lengths / cu_seqlens: device arrays read by the kernels.  lengths_host /
 * cu_seqlens_host: optional host copies; when given, they are validated and used to
 * build an exact, longest-first work list; when NULL the work list covers every tile
 * and the kernels skip empty tiles by reading the device array.
 * Short sequences (seq, or max_len for varlen, at most 32; dim 128; bf16 in; at most 4
 * query heads per kv head) run as one kernel launch with the q/k prologue inside; a
 * varlen sequence found longer than 32 on the device (cu_seqlens_host NULL and a wrong
 * max_len) is reported as TX_EINVAL by tx_sync / tx_finish.
 * stream: a cudaStream_t, or NULL for the context's stream.
 * Returns TX_OK when the work has been queued; errors from inside kernels are reported
 * by tx_sync / tx_finish. */
int tx_attention_padded(void *ctx, const void *q, const void *k, const void *v,
                        const uint32_t *lengths, const uint32_t *lengths_host, void *out,
                        uint32_t batch, uint32_t seq, uint32_t heads, uint32_t kv_heads,
                        uint32_t dim, int in_dtype, int out_dtype, int causal, float scale,
                        const uint16_t *q_norm_w, const uint16_t *k_norm_w, float eps,
                        float theta, void *stream);

int tx_attention_varlen(void *ctx, const void *q, const void *k, const void *v,
                        const int32_t *cu_seqlens, const int32_t *cu_seqlens_host,
                        uint32_t nseq, uint32_t total, uint32_t max_len, void *out,
                        uint32_t heads, uint32_t kv_heads, uint32_t dim, int in_dtype,
                        int out_dtype, int causal, float scale, const uint16_t *q_norm_w,
                        const uint16_t *k_norm_w, float eps, float theta, void *stream);

/* Host-buffer forms of the two entry points above: q, k, v, out, lengths / cu_seqlens and
 * the norm weights are HOST pointers (page-locked memory, e.g. from tx_host_alloc, is
 * copied directly; pageable q/k/v/out go through page-locked staging the context keeps,
 * copied by a few host threads chunk by chunk beside the transfers).  They stand in for the reference's
 * host-side sequence around one attention dispatch -- Buffer uploads (metal.py:94-119),
 * the dispatch (metal.py:532-569) and the read-back (metal.py:650-662) -- in one call.
 * The sequences are split into chunks of whole sequences; chunk i's rows are copied in
 * while chunk i-1 is computed and chunk i-2 copied out, so transfer in both directions
 * overlaps and the kernels hide behind it.  In the padded layout the valid k and v rows
 * are copied, in spans that take short padding gaps between sequences along (fewer
 * copies; padded rows are never attended).  Results equal the
 * device-pointer entry points' bit for bit.  Returns when the output is in `out` (kernel errors included); device
 * memory for the copies is kept by the context and grows to the largest call. */
int tx_attention_padded_host(void *ctx, const void *q, const void *k, const void *v,
                             const uint32_t *lengths, void *out, uint32_t batch, uint32_t seq,
                             uint32_t heads, uint32_t kv_heads, uint32_t dim, int in_dtype,
                             int out_dtype, int causal, float scale, const uint16_t *q_norm_w,
                             const uint16_t *k_norm_w, float eps, float theta);

int tx_attention_varlen_host(void *ctx, const void *q, const void *k, const void *v,
                             const int32_t *cu_seqlens, uint32_t nseq, uint32_t total, void *out,
                             uint32_t heads, uint32_t kv_heads, uint32_t dim, int in_dtype,
                             int out_dtype, int causal, float scale, const uint16_t *q_norm_w,
                             const uint16_t *k_norm_w, float eps, float theta);

/* Bytes the last host-buffer attention call of this context copied: out[0] host to
 * device (q rows, the k/v spans, lengths or cu_seqlens, norm weights, work lists),
 * out[1] device to host (the output rows).  No reference counterpart: the reference's
 * uploads are whole Buffers (metal.py:94-119); this reports what the chunked copies of
 * the two entry points above moved, for throughput accounting. */
int tx_host_copy_bytes(void *ctx, uint64_t *out);

/* Standalone fused q/k prologue (qwen3.py:216-237 as one pass): RMSNorm with bf16
 * weights then split-half RoPE, reading q/k in `in_dtype` and writing bf16 or f32
 * (`out_dtype`) to q_out/k_out (which may alias q/k when the types match).  q (with
 * q_out, q_norm_w) or k (with k_out, k_norm_w) may be NULL to transform only the other.
 * positions: padded layout when cu_seqlens is NULL (rows = batch*seq tokens,
 * position = token % seq), else index within each varlen sequence.
 * lengths (device, padded layout, may be NULL): tokens at positions >= their
 * sequence's length are skipped and their output rows left unwritten -- the rows no
 * attention reads when the output is k. */
int tx_qk_norm_rope(void *ctx, const void *q, const void *k, void *q_out, void *k_out,
                    uint32_t tokens, uint32_t seq, const int32_t *cu_seqlens, uint32_t nseq,
                    const uint32_t *lengths, uint32_t heads, uint32_t kv_heads, uint32_t dim,
                    int in_dtype, int out_dtype, const uint16_t *q_norm_w,
                    const uint16_t *k_norm_w, float eps, float theta, void *stream);

/* Embedding pooling after the last layer (replaces the "pool_project" dispatch,
 * kernels.metal:339-349, and, with norm_w, the final rms_norm before it,
 * qwen3.py:281-290).  For each sequence b, takes one row of x -- the last valid token
 * (first_token = 0, Qwen3 last-token pooling) or the first (first_token = 1, BERT CLS,
 * bert.py:236-244) -- optionally RMS-normalises it over all `cols` columns with the bf16
 * weight norm_w (eps; x * rsqrt(mean(x^2) + eps) * w, as kernels.metal:53-63), and
 * writes its first `dim` columns divided by their L2 norm to out[b, 0:dim] (fp32).
 * x: in_dtype (TX_F32 or TX_BF16), padded [batch, seq, cols] with `lengths` (device
 * u32[batch]), or packed [total, cols] with `cu_seqlens` (device i32[batch+1]; exactly
 * one of the two is non-NULL; seq is ignored for packed).  A sequence without a valid
 * row (length 0, length > seq, empty packed range) gets a NaN row.  dim <= cols.
 * stream: a cudaStream_t, or NULL for the context's stream. */
int tx_pool_project(void *ctx, const void *x, int in_dtype, const uint32_t *lengths,
                    const int32_t *cu_seqlens, float *out, uint32_t batch, uint32_t seq,
                    uint32_t cols, uint32_t dim, int first_token, const uint16_t *norm_w,
                    float eps, void *stream);

/* Allocation-free variant of tx_attention_padded (no counterpart in the reference,
 * whose Metal runtime always owns its buffers).  For callers that may not allocate
 * device memory -- hosts that reserve all memory up front and treat a later
 * cudaMalloc as an error, since it can fail under memory pressure and stall the
 * device -- and that therefore cannot create a context either.  It takes no context.
 * Path: the tensor-core kernel only (bf16 q/k/v on the current device, head_dim 128,
 * at most 64 query heads); q_norm_w (or NULL) applies the fused q RMSNorm + RoPE, while
 * k must already be normalised (tx_qk_norm_rope).  Its only scratch, the work list, is
 * a static device array of 16384 units (one unit = 128 query rows of a pair of query
 * heads, or of one head when the query heads per kv head are odd:
 * batch * heads/2 (or heads) * ceil(seq/128) units); larger problems are rejected with
 * TX_EINVAL before any pointer is used.  The first call on a device looks up that array's
 * device address (with the device current) and loads the kernel's code, which places
 * the array and the code in device memory: make one such call per device at start-up,
 * before memory is reserved and before any stream capture.  All calls share the array
 * and it keeps the last call's contents: calls whose work overlaps on the GPU race.
 * status (required, device int): zeroed by this call, then set by the kernel to
 * TX_ETIMEOUT | site << 8 if a bounded wait gives up; read it after the stream has
 * drained.  Returns TX_OK once queued on `stream` (NULL: the legacy default stream),
 * TX_EINVAL while `stream` is being captured (the work list is copied from host memory
 * that the next call overwrites). */
int tx_attention_padded_noalloc(const void *q, const void *k, const void *v,
                                const uint32_t *lengths, const uint32_t *lengths_host,
                                void *out, uint32_t batch, uint32_t seq, uint32_t heads,
                                uint32_t kv_heads, int out_dtype, int causal, float scale,
                                const uint16_t *q_norm_w, float eps, float theta, int *status,
                                void *stream);

/* ---- the Qwen3 embedding forward around the attention -----------------------------

 * The layer loop of Qwen3Backend.forward (qwen3.py:112-296) is built from these plus
 * tx_attention_varlen and tx_pool_project.  Weights come as the reference stores them
 * (qwen3.py:70-73): uint4 codes `packed` [rows, cols / 8] (code i of a word in bits
 * 4i..4i+3), bf16 `scales` and `biases` [rows, cols / 64]; element (r, c) =
 * code * scale + bias (weight4, kernels.metal:11-19).  All pointers are device pointers;
 * stream NULL: the context's stream. */

/* Epilogues of tx_linear. */
enum {
  TX_LINEAR_STORE_F32 = 0,  /* out fp32 [m, n] = x . w^T */
  TX_LINEAR_STORE_BF16 = 1, /* out bf16 [m, n] */
  TX_LINEAR_ADD_F32 = 2,    /* out fp32 [m, n] += x . w^T (the residual add, qwen3.py:151-152) */
  TX_LINEAR_GATED_BF16 = 3, /* out bf16 [m, n / 2]: silu(gate) * up, w rows interleaved in
                               blocks of 128 gate then 128 up rows (gated4 + silu_gate,
                               kernels.metal:333-337, 609-733); bf16 operands only */
  TX_LINEAR_GELU_SPLIT = 4  /* out = gelu(x . w^T + bias) (erf form, gelu_f32,
                               kernels.metal:381-391) written as the next GEMM's split
                               operand: hi [m, n] then lo [m, n], each in the operand
                               format (bf16, or fp32 holding hi = TF32-rounded value and
                               lo = value - hi) */
};

/* Dequantises a uint4 weight matrix once into bf16 [rows, cols] (out), the operand layout
 * of tx_linear, and, when out_lo is non-NULL, the rounding residue of every weight into
 * out_lo (the lo half of a bf16 pair).  Replaces the per-use decode of weight4
 * (kernels.metal:11-19) inside the reference's linear4* kernels.  cols % 64 == 0; out and
 * out_lo 16-byte aligned. */
int tx_dequant4(void *ctx, const uint32_t *packed, const uint16_t *scales,
                const uint16_t *biases, uint16_t *out, uint16_t *out_lo, uint32_t rows,
                uint32_t cols, void *stream);

/* fp32 x [n] as a bf16 pair: out[i] = bf16(x[i]), out[n + i] = bf16(x[i] - out[i]). */
int tx_split_bf16(void *ctx, const float *x, uint16_t *out, uint64_t n, void *stream);

/* Replaces the "embedding4" dispatch (kernels.metal:21-28): out fp32 [tokens, cols], row
 * t = dequantised row ids[t] of the table.  An id >= vocab gives a NaN row and is reported
 * as TX_EINVAL by the next tx_sync / tx_finish.  cols % 64 == 0. */
int tx_embedding4(void *ctx, const uint32_t *ids, uint32_t tokens, const uint32_t *packed,
                  const uint16_t *scales, const uint16_t *biases, float *out, uint32_t cols,
                  uint32_t vocab, void *stream);

/* Replaces the "rms_norm" dispatch on the hidden rows (kernels.metal:53-63, called at
 * qwen3.py:135-143): out[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * bf16(w), written bf16
 * (out_dtype TX_BF16, the projections' operand) or fp32.  x fp32 [rows, cols], cols % 4
 * == 0. */
int tx_rms_norm_rows(void *ctx, const float *x, const uint16_t *w, void *out, int out_dtype,
                     uint32_t rows, uint32_t cols, float eps, void *stream);

/* Replaces the reference's _linear4 / _gated4 routing (metal.py:416-530) on dequantised
 * weights and its f32 projections matmul_bias_f32* (kernels.metal:438-487, bert.py:127-133):
 * out = x [m, k] times w [n, k] transposed, plus bias (fp32 [n], or NULL), fp32
 * accumulation on tensor cores, epilogue `mode` (TX_LINEAR_*).  fmt TX_BF16: bf16
 * operands; TX_F32: fp32 operands read as TF32.  With x_lo and w_lo (both or neither), the
 * lo parts of split operands, the product is x.w + x.w_lo + x_lo.w: bf16 pairs carry about
 * 16 significant bits of each operand, TF32 pairs (hi = TF32-rounded value, lo = value -
 * hi, see tx_split_tf32) about 22, the fp32 path's accuracy; the gated epilogue then writes a
 * bf16 pair (hi [m, n/2] then lo [m, n/2]).  part: outputs split by columns -- column
 * block p of width `part` goes to its own [m, part] matrix, the p-th of n / part
 * consecutive ones (part == n: one [m, n] matrix).  Needs n and part multiples of 128
 * (256 for the gated epilogue), k a multiple of 64 (bf16) or 32 (TF32), pointers 16-byte
 * aligned; otherwise TX_EINVAL. */
int tx_linear(void *ctx, const void *x, const void *x_lo, const void *w, const void *w_lo,
              const float *bias, void *out, uint32_t m, uint32_t n, uint32_t k, int mode,
              int fmt, uint32_t part, void *stream);

/* The whole forward as one call: the layer loop of Qwen3Backend.forward
 * (qwen3.py:112-296; its per-layer dispatch sequence is qwen3.py:191-280, the final norm
 * and last-token pooling :281-290) queued on the device from native code.  The caller
 * fills the model description once (device pointers to weights already dequantised by
 * tx_dequant4, gate and up rows interleaved for TX_LINEAR_GATED_BF16) and then issues one
 * call per batch; nothing is allocated by the call.  Sequences are packed by cu_seqlens
 * (no padded rows).  Fast mode: bf16 projection operands, the tensor-core attention.
 * Precise mode (`precise` != 0): every projection matrix is followed in memory by its
 * bf16 rounding residues (tx_dequant4 with out_lo = w + n * k), activations enter each
 * projection as bf16 pairs, q/k/v and the attention are fp32. */
typedef struct {
  const uint16_t *input_norm, *post_norm;  /* bf16 [hidden] */
  const uint16_t *q_norm, *k_norm;         /* bf16 [head_dim] */
  const uint16_t *q_proj, *k_proj, *v_proj; /* bf16 [heads|kv_heads * head_dim, hidden] */
  const uint16_t *o_proj;                  /* bf16 [hidden, heads * head_dim] */
  const uint16_t *gate_up;                 /* bf16 [2 * intermediate, hidden], interleaved */
  const uint16_t *down;                    /* bf16 [hidden, intermediate] */
} TxQwen3Layer;

typedef struct {
  uint32_t hidden, intermediate, layers, heads, kv_heads, head_dim, vocab;
  float eps, theta;
  int precise;
  const uint32_t *embed_packed;            /* uint4 table [vocab, hidden / 8] */
  const uint16_t *embed_scales, *embed_biases; /* bf16 [vocab, hidden / 64] */
  const uint16_t *final_norm;              /* bf16 [hidden] */
  const TxQwen3Layer *layer;               /* host array of `layers` entries */
} TxQwen3Model;

/* Bytes of device workspace tx_qwen3_forward needs for `tokens` packed tokens (0 when the
 * model's shapes are not supported: head_dim 128, hidden, heads * head_dim and kv_heads *
 * head_dim multiples of 256, intermediate a multiple of 128). */
uint64_t tx_qwen3_workspace_bytes(const TxQwen3Model *model, uint32_t tokens);

/* Pooled, L2-normalised embeddings `pooled` (device fp32 [nseq, dimensions]) of the token
 * ids `ids` (device uint32 [cu_host[nseq]]) packed by `cu_seqlens` (device int32 [nseq+1],
 * host copy `cu_host`).  `workspace`: device memory of at least tx_qwen3_workspace_bytes
 * bytes, 256-byte aligned.  Queued on `stream` (NULL: the context's stream); errors of the
 * device side (an id >= vocab, a wait that gave up) come from the next tx_sync. */
int tx_qwen3_forward(void *ctx, const TxQwen3Model *model, const uint32_t *ids,
                     const int32_t *cu_seqlens, const int32_t *cu_host, uint32_t nseq,
                     float *pooled, uint32_t dimensions, void *workspace,
                     uint64_t workspace_bytes, void *stream);

/* ---- the BERT (BGE-small) fp32 forward around the head_dim-32 attention -------------

 * BertBackend.forward (bert.py:104-235) is built from these plus tx_linear (fmt TX_F32,
 * TF32 split operands), tx_attention_varlen and tx_pool_project; tx_bert_forward runs the
 * whole loop.  Weights are fp32 as the reference stores them (bert.py:55-66).  All
 * pointers are device pointers; stream NULL: the context's stream. */

/* fp32 x [n] as the split operand of the TF32 GEMM: out[i] = x[i] rounded to TF32 (kept
 * in fp32), out[n + i] = x[i] - out[i] (exact).  n % 4 == 0, 16-byte aligned pointers. */
int tx_split_tf32(void *ctx, const float *x, float *out, uint64_t n, void *stream);

/* Replaces the "layer_norm" dispatch (kernels.metal:362-373) on hidden rows: out[r] =
 * (x[r] - mean) / sqrt(var + eps) * w + b (out may be x), and, when `pair` is non-NULL, the
 * next GEMM's split operand of out: split TX_F32 (TF32 pair, hi [rows, cols] then lo, fp32)
 * or TX_BF16X2 (bf16 pair).  cols at most 1024. */
int tx_layer_norm_rows(void *ctx, const float *x, const float *w, const float *b, float *out,
                       void *pair, int split, uint32_t rows, uint32_t cols, float eps,
                       void *stream);

/* Replaces the "embedding_position" dispatch (kernels.metal:353-361) followed by the
 * embeddings' layer_norm (bert.py:174-190): out[t] = LayerNorm(words[ids[t]] + types[0] +
 * positions[pos(t)]), pos(t) = index of t inside its sequence (packed by cu_seqlens with
 * nseq sequences, or t % seq when cu_seqlens is NULL); `pair` / `split` as in
 * tx_layer_norm_rows.  An id >= vocab or a position >= max_pos gives a NaN row and
 * TX_EINVAL at the next tx_sync. */
int tx_bert_embed(void *ctx, const uint32_t *ids, const int32_t *cu_seqlens, uint32_t nseq,
                  uint32_t seq, uint32_t tokens, const float *words, const float *positions,
                  const float *types, uint32_t vocab, uint32_t max_pos, const float *ln_w,
                  const float *ln_b, float eps, float *out, void *pair, int split, uint32_t cols,
                  void *stream);

/* One encoder layer's weights.  Projection matrices are TF32 split operands of their fp32
 * weights (tx_split_tf32: hi [n, k] then lo [n, k]); qkv is the query, key and value
 * matrices stacked ([3 * hidden, hidden], biases likewise); LayerNorm weights and biases
 * fp32 [hidden]. */
typedef struct {
  const float *qkv_w, *qkv_b;   /* [2][3 hidden, hidden], [3 hidden] */
  const float *o_w, *o_b;       /* attention.output.dense */
  const float *ln1_w, *ln1_b;   /* attention.output.LayerNorm */
  const float *i_w, *i_b;       /* intermediate.dense [2][intermediate, hidden] */
  const float *out_w, *out_b;   /* output.dense [2][hidden, intermediate] */
  const float *ln2_w, *ln2_b;   /* output.LayerNorm */
} TxBertLayer;

typedef struct {
  uint32_t hidden, intermediate, layers, heads, vocab, max_pos;
  float eps;
  int precise;                  /* 1: three TF32 products per GEMM (fp32 accuracy); 0: one */
  const float *words, *positions, *types; /* embedding tables [rows, hidden] */
  const float *ln_w, *ln_b;     /* embeddings.LayerNorm */
  const TxBertLayer *layer;     /* host array of `layers` entries */
} TxBertModel;

/* Bytes of device workspace tx_bert_forward needs for `tokens` packed tokens (0 when the
 * shapes are not supported: hidden and intermediate multiples of 128, hidden at most
 * 1024, hidden % heads == 0). */
uint64_t tx_bert_workspace_bytes(const TxBertModel *model, uint32_t tokens);

/* CLS embeddings `pooled` (device fp32 [nseq, hidden], L2-normalised: pool_project with
 * first_token, kernels.metal:339-349) of token ids `ids` (device uint32 [cu_host[nseq]])
 * packed by `cu_seqlens` (device, host copy `cu_host`): embeddings, then per layer the
 * fused q/k/v projection, bidirectional attention over each sequence's tokens, the output
 * projection added to the residual stream and LayerNorm, the GELU MLP added and LayerNorm
 * (bert.py:191-231).  Nothing is allocated by the call. */
int tx_bert_forward(void *ctx, const TxBertModel *model, const uint32_t *ids,
                    const int32_t *cu_seqlens, const int32_t *cu_host, uint32_t nseq,
                    float *pooled, void *workspace, uint64_t workspace_bytes, void *stream);

/* Number of CUDA devices visible to this process (0 when none or on error): the devices
 * a sharded caller creates one context on each. */
int tx_device_count(void);

/* Waits for all work queued on `stream` (NULL: context stream) and reports kernel
 * errors, including device-side wait timeouts, as a status code. */
int tx_sync(void *ctx, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TESSATTN_H */
