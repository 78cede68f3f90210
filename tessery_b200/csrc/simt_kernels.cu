// Reference-semantics kernels for libtessattn (sm_100a):
//   rms_norm       -- kernels.metal:53-63 (row RMSNorm, bf16 weight)
//   rope           -- kernels.metal:65-74 (split-half rotation, padded position)
//   attention_simt -- kernels.metal:78-103 (per-(query, head) online softmax), the
//                     general fallback: any head_dim <= 256, f32/bf16, padded/varlen
//   qk_norm_rope   -- the q/k RMSNorm + RoPE sequence of qwen3.py:216-237 fused into
//                     one pass that computes the rotation angles once per token.
#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace tx {

// Inverse frequency theta^(-2c/dim), evaluated in double and rounded once to float so
// that every kernel (and the CPU oracle) uses the same float per column.  The angle is
// then the float product position * inv_freq, as kernels.metal:70 forms it in float.
__device__ __forceinline__ float rope_inv_freq(float theta, uint32_t c, uint32_t dim) {
  return (float)pow((double)theta, -2.0 * (double)c / (double)dim);
}

// Sequence index of packed row `tok` (cu is non-decreasing, cu[0] = 0).
__device__ __forceinline__ uint32_t find_seq(const int32_t *cu, uint32_t nseq, uint32_t tok) {
  uint32_t lo = 0, hi = nseq;  // invariant: cu[lo] <= tok < cu[hi]
  while (hi - lo > 1) {
    uint32_t mid = (lo + hi) >> 1;
    if ((uint32_t)cu[mid] <= tok) lo = mid; else hi = mid;
  }
  return lo;
}

// ---- rms_norm: one warp per row (kernels.metal:53-63) --------------------------------
__global__ void rms_norm_kernel(const float *__restrict__ x, const uint16_t *__restrict__ w,
                                float *out, uint32_t rows, uint32_t cols, float eps) {
  uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  uint32_t lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float *xr = x + (size_t)warp * cols;
  float squares = 0.f;
  for (uint32_t c = lane; c < cols; c += 32) { float v = xr[c]; squares += v * v; }
  float inv = 1.0f / sqrtf(warp_sum(squares) / (float)cols + eps);
  for (uint32_t c = lane; c < cols; c += 32)
    out[(size_t)warp * cols + c] = xr[c] * inv * bf16_bits_to_f32(w[c]);
}

cudaError_t launch_rms_norm(const float *x, const uint16_t *w, float *out, uint32_t rows,
                            uint32_t cols, float eps, cudaStream_t stream) {
  if (!rows) return cudaSuccess;
  uint32_t blocks = (rows + 7) / 8;
  rms_norm_kernel<<<blocks, 256, 0, stream>>>(x, w, out, rows, cols, eps);
  return cudaGetLastError();
}

// ---- rope: one thread per rotated pair (kernels.metal:65-74) --------------------------
__global__ void rope_kernel(float *x, uint32_t n, uint32_t heads, uint32_t seq, uint32_t dim,
                            float theta) {
  uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint32_t half = dim / 2, row = i / half, c = i % half;
  uint32_t pos = (row / heads) % seq;
  float angle = (float)pos * rope_inv_freq(theta, c, dim);
  float s, co;
  sincosf(angle, &s, &co);
  size_t base = (size_t)row * dim;
  float a = x[base + c], b = x[base + c + half];
  x[base + c] = a * co - b * s;
  x[base + c + half] = a * s + b * co;
}

cudaError_t launch_rope(float *x, uint32_t n, uint32_t heads, uint32_t seq, uint32_t dim,
                        float theta, cudaStream_t stream) {
  if (!n) return cudaSuccess;
  rope_kernel<<<(n + 255) / 256, 256, 0, stream>>>(x, n, heads, seq, dim, theta);
  return cudaGetLastError();
}

// ---- general attention: one warp per (query row, head) -------------------------------
// Follows kernels.metal:78-103 operation for operation: lane-strided partial dot,
// warp sum, scale, running maximum, exp correction, running denominator.
template <typename TI, typename TO>
__global__ void attention_simt_kernel(AttnProblem p) {
  const TI *q = (const TI *)p.q, *k = (const TI *)p.k, *v = (const TI *)p.v;
  TO *out = (TO *)p.out;
  uint64_t warp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  uint32_t lane = threadIdx.x & 31;
  uint64_t rows = (uint64_t)p.total * p.heads;
  if (warp >= rows) return;
  uint32_t head = (uint32_t)(warp % p.heads);
  uint32_t token = (uint32_t)(warp / p.heads);
  uint32_t kvhead = head / (p.heads / p.kv_heads);
  uint32_t pos, len;
  uint64_t key0;  // packed row index of key 0 of this sequence
  if (p.cu_seqlens) {
    uint32_t s = find_seq(p.cu_seqlens, p.batch, token);
    int32_t start = p.cu_seqlens[s], stop = p.cu_seqlens[s + 1];
    pos = token - (uint32_t)start;
    len = stop > start ? (uint32_t)(stop - start) : 0u;
    key0 = (uint32_t)start;
  } else {
    uint32_t b = token / p.seq;
    pos = token % p.seq;
    len = min(p.lengths[b], p.seq);
    key0 = (uint64_t)b * p.seq;
  }
  uint32_t end = p.causal ? min(pos + 1, len) : len;
  const uint32_t dim = p.dim;
  float qreg[8], accum[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t c = lane + 32 * i;
    qreg[i] = c < dim ? Elem<TI>::load(q, warp * dim + c) : 0.f;
    accum[i] = 0.f;
  }
  float maximum = -INFINITY, denominator = 0.f;
  for (uint32_t key = 0; key < end; ++key) {
    uint64_t kvrow = (key0 + key) * p.kv_heads + kvhead;
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t c = lane + 32 * i;
      if (c < dim) dot += qreg[i] * Elem<TI>::load(k, kvrow * dim + c);
    }
    float score = warp_sum(dot) * p.scale;
    float next = fmaxf(maximum, score);
    float correction = expf(maximum - next), prob = expf(score - next);
    denominator = denominator * correction + prob;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t c = lane + 32 * i;
      if (c < dim) accum[i] = accum[i] * correction + prob * Elem<TI>::load(v, kvrow * dim + c);
    }
    maximum = next;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t c = lane + 32 * i;
    if (c < dim) Elem<TO>::store(out, warp * dim + c, accum[i] / denominator);
  }
}

cudaError_t launch_attention_simt(const AttnProblem &p, cudaStream_t stream) {
  uint64_t rows = (uint64_t)p.total * p.heads;
  if (!rows) return cudaSuccess;
  uint64_t blocks = (rows + 7) / 8;
  if (blocks > 0x7fffffffull) return cudaErrorInvalidValue;
  dim3 grid((unsigned)blocks), block(256);
  if (p.in_dtype == 0 && p.out_dtype == 0)
    attention_simt_kernel<float, float><<<grid, block, 0, stream>>>(p);
  else if (p.in_dtype == 0)
    attention_simt_kernel<float, uint16_t><<<grid, block, 0, stream>>>(p);
  else if (p.out_dtype == 0)
    attention_simt_kernel<uint16_t, float><<<grid, block, 0, stream>>>(p);
  else
    attention_simt_kernel<uint16_t, uint16_t><<<grid, block, 0, stream>>>(p);
  return cudaGetLastError();
}

// ---- fused q/k RMSNorm + RoPE ------------------------------------------------------
// One warp per token (grid-stride).  Lane l holds E = dim/32 consecutive elements
// [E*l, E*l+E); lanes 0..15 hold the first half of the row, lanes 16..31 the second,
// so each rotation pair (c, c+dim/2) sits in lanes l and l^16.  The rotation angles
// depend only on the position, so they are computed once per token and reused for all
// q and k heads.  Rows are processed in groups of kGroup whose loads are all issued
// before any arithmetic, so a warp keeps several row loads in flight.  Arithmetic per
// row follows rms_norm then rope exactly.
constexpr int kGroup = 4;

template <int E, typename TI>
__device__ __forceinline__ void load_row(const TI *in, uint32_t lane, float (&x)[E]) {
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = Elem<TI>::load(in, lane * E + e);
}

template <int E, typename TO>
__device__ __forceinline__ void norm_rope_store(float (&x)[E], TO *out, const uint16_t *w,
                                                const float *co, const float *si, uint32_t lane,
                                                uint32_t dim, float eps) {
  float squares = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) squares += x[e] * x[e];
  float inv = 1.0f / sqrtf(warp_sum(squares) / (float)dim + eps);
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = x[e] * inv * bf16_bits_to_f32(w[lane * E + e]);
  bool first = lane < 16;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
    float a = first ? x[e] : partner;   // element c
    float b = first ? partner : x[e];   // element c + dim/2
    float r = first ? (a * co[e] - b * si[e]) : (a * si[e] + b * co[e]);
    Elem<TO>::store(out, lane * E + e, r);
  }
}

template <int E, typename TI, typename TO>
__device__ __forceinline__ void norm_rope_heads(const TI *in, TO *out, uint32_t nheads,
                                                const uint16_t *w, const float *co,
                                                const float *si, uint32_t lane, uint32_t dim,
                                                float eps) {
  for (uint32_t h0 = 0; h0 < nheads; h0 += kGroup) {
    float x[kGroup][E];
#pragma unroll
    for (int g = 0; g < kGroup; ++g)
      if (h0 + g < nheads) load_row<E, TI>(in + (size_t)(h0 + g) * dim, lane, x[g]);
#pragma unroll
    for (int g = 0; g < kGroup; ++g)
      if (h0 + g < nheads)
        norm_rope_store<E, TO>(x[g], out + (size_t)(h0 + g) * dim, w, co, si, lane, dim, eps);
  }
}

template <int E, typename TI, typename TO>
__global__ void qk_norm_rope_kernel(PrologueProblem p) {
  uint32_t lane = threadIdx.x & 31;
  uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  uint32_t nwarps = (gridDim.x * blockDim.x) >> 5;
  const uint32_t dim = p.dim;
  float inv_freq[E];
#pragma unroll
  for (int e = 0; e < E; ++e) inv_freq[e] = p.inv_freq[(lane % 16) * E + e];
  for (uint32_t tok = warp; tok < p.tokens; tok += nwarps) {
    uint32_t pos;
    if (p.cu_seqlens) {
      pos = tok - (uint32_t)p.cu_seqlens[find_seq(p.cu_seqlens, p.nseq, tok)];
    } else {
      pos = tok % p.seq;
      if (p.lengths && pos >= min(p.lengths[tok / p.seq], p.seq)) continue;
    }
    float co[E], si[E];
#pragma unroll
    for (int e = 0; e < E; ++e) sincosf((float)pos * inv_freq[e], &si[e], &co[e]);
    if (p.q) {
      size_t row = (size_t)tok * p.heads * dim;
      norm_rope_heads<E, TI, TO>((const TI *)p.q + row, (TO *)p.q_out + row, p.heads, p.q_w, co,
                                 si, lane, dim, p.eps);
    }
    if (p.k) {
      size_t row = (size_t)tok * p.kv_heads * dim;
      norm_rope_heads<E, TI, TO>((const TI *)p.k + row, (TO *)p.k_out + row, p.kv_heads, p.k_w,
                                 co, si, lane, dim, p.eps);
    }
  }
}

template <int E>
static cudaError_t launch_prologue_e(const PrologueProblem &p, cudaStream_t stream) {
  uint32_t warps = p.tokens;
  uint32_t blocks = (warps + 7) / 8;
  if (blocks > 148u * 64u) blocks = 148u * 64u;
  if (p.in_dtype == 0 && p.out_dtype == 0)
    qk_norm_rope_kernel<E, float, float><<<blocks, 256, 0, stream>>>(p);
  else if (p.in_dtype == 0)
    qk_norm_rope_kernel<E, float, uint16_t><<<blocks, 256, 0, stream>>>(p);
  else if (p.out_dtype == 0)
    qk_norm_rope_kernel<E, uint16_t, float><<<blocks, 256, 0, stream>>>(p);
  else
    qk_norm_rope_kernel<E, uint16_t, uint16_t><<<blocks, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_qk_norm_rope(const PrologueProblem &problem, cudaStream_t stream) {
  if (!problem.tokens || (!problem.q && !problem.k)) return cudaSuccess;
  if (problem.dim > 256) return cudaErrorInvalidValue;
  // Inverse frequencies once per launch, in double and rounded once to float: the same
  // value rope_inv_freq gives on the device (and the CPU oracle uses).
  PrologueProblem p = problem;
  for (uint32_t c = 0; c < p.dim / 2; ++c)
    p.inv_freq[c] = (float)std::pow((double)p.theta, -2.0 * (double)c / (double)p.dim);
  switch (p.dim) {
    case 32: return launch_prologue_e<1>(p, stream);
    case 64: return launch_prologue_e<2>(p, stream);
    case 128: return launch_prologue_e<4>(p, stream);
    case 256: return launch_prologue_e<8>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tx
