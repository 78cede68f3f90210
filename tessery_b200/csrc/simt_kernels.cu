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

// ---- bf16 head_dim-128 prologue, written for bandwidth -------------------------------
// One pass over the rows of one tensor (q or k).  A block of 4 warps covers 12
// consecutive tokens (padded layout: 12 positions of one sequence, blockIdx.y = the
// sequence, so its length is read once and blocks past it exit); their rows are
// contiguous in memory and arrive in shared memory with one bulk asynchronous copy, so
// the bytes in flight per SM are set by the blocks resident there, not by registers;
// each warp then transforms 3 tokens and writes them straight to global memory (3 per
// warp measured faster than 2 or 4 at the Qwen shapes: more blocks in flight than with
// 4, no second wave as with 2).  Within a
// token, each half-warp owns one 256-byte row (one head) per load, lane l%16 holding the
// 16 bytes of columns 8(l%16)..8(l%16)+7, so every load and store moves 512 contiguous
// bytes per warp.  The rotation partner of column c (c < 64) is column c + 64, held by
// lane l^8: the lanes swap their raw bf16 words and each computes its own output of
// kernels.metal:53-74 (a = x_c * inv * w_c, b = x_{c+64} * inv * w_{c+64}; a*cos - b*sin
// for the first half, a*sin + b*cos for the second), regrouped as
// inv * (own * (w_own * cos) -/+ partner * (w_partner * sin)) so that the per-token
// products are shared by all heads.  The angle is the float product pos * inv_freq[c];
// its sine and cosine come from rope_sincos (a Cody-Waite reduction by 2*pi and the
// hardware approximations, about 2^-21 absolute error).
constexpr int kRowTokensPerWarp = 3;

struct RowPass {
  const uint16_t *in;
  uint16_t *out;
  const uint16_t *w;
  uint32_t nheads;
  uint32_t tokens, seq;
  const int32_t *cu;
  uint32_t nseq;
  const uint32_t *lengths;
  float eps;
  float inv_freq[64];
};

__device__ __forceinline__ void bf16x8_unpack(const uint4 &v, float (&f)[8]) {
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t w = e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w;
    f[2 * e] = __uint_as_float(w << 16);
    f[2 * e + 1] = __uint_as_float(w & 0xffff0000u);
  }
}

__device__ __forceinline__ uint64_t pf2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t pf2_bits(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
__device__ __forceinline__ float2 pf2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t pfma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t pmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// The two bf16 of a word as a float pair (lo first).
__device__ __forceinline__ uint64_t bf16x2_pf2(uint32_t w) { return pf2_bits(w << 16, w & 0xffff0000u); }


template <int NP>  // row pairs per token: ceil(nheads / 2)
__global__ void __launch_bounds__(128) norm_rope_rows_bf16_kernel(RowPass p) {
  // The attention kernel that follows may be launched early (programmatic dependent
  // launch); it waits for this grid's completion before it reads what this one writes.
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ __align__(128) uint8_t rows_s[];  // the block's token rows
  __shared__ int32_t cu_s[1025];
  __shared__ __align__(8) uint64_t full_bar;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t l16 = lane & 15, half = lane >> 4, g = l16 & 7;
  const bool first = l16 < 8;
  constexpr uint32_t kBlockTokens = 4 * kRowTokensPerWarp;
  // Tokens of this block: [tb, tb + nb) of one sequence (padded) or of the packed rows.
  uint32_t tb, nb, pos0 = 0;
  if (p.cu) {
    tb = blockIdx.x * kBlockTokens;
    if (tb >= p.tokens) return;
    nb = min(kBlockTokens, p.tokens - tb);
    if (p.nseq < 1025)
      for (uint32_t i = threadIdx.x; i <= p.nseq; i += blockDim.x) cu_s[i] = p.cu[i];
  } else {
    const uint32_t b = blockIdx.y;
    const uint32_t len = p.lengths ? min(p.lengths[b], p.seq) : p.seq;
    pos0 = blockIdx.x * kBlockTokens;
    if (pos0 >= len) return;
    nb = min(kBlockTokens, len - pos0);
    tb = b * p.seq + pos0;
  }
  const uint32_t row_bytes = p.nheads * 256;
  const uint32_t full = (uint32_t)__cvta_generic_to_shared(&full_bar);
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(full) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // One bulk copy of the block's consecutive token rows into shared memory.
    const uint32_t bytes = nb * row_bytes;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(full), "r"(bytes)
                 : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            (uint32_t)__cvta_generic_to_shared(rows_s)),
        "l"(p.in + (size_t)tb * p.nheads * 128), "r"(bytes), "r"(full)
        : "memory");
  }
  // Weights of this lane's columns and of its partner's, and its inverse frequencies.
  const uint4 wo = __ldg(reinterpret_cast<const uint4 *>(p.w) + l16);
  const uint4 wp = __ldg(reinterpret_cast<const uint4 *>(p.w) + (l16 ^ 8));
  float wof[8], wpf[8], invf[8];
  bf16x8_unpack(wo, wof);
  bf16x8_unpack(wp, wpf);
#pragma unroll
  for (int e = 0; e < 8; ++e) invf[e] = p.inv_freq[8 * g + e];
  // Bounded wait for the copy (it completes unless the copy itself failed).
  {
    uint32_t done = 0;
    const long long t0 = clock64();
    while (!done) {
      asm volatile(
          "{\n\t.reg .pred q;\n\tmbarrier.try_wait.parity.shared::cta.b64 q, [%1], 0;\n\t"
          "selp.u32 %0, 1, 0, q;\n\t}"
          : "=r"(done)
          : "r"(full)
          : "memory");
      if (!done && clock64() - t0 > 2000000000ll) return;
    }
  }
  auto position = [&](uint32_t tok) -> uint32_t {
    if (!p.cu) return pos0 + (tok - tb);
    uint32_t lo = 0, hi = p.nseq;
    if (p.nseq < 1025) {
      while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if ((uint32_t)cu_s[mid] <= tok) lo = mid; else hi = mid;
      }
      return tok - (uint32_t)cu_s[lo];
    }
    return tok - (uint32_t)p.cu[find_seq(p.cu, p.nseq, tok)];
  };
  const uint32_t srow0 = (uint32_t)__cvta_generic_to_shared(rows_s);
#pragma unroll 1
  for (uint32_t i = warp * kRowTokensPerWarp; i < min((warp + 1) * kRowTokensPerWarp, nb); ++i) {
    const uint32_t tok = tb + i;
    uint4 x[NP];
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      const uint32_t head = 2 * j + half;
      if (head < p.nheads) {
        const uint32_t addr = srow0 + i * row_bytes + head * 256 + l16 * 16;
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(x[j].x), "=r"(x[j].y), "=r"(x[j].z), "=r"(x[j].w)
                     : "r"(addr));
      } else {
        x[j] = make_uint4(0, 0, 0, 0);
      }
    }
    const float fpos = (float)position(tok);
    uint64_t c1[4], c2[4];  // pairs of w_own * cos and -/+ w_partner * sin
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float sn0, cs0, sn1, cs1;
      rope_sincos(fpos * invf[2 * e], &sn0, &cs0);
      rope_sincos(fpos * invf[2 * e + 1], &sn1, &cs1);
      c1[e] = pf2(wof[2 * e] * cs0, wof[2 * e + 1] * cs1);
      c2[e] = first ? pf2(-(wpf[2 * e] * sn0), -(wpf[2 * e + 1] * sn1))
                    : pf2(wpf[2 * e] * sn0, wpf[2 * e + 1] * sn1);
    }
    uint16_t *orow = p.out + (size_t)tok * p.nheads * 128;
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      const uint32_t head = 2 * j + half;
      const uint32_t xw[4] = {x[j].x, x[j].y, x[j].z, x[j].w};
      uint64_t a[4], b[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        a[e] = bf16x2_pf2(xw[e]);
        b[e] = bf16x2_pf2(__shfl_xor_sync(0xffffffffu, xw[e], 8));
      }
      uint64_t ss2 = pmul2(a[0], a[0]);
#pragma unroll
      for (int e = 1; e < 4; ++e) ss2 = pfma2(a[e], a[e], ss2);
      const float2 ssp = pf2_unpack(ss2);
      float ss = ssp.x + ssp.y;
      ss += __shfl_xor_sync(0xffffffffu, ss, 8);
      ss += __shfl_xor_sync(0xffffffffu, ss, 4);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      const float inv = 1.0f / sqrtf(ss / 128.0f + p.eps);
      const uint64_t inv2 = pf2(inv, inv);
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 r = pf2_unpack(pmul2(inv2, pfma2(b[e], c2[e], pmul2(a[e], c1[e]))));
        o[e] = pack_bf16x2(r.x, r.y);
      }
      if (head < p.nheads)
        reinterpret_cast<uint4 *>(orow + (size_t)head * 128)[l16] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

template <int NP>
static cudaError_t launch_rows(const RowPass &rp, const PrologueProblem &p, cudaStream_t stream) {
  constexpr uint32_t kBlockTokens = 4 * kRowTokensPerWarp;
  dim3 grid;
  if (rp.cu) {
    grid = dim3((rp.tokens + kBlockTokens - 1) / kBlockTokens, 1, 1);
  } else {
    if (p.tokens % p.seq) return cudaErrorInvalidValue;
    grid = dim3((rp.seq + kBlockTokens - 1) / kBlockTokens, rp.tokens / rp.seq, 1);
    if (grid.y > 65535u) return cudaErrorInvalidValue;
  }
  const uint32_t smem = kBlockTokens * rp.nheads * 256;
  // The 48 KB default covers static and dynamic shared memory together (the kernel's
  // static arrays take ~4 KB): opt in above that.
  if (smem + 8 * 1024 > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(norm_rope_rows_bf16_kernel<NP>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  norm_rope_rows_bf16_kernel<NP><<<grid, 128, smem, stream>>>(rp);
  return cudaGetLastError();
}

static cudaError_t launch_rows_pass(const void *in, void *out, const uint16_t *w, uint32_t nheads,
                                    const PrologueProblem &p, cudaStream_t stream) {
  RowPass rp{};
  rp.in = (const uint16_t *)in;
  rp.out = (uint16_t *)out;
  rp.w = w;
  rp.nheads = nheads;
  rp.tokens = p.tokens;
  rp.seq = p.seq;
  rp.cu = p.cu_seqlens;
  rp.nseq = p.nseq;
  rp.lengths = p.lengths;
  rp.eps = p.eps;
  for (int c = 0; c < 64; ++c) rp.inv_freq[c] = p.inv_freq[c];
  switch ((nheads + 1) / 2) {
    case 1: return launch_rows<1>(rp, p, stream);
    case 2: return launch_rows<2>(rp, p, stream);
    case 3: return launch_rows<3>(rp, p, stream);
    case 4: return launch_rows<4>(rp, p, stream);
    case 5: case 6: return launch_rows<6>(rp, p, stream);
    default: return launch_rows<8>(rp, p, stream);
  }
}

cudaError_t launch_qk_norm_rope(const PrologueProblem &problem, cudaStream_t stream) {
  if (!problem.tokens || (!problem.q && !problem.k)) return cudaSuccess;
  if (problem.dim > 256) return cudaErrorInvalidValue;
  // Inverse frequencies once per launch, in double and rounded once to float: the same
  // value rope_inv_freq gives on the device (and the CPU oracle uses).
  PrologueProblem p = problem;
  for (uint32_t c = 0; c < p.dim / 2; ++c)
    p.inv_freq[c] = (float)std::pow((double)p.theta, -2.0 * (double)c / (double)p.dim);
  // bf16 head_dim 128 with up to 16 heads: one bandwidth-oriented pass per tensor.
  const bool fast = p.dim == 128 && p.in_dtype == 1 && p.out_dtype == 1 &&
                    (!p.q || (p.heads <= 16 && (uintptr_t)p.q % 16 == 0 &&
                              (uintptr_t)p.q_out % 16 == 0 && (uintptr_t)p.q_w % 16 == 0)) &&
                    (!p.k || (p.kv_heads <= 16 && (uintptr_t)p.k % 16 == 0 &&
                              (uintptr_t)p.k_out % 16 == 0 && (uintptr_t)p.k_w % 16 == 0)) &&
                    (p.cu_seqlens || (p.seq && p.tokens % p.seq == 0 && p.tokens / p.seq <= 65535u));
  if (fast) {
    cudaError_t e = cudaSuccess;
    if (p.q) e = launch_rows_pass(p.q, p.q_out, p.q_w, p.heads, p, stream);
    if (e == cudaSuccess && p.k) e = launch_rows_pass(p.k, p.k_out, p.k_w, p.kv_heads, p, stream);
    return e;
  }
  switch (p.dim) {
    case 32: return launch_prologue_e<1>(p, stream);
    case 64: return launch_prologue_e<2>(p, stream);
    case 128: return launch_prologue_e<4>(p, stream);
    case 256: return launch_prologue_e<8>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tx
