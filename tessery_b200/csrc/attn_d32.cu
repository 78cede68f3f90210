// Attention for head_dim 32, fp32 arithmetic on fp32 or bf16 inputs (BERT/BGE-small shapes: 12 heads x 32, bidirectional,
// key-padding mask by length), the operator of bert.py:196-204 dispatched through
// MetalRuntime._attention (metal.py:532-569).
//
// Semantics are those of kernels.metal:78-103 (query at position p of a sequence of
// length n attends to [0, causal ? min(p+1, n) : n); padded query rows included).
//
// Layout of the work: one CTA of 128 threads per (query block of 128 rows, head,
// sequence).  K and V rows of the sequence are staged through shared memory in chunks
// of 128 keys with 128-bit coalesced loads (a 32-float row is exactly 128 bytes); each
// pair of threads owns two query rows, one half of the head dimension each (q and the
// output accumulators in registers, as packed float pairs), and reads the staged
// key/value rows as shared-memory broadcasts.  Softmax is online over blocks of 8 keys.
// With padded query rows counted the work is ~23 FLOP per byte of I/O, above the part's
// fp32 ridge, so the kernel is written for FMA throughput: packed f32x2 FMAs, two rows
// per shared-memory read, exp2 on the special-function unit.
#include "common.cuh"
#include "kernels.h"

namespace tx {

namespace {
constexpr int kD = 32;
constexpr int kRows = 128;   // query rows per CTA (one per thread)
constexpr int kChunk = 128;  // keys staged per shared-memory chunk
constexpr int kBlock = 8;    // keys per online-softmax step
}  // namespace

__device__ __forceinline__ uint32_t d32_find_seq(const int32_t *cu, uint32_t nseq, uint32_t tok) {
  uint32_t lo = 0, hi = nseq;
  while (hi - lo > 1) {
    uint32_t mid = (lo + hi) >> 1;
    if ((uint32_t)cu[mid] <= tok) lo = mid; else hi = mid;
  }
  return lo;
}

// Eight consecutive elements (16-byte aligned for f32 pairs of float4, 16-byte for bf16)
// as floats.
__device__ __forceinline__ void load8(const float *p, float (&x)[8]) {
  const float4 a = ((const float4 *)p)[0], b = ((const float4 *)p)[1];
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}
__device__ __forceinline__ void load8(const uint16_t *p, float (&x)[8]) {
  const uint4 a = *(const uint4 *)p;
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = __uint_as_float(w[i] << 16);
    x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// Packed pairs of floats (Blackwell f32x2: two lanes per instruction, each rounded as
// the scalar instruction rounds it).
__device__ __forceinline__ uint64_t d32_f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 d32_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t d32_fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t d32_mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float d32_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Dot products of two rows' 16 query elements (8 packed pairs each) with 16 staged key
// elements, read once for both rows.
__device__ __forceinline__ void d32_dot16x2(const uint64_t (&qa)[8], const uint64_t (&qb)[8],
                                            const float *kr, float *da, float *db) {
  uint64_t a0 = d32_f2(0.f, 0.f), a1 = a0, b0 = a0, b1 = a0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 t = ((const float4 *)kr)[i];
    const uint64_t k0 = d32_f2(t.x, t.y), k1 = d32_f2(t.z, t.w);
    a0 = d32_fma2(qa[2 * i], k0, a0);
    a1 = d32_fma2(qa[2 * i + 1], k1, a1);
    b0 = d32_fma2(qb[2 * i], k0, b0);
    b1 = d32_fma2(qb[2 * i + 1], k1, b1);
  }
  const float2 x0 = d32_unpack(a0), x1 = d32_unpack(a1), y0 = d32_unpack(b0),
               y1 = d32_unpack(b1);
  *da = (x0.x + x0.y) + (x1.x + x1.y);
  *db = (y0.x + y0.y) + (y1.x + y1.y);
}

// Thread t works on query rows 2(t/2) and 2(t/2)+1 of the CTA's 128 and on head-dimension
// half t%2 (16 of the 32 elements): each staged K or V row read from shared memory feeds
// both rows, the two halves of a dot product meet in one shuffle, and the accumulators
// of P.V stay split by half.  Scores are in log2 units (q is pre-multiplied by
// scale * log2(e)), the online softmax keeps a lazily updated reference maximum per row
// (the accumulators are rescaled only when a block's maximum exceeds it by more than 8),
// so every probability is at most 2^8 and the normalised result is unchanged.
template <typename TI, typename TO>
__global__ void __launch_bounds__(kRows, 4) attention_d32_kernel(AttnProblem p) {
  __shared__ __align__(16) float ks[kChunk * kD];
  __shared__ __align__(16) float vs[kChunk * kD];
  const TI *q = (const TI *)p.q, *k = (const TI *)p.k, *v = (const TI *)p.v;
  TO *out = (TO *)p.out;
  const uint32_t qblock = blockIdx.x, head = blockIdx.y, seqi = blockIdx.z;
  const uint32_t kvhead = head / (p.heads / p.kv_heads);
  const uint32_t tid = threadIdx.x, half = tid & 1;
  uint32_t len, rows;  // valid keys; query rows present in the layout
  uint64_t base;       // row index of position 0
  if (p.cu_seqlens) {
    int32_t a = p.cu_seqlens[seqi], b = p.cu_seqlens[seqi + 1];
    len = b > a ? (uint32_t)(b - a) : 0u;
    rows = len;
    base = (uint32_t)a;
  } else {
    len = min(p.lengths[seqi], p.seq);
    rows = p.seq;
    base = (uint64_t)seqi * p.seq;
  }
  const uint32_t q0 = qblock * kRows;
  if (q0 >= rows) return;
  const uint32_t pos0 = q0 + (tid & ~1u), pos1 = pos0 + 1;
  const bool act0 = pos0 < rows, act1 = pos1 < rows;
  const uint32_t end0 = act0 ? (p.causal ? min(pos0 + 1, len) : len) : 0u;
  const uint32_t end1 = act1 ? (p.causal ? min(pos1 + 1, len) : len) : 0u;
  // Keys needed by any row of this CTA.
  const uint32_t last = min(q0 + kRows, rows) - 1;
  const uint32_t kend = p.causal ? min(last + 1, len) : len;
  const float qs = p.scale * 1.4426950408889634f;

  uint64_t qa[8], qb[8];  // rows 0 and 1, elements 16*half .. 16*half+15, scaled
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const bool act = r ? act1 : act0;
    uint64_t(&qr)[8] = r ? qb : qa;
    if (act) {
      const TI *qp = q + ((base + (r ? pos1 : pos0)) * p.heads + head) * kD + 16 * half;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        float t[8];
        load8(qp + 8 * i, t);
#pragma unroll
        for (int e = 0; e < 4; ++e) qr[4 * i + e] = d32_f2(t[2 * e] * qs, t[2 * e + 1] * qs);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) qr[i] = d32_f2(0.f, 0.f);
    }
  }
  uint64_t acc0[8], acc1[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc0[i] = acc1[i] = d32_f2(0.f, 0.f);
  float m0 = -INFINITY, l0 = 0.f, m1 = -INFINITY, l1 = 0.f;
  // The warp's largest key bound (end is non-decreasing in the lane for causal rows).
  uint32_t wend = max(end0, end1);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wend = max(wend, __shfl_xor_sync(0xffffffffu, wend, o));

  for (uint32_t c0 = 0; c0 < kend; c0 += kChunk) {
    const uint32_t cn = min(kChunk, kend - c0);
    __syncthreads();  // previous chunk fully consumed
    // Stage K and V rows [c0, c0+cn) as fp32: 4 groups of 8 elements per row
    // (128-bit loads for bf16, 2 x 128-bit for f32), consecutive threads on consecutive
    // groups so the row reads coalesce.
    for (uint32_t i = tid; i < cn * (kD / 8); i += kRows) {
      uint32_t r = i / (kD / 8), c8 = i % (kD / 8);
      uint64_t row = ((base + c0 + r) * p.kv_heads + kvhead) * kD + c8 * 8;
      float t[8];
      load8(k + row, t);
      ((float4 *)ks)[2 * i] = make_float4(t[0], t[1], t[2], t[3]);
      ((float4 *)ks)[2 * i + 1] = make_float4(t[4], t[5], t[6], t[7]);
      load8(v + row, t);
      ((float4 *)vs)[2 * i] = make_float4(t[0], t[1], t[2], t[3]);
      ((float4 *)vs)[2 * i + 1] = make_float4(t[4], t[5], t[6], t[7]);
    }
    __syncthreads();
    if (wend <= c0) continue;
    const uint32_t stop = min(cn, wend - c0);
    for (uint32_t j0 = 0; j0 < stop; j0 += kBlock) {
      float s0[kBlock], s1[kBlock];
      // Blocks wholly inside both rows' key ranges need no mask (warp-uniform test).
      const bool full = __all_sync(0xffffffffu, c0 + j0 + kBlock <= min(end0, end1));
#pragma unroll
      for (int j = 0; j < kBlock; ++j) {
        const float *kr = ks + (j0 + j) * kD + 16 * half;
        float d0, d1;
        d32_dot16x2(qa, qb, kr, &d0, &d1);
        d0 += __shfl_xor_sync(0xffffffffu, d0, 1);
        d1 += __shfl_xor_sync(0xffffffffu, d1, 1);
        const uint32_t key = c0 + j0 + j;
        s0[j] = full || key < end0 ? d0 : -INFINITY;
        s1[j] = full || key < end1 ? d1 : -INFINITY;
      }
      float mb0 = s0[0], mb1 = s1[0];
#pragma unroll
      for (int j = 1; j < kBlock; ++j) {
        mb0 = fmaxf(mb0, s0[j]);
        mb1 = fmaxf(mb1, s1[j]);
      }
      if (mb0 > m0 + 8.0f) {  // also the first block with a valid key (m0 = -inf)
        const float c = d32_ex2(m0 - mb0);
        const uint64_t c2 = d32_f2(c, c);
        l0 *= c;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc0[i] = d32_mul2(acc0[i], c2);
        m0 = mb0;
      }
      if (mb1 > m1 + 8.0f) {
        const float c = d32_ex2(m1 - mb1);
        const uint64_t c2 = d32_f2(c, c);
        l1 *= c;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc1[i] = d32_mul2(acc1[i], c2);
        m1 = mb1;
      }
#pragma unroll
      for (int j = 0; j < kBlock; ++j) {
        const float p0 = d32_ex2(s0[j] - m0), p1 = d32_ex2(s1[j] - m1);
        l0 += p0;
        l1 += p1;
        const uint64_t p02 = d32_f2(p0, p0), p12 = d32_f2(p1, p1);
        const float4 *vr = (const float4 *)(vs + (j0 + j) * kD + 16 * half);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 t = vr[i];
          const uint64_t va = d32_f2(t.x, t.y), vb = d32_f2(t.z, t.w);
          acc0[2 * i] = d32_fma2(p02, va, acc0[2 * i]);
          acc0[2 * i + 1] = d32_fma2(p02, vb, acc0[2 * i + 1]);
          acc1[2 * i] = d32_fma2(p12, va, acc1[2 * i]);
          acc1[2 * i + 1] = d32_fma2(p12, vb, acc1[2 * i + 1]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (!(r ? act1 : act0)) continue;
    const float inv = 1.0f / (r ? l1 : l0);
    const uint64_t(&acc)[8] = r ? acc1 : acc0;
    float o[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 t = d32_unpack(acc[i]);
      o[2 * i] = t.x * inv;
      o[2 * i + 1] = t.y * inv;
    }
    TO *op = out + ((base + (r ? pos1 : pos0)) * p.heads + head) * kD + 16 * half;
    if constexpr (sizeof(TO) == 4) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        ((float4 *)op)[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 2; ++i)
        ((uint4 *)op)[i] = make_uint4(pack_bf16x2(o[8 * i], o[8 * i + 1]),
                                      pack_bf16x2(o[8 * i + 2], o[8 * i + 3]),
                                      pack_bf16x2(o[8 * i + 4], o[8 * i + 5]),
                                      pack_bf16x2(o[8 * i + 6], o[8 * i + 7]));
    }
  }
}

cudaError_t launch_attention_d32(const AttnProblem &p, cudaStream_t stream) {
  if (p.dim != kD) return cudaErrorInvalidValue;
  if (!p.batch || !p.heads) return cudaSuccess;
  uint32_t qblocks = (p.seq + kRows - 1) / kRows;
  if (!qblocks) return cudaSuccess;
  if (p.batch > 65535u || p.heads > 65535u) return cudaErrorInvalidValue;
  dim3 grid(qblocks, p.heads, p.batch);
  if (p.in_dtype == 0 && p.out_dtype == 0)
    attention_d32_kernel<float, float><<<grid, kRows, 0, stream>>>(p);
  else if (p.in_dtype == 0)
    attention_d32_kernel<float, uint16_t><<<grid, kRows, 0, stream>>>(p);
  else if (p.out_dtype == 0)
    attention_d32_kernel<uint16_t, float><<<grid, kRows, 0, stream>>>(p);
  else
    attention_d32_kernel<uint16_t, uint16_t><<<grid, kRows, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace tx
