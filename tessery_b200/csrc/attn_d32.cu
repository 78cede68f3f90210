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
// thread owns one query row (q and the output accumulator in registers) and reads the
// staged key/value rows as shared-memory broadcasts.  Softmax is online over blocks of
// 8 keys.  At head_dim 32 the arithmetic intensity is about 12 FLOP/byte, near the fp32
// ridge of the part, so the kernel is written to keep HBM streaming, not for tensor
// cores.
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

template <typename TI, typename TO>
__global__ void __launch_bounds__(kRows) attention_d32_kernel(AttnProblem p) {
  __shared__ __align__(16) float ks[kChunk * kD];
  __shared__ __align__(16) float vs[kChunk * kD];
  const TI *q = (const TI *)p.q, *k = (const TI *)p.k, *v = (const TI *)p.v;
  TO *out = (TO *)p.out;
  const uint32_t qblock = blockIdx.x, head = blockIdx.y, seqi = blockIdx.z;
  const uint32_t kvhead = head / (p.heads / p.kv_heads);
  const uint32_t tid = threadIdx.x;
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
  const uint32_t pos = q0 + tid;
  const bool active = pos < rows;
  const uint32_t end = active ? (p.causal ? min(pos + 1, len) : len) : 0u;
  // Keys needed by any row of this CTA.
  const uint32_t last = min(q0 + kRows, rows) - 1;
  const uint32_t kend = p.causal ? min(last + 1, len) : len;

  float qr[kD], acc[kD];
  if (active) {
    const TI *qp = q + ((base + pos) * p.heads + head) * kD;
#pragma unroll
    for (int i = 0; i < kD / 8; ++i) {
      float t[8];
      load8(qp + 8 * i, t);
#pragma unroll
      for (int e = 0; e < 8; ++e) qr[8 * i + e] = t[e];
    }
  } else {
#pragma unroll
    for (int i = 0; i < kD; ++i) qr[i] = 0.f;
  }
#pragma unroll
  for (int i = 0; i < kD; ++i) acc[i] = 0.f;
  float m = -INFINITY, l = 0.f;
  // The warp's largest key bound (end is non-decreasing in the lane for causal rows).
  uint32_t wend = end;
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
      float s[kBlock];
#pragma unroll
      for (int j = 0; j < kBlock; ++j) {
        const float4 *kr = (const float4 *)(ks + (j0 + j) * kD);
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < kD / 4; ++i) {
          float4 t = kr[i];
          dot += qr[4 * i] * t.x;
          dot += qr[4 * i + 1] * t.y;
          dot += qr[4 * i + 2] * t.z;
          dot += qr[4 * i + 3] * t.w;
        }
        uint32_t key = c0 + j0 + j;
        s[j] = (key < end) ? dot * p.scale : -INFINITY;
      }
      float mb = s[0];
#pragma unroll
      for (int j = 1; j < kBlock; ++j) mb = fmaxf(mb, s[j]);
      float mn = fmaxf(m, mb);
      if (mn == -INFINITY) continue;  // no valid key yet for this row
      float corr = expf(m - mn);
      l *= corr;
#pragma unroll
      for (int i = 0; i < kD; ++i) acc[i] *= corr;
#pragma unroll
      for (int j = 0; j < kBlock; ++j) {
        float pj = expf(s[j] - mn);
        l += pj;
        const float4 *vr = (const float4 *)(vs + (j0 + j) * kD);
#pragma unroll
        for (int i = 0; i < kD / 4; ++i) {
          float4 t = vr[i];
          acc[4 * i] += pj * t.x;
          acc[4 * i + 1] += pj * t.y;
          acc[4 * i + 2] += pj * t.z;
          acc[4 * i + 3] += pj * t.w;
        }
      }
      m = mn;
    }
  }
  if (active) {
    float inv = 1.0f / l;
    TO *op = out + ((base + pos) * p.heads + head) * kD;
    if constexpr (sizeof(TO) == 4) {
#pragma unroll
      for (int i = 0; i < kD / 4; ++i)
        ((float4 *)op)[i] = make_float4(acc[4 * i] * inv, acc[4 * i + 1] * inv,
                                        acc[4 * i + 2] * inv, acc[4 * i + 3] * inv);
    } else {
#pragma unroll
      for (int i = 0; i < kD / 8; ++i)
        ((uint4 *)op)[i] = make_uint4(pack_bf16x2(acc[8 * i] * inv, acc[8 * i + 1] * inv),
                                      pack_bf16x2(acc[8 * i + 2] * inv, acc[8 * i + 3] * inv),
                                      pack_bf16x2(acc[8 * i + 4] * inv, acc[8 * i + 5] * inv),
                                      pack_bf16x2(acc[8 * i + 6] * inv, acc[8 * i + 7] * inv));
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
