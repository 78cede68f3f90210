// Pooling of the encoder's final hidden states into embeddings: one row per sequence
// (the last valid token, or the first token for CLS pooling), optionally RMS-normalised
// with the model's final norm weight, then L2-normalised over its first `dim` columns.
//
//   pool_project   kernels.metal:339-349 (row = batch*seq + (first ? 0 : len-1);
//                  out = x[row, :dim] / ||x[row, :dim]||)
//   final norm     qwen3.py:281-290 runs rms_norm (kernels.metal:53-63) over every token
//                  and then pools; only the pooled rows reach the output, so the fused
//                  form normalises just those rows, with the same per-row arithmetic.
//   CLS pooling    bert.py:236-244 (first_token = 1, no norm).
//
// One warp per sequence.  Rows of up to 1024 columns that are 16-byte aligned (cols a
// multiple of 4 for fp32, 8 for bf16) are loaded whole into registers with vector loads,
// so a row costs one memory round trip; other rows are walked in strided passes.  A
// sequence with no valid row (length 0, length > seq, or an empty packed range) gets a
// NaN row: the reference would read outside the sequence there.
#include "common.cuh"
#include "kernels.h"

namespace tx {

namespace {

__device__ __forceinline__ float load1(const float *x, uint64_t i) { return x[i]; }
__device__ __forceinline__ float load1(const uint16_t *x, uint64_t i) {
  return bf16_bits_to_f32(x[i]);
}

template <typename TI>
__device__ __forceinline__ void load4(const TI *row, uint32_t c, float (&v)[4]) {
  if constexpr (sizeof(TI) == 4) {
    const float4 t = *(const float4 *)(row + c);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else {
    const uint2 t = *(const uint2 *)(row + c);
    v[0] = __uint_as_float(t.x << 16); v[1] = __uint_as_float(t.x & 0xffff0000u);
    v[2] = __uint_as_float(t.y << 16); v[3] = __uint_as_float(t.y & 0xffff0000u);
  }
}

// Element c of the row after the optional RMSNorm: (x * inv_rms) * w, the order of
// rms_norm_kernel.
__device__ __forceinline__ float normed(float x, float inv, const uint16_t *w, uint32_t c) {
  return w ? x * inv * bf16_bits_to_f32(w[c]) : x;
}

constexpr int kHeld = 8;  // float4 groups per lane held in registers: rows up to 1024 cols

template <typename TI>
__global__ void __launch_bounds__(128) pool_project_kernel(PoolProblem p) {
  const uint32_t b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t lane = threadIdx.x & 31;
  if (b >= p.batch) return;
  float *out = p.out + (uint64_t)b * p.dim;
  int64_t row = -1;
  if (p.cu_seqlens) {
    const int32_t s = p.cu_seqlens[b], e = p.cu_seqlens[b + 1];
    if (e > s) row = p.first_token ? s : e - 1;
  } else {
    const uint32_t len = p.lengths[b];
    if (p.first_token ? p.seq > 0 : (len > 0 && len <= p.seq))
      row = (int64_t)b * p.seq + (p.first_token ? 0 : len - 1);
  }
  if (row < 0) {
    for (uint32_t c = lane; c < p.dim; c += 32) out[c] = __int_as_float(0x7fc00000);
    return;
  }
  const TI *x = (const TI *)p.x + (uint64_t)row * p.cols;
  const bool vec = p.vector_ok;
  const uint16_t *w = p.norm_w;

  if (vec && p.cols <= 128 * kHeld) {
    // The whole row in registers: every load is issued before the first use, so the row
    // costs one memory round trip.
    float v[kHeld][4];
#pragma unroll
    for (int i = 0; i < kHeld; ++i) {
      const uint32_t c = 4 * lane + 128 * i;
      if (c < p.cols) load4(x, c, v[i]);
      else v[i][0] = v[i][1] = v[i][2] = v[i][3] = 0.f;
    }
    float inv = 1.f;
    if (w) {
      float sq = 0.f;
#pragma unroll
      for (int i = 0; i < kHeld; ++i)
        sq += v[i][0] * v[i][0] + v[i][1] * v[i][1] + v[i][2] * v[i][2] + v[i][3] * v[i][3];
      inv = 1.0f / sqrtf(warp_sum(sq) / (float)p.cols + p.eps);
#pragma unroll
      for (int i = 0; i < kHeld; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t c = 4 * lane + 128 * i + e;
          v[i][e] = c < p.cols ? normed(v[i][e], inv, w, c) : 0.f;
        }
    }
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < kHeld; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (4 * lane + 128 * i + e < p.dim) sq += v[i][e] * v[i][e];
    const float scale = 1.0f / sqrtf(warp_sum(sq));
    const bool out_vec = p.dim % 4 == 0 && ((uintptr_t)p.out & 15) == 0;
#pragma unroll
    for (int i = 0; i < kHeld; ++i) {
      const uint32_t c = 4 * lane + 128 * i;
      if (out_vec && c + 4 <= p.dim) {
        *(float4 *)(out + c) = make_float4(v[i][0] * scale, v[i][1] * scale, v[i][2] * scale,
                                           v[i][3] * scale);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (c + e < p.dim) out[c + e] = v[i][e] * scale;
      }
    }
    return;
  }

  // RMS of the whole row (only when the final norm is fused).
  float inv = 1.f;
  if (w) {
    float sq = 0.f;
    if (vec) {
      for (uint32_t c = 4 * lane; c < p.cols; c += 128) {
        float v[4];
        load4(x, c, v);
        sq += v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
      }
    } else {
      for (uint32_t c = lane; c < p.cols; c += 32) { float v = load1(x, c); sq += v * v; }
    }
    inv = 1.0f / sqrtf(warp_sum(sq) / (float)p.cols + p.eps);
  }
  // L2 norm of the first dim columns.
  float sq = 0.f;
  if (vec) {
    for (uint32_t c = 4 * lane; c < p.dim; c += 128) {
      float v[4];
      load4(x, c, v);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (c + i < p.dim) { float y = normed(v[i], inv, w, c + i); sq += y * y; }
    }
  } else {
    for (uint32_t c = lane; c < p.dim; c += 32) {
      float y = normed(load1(x, c), inv, w, c);
      sq += y * y;
    }
  }
  const float scale = 1.0f / sqrtf(warp_sum(sq));
  for (uint32_t c = lane; c < p.dim; c += 32) out[c] = normed(load1(x, c), inv, w, c) * scale;
}

}  // namespace

cudaError_t launch_pool_project(const PoolProblem &p, cudaStream_t stream) {
  if (!p.batch || !p.dim) return cudaSuccess;
  if (p.dim > p.cols || (p.in_dtype != 0 && p.in_dtype != 1)) return cudaErrorInvalidValue;
  PoolProblem q = p;
  const uint32_t vec_cols = p.in_dtype == 0 ? 4u : 8u;
  q.vector_ok = (p.cols % vec_cols == 0) && ((uintptr_t)p.x % 16 == 0);
  const uint32_t blocks = (p.batch + 3) / 4;
  if (p.in_dtype == 0)
    pool_project_kernel<float><<<blocks, 128, 0, stream>>>(q);
  else
    pool_project_kernel<uint16_t><<<blocks, 128, 0, stream>>>(q);
  return cudaGetLastError();
}

}  // namespace tx
