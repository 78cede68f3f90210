// Device operations of the Qwen3 embedding forward around the attention and the GEMMs:
// uint4 affine dequantisation of weight matrices, the uint4 token embedding, and the row
// RMSNorm that feeds the projections.
//
// Weights are stored as in the reference (qwen3.py:70-73): `packed` [rows, cols / 8]
// uint32 (eight 4-bit codes per word, code i of a word in bits 4i..4i+3), `scales` and
// `biases` [rows, cols / 64] bf16; element (r, c) = code * scale[r, c / 64] + bias[r, c / 64]
// (weight4, kernels.metal:11-19), computed in fp32.
#include <cuda_runtime.h>

#include "../../include/tessattn.h"
#include "common.cuh"
#include "kernels.h"

namespace tx {
namespace {

__device__ __forceinline__ float dequant(uint32_t word, int i, float scale, float bias) {
  return (float)((word >> (4 * i)) & 15u) * scale + bias;
}

// One thread per packed word: its eight weights, written as eight bf16 (16 bytes).
// With out_lo, also the rounding residue of each weight as bf16 (the lo half of a bf16
// pair whose hi half is `out`).
__global__ void dequant4_kernel(const uint32_t *packed, const uint16_t *scales,
                                const uint16_t *biases, uint16_t *out, uint16_t *out_lo,
                                uint32_t rows, uint32_t cols) {
  const uint32_t words_per_row = cols / 8;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)rows * words_per_row) return;
  const uint32_t r = (uint32_t)(i / words_per_row), wc = (uint32_t)(i % words_per_row);
  const uint32_t g = r * (cols / 64) + wc / 8;
  const float s = bf16_bits_to_f32(scales[g]), b = bf16_bits_to_f32(biases[g]);
  const uint32_t word = packed[i];
  uint32_t o[4], ol[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float a = dequant(word, 2 * e, s, b), c = dequant(word, 2 * e + 1, s, b);
    o[e] = pack_bf16x2(a, c);
    ol[e] = pack_bf16x2(a - __uint_as_float(o[e] << 16), c - __uint_as_float(o[e] & 0xffff0000u));
  }
  reinterpret_cast<uint4 *>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  if (out_lo) reinterpret_cast<uint4 *>(out_lo)[i] = make_uint4(ol[0], ol[1], ol[2], ol[3]);
}

// embedding4 (kernels.metal:21-28): out[t, c] = weight(ids[t], c), fp32.  One warp per
// token, each lane a packed word at a time.  An id at or past `vocab` gives a NaN row and
// reports a bad argument.
__global__ void embedding4_kernel(const uint32_t *ids, uint32_t tokens, const uint32_t *packed,
                                  const uint16_t *scales, const uint16_t *biases, float *out,
                                  uint32_t cols, uint32_t vocab, int *status) {
  const uint32_t t = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (t >= tokens) return;
  const uint32_t id = ids[t];
  float *orow = out + (size_t)t * cols;
  if (id >= vocab) {
    for (uint32_t c = lane; c < cols; c += 32) orow[c] = __int_as_float(0x7fc00000);
    if (lane == 0) report_status(status, kStatusBadArg);
    return;
  }
  const uint32_t *prow = packed + (size_t)id * (cols / 8);
  for (uint32_t wc = lane; wc < cols / 8; wc += 32) {
    const uint32_t g = id * (cols / 64) + wc / 8;
    const float s = bf16_bits_to_f32(scales[g]), b = bf16_bits_to_f32(biases[g]);
    const uint32_t word = prow[wc];
    float4 lo, hi;
    lo.x = dequant(word, 0, s, b); lo.y = dequant(word, 1, s, b);
    lo.z = dequant(word, 2, s, b); lo.w = dequant(word, 3, s, b);
    hi.x = dequant(word, 4, s, b); hi.y = dequant(word, 5, s, b);
    hi.z = dequant(word, 6, s, b); hi.w = dequant(word, 7, s, b);
    reinterpret_cast<float4 *>(orow)[2 * wc] = lo;
    reinterpret_cast<float4 *>(orow)[2 * wc + 1] = hi;
  }
}

// rms_norm (kernels.metal:53-63) over rows of fp32 x: x * rsqrt(mean(x^2) + eps) * bf16(w),
// written as fp32 (kOut 0), bf16 (1, the projections' operand) or a bf16 pair (2: hi at
// out, the rounding residue at out + rows * cols).  One warp per row; cols % 4 == 0.
template <int kOut>
__global__ void rms_norm_rows_kernel(const float *x, const uint16_t *w, void *out, uint32_t rows,
                                     uint32_t cols, float eps) {
  const uint32_t row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)row * cols);
  float ss = 0.f;
  for (uint32_t c = lane; c < cols / 4; c += 32) {
    const float4 v = xr[c];
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)cols + eps);
  for (uint32_t c = lane; c < cols / 4; c += 32) {
    const float4 v = xr[c];
    const uint2 wb = reinterpret_cast<const uint2 *>(w)[c];
    const float a = v.x * inv * __uint_as_float(wb.x << 16);
    const float b = v.y * inv * __uint_as_float(wb.x & 0xffff0000u);
    const float d = v.z * inv * __uint_as_float(wb.y << 16);
    const float e = v.w * inv * __uint_as_float(wb.y & 0xffff0000u);
    if (kOut == 0) {
      reinterpret_cast<float4 *>(static_cast<float *>(out) + (size_t)row * cols)[c] =
          make_float4(a, b, d, e);
    } else {
      uint16_t *o16 = static_cast<uint16_t *>(out);
      const uint32_t h0 = pack_bf16x2(a, b), h1 = pack_bf16x2(d, e);
      reinterpret_cast<uint2 *>(o16 + (size_t)row * cols)[c] = make_uint2(h0, h1);
      if (kOut == 2)
        reinterpret_cast<uint2 *>(o16 + (size_t)rows * cols + (size_t)row * cols)[c] = make_uint2(
            pack_bf16x2(a - __uint_as_float(h0 << 16), b - __uint_as_float(h0 & 0xffff0000u)),
            pack_bf16x2(d - __uint_as_float(h1 << 16), e - __uint_as_float(h1 & 0xffff0000u)));
    }
  }
}

}  // namespace

cudaError_t launch_dequant4(const uint32_t *packed, const uint16_t *scales,
                            const uint16_t *biases, uint16_t *out, uint16_t *out_lo, uint32_t rows,
                            uint32_t cols, cudaStream_t stream) {
  if (!rows || !cols || cols % 64) return cudaErrorInvalidValue;
  const size_t words = (size_t)rows * (cols / 8);
  const uint32_t block = 256;
  const size_t grid = (words + block - 1) / block;
  if (grid > 0x7fffffffu) return cudaErrorInvalidValue;
  dequant4_kernel<<<(uint32_t)grid, block, 0, stream>>>(packed, scales, biases, out, out_lo, rows,
                                                        cols);
  return cudaGetLastError();
}

cudaError_t launch_embedding4(const uint32_t *ids, uint32_t tokens, const uint32_t *packed,
                              const uint16_t *scales, const uint16_t *biases, float *out,
                              uint32_t cols, uint32_t vocab, int *status, cudaStream_t stream) {
  if (!tokens) return cudaSuccess;
  if (!cols || cols % 64) return cudaErrorInvalidValue;
  const uint32_t warps = 8;
  embedding4_kernel<<<(tokens + warps - 1) / warps, 32 * warps, 0, stream>>>(
      ids, tokens, packed, scales, biases, out, cols, vocab, status);
  return cudaGetLastError();
}

cudaError_t launch_rms_norm_rows(const float *x, const uint16_t *w, void *out, int out_kind,
                                 uint32_t rows, uint32_t cols, float eps, cudaStream_t stream) {
  if (!rows) return cudaSuccess;
  if (!cols || cols % 4) return cudaErrorInvalidValue;
  const uint32_t warps = 8, grid = (rows + warps - 1) / warps;
  if (out_kind == 2)
    rms_norm_rows_kernel<2><<<grid, 32 * warps, 0, stream>>>(x, w, out, rows, cols, eps);
  else if (out_kind == 1)
    rms_norm_rows_kernel<1><<<grid, 32 * warps, 0, stream>>>(x, w, out, rows, cols, eps);
  else
    rms_norm_rows_kernel<0><<<grid, 32 * warps, 0, stream>>>(x, w, out, rows, cols, eps);
  return cudaGetLastError();
}

namespace {
// out[i] = bf16(x[i]), out[n + i] = bf16(x[i] - out[i]): fp32 values as bf16 pairs.
__global__ void split_bf16_kernel(const float *x, uint16_t *out, uint64_t n) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = x[i];
  const uint16_t hi = f32_to_bf16_bits(v);
  out[i] = hi;
  out[n + i] = f32_to_bf16_bits(v - bf16_bits_to_f32(hi));
}
}  // namespace

cudaError_t launch_split_bf16(const float *x, uint16_t *out, uint64_t n, cudaStream_t stream) {
  if (!n) return cudaSuccess;
  if ((n + 255) / 256 > 0x7fffffffu) return cudaErrorInvalidValue;
  split_bf16_kernel<<<(uint32_t)((n + 255) / 256), 256, 0, stream>>>(x, out, n);
  return cudaGetLastError();
}

}  // namespace tx

// ---- fp32 kernels behind the reference's dispatch names (the Params-block route) --------
namespace tx {
namespace {

// linear4 semantics (kernels.metal:32-51), fp32: out[t, n] = sum_c x[t, c] * weight(n, c)
// for tokens t in [t0, t1).  One warp per (group of four tokens, output channel), lanes
// striding over the inputs, a warp sum at the end.
__global__ void linear4_f32_kernel(const float *x, const uint32_t *packed, const uint16_t *scales,
                                   const uint16_t *biases, float *out, uint32_t t0, uint32_t t1,
                                   uint32_t cols, uint32_t k) {
  const uint64_t gw = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t groups = ((uint64_t)(t1 - t0) + 3) / 4;
  if (gw >= groups * cols) return;
  const uint32_t channel = (uint32_t)(gw % cols), token = t0 + 4 * (uint32_t)(gw / cols);
  float total[4] = {0.f, 0.f, 0.f, 0.f};
  for (uint32_t c = lane; c < k; c += 32) {
    const uint32_t word = packed[(size_t)channel * (k / 8) + c / 8];
    const uint32_t g = channel * (k / 64) + c / 64;
    const float w = dequant(word, (int)(c % 8), bf16_bits_to_f32(scales[g]), bf16_bits_to_f32(biases[g]));
#pragma unroll
    for (int t = 0; t < 4; ++t)
      if (token + t < t1) total[t] += x[(size_t)(token + t) * k + c] * w;
  }
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const float sum = warp_sum(total[t]);
    if (lane == 0 && token + t < t1) out[(size_t)(token + t) * cols + channel] = sum;
  }
}

// silu_gate (kernels.metal:333-337): gate = gate / (1 + exp(-gate)) * up; add (:300-304).
__global__ void silu_gate_kernel(float *gate, const float *up, uint64_t n) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float g = gate[i];
    gate[i] = (g / (1.0f + expf(-g))) * up[i];
  }
}
__global__ void add_kernel(const float *a, const float *b, float *out, uint64_t n) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = a[i] + b[i];
}

}  // namespace

cudaError_t launch_linear4_f32(const float *x, const uint32_t *packed, const uint16_t *scales,
                               const uint16_t *biases, float *out, uint32_t t0, uint32_t t1,
                               uint32_t cols, uint32_t k, cudaStream_t stream) {
  if (t1 <= t0) return cudaSuccess;
  if (!cols || !k || k % 64) return cudaErrorInvalidValue;
  const uint64_t warps = (((uint64_t)(t1 - t0) + 3) / 4) * cols;
  const uint64_t grid = (warps * 32 + 255) / 256;
  if (grid > 0x7fffffffu) return cudaErrorInvalidValue;
  linear4_f32_kernel<<<(uint32_t)grid, 256, 0, stream>>>(x, packed, scales, biases, out, t0, t1,
                                                          cols, k);
  return cudaGetLastError();
}

cudaError_t launch_silu_gate(float *gate, const float *up, uint64_t n, cudaStream_t stream) {
  if (!n) return cudaSuccess;
  silu_gate_kernel<<<(uint32_t)((n + 255) / 256), 256, 0, stream>>>(gate, up, n);
  return cudaGetLastError();
}

cudaError_t launch_add(const float *a, const float *b, float *out, uint64_t n,
                       cudaStream_t stream) {
  if (!n) return cudaSuccess;
  add_kernel<<<(uint32_t)((n + 255) / 256), 256, 0, stream>>>(a, b, out, n);
  return cudaGetLastError();
}

}  // namespace tx
