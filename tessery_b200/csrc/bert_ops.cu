// Row kernels of the BERT fp32 forward around the head_dim-32 attention (the reference's
// BertBackend.forward, src/metal_inference/bert.py:104-235), and the reference kernels its
// Params-block dispatch names (kernels.metal:300-391, 438-487) for callers that drive this
// library through tx_dispatch.
//
//   bert_embed_norm_kernel  embedding_position (kernels.metal:353-361) fused with the
//                           embeddings' layer_norm (:362-373): word + token type 0 +
//                           absolute position, then LayerNorm; one warp per token
//   layer_norm_rows_kernel  layer_norm of hidden rows (one warp per row), writing the fp32
//                           row and, optionally, the next GEMM's split operand
//   split_tf32_kernel       v -> (hi = v rounded to TF32, lo = v - hi), the operand pair of
//                           the fp32 tensor-core GEMM
//   gelu_kernel, add_bias_kernel, embedding_position_kernel, matmul_f32_kernel,
//   transpose_kernel, silu_kernel
//                           the reference's elementwise / SIMT kernels for tx_dispatch
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>

#include "../../include/tessattn.h"
#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace tx {

namespace {

constexpr int kMaxPerLane = 32;  // rows of up to 1024 columns stay in registers
// The row kernels are instantiated per columns-per-lane bucket (kPer = 4, 8, 12, 16, 24 or
// 32: rows of up to 32 kPer columns), so that a row takes no more registers than it needs
// (one 32-entry array for every width left the LayerNorm at 149 registers and one block
// per SM).

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// LayerNorm of a row held as v[i] = x[lane + 32 i] (columns below `cols`), in place
// (kernels.metal:362-373: the mean, then the mean of squared deviations,
// inv = 1/sqrt(var + eps), (x - mean) * inv * w + b).
template <int kPer>
__device__ __forceinline__ void norm_row(float (&v)[kPer], uint32_t cols, const float *w,
                                         const float *b, float eps) {
  const uint32_t lane = threadIdx.x & 31;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    if (lane + 32 * i < cols) s += v[i];
  const float mean = warp_sum(s) / (float)cols;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    if (lane + 32 * i < cols) {
      const float d = v[i] - mean;
      q += d * d;
    }
  const float inv = 1.0f / sqrtf(warp_sum(q) / (float)cols + eps);
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const uint32_t c = lane + 32 * i;
    if (c < cols) v[i] = (v[i] - mean) * inv * w[c] + b[c];
  }
}

// Row r of the split operand `pair` (hi [rows, cols] then lo [rows, cols]): TF32 pair in
// fp32 containers (split == TX_F32) or a bf16 pair (split == TX_BF16X2).
template <int kPer>
__device__ __forceinline__ void write_split(const float (&v)[kPer], uint32_t cols,
                                            uint32_t rows, uint32_t r, void *pair, int split) {
  const uint32_t lane = threadIdx.x & 31;
  const size_t plane = (size_t)rows * cols;
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    if (lane + 32 * i < cols) {
      const size_t at = (size_t)r * cols + lane + 32 * i;
      if (split == TX_F32) {
        const float h = ptx::tf32_round(v[i]);
        static_cast<float *>(pair)[at] = h;
        static_cast<float *>(pair)[plane + at] = v[i] - h;
      } else {
        const __nv_bfloat16 h = __float2bfloat16_rn(v[i]);
        static_cast<__nv_bfloat16 *>(pair)[at] = h;
        static_cast<__nv_bfloat16 *>(pair)[plane + at] =
            __float2bfloat16_rn(v[i] - __bfloat162float(h));
      }
    }
}

// Position of token t: its index inside its packed sequence (cu_seqlens, binary search),
// or t % seq in the padded layout (the reference's (token % seq), kernels.metal:360).
__device__ __forceinline__ uint32_t position_of(uint32_t t, const int32_t *cu, uint32_t nseq,
                                                uint32_t seq) {
  if (!cu) return t % seq;
  uint32_t lo = 0, hi = nseq;  // cu[lo] <= t < cu[hi]
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) >> 1;
    if ((uint32_t)cu[mid] <= t) lo = mid; else hi = mid;
  }
  return t - (uint32_t)cu[lo];
}

template <int kPer>
__global__ void __launch_bounds__(256) bert_embed_norm_kernel(BertEmbedProblem p) {
  const uint32_t t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= p.tokens) return;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t id = p.ids[t];
  const uint32_t pos = position_of(t, p.cu, p.nseq, p.seq);
  float v[kPer];
  if (id >= p.vocab || pos >= p.max_pos) {
    // An id or position outside the tables: a NaN row, reported as an invalid argument.
    if (lane == 0) report_status(p.status, TX_EINVAL);
#pragma unroll
    for (int i = 0; i < kPer; ++i) v[i] = __int_as_float(0x7fc00000);
  } else {
    const float *wr = p.words + (size_t)id * p.cols, *pr = p.positions + (size_t)pos * p.cols;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const uint32_t c = lane + 32 * i;
      if (c < p.cols) v[i] = (wr[c] + p.types[c]) + pr[c];  // kernels.metal:360, type 0
    }
    norm_row(v, p.cols, p.ln_w, p.ln_b, p.eps);
  }
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const uint32_t c = lane + 32 * i;
    if (c < p.cols) p.out[(size_t)t * p.cols + c] = v[i];
  }
  if (p.pair) write_split(v, p.cols, p.tokens, t, p.pair, p.split);
}

template <int kPer>
__global__ void __launch_bounds__(256) layer_norm_rows_kernel(const float *x, const float *w,
                                                              const float *b, float *out,
                                                              void *pair, int split,
                                                              uint32_t rows, uint32_t cols,
                                                              float eps) {
  const uint32_t r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const uint32_t lane = threadIdx.x & 31;
  float v[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const uint32_t c = lane + 32 * i;
    if (c < cols) v[i] = x[(size_t)r * cols + c];
  }
  norm_row(v, cols, w, b, eps);
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const uint32_t c = lane + 32 * i;
    if (c < cols) out[(size_t)r * cols + c] = v[i];
  }
  if (pair) write_split(v, cols, rows, r, pair, split);
}

__global__ void split_tf32_kernel(const float4 *x, float4 *out, uint64_t n4) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n4;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const float4 v = x[i];
    const float4 h = make_float4(ptx::tf32_round(v.x), ptx::tf32_round(v.y),
                                 ptx::tf32_round(v.z), ptx::tf32_round(v.w));
    out[i] = h;
    out[n4 + i] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
  }
}

// ---- the reference's kernels for tx_dispatch (kernels.metal:300-391, 438-487) ---------

// gelu_f32 (kernels.metal:381-391): the erf form with Abramowitz-Stegun 7.1.26, in place.
__global__ void gelu_kernel(float *x, uint32_t n) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = gelu_erf(x[i]);
}

// add_bias (kernels.metal:376-379): x[i] += bias[i % cols].
__global__ void add_bias_kernel(float *x, const float *bias, uint32_t n, uint32_t cols) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] += bias[i % cols];
}

// silu_f32 (kernels.metal:328-331).
__global__ void silu_kernel(const float *x, float *out, uint32_t n) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = x[i] / (1.0f + expf(-x[i]));
}

// transpose_f32 (kernels.metal:323-326): out[c * rows + r] = x[r * cols + c].
__global__ void transpose_kernel(const float *x, float *out, uint32_t rows, uint32_t cols) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i < (uint64_t)rows * cols) out[(i % cols) * rows + i / cols] = x[i];
}

// embedding_position (kernels.metal:353-361), padded layout, no normalisation.
__global__ void embedding_position_kernel(const uint32_t *ids, const float *words,
                                          const float *positions, const float *types,
                                          float *out, uint32_t n, uint32_t cols, uint32_t seq) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t token = i / cols, c = i % cols;
  out[i] = (words[(size_t)ids[token] * cols + c] + types[c]) +
           positions[(size_t)(token % seq) * cols + c];
}

// matmul_f32 / matmul_bias_f32 and their tiled variants (kernels.metal:306-321, 392-487):
// out[r, c] = sum_k a[r, k] bt[c, k] (+ bias[c]) for rows [row0, rows), fp32 FMA with
// 32 x 32 output tiles staged through shared memory.  Each step of 32 products is summed
// on its own and then added to the total, as the reference's chunk32 kernels do to bound
// the accumulation error over long K (kernels.metal:416-436).
__global__ void matmul_f32_kernel(const float *a, const float *bt, const float *bias,
                                  float *out, uint32_t row0, uint32_t rows, uint32_t cols,
                                  uint32_t k) {
  __shared__ float as[32][33], bs[32][33];
  const uint32_t tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  const uint32_t r0 = row0 + blockIdx.y * 32, c0 = blockIdx.x * 32;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (uint32_t k0 = 0; k0 < k; k0 += 32) {
    for (uint32_t i = ty; i < 32; i += 8) {
      const uint32_t r = r0 + i, c = c0 + i, kk = k0 + tx;
      as[i][tx] = (r < rows && kk < k) ? a[(size_t)r * k + kk] : 0.f;
      bs[i][tx] = (c < cols && kk < k) ? bt[(size_t)c * k + kk] : 0.f;
    }
    __syncthreads();
    float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (uint32_t kk = 0; kk < 32; ++kk) {
      const float bv = bs[tx][kk];
#pragma unroll
      for (int j = 0; j < 4; ++j) part[j] = fmaf(as[ty + 8 * j][kk], bv, part[j]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j] += part[j];
    __syncthreads();
  }
  const uint32_t c = c0 + tx;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t r = r0 + ty + 8 * j;
    if (r < rows && c < cols) out[(size_t)r * cols + c] = acc[j] + (bias ? bias[c] : 0.f);
  }
}

}  // namespace

// ---- launchers ------------------------------------------------------------------------

bool bert_cols_ok(uint32_t cols) { return cols && cols <= 32 * kMaxPerLane; }

// Calls f(std::integral_constant<int, kPer>) for the smallest bucket that holds `cols`.
template <class F>
cudaError_t with_per_lane(uint32_t cols, F &&f) {
  const uint32_t per = (cols + 31) / 32;
  if (per <= 4) return f(std::integral_constant<int, 4>());
  if (per <= 8) return f(std::integral_constant<int, 8>());
  if (per <= 12) return f(std::integral_constant<int, 12>());
  if (per <= 16) return f(std::integral_constant<int, 16>());
  if (per <= 24) return f(std::integral_constant<int, 24>());
  return f(std::integral_constant<int, 32>());
}

cudaError_t launch_bert_embed(const BertEmbedProblem &p, cudaStream_t stream) {
  if (!bert_cols_ok(p.cols)) return cudaErrorInvalidValue;
  if (!p.tokens) return cudaSuccess;
  return with_per_lane(p.cols, [&](auto per) {
    bert_embed_norm_kernel<decltype(per)::value><<<(p.tokens + 7) / 8, 256, 0, stream>>>(p);
    return cudaGetLastError();
  });
}

cudaError_t launch_layer_norm_rows(const float *x, const float *w, const float *b, float *out,
                                   void *pair, int split, uint32_t rows, uint32_t cols, float eps,
                                   cudaStream_t stream) {
  if (!bert_cols_ok(cols)) return cudaErrorInvalidValue;
  if (!rows) return cudaSuccess;
  return with_per_lane(cols, [&](auto per) {
    layer_norm_rows_kernel<decltype(per)::value>
        <<<(rows + 7) / 8, 256, 0, stream>>>(x, w, b, out, pair, split, rows, cols, eps);
    return cudaGetLastError();
  });
}

cudaError_t launch_split_tf32(const float *x, float *out, uint64_t n, cudaStream_t stream) {
  if (n % 4 || (uintptr_t)x % 16 || (uintptr_t)out % 16) return cudaErrorInvalidValue;
  if (!n) return cudaSuccess;
  const uint64_t n4 = n / 4;
  const uint32_t blocks = (uint32_t)std::min<uint64_t>((n4 + 255) / 256, 148u * 16u);
  split_tf32_kernel<<<blocks, 256, 0, stream>>>((const float4 *)x, (float4 *)out, n4);
  return cudaGetLastError();
}

cudaError_t launch_gelu(float *x, uint32_t n, cudaStream_t stream) {
  if (!n) return cudaSuccess;
  gelu_kernel<<<(n + 255) / 256, 256, 0, stream>>>(x, n);
  return cudaGetLastError();
}

cudaError_t launch_add_bias(float *x, const float *bias, uint32_t n, uint32_t cols,
                            cudaStream_t stream) {
  if (!n) return cudaSuccess;
  if (!cols) return cudaErrorInvalidValue;
  add_bias_kernel<<<(n + 255) / 256, 256, 0, stream>>>(x, bias, n, cols);
  return cudaGetLastError();
}

cudaError_t launch_silu(const float *x, float *out, uint32_t n, cudaStream_t stream) {
  if (!n) return cudaSuccess;
  silu_kernel<<<(n + 255) / 256, 256, 0, stream>>>(x, out, n);
  return cudaGetLastError();
}

cudaError_t launch_transpose(const float *x, float *out, uint32_t rows, uint32_t cols,
                             cudaStream_t stream) {
  const uint64_t n = (uint64_t)rows * cols;
  if (!n) return cudaSuccess;
  transpose_kernel<<<(uint32_t)((n + 255) / 256), 256, 0, stream>>>(x, out, rows, cols);
  return cudaGetLastError();
}

cudaError_t launch_embedding_position(const uint32_t *ids, const float *words,
                                      const float *positions, const float *types, float *out,
                                      uint32_t n, uint32_t cols, uint32_t seq,
                                      cudaStream_t stream) {
  if (!n) return cudaSuccess;
  if (!cols || !seq) return cudaErrorInvalidValue;
  embedding_position_kernel<<<(n + 255) / 256, 256, 0, stream>>>(ids, words, positions, types,
                                                                 out, n, cols, seq);
  return cudaGetLastError();
}

cudaError_t launch_matmul_f32(const float *a, const float *bt, const float *bias, float *out,
                              uint32_t row0, uint32_t rows, uint32_t cols, uint32_t k,
                              cudaStream_t stream) {
  if (row0 >= rows || !cols) return cudaSuccess;
  const dim3 grid((cols + 31) / 32, (rows - row0 + 31) / 32);
  matmul_f32_kernel<<<grid, 256, 0, stream>>>(a, bt, bias, out, row0, rows, cols, k);
  return cudaGetLastError();
}

}  // namespace tx
