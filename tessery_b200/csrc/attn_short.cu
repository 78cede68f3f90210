// Short-sequence attention for head_dim 128 with bf16 q/k/v: the Qwen3 causal GQA operator
// of qwen3.py:238-245 (semantics of kernels.metal:78-103) with the q/k RMSNorm + RoPE of
// qwen3.py:216-237 (kernels.metal:53-74) fused in front, for batches whose sequences are
// at most 32 tokens long (the short-tail shape).
//
// At these lengths a whole (sequence, kv head) problem fits in one CTA's shared memory:
// the K and V rows of the sequence and the Q rows of every query head that reads them.
// One CTA (8 warps) per (sequence, kv head) loads them once, normalises and rotates q and
// k in shared memory (k rows are used by exactly this CTA, so the k prologue needs no
// separate pass),
// computes S = Q K^T, the masked softmax and O = P V with register-level tensor-core
// MMAs (mma.sync m16n8k16, bf16 operands, fp32 accumulators: each warp owns 16 query
// rows, S stays in registers and becomes the A operand of P V), and writes O.  No
// tensor-memory set-up, no work list and no prologue launch: the whole operator is one
// launch whose time is a few global-memory round trips.
//
// Numerics: q and k after the prologue and P are bf16 operands, as on the tcgen05 path;
// scores, softmax statistics and O are fp32; exp2 on the special-function unit.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace tx {
namespace sh {

constexpr uint32_t kMaxRows = 32;   // rows (and keys) per sequence
constexpr uint32_t kMaxGroup = 4;   // query heads per kv head
constexpr uint32_t kThreads = 256;
constexpr uint32_t kRS = 136;       // row stride (bf16) of the Q, K and V tiles: rows 4 banks apart

struct Params {
  const uint16_t *q, *k, *v;
  void *out;
  const uint32_t *lengths;  // padded layout
  const int32_t *cu;        // varlen layout
  uint32_t seq, heads, kv_heads, group;
  int out_bf16, causal;
  float scale_log2;
  const uint16_t *q_w, *k_w;
  float eps;
  int *status;
  float inv_freq[64];
};

// Shared-memory bytes for a group of g query heads: Q, K and V (bf16, kRS), then the raw
// bf16 rows of k and q as loaded.
__host__ __device__ constexpr uint32_t smem_bytes(uint32_t g) {
  return (g * kMaxRows * kRS + 2 * kMaxRows * kRS) * 2 + (1 + g) * kMaxRows * 256;
}

// D = A B + D for one m16n8k16 tile (bf16 A and B, fp32 accumulators).
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(kThreads) attn_short_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const uint32_t s = blockIdx.x, kvh = blockIdx.y;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t tok0, n, rows;
  if (p.cu) {
    const int32_t a = p.cu[s], b = p.cu[s + 1];
    tok0 = (uint32_t)a;
    n = b > a ? (uint32_t)(b - a) : 0u;
    rows = n;
  } else {
    tok0 = s * p.seq;
    n = min(p.lengths[s], p.seq);
    rows = p.seq;
  }
  if (rows > kMaxRows) {  // a sequence longer than the maximum this kernel was chosen for
    if (threadIdx.x == 0) report_status(p.status, kStatusBadArg);
    return;
  }
  if (!rows) return;
  const uint32_t G = p.group, R = G * rows;
  uint16_t *Qs = reinterpret_cast<uint16_t *>(smem);  // [G*rows][kRS] bf16
  uint16_t *Ks = Qs + G * kMaxRows * kRS;             // [n][kRS]
  uint16_t *Vs = Ks + kMaxRows * kRS;                 // [32][kRS]: V rows, zero past n
  uint16_t *raw = Vs + kMaxRows * kRS;                // [n+R][128] bf16: k, q as loaded
  const float f0 = p.inv_freq[2 * lane], f1 = p.inv_freq[2 * lane + 1];
  // Head (within the group) of Q-tile row r < R, without a division (G <= 4).
  auto head_of = [&](uint32_t r) -> uint32_t {
    return (uint32_t)(r >= rows) + (uint32_t)(r >= 2 * rows) + (uint32_t)(r >= 3 * rows);
  };

  // Raw rows k (n) and q (G heads x rows) into shared memory, v rows (n) straight into
  // their tile: every 16-byte piece is an asynchronous copy, all in flight at once (one
  // memory latency for the whole load).
  const uint32_t staged = n + R;
  for (uint32_t c = threadIdx.x; c < (staged + n) * 16; c += kThreads) {
    const uint32_t i = c >> 4, piece = c & 15;
    const uint16_t *src;
    uint16_t *dst;
    if (i < n) {
      src = p.k + ((size_t)(tok0 + i) * p.kv_heads + kvh) * 128;
      dst = raw + i * 128;
    } else if (i < staged) {
      const uint32_t r = i - n, g = head_of(r);
      src = p.q + ((size_t)(tok0 + r - g * rows) * p.heads + kvh * G + g) * 128;
      dst = raw + i * 128;
    } else {
      src = p.v + ((size_t)(tok0 + i - staged) * p.kv_heads + kvh) * 128;
      dst = Vs + (i - staged) * kRS;
    }
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(dst + piece * 8)),
                 "l"(src + piece * 8)
                 : "memory");
  }
  // V rows n..31 are zero (P is zero there too, but 0 * garbage need not be).
  for (uint32_t c = threadIdx.x; c < (kMaxRows - n) * 64; c += kThreads)
    reinterpret_cast<uint32_t *>(Vs + (n + (c >> 6)) * kRS)[c & 63] = 0u;
  // This lane's RMSNorm weight words for q and k.
  uint32_t wq_l = 0, wq_h = 0, wk_l = 0, wk_h = 0;
  if (p.q_w) {
    wq_l = reinterpret_cast<const uint32_t *>(p.q_w)[lane];
    wq_h = reinterpret_cast<const uint32_t *>(p.q_w)[32 + lane];
  }
  if (p.k_w) {
    wk_l = reinterpret_cast<const uint32_t *>(p.k_w)[lane];
    wk_h = reinterpret_cast<const uint32_t *>(p.k_w)[32 + lane];
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  // q and k normalised and rotated (rounded to bf16).  Each warp takes four
  // rows at a time (rows i, i+W, i+2W, i+3W of the staged list, W warps) whose reductions
  // and sin/cos evaluations interleave.
  for (uint32_t i0 = warp; i0 < staged; i0 += 4 * (kThreads / 32)) {
    float x[4][4], ss[4];
    bool norm[4];
    uint32_t wl[4], wh[4], pos[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t i = i0 + u * (kThreads / 32);
      const bool live = i < staged;
      const uint32_t lo = live ? reinterpret_cast<const uint32_t *>(raw + i * 128)[lane] : 0u;
      const uint32_t hi = live ? reinterpret_cast<const uint32_t *>(raw + i * 128)[32 + lane] : 0u;
      x[u][0] = __uint_as_float(lo << 16);
      x[u][1] = __uint_as_float(lo & 0xffff0000u);
      x[u][2] = __uint_as_float(hi << 16);
      x[u][3] = __uint_as_float(hi & 0xffff0000u);
      const bool is_k = i < n;
      norm[u] = live && (is_k ? p.k_w != nullptr : p.q_w != nullptr);
      wl[u] = is_k ? wk_l : wq_l;
      wh[u] = is_k ? wk_h : wq_h;
      pos[u] = is_k ? i : (i - n) - head_of(i - n) * rows;
      ss[u] = x[u][0] * x[u][0] + x[u][1] * x[u][1] + x[u][2] * x[u][2] + x[u][3] * x[u][3];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < 4; ++u) ss[u] += __shfl_xor_sync(0xffffffffu, ss[u], o);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t i = i0 + u * (kThreads / 32);
      if (i >= staged) continue;
      if (norm[u]) {
        const float inv = rsqrtf(ss[u] / 128.0f + p.eps);
        const float ya0 = x[u][0] * inv * __uint_as_float(wl[u] << 16);
        const float ya1 = x[u][1] * inv * __uint_as_float(wl[u] & 0xffff0000u);
        const float yb0 = x[u][2] * inv * __uint_as_float(wh[u] << 16);
        const float yb1 = x[u][3] * inv * __uint_as_float(wh[u] & 0xffff0000u);
        float s0, c0, s1, c1;
        rope_sincos((float)pos[u] * f0, &s0, &c0);
        rope_sincos((float)pos[u] * f1, &s1, &c1);
        x[u][0] = ya0 * c0 - yb0 * s0;
        x[u][2] = ya0 * s0 + yb0 * c0;
        x[u][1] = ya1 * c1 - yb1 * s1;
        x[u][3] = ya1 * s1 + yb1 * c1;
      }
      uint16_t *dst = i < n ? Ks + i * kRS : Qs + (i - n) * kRS;
      reinterpret_cast<uint32_t *>(dst)[lane] = pack_bf16x2(x[u][0], x[u][1]);
      reinterpret_cast<uint32_t *>(dst)[32 + lane] = pack_bf16x2(x[u][2], x[u][3]);
    }
  }
  __syncthreads();

  // Each warp: tiles of 16 query rows.  Fragment layout of m16n8k16 (g = lane / 4,
  // t = lane % 4): A holds rows g and g+8, columns 2t, 2t+1 (+8); B holds column g, rows
  // 2t, 2t+1 (+8); C holds rows g and g+8, columns 2t, 2t+1.
  const uint32_t g = lane >> 2, t = lane & 3;
  const uint32_t *Qw = reinterpret_cast<const uint32_t *>(Qs);
  const uint32_t *Kw = reinterpret_cast<const uint32_t *>(Ks);
  // Lane l addresses row 16kk + l%16 of V at columns 8nt + 8(l/16) for the transposing
  // matrix load of two B fragments pairs (column blocks nt and nt+1).
  const uint32_t vaddr = (uint32_t)__cvta_generic_to_shared(Vs + (lane & 15) * kRS + 8 * (lane >> 4));
  const uint32_t nkt = (n + 7) / 8, nkk = (n + 15) / 16;  // key tiles of 8 / steps of 16
  for (uint32_t row0 = warp * 16; row0 < R; row0 += kThreads / 2) {
    const uint32_t ra = min(row0 + g, R - 1), rb = min(row0 + g + 8, R - 1);
    float sacc[4][4];
#pragma unroll
    for (int kt = 0; kt < 4; ++kt)
#pragma unroll
      for (int e = 0; e < 4; ++e) sacc[kt][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {  // 16 dims per step
      const uint32_t a0 = Qw[ra * (kRS / 2) + ks * 8 + t], a1 = Qw[rb * (kRS / 2) + ks * 8 + t];
      const uint32_t a2 = Qw[ra * (kRS / 2) + ks * 8 + 4 + t];
      const uint32_t a3 = Qw[rb * (kRS / 2) + ks * 8 + 4 + t];
#pragma unroll
      for (int kt = 0; kt < 4; ++kt) {
        if (kt < (int)nkt) {
          const uint32_t key = min(kt * 8 + g, n - 1);
          mma16816(sacc[kt], a0, a1, a2, a3, Kw[key * (kRS / 2) + ks * 8 + t],
                   Kw[key * (kRS / 2) + ks * 8 + 4 + t]);
        }
      }
    }
    // Masked softmax over the keys of rows g (e = 0, 1) and g+8 (e = 2, 3); the four
    // lanes of a quad hold one row's columns.
    float m[2], l[2];
    uint32_t end[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t r = row0 + g + 8 * h;
      const uint32_t qi = r < R ? r - head_of(r) * rows : 0u;
      // Keys [0, end): the causal prefix of the row's position; a padded row (position
      // at or past the length) sees the whole sequence.
      end[h] = p.causal ? min(qi + 1, n) : n;
      m[h] = -INFINITY;
#pragma unroll
      for (int kt = 0; kt < 4; ++kt)
#pragma unroll
        for (int e = 0; e < 2; ++e)
          if (kt * 8 + 2 * t + e < end[h]) m[h] = fmaxf(m[h], sacc[kt][2 * h + e]);
      m[h] = fmaxf(m[h], __shfl_xor_sync(0xffffffffu, m[h], 1));
      m[h] = fmaxf(m[h], __shfl_xor_sync(0xffffffffu, m[h], 2));
      const float ms = end[h] ? m[h] * p.scale_log2 : 0.f;
      l[h] = 0.f;
#pragma unroll
      for (int kt = 0; kt < 4; ++kt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float pr = 0.f;
          if (kt * 8 + 2 * t + e < end[h])
            asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(pr) : "f"(fmaf(sacc[kt][2 * h + e], p.scale_log2, -ms)));
          sacc[kt][2 * h + e] = pr;
          l[h] += pr;
        }
      l[h] += __shfl_xor_sync(0xffffffffu, l[h], 1);
      l[h] += __shfl_xor_sync(0xffffffffu, l[h], 2);
    }
    // O = P V: P (bf16) straight from the S accumulators as the A operand.
    float oacc[16][4];
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) oacc[nt][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      if (kk < (int)nkk) {
        const uint32_t a0 = pack_bf16x2(sacc[2 * kk][0], sacc[2 * kk][1]);
        const uint32_t a1 = pack_bf16x2(sacc[2 * kk][2], sacc[2 * kk][3]);
        const uint32_t a2 = pack_bf16x2(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
        const uint32_t a3 = pack_bf16x2(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
#pragma unroll
        for (int nt = 0; nt < 16; nt += 2) {
          uint32_t b[4];
          asm volatile(
              "ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
              : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3])
              : "r"(vaddr + (kk * 16 * kRS + nt * 8) * 2));
          mma16816(oacc[nt], a0, a1, a2, a3, b[0], b[1]);
          mma16816(oacc[nt + 1], a0, a1, a2, a3, b[2], b[3]);
        }
      }
    }
    // Normalise and store rows g and g+8 of the tile (columns 8nt + 2t, 2t+1).
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t r = row0 + g + 8 * h;
      if (r >= R) continue;
      const uint32_t gq = head_of(r), qi = r - gq * rows;
      // No valid key: 0/0, as the reference's running sums give.
      const float inv = l[h] > 0.f ? 1.0f / l[h] : __int_as_float(0x7fc00000);
      const size_t o = ((size_t)(tok0 + qi) * p.heads + kvh * G + gq) * 128 + 2 * t;
      if (p.out_bf16) {
        uint32_t *dst = reinterpret_cast<uint32_t *>(static_cast<uint16_t *>(p.out) + o);
#pragma unroll
        for (int nt = 0; nt < 16; ++nt)
          dst[nt * 4] = l[h] > 0.f ? pack_bf16x2(oacc[nt][2 * h] * inv, oacc[nt][2 * h + 1] * inv)
                                   : 0x7fc07fc0u;
      } else {
        float2 *dst = reinterpret_cast<float2 *>(static_cast<float *>(p.out) + o);
#pragma unroll
        for (int nt = 0; nt < 16; ++nt)
          dst[nt * 4] = make_float2(oacc[nt][2 * h] * inv, oacc[nt][2 * h + 1] * inv);
      }
    }
  }
}

}  // namespace sh

bool short_attention_supported(const AttnProblem &p) {
  if (p.dim != 128 || p.in_dtype != 1 || p.scale <= 0.f) return false;
  if (!p.kv_heads || p.heads % p.kv_heads || p.heads / p.kv_heads > sh::kMaxGroup) return false;
  if (!p.seq || p.seq > sh::kMaxRows) return false;
  if (p.batch > 0x7fffffffu || p.kv_heads > 65535u) return false;
  if ((uintptr_t)p.q % 16 || (uintptr_t)p.k % 16 || (uintptr_t)p.v % 16 || (uintptr_t)p.out % 16)
    return false;
  return true;
}

cudaError_t launch_attention_short(const AttnProblem &p, const uint16_t *q_w, const uint16_t *k_w,
                                   float eps, float theta, int *status, cudaStream_t stream) {
  sh::Params k{};
  k.q = static_cast<const uint16_t *>(p.q);
  k.k = static_cast<const uint16_t *>(p.k);
  k.v = static_cast<const uint16_t *>(p.v);
  k.out = p.out;
  k.lengths = p.lengths;
  k.cu = p.cu_seqlens;
  k.seq = p.seq;
  k.heads = p.heads;
  k.kv_heads = p.kv_heads;
  k.group = p.heads / p.kv_heads;
  k.out_bf16 = p.out_dtype == 1;
  k.causal = p.causal;
  k.scale_log2 = p.scale * 1.4426950408889634f;
  k.q_w = q_w;
  k.k_w = k_w;
  k.eps = eps;
  k.status = status;
  // Inverse frequencies in double, rounded once to float (as the other prologue paths);
  // the table of the last theta is kept, so repeated calls skip the pow evaluations.
  static thread_local float last_theta = 0.f, table[64];
  if (theta != last_theta) {
    for (int c = 0; c < 64; ++c) table[c] = (float)std::pow((double)theta, -2.0 * c / 128.0);
    last_theta = theta;
  }
  std::copy(table, table + 64, k.inv_freq);
  // The shared-memory limit is raised once per device, to the largest group's size.
  static bool raised[256] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 256) return cudaErrorInvalidDevice;
  if (!raised[dev]) {
    e = cudaFuncSetAttribute(sh::attn_short_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sh::smem_bytes(sh::kMaxGroup));
    if (e != cudaSuccess) return e;
    raised[dev] = true;
  }
  const size_t smem = sh::smem_bytes(k.group);
  sh::attn_short_kernel<<<dim3(p.batch, p.kv_heads), sh::kThreads, smem, stream>>>(k);
  return cudaGetLastError();
}

}  // namespace tx
