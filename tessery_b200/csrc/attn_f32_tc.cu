// Attention for head_dim 128 with fp32 inputs and output: the call the reference's Qwen3
// adapter makes (qwen3.py:238-245, MetalRuntime._attention with float buffers,
// metal.py:532-569), which the reference serves with its F32 SIMD-group-MMA tiled kernel
// (kernels.metal:108-170), with the semantics of kernels.metal:78-103 (a query at position
// p of a sequence of length n attends to [0, causal ? min(p + 1, n) : n); padded query
// rows included).
//
// Scores on the tensor cores, the rest on the FP32 pipe.  One CTA (8 warps) per (128
// query rows, head, sequence); per tile of 64 keys:
//   - each warp stages 16 rows a row at a time (lane l: floats 4l..4l+3, so every load
//     is one coalesced 512-byte row): the CTA's query rows once (scaled by
//     scale * log2(e)), then per tile warps 0-3 the key rows and warps 4-7 the value rows.
//     Query and key rows are split into TF32 pairs (hi = value rounded to TF32, lo =
//     value - hi) and stored in the 128-byte-swizzled K-major layout, one 32-float column
//     block per 128-byte row; value rows are stored whole, the odd 32-float quarters with
//     their 16-byte chunks permuted (chunk i at i ^ 4) so that the two quarters a warp
//     reads at once fall on different banks;
//   - one thread issues the scores with tcgen05.mma kind::tf32 (M=128, N=64, K=8) into
//     three accumulators of 64 tensor-memory columns: Qhi.Khi over columns 0-63 of the
//     head dimension, Qhi.Khi over columns 64-127, and the corrections Qhi.Klo + Qlo.Khi
//     (2^-11 of the scores' size), so that no main product takes more than 8 updates (the
//     tensor core's fp32 accumulation loses bits on long chains) -- about 22 significant
//     bits per operand;
//   - warps w and w + 4 both take query rows 32 (w % 4) .. + 31 (tensor-memory lanes of
//     warp w % 4), each thread one row: it adds the row's three partial scores 16 keys at
//     a time, takes masked chunk maxima and forms exp2(s - m); threads 2i and 2i+1
//     exchange these and each accumulates both rows' p * v for one quarter of the head
//     dimension (32 columns: warps 0-3 the first half, warps 4-7 the second) with packed
//     f32x2 FMAs, every value row read as a shared-memory broadcast feeding two rows; the
//     softmax is online across tiles with a lazily updated reference maximum (rescaled
//     only when a chunk maximum exceeds it by more than 8), so every probability stays at
//     most 2^8.
// Key and value rows at or past a sequence's end are never read (zeros are staged).  The
// single wait (scores ready) is bounded; a wait that gives up records
// TX_ETIMEOUT | site << 8 and the CTA returns after its MMAs drained.
#include <cuda.h>

#include "../../include/tessattn.h"
#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace tx {
namespace f32tc {

using namespace ptx;

constexpr int kRows = 128;  // query rows per CTA = tensor-memory lanes
constexpr int kThreads = 256;  // two threads per query row (each half of the head dimension)
constexpr int kKeys = 64;   // keys per tile (N of the score MMA)
constexpr int kD = 128;
constexpr uint32_t kQBlock = kRows * 128;  // one 32-column block of Q: 128 rows x 128 B
constexpr uint32_t kKBlock = kKeys * 128;  // one 32-column block of K: 64 rows x 128 B
// Shared memory: Q hi, Q lo (4 blocks each), K hi, K lo (4 blocks each), V, barrier.
constexpr uint32_t kOffQ = 0, kOffQlo = 4 * kQBlock, kOffK = 8 * kQBlock,
                   kOffKlo = kOffK + 4 * kKBlock, kOffV = kOffKlo + 4 * kKBlock,
                   kOffBar = kOffV + kKeys * kD * 4;
constexpr uint32_t kSmemBytes = kOffBar + 1024 + 64;  // + alignment slack
static_assert(kSmemBytes <= 232448, "shared memory budget");
constexpr uint32_t kTmemCols = 256;  // three 64-column accumulators
constexpr long long kWaitCycles = 2000000000ll;
// kind::tf32: D = f32 (bit 4), A and B TF32 (2 at bits 7 and 10), K-major, N >> 3 at bit
// 17, M >> 4 at bit 24.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kKeys >> 3) << 17) |
                            ((uint32_t)(kRows >> 4) << 24);
constexpr int kSiteScores = 1;


// Rows r0..r0+15 of a tile into shared memory, one warp, a row at a time: row r is read
// from src + r * stride (lane l: floats 4l..4l+3); rows at or past `nvalid` are zeros.
// kSplit: scaled by `scale`, split into TF32 pairs and stored swizzled (column block
// b = l / 8 of row r at hi/lo + b * blk + r * 128, 16-byte chunk j = l % 8 at chunk
// j ^ (r % 8)); otherwise stored whole at hi + r * 512, chunk l at l ^ 4 when l / 8 is odd.
template <bool kSplit>
__device__ __forceinline__ void stage_rows(const float *src, uint64_t stride, uint32_t r0,
                                           uint32_t nvalid, float scale, uint32_t hi,
                                           uint32_t lo, uint32_t blk, uint32_t lane) {
  const uint32_t b = lane >> 3, j = lane & 7;
#pragma unroll 1
  for (uint32_t i0 = 0; i0 < 16; i0 += 8) {
    float4 x[8];
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) {
      const uint32_t r = r0 + i0 + i;
      x[i] = r < nvalid ? __ldg(reinterpret_cast<const float4 *>(src + r * stride) + lane)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) {
      const uint32_t r = r0 + i0 + i;
      if (kSplit) {
        const float4 t = make_float4(x[i].x * scale, x[i].y * scale, x[i].z * scale,
                                     x[i].w * scale);
        const float h0 = tf32_round(t.x), h1 = tf32_round(t.y), h2 = tf32_round(t.z),
                    h3 = tf32_round(t.w);
        const uint32_t off = b * blk + r * 128 + ((j ^ (r & 7)) << 4);
        st_shared_v4(hi + off, __float_as_uint(h0), __float_as_uint(h1), __float_as_uint(h2),
                     __float_as_uint(h3));
        st_shared_v4(lo + off, __float_as_uint(t.x - h0), __float_as_uint(t.y - h1),
                     __float_as_uint(t.z - h2), __float_as_uint(t.w - h3));
      } else {
        st_shared_v4(hi + r * (kD * 4) + ((lane ^ ((lane >> 1) & 4)) << 4), __float_as_uint(x[i].x),
                     __float_as_uint(x[i].y), __float_as_uint(x[i].z), __float_as_uint(x[i].w));
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1) attn_f32_tc_kernel(AttnProblem p, int *status) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned window for the swizzled blocks.
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t *smem = smem_raw + (sbase - raw);
  const uint32_t bar = sbase + kOffBar;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffBar + 8);
  const float *vs = reinterpret_cast<const float *>(smem + kOffV);

  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, h = tid & 1;
  // Query row of this thread within the CTA (tensor-memory lane) and its column quarter.
  const uint32_t quad = warp & 3, row = quad * 32 + lane, quarter = (warp >> 2) * 2 + h;
  const uint32_t qblock = blockIdx.x, head = blockIdx.y, seqi = blockIdx.z;
  const uint32_t kvhead = head / (p.heads / p.kv_heads);
  uint32_t len, rows;
  uint64_t base;
  if (p.cu_seqlens) {
    const int32_t a = p.cu_seqlens[seqi], b = p.cu_seqlens[seqi + 1];
    len = b > a ? (uint32_t)(b - a) : 0u;
    rows = len;
    base = (uint32_t)a;
  } else {
    len = min(p.lengths[seqi], p.seq);
    rows = p.seq;
    base = (uint64_t)seqi * p.seq;
  }
  const uint32_t q0 = qblock * kRows;
  if (q0 >= rows) return;  // uniform over the CTA
  const uint32_t pos = q0 + row;
  const uint32_t end = pos < rows ? (p.causal ? min(pos + 1, len) : len) : 0u;
  const uint32_t last = min(q0 + kRows, rows) - 1;
  const uint32_t kend = p.causal ? min(last + 1, len) : len;
  const float *q = static_cast<const float *>(p.q), *k = static_cast<const float *>(p.k),
              *v = static_cast<const float *>(p.v);
  float *out = static_cast<float *>(p.out);
  const uint64_t kv_stride = (uint64_t)p.kv_heads * kD;

  if (tid == 0) {
    mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // The CTA's query rows, pre-scaled into log2 units, as TF32 pairs.
  stage_rows<true>(q + ((base + q0) * p.heads + head) * kD, (uint64_t)p.heads * kD, warp * 16,
                   rows - q0, p.scale * 1.4426950408889634f, sbase + kOffQ, sbase + kOffQlo,
                   kQBlock, lane);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem + ((quad * 32u) << 16);

  // Threads 2i and 2i+1 (rows 2i and 2i+1) share the output accumulators of both rows,
  // each for one quarter of the head dimension; each keeps its own row's softmax state.
  uint64_t acc_e[16], acc_o[16];  // rows 2i and 2i+1, columns 32q..32q+31, packed pairs
#pragma unroll
  for (int i = 0; i < 16; ++i) acc_e[i] = acc_o[i] = f2(0.f, 0.f);
  float m = -INFINITY, l = 0.f;
  bool ok = true;
  uint32_t phase = 0;
  for (uint32_t c0 = 0; c0 < kend; c0 += kKeys, phase ^= 1) {
    // Key rows (warps 0-3, split) and value rows (warps 4-7) of the tile; rows past the end
    // are zeros.
    {
      const float *src = (warp < 4 ? k : v) + ((base + c0) * p.kv_heads + kvhead) * kD;
      if (warp < 4)
        stage_rows<true>(src, kv_stride, warp * 16, kend - c0, 1.0f, sbase + kOffK,
                         sbase + kOffKlo, kKBlock, lane);
      else
        stage_rows<false>(src, kv_stride, (warp - 4) * 16, kend - c0, 1.0f, sbase + kOffV, 0u,
                          0u, lane);
    }
    fence_proxy_async();  // generic stores seen by the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
#pragma unroll
      for (uint32_t dc = 0; dc < 4; ++dc) {  // 32-column block of the head dimension
        const uint64_t qd = sw128_desc(sbase + kOffQ + dc * kQBlock, 16, 1024);
        const uint64_t qld = sw128_desc(sbase + kOffQlo + dc * kQBlock, 16, 1024);
        const uint64_t kd = sw128_desc(sbase + kOffK + dc * kKBlock, 16, 1024);
        const uint64_t kld = sw128_desc(sbase + kOffKlo + dc * kKBlock, 16, 1024);
        const uint32_t main_acc = tmem + (dc >> 1) * kKeys, corr = tmem + 2 * kKeys;
#pragma unroll
        for (uint32_t ks = 0; ks < 4; ++ks) {  // 8 elements = 32 bytes of the swizzled row
          const uint64_t o = (uint64_t)(ks * 2);
          umma_tf32(main_acc, qd + o, kd + o, kIdesc, ((dc & 1) | ks) ? 1u : 0u);
          umma_tf32(corr, qd + o, kld + o, kIdesc, (dc | ks) ? 1u : 0u);
          umma_tf32(corr, qld + o, kd + o, kIdesc, 1u);
        }
      }
      umma_commit(bar);
    }
    // Scores ready (bounded wait).
    {
      const long long t0 = clock64();
      while (!mbar_test(bar, phase) && ok)
        if (clock64() - t0 > kWaitCycles) ok = false;
    }
    if (!__syncthreads_and(ok)) {
      // The issued MMAs complete by themselves: wait for them before the columns are
      // freed, then return without output.
      if (tid == 0) report_status(status, kStatusTimeout | (kSiteScores << 8));
      const long long t0 = clock64();
      while (!mbar_test(bar, phase) && clock64() - t0 < kWaitCycles) {
      }
      ok = false;
      break;
    }
    tc_fence_after();
    // This row's scores, 16 keys at a time: the three partial sums added, masked maximum of
    // the chunk (the reference maximum moves only when it exceeds it by more than 8), then
    // exp2(s - m) * v.
    const int valid = (int)min(max((int)end - (int)c0, 0), kKeys);
#pragma unroll 1
    for (int c = 0; c < kKeys / 16; ++c) {
      if (c0 + c * 16 >= kend) break;  // uniform: no row has keys there
      float s[16];
      {
        uint32_t a[16], b[16];
        tmem_ld16(tS + c * 16, a);
        tmem_ld16(tS + kKeys + c * 16, b);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 16; ++t) s[t] = __uint_as_float(a[t]) + __uint_as_float(b[t]);
        tmem_ld16(tS + 2 * kKeys + c * 16, a);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 16; ++t) s[t] += __uint_as_float(a[t]);
      }
      float mc = -INFINITY;
#pragma unroll
      for (int t = 0; t < 16; ++t)
        if (c * 16 + t < valid) mc = fmaxf(mc, s[t]);
      float cr = 1.0f;  // rescale factor of this thread's row (1: none)
      if (mc > m + 8.0f) {  // also the first chunk with a valid key (m = -inf)
        cr = ex2(m - mc);
        l *= cr;
        m = mc;
      }
      const float cr_pair = __shfl_xor_sync(0xffffffffu, cr, 1);
      if (__any_sync(0xffffffffu, cr != 1.0f || cr_pair != 1.0f)) {
        const float ce = h ? cr_pair : cr, co = h ? cr : cr_pair;
        const uint64_t ce2 = f2(ce, ce), co2 = f2(co, co);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          acc_e[i] = mul2(acc_e[i], ce2);
          acc_o[i] = mul2(acc_o[i], co2);
        }
      }
      // This thread's quarter of the value rows: chunk i sits at chunk i ^ 4h, i.e. at
      // va_lo + 4i for i < 4 and at va_hi + 4i for i >= 4.
      const float *vq = vs + c * 16 * kD + 32 * quarter;
      const float *va_lo = vq + 16 * h, *va_hi = vq - 16 * h;
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const float pj = c * 16 + t < valid ? ex2(s[t] - m) : 0.f;
        l += pj;
        const float pp = __shfl_xor_sync(0xffffffffu, pj, 1);
        const float pe = h ? pp : pj, po = h ? pj : pp;
        const uint64_t pe2 = f2(pe, pe), po2 = f2(po, po);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 vv = *reinterpret_cast<const float4 *>((i < 4 ? va_lo : va_hi) + t * kD + 4 * i);
          const uint64_t va = f2(vv.x, vv.y), vb = f2(vv.z, vv.w);
          acc_e[2 * i] = fma2(pe2, va, acc_e[2 * i]);
          acc_e[2 * i + 1] = fma2(pe2, vb, acc_e[2 * i + 1]);
          acc_o[2 * i] = fma2(po2, va, acc_o[2 * i]);
          acc_o[2 * i + 1] = fma2(po2, vb, acc_o[2 * i + 1]);
        }
      }
    }
    // Shared memory and the score columns are reused by the next tile.
    tc_fence_before();
    __syncthreads();
  }
  {
    // This thread's quarter of rows 2i and 2i+1 (zero valid keys: 0/0, as the reference's
    // sums give).
    const float l_pair = __shfl_xor_sync(0xffffffffu, l, 1);
    const float inv_e = 1.0f / (h ? l_pair : l), inv_o = 1.0f / (h ? l : l_pair);
    const uint32_t pos_e = q0 + (row & ~1u);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint32_t prow = pos_e + r;
      if (!ok || prow >= rows) continue;
      const uint64_t(&a)[16] = r ? acc_o : acc_e;
      const float inv = r ? inv_o : inv_e;
      float4 *op =
          reinterpret_cast<float4 *>(out + ((base + prow) * p.heads + head) * kD + 32 * quarter);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 x0 = f2_unpack(a[2 * i]), x1 = f2_unpack(a[2 * i + 1]);
        op[i] = make_float4(x0.x * inv, x0.y * inv, x1.x * inv, x1.y * inv);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
}

}  // namespace f32tc

bool f32_tc_supported(const AttnProblem &p) {
  return p.dim == 128 && p.in_dtype == TX_F32 && p.out_dtype == TX_F32 && p.kv_heads &&
         p.heads % p.kv_heads == 0 && p.batch <= 65535u && p.heads <= 65535u &&
         (uintptr_t)p.q % 16 == 0 && (uintptr_t)p.k % 16 == 0 && (uintptr_t)p.v % 16 == 0 &&
         (uintptr_t)p.out % 16 == 0 && p.scale > 0.f;
}

cudaError_t launch_attention_f32_tc(const AttnProblem &p, int *status, cudaStream_t stream) {
  if (!f32_tc_supported(p)) return cudaErrorInvalidValue;
  const uint32_t qblocks = (p.seq + f32tc::kRows - 1) / f32tc::kRows;
  if (!qblocks || qblocks > 65535u) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(f32tc::attn_f32_tc_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)f32tc::kSmemBytes);
  if (e != cudaSuccess) return e;
  const dim3 grid(qblocks, p.heads, p.batch);
  f32tc::attn_f32_tc_kernel<<<grid, f32tc::kThreads, f32tc::kSmemBytes, stream>>>(p, status);
  return cudaGetLastError();
}

}  // namespace tx
