// Attention for head_dim 32 with fp32 inputs and output (BERT/BGE-small: 12 heads x 32,
// bidirectional, key-padding mask by length), the operator of bert.py:196-204 dispatched
// through MetalRuntime._attention (metal.py:532-569), with the semantics of
// kernels.metal:78-103 (a query at position p of a sequence of length n attends to
// [0, causal ? min(p + 1, n) : n); padded query rows included).
//
// The scores go to the tensor cores, the rest stays on the FP32 pipe: with padded query
// rows counted the head_dim-32 problem is ~23 FLOP per byte of I/O, above the fp32 SIMT
// ridge, and half of those FLOPs are Q.K^T.  Per CTA (one per 128 query rows, head,
// sequence), per tile of 128 keys:
//   - every thread loads one query row (once) and one key row, scales q by
//     scale * log2(e), splits each value into a TF32 pair (hi = value rounded to TF32,
//     lo = value - hi) and stores both parts into shared memory in the 128-byte-swizzled
//     K-major layout the tensor core reads (a 32-float row is one 128-byte row); value
//     rows are stored as they are;
//   - one thread issues S = Qhi.Khi + Qhi.Klo + Qlo.Khi (tcgen05.mma kind::tf32,
//     M=128, N=128, K=8, twelve instructions) into 128 tensor-memory columns: about 22
//     significant bits per operand, so the scores carry fp32-level error;
//   - thread t (tensor-memory lane t = query row t) reads its row of S, takes the
//     masked maximum and forms exp2(s - m); threads 2i and 2i+1 exchange these and each
//     accumulates both rows' p * v for its half of the head dimension with packed f32x2
//     FMAs (every value row read as a shared-memory broadcast feeds two rows); the
//     softmax is online across tiles with a lazily updated reference maximum (rescaled
//     only when a chunk maximum exceeds it by more than 8), so every probability stays
//     at most 2^8.
// Key and value rows at or past a sequence's end are never read (zeros are staged), so
// padded rows may hold anything.  The single wait (scores ready) is bounded; a wait that
// gives up records TX_ETIMEOUT | site << 8 and the CTA returns after its MMAs drained.
#include <cuda.h>

#include "../../include/tessattn.h"
#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace tx {
namespace d32tc {

using namespace ptx;

constexpr int kRows = 128;       // query rows per CTA = threads = tensor-memory lanes
constexpr int kKeys = 128;       // keys per tile (N of the score MMA)
constexpr uint32_t kTile = kRows * 128;  // one operand part: 128 rows x 128 bytes
// Shared memory: Q hi, Q lo, K hi, K lo (swizzled, 16 KB each), V (16 KB), barrier.
constexpr uint32_t kOffQ = 0, kOffQlo = kTile, kOffK = 2 * kTile, kOffKlo = 3 * kTile,
                   kOffV = 4 * kTile, kOffBar = 5 * kTile;
constexpr uint32_t kSmemBytes = kOffBar + 1024 + 64;  // + alignment slack
constexpr uint32_t kTmemCols = 128;
constexpr long long kWaitCycles = 2000000000ll;
// kind::tf32: D = f32 (bit 4), A and B TF32 (2 at bits 7 and 10), K-major, N >> 3 at bit
// 17, M >> 4 at bit 24.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kKeys >> 3) << 17) |
                            ((uint32_t)(kRows >> 4) << 24);
constexpr int kSiteScores = 1;

// Stores a 32-float row (r of 128) as a TF32 pair into the swizzled hi and lo tiles:
// 16-byte chunk j of row r sits at chunk j ^ (r % 8) of the row's 128 bytes.
__device__ __forceinline__ void store_split_row(uint32_t hi_tile, uint32_t lo_tile, uint32_t r,
                                                const float (&x)[32]) {
  const uint32_t row = r * 128, sw = r & 7;
#pragma unroll
  for (uint32_t j = 0; j < 8; ++j) {
    float h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      h[e] = tf32_round(x[4 * j + e]);
      l[e] = x[4 * j + e] - h[e];
    }
    const uint32_t off = row + ((j ^ sw) << 4);
    st_shared_v4(hi_tile + off, __float_as_uint(h[0]), __float_as_uint(h[1]),
                 __float_as_uint(h[2]), __float_as_uint(h[3]));
    st_shared_v4(lo_tile + off, __float_as_uint(l[0]), __float_as_uint(l[1]),
                 __float_as_uint(l[2]), __float_as_uint(l[3]));
  }
}

__device__ __forceinline__ void load_row(const float *p, bool ok, float (&x)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 t = ok ? __ldg(reinterpret_cast<const float4 *>(p) + j)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
    x[4 * j] = t.x, x[4 * j + 1] = t.y, x[4 * j + 2] = t.z, x[4 * j + 3] = t.w;
  }
}

__global__ void __launch_bounds__(kRows, 2) attn_d32_tc_kernel(AttnProblem p, int *status) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned window for the swizzled tiles.
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t *smem = smem_raw + (sbase - raw);
  const uint32_t bar = sbase + kOffBar;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffBar + 8);
  const float *vs = reinterpret_cast<const float *>(smem + kOffV);

  const uint32_t tid = threadIdx.x, warp = tid >> 5;
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
  const uint32_t pos = q0 + tid;
  const bool act = pos < rows;
  const uint32_t end = act ? (p.causal ? min(pos + 1, len) : len) : 0u;
  const uint32_t last = min(q0 + kRows, rows) - 1;
  const uint32_t kend = p.causal ? min(last + 1, len) : len;
  const float *q = static_cast<const float *>(p.q), *k = static_cast<const float *>(p.k),
              *v = static_cast<const float *>(p.v);
  float *out = static_cast<float *>(p.out);

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
  // This thread's query row, pre-scaled into log2 units, as a TF32 pair.
  {
    float x[32];
    load_row(q + ((base + pos) * p.heads + head) * 32, act, x);
    const float qs = p.scale * 1.4426950408889634f;
#pragma unroll
    for (int e = 0; e < 32; ++e) x[e] *= qs;
    store_split_row(sbase + kOffQ, sbase + kOffQlo, tid, x);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem + ((warp * 32u) << 16);

  // Threads 2i and 2i+1 (rows 2i and 2i+1) share the output accumulators of both rows,
  // each for one half of the head dimension (h), so every value-row read from shared
  // memory feeds two rows; each thread keeps the softmax state of its own row.
  const uint32_t h = tid & 1;
  uint64_t acc_e[8], acc_o[8];  // rows 2i and 2i+1, columns 16h..16h+15, packed pairs
#pragma unroll
  for (int i = 0; i < 8; ++i) acc_e[i] = acc_o[i] = f2(0.f, 0.f);
  float m = -INFINITY, l = 0.f;
  bool ok = true;
  uint32_t phase = 0;
  for (uint32_t c0 = 0; c0 < kend; c0 += kKeys, phase ^= 1) {
    // Stage key row c0 + tid (split) and value row c0 + tid; rows past the end are zeros.
    {
      const uint32_t key = c0 + tid;
      const bool kin = key < kend;
      const uint64_t row = ((base + key) * p.kv_heads + kvhead) * 32;
      float x[32];
      load_row(k + row, kin, x);
      store_split_row(sbase + kOffK, sbase + kOffKlo, tid, x);
      load_row(v + row, kin, x);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        st_shared_v4(sbase + kOffV + tid * 128 + j * 16, __float_as_uint(x[4 * j]),
                     __float_as_uint(x[4 * j + 1]), __float_as_uint(x[4 * j + 2]),
                     __float_as_uint(x[4 * j + 3]));
    }
    fence_proxy_async();  // generic stores seen by the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      const uint64_t qd = sw128_desc(sbase + kOffQ, 16, 1024), qld = sw128_desc(sbase + kOffQlo, 16, 1024);
      const uint64_t kd = sw128_desc(sbase + kOffK, 16, 1024), kld = sw128_desc(sbase + kOffKlo, 16, 1024);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {  // 8 elements of K = 32 bytes of the swizzled row
        const uint64_t o = (uint64_t)(ks * 2);
        umma_tf32(tmem, qd + o, kd + o, kIdesc, ks > 0 ? 1u : 0u);
        umma_tf32(tmem, qd + o, kld + o, kIdesc, 1u);
        umma_tf32(tmem, qld + o, kd + o, kIdesc, 1u);
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
    // This row's scores, 32 keys at a time: masked maximum of the chunk (the reference
    // maximum moves only when it exceeds it by more than 8), then exp2(s - m) * v.
    const int valid = (int)min(max((int)end - (int)c0, 0), kKeys);
#pragma unroll 1
    for (int c = 0; c < kKeys / 32; ++c) {
      if (c0 + c * 32 >= kend) break;  // uniform: no row has keys there
      uint32_t r[32];
      tmem_ld32(tS + c * 32, r);
      tmem_ld_wait();
      float mc = -INFINITY;
#pragma unroll
      for (int t = 0; t < 32; ++t)
        if (c * 32 + t < valid) mc = fmaxf(mc, __uint_as_float(r[t]));
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
        for (int i = 0; i < 8; ++i) {
          acc_e[i] = mul2(acc_e[i], ce2);
          acc_o[i] = mul2(acc_o[i], co2);
        }
      }
      const float *vc = vs + c * 32 * 32 + 16 * h;
#pragma unroll
      for (int t = 0; t < 32; ++t) {
        const float pj = c * 32 + t < valid ? ex2(__uint_as_float(r[t]) - m) : 0.f;
        l += pj;
        const float pp = __shfl_xor_sync(0xffffffffu, pj, 1);
        const float pe = h ? pp : pj, po = h ? pj : pp;
        const uint64_t pe2 = f2(pe, pe), po2 = f2(po, po);
        const float4 *vr = reinterpret_cast<const float4 *>(vc + t * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 vv = vr[i];
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
    // This thread's half of rows 2i and 2i+1 (zero valid keys: 0/0, as the reference's
    // sums give).
    const float l_pair = __shfl_xor_sync(0xffffffffu, l, 1);
    const float inv_e = 1.0f / (h ? l_pair : l), inv_o = 1.0f / (h ? l : l_pair);
    const uint32_t pos_e = q0 + (tid & ~1u);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint32_t prow = pos_e + r;
      if (!ok || prow >= rows) continue;
      const uint64_t(&a)[8] = r ? acc_o : acc_e;
      const float inv = r ? inv_o : inv_e;
      float4 *op =
          reinterpret_cast<float4 *>(out + ((base + prow) * p.heads + head) * 32 + 16 * h);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
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

}  // namespace d32tc

bool d32_tc_supported(const AttnProblem &p) {
  return p.dim == 32 && p.in_dtype == TX_F32 && p.out_dtype == TX_F32 && p.kv_heads &&
         p.heads % p.kv_heads == 0 && p.batch <= 65535u && p.heads <= 65535u &&
         (uintptr_t)p.q % 16 == 0 && (uintptr_t)p.k % 16 == 0 && (uintptr_t)p.v % 16 == 0 &&
         (uintptr_t)p.out % 16 == 0 && p.scale > 0.f;
}

cudaError_t launch_attention_d32_tc(const AttnProblem &p, int *status, cudaStream_t stream) {
  if (!d32_tc_supported(p)) return cudaErrorInvalidValue;
  const uint32_t qblocks = (p.seq + d32tc::kRows - 1) / d32tc::kRows;
  if (!qblocks || qblocks > 65535u) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(d32tc::attn_d32_tc_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)d32tc::kSmemBytes);
  if (e != cudaSuccess) return e;
  const dim3 grid(qblocks, p.heads, p.batch);
  d32tc::attn_d32_tc_kernel<<<grid, d32tc::kRows, d32tc::kSmemBytes, stream>>>(p, status);
  return cudaGetLastError();
}

}  // namespace tx
