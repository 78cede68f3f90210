// Attention for head_dim 32 with fp32 inputs and output (BERT/BGE-small: 12 heads x 32,
// bidirectional, key-padding mask by length), the operator of bert.py:196-204 dispatched
// through MetalRuntime._attention (metal.py:532-569), with the semantics of
// kernels.metal:78-103 (a query at position p of a sequence of length n attends to
// [0, causal ? min(p + 1, n) : n); padded query rows included).
//
// Both products on the tensor cores, as three-product TF32 splits (hi = value rounded to
// TF32, lo = value - hi; hi.hi + hi.lo + lo.hi keeps about 22 significant bits per
// operand, fp32-level error); the FP32 pipe keeps only the softmax.  With padded query
// rows counted the head_dim-32 problem is ~23 FLOP per byte of I/O, and on the FP32 pipe
// alone P.V by itself would take longer than the HBM traffic.  One CTA (4 warps, thread t
// = query row t = tensor-memory lane t) per (128 query rows, head, sequence); per tile of
// T keys (T = 64, two CTAs per SM, for launches within one wave; T = 32, three CTAs per
// SM, beyond):
//   - thread t stages query row t once (scaled by scale * log2(e)), then per tile
//     threads [0, T) key row c0 + t and threads [T, 2T) value row c0 + t - T, as TF32
//     pairs in the 128-byte-swizzled K-major layouts the tensor core reads: Q and K one
//     128-byte row per token, V transposed (V^T: one row per head-dimension column, 32
//     keys per 128-byte block).  Two K/V buffers: tile j + 2 is staged once P.V of tile
//     j has run, tile j + 1 is in place when Q.K^T of tile j + 1 is issued;
//   - one thread issues S = Qhi.Khi + Qhi.Klo + Qlo.Khi (M=128, N=T, K=8, twelve
//     instructions) into T tensor-memory columns;
//   - thread t reads its row of S, takes the masked tile maximum (the reference maximum
//     moves only when it exceeds it by more than 8, so every probability stays at most
//     2^8), forms p = exp2(s - m) and writes its TF32 pair into tensor memory, hi over S
//     and lo beside it;
//   - one thread issues O_t = Phi.Vhi (into 32 columns) and Phi.Vlo + Plo.Vhi (into 32
//     more) with P as the tensor-memory A operand (M=128, N=32, K=8, 3T/8 instructions);
//   - with the next tile's scores thread t reads both partial outputs of the previous
//     tile and adds them to its row's fp32 accumulators, rescaled with the maximum.
// Key and value rows at or past a sequence's end are never read (zeros are staged), so
// padded rows may hold anything.  Every wait is bounded; a wait that gives up records
// TX_ETIMEOUT | site << 8 and the CTA returns once the products it issued have drained.
#include <cuda.h>

#include "../../include/tessattn.h"
#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace tx {
namespace d32tc {

using namespace ptx;

constexpr int kRows = 128;  // query rows per CTA = threads = tensor-memory lanes
constexpr int kD = 32;
constexpr uint32_t kQPart = kRows * 128;   // Q hi or lo: 128 rows x 128 B
constexpr uint32_t kVBlock = kD * 128;     // V^T block of 32 keys: 32 rows x 128 B
constexpr uint32_t kOffQ = 0, kOffQlo = kQPart, kOffKV = 2 * kQPart;
constexpr long long kWaitCycles = 2000000000ll;
// kind::tf32: D = f32 (bit 4), A and B TF32 (2 at bits 7 and 10), K-major, N >> 3 at bit
// 17, M >> 4 at bit 24.
constexpr uint32_t idesc_tf32(uint32_t n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((n >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);
}
constexpr int kSiteScores = 1, kSiteOutput = 2;

// Layout for tiles of kKeys keys (N of the score MMA, K of the output MMA): 64-key tiles
// take fewer round trips per CTA (the one-wave latency case), 32-key tiles fit three
// CTAs per SM (128 tensor-memory columns, 65 KB of shared memory, <= 168 registers).
template <int kKeys>
struct Cfg {
  static_assert(kKeys == 32 || kKeys == 64, "tile of 32 or 64 keys");
  static constexpr int kChunks = kKeys / 32;            // 32-column chunks of a score row
  static constexpr uint32_t kKPart = kKeys * 128;       // K hi or lo: 128 B per key
  static constexpr uint32_t kVPart = kChunks * kVBlock;  // V^T hi or lo: a block per 32 keys
  static constexpr uint32_t kKVBuf = 2 * kKPart + 2 * kVPart;  // K hi, K lo, V^T hi, V^T lo
  // Shared memory: Q hi, Q lo, then two K/V buffers, then the barriers.
  static constexpr uint32_t kOffBar = kOffKV + 2 * kKVBuf;
  static constexpr uint32_t kSmemBytes = kOffBar + 1024 + 64;  // + alignment slack
  // Tensor memory: S / P hi [0, kKeys), P lo [kKeys, 2 kKeys), O main and O corr.
  static constexpr uint32_t kColPlo = kKeys, kColOm = 2 * kKeys, kColOc = 2 * kKeys + kD;
  static constexpr uint32_t kTmemCols = kColOc + kD <= 128 ? 128 : 256;  // a power of two
  static constexpr int kCtasPerSm = kTmemCols == 128 ? 3 : 2;
  static constexpr uint32_t kIdescQK = idesc_tf32(kKeys), kIdescPV = idesc_tf32(kD);
};

// D (+)= A B, A (TF32, lane = row, one element per column) read from tensor memory.
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// A 32-float row (8 float4 from global memory, or zeros), scaled.
__device__ __forceinline__ void load_row(const float *src, bool ok, float scale,
                                         float4 (&x)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float4 t = ok ? __ldg(reinterpret_cast<const float4 *>(src) + j)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
    x[j] = make_float4(t.x * scale, t.y * scale, t.z * scale, t.w * scale);
  }
}

// Row r of a K-major operand (128 B per row) as a TF32 pair: 16-byte chunk j of row r at
// chunk j ^ (r % 8).
__device__ __forceinline__ void store_split_row(uint32_t hi, uint32_t lo, uint32_t r,
                                                const float4 (&x)[8]) {
  const uint32_t row = r * 128, sw = r & 7;
#pragma unroll
  for (uint32_t j = 0; j < 8; ++j) {
    const float h0 = tf32_round(x[j].x), h1 = tf32_round(x[j].y), h2 = tf32_round(x[j].z),
                h3 = tf32_round(x[j].w);
    const uint32_t off = row + ((j ^ sw) << 4);
    st_shared_v4(hi + off, __float_as_uint(h0), __float_as_uint(h1), __float_as_uint(h2),
                 __float_as_uint(h3));
    st_shared_v4(lo + off, __float_as_uint(x[j].x - h0), __float_as_uint(x[j].y - h1),
                 __float_as_uint(x[j].z - h2), __float_as_uint(x[j].w - h3));
  }
}

// Value row `key` (of 64) as column `key` of V^T, a TF32 pair: V^T row d (head-dimension
// column d) holds the keys of a 32-key block in 128 bytes, 16-byte chunk j (keys 4j..4j+3
// of the block) at chunk j ^ (d % 8).  Threads of a warp hold 32 consecutive keys, so
// each 4-byte store of a warp fills one 128-byte row without bank conflicts.
__device__ __forceinline__ void store_split_col(uint32_t hi, uint32_t lo, uint32_t key,
                                                const float4 (&x)[8]) {
  const uint32_t blk = (key >> 5) * kVBlock, k = key & 31, j = k >> 2, e = (k & 3) * 4;
#pragma unroll
  for (uint32_t c = 0; c < 8; ++c) {
    const float v[4] = {x[c].x, x[c].y, x[c].z, x[c].w};
#pragma unroll
    for (uint32_t i = 0; i < 4; ++i) {
      const uint32_t d = 4 * c + i;
      const uint32_t off = blk + d * 128 + ((j ^ (d & 7)) << 4) + e;
      const float h = tf32_round(v[i]);
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(hi + off), "r"(__float_as_uint(h)));
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(lo + off), "r"(__float_as_uint(v[i] - h)));
    }
  }
}

template <int kKeys>
__global__ void __launch_bounds__(kRows, Cfg<kKeys>::kCtasPerSm)
    attn_d32_tc_kernel(AttnProblem p, int *status) {
  using C = Cfg<kKeys>;
  constexpr int kChunks = C::kChunks;
  constexpr uint32_t kKPart = C::kKPart, kVPart = C::kVPart, kKVBuf = C::kKVBuf,
                     kOffBar = C::kOffBar, kColPlo = C::kColPlo, kColOm = C::kColOm,
                     kColOc = C::kColOc, kTmemCols = C::kTmemCols, kIdescQK = C::kIdescQK,
                     kIdescPV = C::kIdescPV;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned window for the swizzled operands.
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t *smem = smem_raw + (sbase - raw);
  const uint32_t bar_s = sbase + kOffBar, bar_o = bar_s + 8, bar_d = bar_s + 16;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffBar + 24);

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
  const uint32_t ntiles = (kend + kKeys - 1) / kKeys;
  const float *q = static_cast<const float *>(p.q), *k = static_cast<const float *>(p.k),
              *v = static_cast<const float *>(p.v);
  float *out = static_cast<float *>(p.out);

  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    mbar_init(bar_d, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // Tile j of keys for K/V buffer j % 2: threads [0, kKeys) a key row, [kKeys, 2 kKeys) a
  // value row;
  // rows at or past kend are zeros.  Loads and stores are separate steps so that the
  // first tiles' loads are all in flight at once.
  const uint32_t r_kv = tid & (kKeys - 1);
  auto load_tile = [&](uint32_t j, float4 (&x)[8]) {
    const uint32_t key = j * kKeys + r_kv;
    const uint64_t row = ((base + key) * p.kv_heads + kvhead) * kD;
    load_row((tid < (uint32_t)kKeys ? k : v) + row, key < kend && tid < 2u * kKeys, 1.0f, x);
  };
  auto store_tile = [&](uint32_t j, const float4 (&x)[8]) {
    const uint32_t buf = sbase + kOffKV + (j & 1) * kKVBuf;
    if (tid < (uint32_t)kKeys)
      store_split_row(buf, buf + kKPart, r_kv, x);
    else if (tid < 2u * kKeys)
      store_split_col(buf + 2 * kKPart, buf + 2 * kKPart + kVPart, r_kv, x);
  };
  auto stage = [&](uint32_t j) {
    float4 x[8];
    load_tile(j, x);
    store_tile(j, x);
  };
  {
    float4 xq[8], x0[8], x1[8];
    load_row(q + ((base + pos) * p.heads + head) * kD, act, p.scale * 1.4426950408889634f, xq);
    load_tile(0, x0);  // rows past kend (no tile) are zeros and never stored
    load_tile(1, x1);
    store_split_row(sbase + kOffQ, sbase + kOffQlo, tid, xq);
    if (ntiles > 0) store_tile(0, x0);
    if (ntiles > 1) store_tile(1, x1);
  }
  fence_proxy_async();  // generic stores seen by the tensor core
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tL = tmem + ((warp * 32u) << 16);  // this warp's lanes

  // S = Q K_j^T, three TF32 products over the 32 columns (4 steps of 8).
  auto issue_qk = [&](uint32_t j) {
    const uint32_t buf = sbase + kOffKV + (j & 1) * kKVBuf;
    const uint64_t qd = sw128_desc(sbase + kOffQ, 16, 1024);
    const uint64_t qld = sw128_desc(sbase + kOffQlo, 16, 1024);
    const uint64_t kd = sw128_desc(buf, 16, 1024), kld = sw128_desc(buf + kKPart, 16, 1024);
#pragma unroll
    for (uint32_t ks = 0; ks < 4; ++ks) {
      const uint64_t o = (uint64_t)(ks * 2);  // 8 elements = 32 bytes of the swizzled row
      umma_tf32(tmem, qd + o, kd + o, kIdescQK, ks > 0 ? 1u : 0u);
      umma_tf32(tmem, qd + o, kld + o, kIdescQK, 1u);
      umma_tf32(tmem, qld + o, kd + o, kIdescQK, 1u);
    }
    umma_commit(bar_s);
  };
  // O_j = P V_j over the tile's keys (steps of 8): Phi.Vhi into the main columns,
  // Phi.Vlo + Plo.Vhi into the correction columns.
  auto issue_pv = [&](uint32_t j) {
    const uint32_t vb = sbase + kOffKV + (j & 1) * kKVBuf + 2 * kKPart;
#pragma unroll
    for (uint32_t ks = 0; ks < kKeys / 8; ++ks) {
      const uint32_t blk = (ks >> 2) * kVBlock;
      const uint64_t o = (uint64_t)((ks & 3) * 2);
      const uint64_t vd = sw128_desc(vb + blk, 16, 1024) + o;
      const uint64_t vld = sw128_desc(vb + kVPart + blk, 16, 1024) + o;
      umma_tf32_ts(tmem + kColOm, tmem + 8 * ks, vd, kIdescPV, ks > 0 ? 1u : 0u);
      umma_tf32_ts(tmem + kColOc, tmem + 8 * ks, vld, kIdescPV, ks > 0 ? 1u : 0u);
      umma_tf32_ts(tmem + kColOc, tmem + kColPlo + 8 * ks, vd, kIdescPV, 1u);
    }
    umma_commit(bar_o);
  };
  // Bounded wait for phase `parity` of barrier b.
  auto wait_bar = [&](uint32_t b, uint32_t parity) -> bool {
    const long long t0 = clock64();
    while (!mbar_test(b, parity))
      if (clock64() - t0 > kWaitCycles) return false;
    return true;
  };

  if (tid == 0 && ntiles > 0) issue_qk(0);
  float acc[kD];
#pragma unroll
  for (int d = 0; d < kD; ++d) acc[d] = 0.f;
  float m = -INFINITY, l = 0.f;
  bool ok = true;
  int site = 0;
  for (uint32_t j = 0; j < ntiles; ++j) {
    // S_j ready: committed after P.V of tile j - 1, so that one ran too.
    if (!__syncthreads_and(wait_bar(bar_s, j & 1))) {
      ok = false;
      site = kSiteScores;
      break;
    }
    tc_fence_after();
    uint32_t sr[kKeys];
#pragma unroll
    for (int c = 0; c < kChunks; ++c)
      tmem_ld32(tL + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(sr + 32 * c));
    if (j > 0) {  // tile j - 1's partial outputs into the accumulators
      uint32_t om[32], oc[32];
      tmem_ld32(tL + kColOm, om);
      tmem_ld32(tL + kColOc, oc);
      tmem_ld_wait();
#pragma unroll
      for (int d = 0; d < kD; ++d) acc[d] += __uint_as_float(om[d]) + __uint_as_float(oc[d]);
    } else {
      tmem_ld_wait();
    }
    const int valid = (int)min(max((int)end - (int)(j * kKeys), 0), kKeys);
    float mc = -INFINITY;
#pragma unroll
    for (int t = 0; t < kKeys; ++t)
      if (t < valid) mc = fmaxf(mc, __uint_as_float(sr[t]));
    if (mc > m + 8.0f) {  // also the first tile with a valid key (m = -inf)
      const float cr = ex2(m - mc);
      l *= cr;
#pragma unroll
      for (int d = 0; d < kD; ++d) acc[d] *= cr;
      m = mc;
    }
    // P as a TF32 pair: hi over S, lo beside it (32 keys at a time).
#pragma unroll
    for (int h = 0; h < kChunks; ++h) {
      uint32_t ph[32], pl[32];
#pragma unroll
      for (int t = 0; t < 32; ++t) {
        const float pj = 32 * h + t < valid ? ex2(__uint_as_float(sr[32 * h + t]) - m) : 0.f;
        l += pj;
        const float hi = tf32_round(pj);
        ph[t] = __float_as_uint(hi);
        pl[t] = __float_as_uint(pj - hi);
      }
      tmem_st32(tL + 32 * h, ph);
      tmem_st32(tL + kColPlo + 32 * h, pl);
    }
    tmem_st_wait();
    tc_fence_before();
    __syncthreads();  // P complete in every lane; tile j + 1 staged
    tc_fence_after();
    if (tid == 0) {
      issue_pv(j);
      if (j + 1 < ntiles) issue_qk(j + 1);
    }
    if (j + 2 < ntiles) {
      // Tile j + 2 into this tile's buffer once P.V of tile j (the last reader) ran; the
      // next iteration's barrier orders the stores before its Q.K^T is issued.
      if (!__syncthreads_and(wait_bar(bar_o, j & 1))) {
        ok = false;
        site = kSiteOutput;
        break;
      }
      stage(j + 2);
      fence_proxy_async();
    }
  }
  if (ok && ntiles > 0) {
    // The last tile's partial outputs.
    if (__syncthreads_and(wait_bar(bar_o, (ntiles - 1) & 1))) {
      tc_fence_after();
      uint32_t om[32], oc[32];
      tmem_ld32(tL + kColOm, om);
      tmem_ld32(tL + kColOc, oc);
      tmem_ld_wait();
#pragma unroll
      for (int d = 0; d < kD; ++d) acc[d] += __uint_as_float(om[d]) + __uint_as_float(oc[d]);
    } else {
      ok = false;
      site = kSiteOutput;
    }
  }
  if (!ok) {
    // Every product issued completes by itself: wait for them (one commit tracks all of
    // the issuing thread's) before the columns are freed; no output.
    if (tid == 0) {
      report_status(status, kStatusTimeout | (site << 8));
      umma_commit(bar_d);
      wait_bar(bar_d, 0);
    }
  } else if (act) {
    // Zero valid keys: 0/0, as the reference's sums give.
    const float inv = 1.0f / l;
    float4 *op = reinterpret_cast<float4 *>(out + ((base + pos) * p.heads + head) * kD);
#pragma unroll
    for (int c = 0; c < 8; ++c)
      op[c] = make_float4(acc[4 * c] * inv, acc[4 * c + 1] * inv, acc[4 * c + 2] * inv,
                          acc[4 * c + 3] * inv);
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

namespace {
template <int kKeys>
cudaError_t launch_d32_tc(const AttnProblem &p, int *status, cudaStream_t stream, dim3 grid) {
  constexpr uint32_t bytes = d32tc::Cfg<kKeys>::kSmemBytes;
  cudaError_t e = cudaFuncSetAttribute(d32tc::attn_d32_tc_kernel<kKeys>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return e;
  d32tc::attn_d32_tc_kernel<kKeys><<<grid, d32tc::kRows, bytes, stream>>>(p, status);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_attention_d32_tc(const AttnProblem &p, int *status, cudaStream_t stream,
                                    int num_sms) {
  if (!d32_tc_supported(p)) return cudaErrorInvalidValue;
  const uint32_t qblocks = (p.seq + d32tc::kRows - 1) / d32tc::kRows;
  if (!qblocks || qblocks > 65535u) return cudaErrorInvalidValue;
  const dim3 grid(qblocks, p.heads, p.batch);
  // Within one wave at two CTAs per SM the CTA's own latency decides: 64-key tiles (BGE
  // config 1: 14.9 us against 18.4); beyond, three CTAs per SM with 32-key tiles (batch
  // 4096: 1.44 ms against 1.68).
  const uint64_t ctas = (uint64_t)qblocks * p.heads * p.batch;
  if (ctas <= 2ull * (uint64_t)num_sms) return launch_d32_tc<64>(p, status, stream, grid);
  return launch_d32_tc<32>(p, status, stream, grid);
}

}  // namespace tx
