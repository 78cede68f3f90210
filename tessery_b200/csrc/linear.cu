// Blackwell (sm_100a) tensor-core GEMM for the projections around the attention:
// out = x . w^T (+ bias) with x [M, K] (row-major, tokens x input channels) and w [N, K]
// (row-major, output channels x input channels -- the layout of the reference's weights,
// qwen3.py:70-73 once dequantised, bert.py:55-58), fp32 accumulation in tensor memory.
// It stands in for the reference's linear4* kernels (kernels.metal:32-51, 491-608,
// 658-773), with the gated epilogue for gated4* plus silu_gate (kernels.metal:333-337,
// 609-733), and for matmul_f32* / matmul_bias_f32* (kernels.metal:306-321, 392-487).
//
// Operand formats: bf16 (kind::f16, K = 16 per instruction, 64 elements per 128-byte
// row) or fp32 read as TF32 (kind::tf32, K = 8, 32 elements per row).  With the lo parts
// of split operands (v = hi + lo) the product is x.w + x.w_lo (2 passes) or
// x.w + x.w_lo + x_lo.w (3 passes): bf16 pairs carry about 16 significant bits of each
// operand, TF32 pairs (hi = v rounded to TF32, lo = v - hi) about 22, which is the fp32
// path's accuracy.
//
// Tile 128 x BN (BN = 256 or 128; two CTAs per SM for bf16 with one product), K through a
// ring of shared-memory stages filled by TMA
// (128-byte swizzle); one elected thread issues tcgen05.mma (M=128, N=BN) into BN
// tensor-memory columns (2 BN with split operands: the main product and the two
// corrections accumulate apart); four epilogue warps (one per 32-lane quarter of tensor memory,
// thread = output row) read the accumulator, add the bias (fp32 [N], optional) and apply
// the epilogue:
//   kStoreF32   out[m, n] = acc                       (fp32)
//   kStoreBf16  out[m, n] = bf16(acc)                 (bf16)
//   kAddF32     out[m, n] += acc                      (the residual stream, qwen3.py:151-152,
//                                                      bert.py:211-217)
//   kGatedBf16  out[m, 128 t + j] = bf16(silu(acc[j]) * acc[128 + j]) for tile t, j < 128:
//               the weight rows are interleaved so that each 256-row block holds 128 gate
//               rows then the matching 128 up rows (interleave_gate_up on the host side);
//               a bf16 pair (hi [M, N/2] then lo) with split operands
//   kGeluSplit  gelu(acc) (the erf form of gelu_f32, kernels.metal:381-391) written as the
//               next GEMM's split operand: hi [M, N] then lo [M, N], in this GEMM's format
// Outputs may be split by columns: with `part` < N, column block [p*part, (p+1)*part) is
// written to its own [M, part] matrix, the p-th of `N / part` consecutive ones (a fused
// q/k/v projection writing q, k and v).  Rows past M are read as zeros (TMA bounds) and
// never stored.  Every wait is bounded; a wait that gives up records
// TX_ETIMEOUT | site << 8 in the status word and the roles drain what they issued before
// tensor memory is freed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "../../include/tessattn.h"
#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace tx {
namespace gemm {

using namespace ptx;

constexpr int kBM = 128;
constexpr int kMaxStages = 4;
constexpr uint32_t kSmemBudget = 232448;
constexpr int kThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr long long kDrainCycles = 2000000000ll;

// Shared-memory ring and instruction descriptor per operand format, tile width and number
// of products (1: x.w, 2: + x.w_lo, 3: + x_lo.w).
template <bool kTf32, int kBN, int kPasses>
struct Cfg {
  static constexpr uint32_t kBK = kTf32 ? 32 : 64;  // K elements per 128-byte row
  static constexpr uint32_t kABytes = kBM * 128;
  static constexpr uint32_t kBBytes = kBN * 128;
  static constexpr uint32_t kAParts = kPasses == 3 ? 2 : 1;
  static constexpr uint32_t kBParts = kPasses == 1 ? 1 : 2;
  static constexpr uint32_t kStageBytes = kAParts * kABytes + kBParts * kBBytes;
  // bf16 with one product: two CTAs per SM (each holds at most 256 TMEM columns), so one
  // CTA's epilogue runs beside the other's products (measured: the Qwen3 forward went from
  // 12.7 to 11.5 ms per 32 texts against one CTA with a 4-stage ring).
  static constexpr int kCtas = (!kTf32 && kPasses == 1) ? 2 : 1;
  static constexpr int kFit = (int)((kSmemBudget / kCtas - 1024 - 256) / kStageBytes);
  static constexpr int kStages = kFit < kMaxStages ? kFit : kMaxStages;
  static constexpr uint32_t kOffAlo = kABytes, kOffB = kAParts * kABytes,
                            kOffBlo = kOffB + kBBytes;
  static constexpr uint32_t kOffBars = kStages * kStageBytes;
  static constexpr uint32_t kSmemBytes = kOffBars + 256;
  // With split operands the two small correction products accumulate in their own BN
  // columns (after the main product's), so the large main sum takes a third of the
  // accumulator updates; the epilogue adds the two.  TF32 with split operands (the fp32
  // path, BN = 128) goes further: the main product is summed in partial sums of
  // kChunkSteps K steps, alternately in two column blocks, and the epilogue warps add the
  // partials in registers as they complete (the reference's f32 projections reset their
  // partial sums every 32 products for the same reason, kernels.metal:416-436); the
  // corrections follow in the third block.
  static constexpr bool kChunked = kTf32 && kPasses == 3 && kBN == 128;
  static constexpr uint32_t kChunkSteps = 4;  // 128 products of K per partial sum
  static constexpr uint32_t kCorrCol = kChunked ? 2 * kBN : kBN;
  static constexpr uint32_t kTmemCols = kChunked ? 512 : kPasses == 3 ? 2 * kBN : kBN;
  // D = f32 (bit 4); A and B formats at bits 7 and 10 (bf16 1, tf32 2), both K-major;
  // N >> 3 at bit 17, M >> 4 at bit 24.
  static constexpr uint32_t kFmt = kTf32 ? 2u : 1u;
  static constexpr uint32_t kIdesc = (1u << 4) | (kFmt << 7) | (kFmt << 10) |
                                     ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
  static_assert(kStages >= 2, "at least two ring stages");
  static_assert(kSmemBytes <= kSmemBudget, "shared memory budget");
};

enum : uint32_t { kBarFull = 0, kBarEmpty = kMaxStages, kBarAccum = 2 * kMaxStages,
                  kBarDrain = kBarAccum + 1,
                  kBarPartFull = kBarDrain + 1,   // + block: a partial sum is complete
                  kBarPartFree = kBarPartFull + 2,  // + block: the epilogue has read it
                  kNumBars = kBarPartFree + 2 };
enum : int { kSiteEmpty = 1, kSiteFull = 2, kSiteAccum = 3, kSitePartFree = 4, kSitePartFull = 5 };

struct Params {
  uint32_t m, n, k;
  uint32_t part;        // output column-block width (n: one [m, n] matrix)
  void *out;
  const float *bias;    // fp32 [n] or NULL
  int *status;
  long long wait_cycles;
};

// Bounded wait; gives up (status, CTA abort flag) after `limit` cycles.
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                         int *status, int site, long long limit) {
  if (mbar_test(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_test(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > limit) {
      *abort_flag = 1;
      report_status(status, kStatusTimeout | (site << 8));
      return false;
    }
  }
}
__device__ __forceinline__ void drain_bar(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_test(bar, parity) && clock64() - t0 < kDrainCycles) {
  }
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + __expf(-g)); }

template <int kMode, bool kTf32, int kBN, int kPasses>
__global__ void __launch_bounds__(kThreads, Cfg<kTf32, kBN, kPasses>::kCtas)
    linear_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_xlo,
                  const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_wlo,
                  const __grid_constant__ Params p) {
  using C = Cfg<kTf32, kBN, kPasses>;
  constexpr int kStages = C::kStages;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_addr(smem);
  if (sbase & 1023u) {
    if (threadIdx.x == 0) report_status(p.status, kStatusBadArg);
    return;
  }
  const uint32_t bars = sbase + C::kOffBars;
  auto bar = [&](uint32_t i) { return bars + 8u * i; };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::kOffBars + 8 * kNumBars);
  volatile int *abort_flag =
      reinterpret_cast<volatile int *>(smem + C::kOffBars + 8 * kNumBars + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM;
  const uint32_t nk = p.k / C::kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kBarFull + s), 1);
      mbar_init(bar(kBarEmpty + s), 1);
    }
    mbar_init(bar(kBarAccum), 1);
    mbar_init(bar(kBarDrain), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(kBarPartFull + b), 1);
      mbar_init(bar(kBarPartFree + b), 128);  // every epilogue thread
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_w);
    if (kPasses == 3) prefetch_tmap(&tm_xlo);
    if (kPasses > 1) prefetch_tmap(&tm_wlo);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer: K step kb into ring slot kb % kStages ----
    if (lane == 0) {
      bool ok = true;
      uint32_t fills = 0;  // fills issued so far
      for (uint32_t kb = 0; ok && kb < nk; ++kb) {
        const uint32_t s = kb % kStages, round = kb / kStages;
        if (round > 0 && !(ok = wait_bar(bar(kBarEmpty + s), (round - 1) & 1, abort_flag,
                                         p.status, kSiteEmpty, p.wait_cycles)))
          break;
        const uint32_t dst = sbase + s * C::kStageBytes;
        mbar_expect_tx(bar(kBarFull + s), C::kStageBytes);
        const int kx = (int)(kb * C::kBK);
        tma_load_2d(dst, &tm_x, bar(kBarFull + s), kx, (int)m0);
        if (kPasses == 3) tma_load_2d(dst + C::kOffAlo, &tm_xlo, bar(kBarFull + s), kx, (int)m0);
        tma_load_2d(dst + C::kOffB, &tm_w, bar(kBarFull + s), kx, (int)n0);
        if (kPasses > 1) tma_load_2d(dst + C::kOffBlo, &tm_wlo, bar(kBarFull + s), kx, (int)n0);
        ++fills;
      }
      if (!ok) {
        // Every issued fill completes by itself: wait for the latest fill of each slot.
        for (uint32_t s = 0; s < (uint32_t)kStages && s < fills; ++s) {
          uint32_t last = s;
          while (last + kStages < fills) last += kStages;
          drain_bar(bar(kBarFull + s), (last / kStages) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      bool ok = true, issued = false;
      auto mma = [&](uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
        if (kTf32)
          umma_tf32(d, a, b, C::kIdesc, acc);
        else
          umma(d, a, b, C::kIdesc, acc);
      };
      const uint32_t corr = tmem + C::kCorrCol;
      for (uint32_t kb = 0; ok && kb < nk; ++kb) {
        const uint32_t s = kb % kStages;
        if (!(ok = wait_bar(bar(kBarFull + s), (kb / kStages) & 1, abort_flag, p.status,
                            kSiteFull, p.wait_cycles)))
          break;
        // Partial-sum block of this K step (chunked): wait until the epilogue has read the
        // partial it last held.
        const uint32_t chunk = kb / C::kChunkSteps, pb = chunk & 1;
        const bool chunk_first = kb % C::kChunkSteps == 0;
        if (C::kChunked && chunk_first && chunk >= 2 &&
            !(ok = wait_bar(bar(kBarPartFree + pb), ((chunk >> 1) - 1) & 1, abort_flag,
                            p.status, kSitePartFree, p.wait_cycles)))
          break;
        const uint32_t main_acc = C::kChunked ? tmem + pb * kBN : tmem;
        tc_fence_after();
        const uint32_t st = sbase + s * C::kStageBytes;
        const uint64_t ad = sw128_desc(st, 16, 1024), bd = sw128_desc(st + C::kOffB, 16, 1024);
        const uint64_t adl = sw128_desc(st + C::kOffAlo, 16, 1024);
        const uint64_t bdl = sw128_desc(st + C::kOffBlo, 16, 1024);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {  // one instruction's K = 32 bytes of the swizzled row
          const uint64_t o = (uint64_t)(ks * 2);
          const uint32_t first = (kb > 0 || ks > 0) ? 1u : 0u;
          mma(main_acc, ad + o, bd + o, C::kChunked ? (chunk_first && ks == 0 ? 0u : 1u) : first);
          if (kPasses == 3) {
            mma(corr, ad + o, bdl + o, first);
            mma(corr, adl + o, bd + o, 1u);
          }
        }
        umma_commit(bar(kBarEmpty + s));
        if (C::kChunked && (kb % C::kChunkSteps == C::kChunkSteps - 1 || kb + 1 == nk))
          umma_commit(bar(kBarPartFull + pb));
        issued = true;
      }
      if (ok) umma_commit(bar(kBarAccum));
      if (issued) {
        umma_commit(bar(kBarDrain));
        drain_bar(bar(kBarDrain), 0);
      }
    }
    __syncwarp();
  } else {
    // ---- epilogue: thread = output row of the tile (tensor-memory lane) ----
    const uint32_t quarter = (uint32_t)warp & 3;
    const uint32_t r = quarter * 32 + lane;
    const uint32_t m = m0 + r;
    const uint32_t tl = tmem + ((quarter * 32u) << 16);
    // Chunked: this row's main sum, added up from the partial sums as they complete.
    float part_sum[C::kChunked ? kBN : 1];
    bool ok = true;
    if constexpr (C::kChunked) {
#pragma unroll
      for (int t = 0; t < kBN; ++t) part_sum[t] = 0.f;
      const uint32_t chunks = (nk + C::kChunkSteps - 1) / C::kChunkSteps;
      for (uint32_t c = 0; ok && c < chunks; ++c) {
        const uint32_t pb = c & 1;
        ok = __all_sync(0xffffffffu, wait_bar(bar(kBarPartFull + pb), (c >> 1) & 1, abort_flag,
                                              p.status, kSitePartFull, p.wait_cycles));
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int q = 0; q < kBN / 32; ++q) {
          uint32_t a[32];
          tmem_ld32(tl + pb * kBN + q * 32, a);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 32; ++t) part_sum[q * 32 + t] += __uint_as_float(a[t]);
        }
        tc_fence_before();
        mbar_arrive(bar(kBarPartFree + pb));
      }
    }
    ok = ok && __all_sync(0xffffffffu, wait_bar(bar(kBarAccum), 0, abort_flag, p.status,
                                                kSiteAccum, p.wait_cycles));
    // Output matrix of this tile's column block, its row stride and first column.
    const uint32_t blk = n0 / p.part, col0 = n0 % p.part;
    // Accumulator columns [col, col + 32) of this thread's row: the main sum plus, with
    // split operands, the correction sum.
    auto load_acc = [&](uint32_t col, float (&v)[32]) {
      uint32_t a[32];
      if constexpr (C::kChunked) {
        tmem_ld32(tl + C::kCorrCol + col, a);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) v[t] = part_sum[col + t] + __uint_as_float(a[t]);
        return;
      }
      tmem_ld32(tl + col, a);
      if (kPasses == 3) {
        uint32_t b[32];
        tmem_ld32(tl + C::kCorrCol + col, b);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) v[t] = __uint_as_float(a[t]) + __uint_as_float(b[t]);
      } else {
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) v[t] = __uint_as_float(a[t]);
      }
    };
    if (ok) {
      tc_fence_after();
      if (kMode == TX_LINEAR_GATED_BF16) {
        uint16_t *orow = static_cast<uint16_t *>(p.out) + (size_t)m * (p.n / 2) + n0 / 2;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {  // gate columns 32c.., up columns 128 + 32c..
          float g[32], u[32];
          load_acc(c * 32, g);
          load_acc(128 + c * 32, u);
          if (m < p.m) {
            uint32_t w[16], wl[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) {
              const float a = silu(g[2 * t]) * u[2 * t];
              const float b = silu(g[2 * t + 1]) * u[2 * t + 1];
              w[t] = pack_bf16x2(a, b);
              if (kPasses > 1)  // the rounding residue, as the lo half of a bf16 pair
                wl[t] = pack_bf16x2(a - bf16_lo(w[t]), b - bf16_hi(w[t]));
            }
            uint4 *o = reinterpret_cast<uint4 *>(orow + c * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) o[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
            if (kPasses > 1) {
              uint4 *ol = reinterpret_cast<uint4 *>(orow + (size_t)p.m * (p.n / 2) + c * 32);
#pragma unroll
              for (int q = 0; q < 4; ++q)
                ol[q] = make_uint4(wl[4 * q], wl[4 * q + 1], wl[4 * q + 2], wl[4 * q + 3]);
            }
          }
        }
      } else {
        const size_t plane = (size_t)p.m * p.part;  // elements of one output matrix
        // (fully unrolled when chunked: the row's sums are indexed by the column)
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) {
          float v[32];
          load_acc(c * 32, v);
          if (m >= p.m) continue;
          if (p.bias) {
            const float4 *b4 = reinterpret_cast<const float4 *>(p.bias + n0 + c * 32);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 b = __ldg(b4 + q);
              v[4 * q] += b.x;
              v[4 * q + 1] += b.y;
              v[4 * q + 2] += b.z;
              v[4 * q + 3] += b.w;
            }
          }
          const size_t off = blk * plane + (size_t)m * p.part + col0 + c * 32;
          if (kMode == TX_LINEAR_STORE_BF16 || (kMode == TX_LINEAR_GELU_SPLIT && !kTf32)) {
            if (kMode == TX_LINEAR_GELU_SPLIT) {
#pragma unroll
              for (int t = 0; t < 32; ++t) v[t] = gelu_erf(v[t]);
            }
            uint32_t w[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) w[t] = pack_bf16x2(v[2 * t], v[2 * t + 1]);
            uint4 *o = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.out) + off);
#pragma unroll
            for (int q = 0; q < 4; ++q) o[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
            if (kMode == TX_LINEAR_GELU_SPLIT && kPasses > 1) {
#pragma unroll
              for (int t = 0; t < 16; ++t)
                w[t] = pack_bf16x2(v[2 * t] - bf16_lo(w[t]), v[2 * t + 1] - bf16_hi(w[t]));
              uint4 *ol = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.out) + plane + off);
#pragma unroll
              for (int q = 0; q < 4; ++q)
                ol[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
            }
          } else if (kMode == TX_LINEAR_GELU_SPLIT) {  // TF32 pair: hi then lo, fp32 each
            float *oh = static_cast<float *>(p.out) + off;
            float *ol = oh + plane;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float h[4], l[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float g = gelu_erf(v[4 * q + e]);
                h[e] = tf32_round(g);
                l[e] = g - h[e];
              }
              reinterpret_cast<float4 *>(oh)[q] = make_float4(h[0], h[1], h[2], h[3]);
              reinterpret_cast<float4 *>(ol)[q] = make_float4(l[0], l[1], l[2], l[3]);
            }
          } else {
            float4 *o = reinterpret_cast<float4 *>(static_cast<float *>(p.out) + off);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float4 val = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
              if (kMode == TX_LINEAR_ADD_F32) {
                const float4 old = o[q];
                val.x = old.x + val.x;
                val.y = old.y + val.y;
                val.z = old.z + val.z;
                val.w = old.w + val.w;
              }
              o[q] = val;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(C::kTmemCols)
                 : "memory");
}

}  // namespace gemm

// ---- host side ----------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)ptr;
  }
  return fn;
}

// 2-D map over a row-major [rows, cols] matrix of bf16 or fp32; a box is one 128-byte row
// of K (64 bf16 or 32 fp32) x box_rows rows, in the 128-byte swizzle.
bool make_map_2d(CUtensorMap *map, const void *base, uint32_t rows, uint32_t cols,
                 uint32_t box_rows, bool fp32) {
  auto fn = encode_fn();
  if (!fn) return false;
  const uint32_t esz = fp32 ? 4 : 2;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * esz};
  cuuint32_t box[2] = {128 / esz, box_rows};
  cuuint32_t elem[2] = {1, 1};
  return fn(map, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
            const_cast<void *>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int kMode, bool kTf32, int kBN, int kPasses>
cudaError_t launch_one(const CUtensorMap (&maps)[4], const gemm::Params &prm, dim3 grid,
                       cudaStream_t stream) {
  constexpr uint32_t smem = gemm::Cfg<kTf32, kBN, kPasses>::kSmemBytes;
  auto kernel = gemm::linear_kernel<kMode, kTf32, kBN, kPasses>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  kernel<<<grid, gemm::kThreads, smem, stream>>>(maps[0], maps[1], maps[2], maps[3], prm);
  return cudaGetLastError();
}

template <bool kTf32, int kBN, int kPasses>
cudaError_t launch_mode(int mode, const CUtensorMap (&maps)[4], const gemm::Params &prm,
                        dim3 grid, cudaStream_t stream) {
  switch (mode) {
    case TX_LINEAR_STORE_F32:
      return launch_one<TX_LINEAR_STORE_F32, kTf32, kBN, kPasses>(maps, prm, grid, stream);
    case TX_LINEAR_ADD_F32:
      return launch_one<TX_LINEAR_ADD_F32, kTf32, kBN, kPasses>(maps, prm, grid, stream);
    case TX_LINEAR_GELU_SPLIT:
      return launch_one<TX_LINEAR_GELU_SPLIT, kTf32, kBN, kPasses>(maps, prm, grid, stream);
    default:
      break;
  }
  if constexpr (!kTf32) {
    if (mode == TX_LINEAR_STORE_BF16)
      return launch_one<TX_LINEAR_STORE_BF16, false, kBN, kPasses>(maps, prm, grid, stream);
    if constexpr (kBN == 256)
      if (mode == TX_LINEAR_GATED_BF16)
        return launch_one<TX_LINEAR_GATED_BF16, false, 256, kPasses>(maps, prm, grid, stream);
  }
  return cudaErrorInvalidValue;
}

template <bool kTf32>
cudaError_t launch_format(int mode, uint32_t bn, bool split, const CUtensorMap (&maps)[4],
                          const gemm::Params &prm, dim3 grid, cudaStream_t stream) {
  if (bn == 256)
    return split ? launch_mode<kTf32, 256, 3>(mode, maps, prm, grid, stream)
                 : launch_mode<kTf32, 256, 1>(mode, maps, prm, grid, stream);
  return split ? launch_mode<kTf32, 128, 3>(mode, maps, prm, grid, stream)
               : launch_mode<kTf32, 128, 1>(mode, maps, prm, grid, stream);
}

}  // namespace

uint32_t linear_tile_n(uint32_t n, uint32_t part, int mode) {
  if (mode == TX_LINEAR_GATED_BF16) return n % 256 == 0 && part == n ? 256u : 0u;
  if (n % 256 == 0 && part % 256 == 0) return 256;
  if (n % 128 == 0 && part % 128 == 0) return 128;
  return 0;
}

bool linear_supported(uint32_t m, uint32_t n, uint32_t k, int mode, int fmt, uint32_t part,
                      const void *x, const void *w, const void *out) {
  if (!m || !n || !k || !part || n % part) return false;
  if (fmt != TX_BF16 && fmt != TX_F32) return false;
  if (k % (fmt == TX_F32 ? 32u : 64u)) return false;
  if (m > 0x7fffffffu || (uint64_t)(m + gemm::kBM - 1) / gemm::kBM > 65535u) return false;
  if (mode < TX_LINEAR_STORE_F32 || mode > TX_LINEAR_GELU_SPLIT) return false;
  if (fmt == TX_F32 && (mode == TX_LINEAR_STORE_BF16 || mode == TX_LINEAR_GATED_BF16))
    return false;
  if (!linear_tile_n(n, part, mode)) return false;
  return (uintptr_t)x % 16 == 0 && (uintptr_t)w % 16 == 0 && (uintptr_t)out % 16 == 0;
}

cudaError_t launch_linear(const void *x, const void *x_lo, const void *w, const void *w_lo,
                          const float *bias, void *out, uint32_t m, uint32_t n, uint32_t k,
                          int mode, int fmt, uint32_t part, int *status, long long wait_cycles,
                          cudaStream_t stream) {
  if (!linear_supported(m, n, k, mode, fmt, part, x, w, out)) return cudaErrorInvalidValue;
  if (!x_lo != !w_lo || (uintptr_t)x_lo % 16 || (uintptr_t)w_lo % 16 || (uintptr_t)bias % 16)
    return cudaErrorInvalidValue;
  if (bias && mode == TX_LINEAR_GATED_BF16) return cudaErrorInvalidValue;
  const bool f32 = fmt == TX_F32;
  // fp32 with split operands: 128-column tiles, whose main sums are chunked (see Cfg).
  const uint32_t bn = f32 && x_lo ? 128u : linear_tile_n(n, part, mode);
  CUtensorMap maps[4];
  if (!make_map_2d(&maps[0], x, m, k, gemm::kBM, f32) || !make_map_2d(&maps[2], w, n, k, bn, f32))
    return cudaErrorInvalidValue;
  maps[1] = maps[0];
  maps[3] = maps[2];
  if (x_lo && (!make_map_2d(&maps[1], x_lo, m, k, gemm::kBM, f32) ||
               !make_map_2d(&maps[3], w_lo, n, k, bn, f32)))
    return cudaErrorInvalidValue;
  gemm::Params prm;
  prm.m = m;
  prm.n = n;
  prm.k = k;
  prm.part = part;
  prm.out = out;
  prm.bias = bias;
  prm.status = status;
  prm.wait_cycles = wait_cycles > 0 ? wait_cycles : 2000000000ll;
  const dim3 grid(n / bn, (m + gemm::kBM - 1) / gemm::kBM);
  return f32 ? launch_format<true>(mode, bn, x_lo != nullptr, maps, prm, grid, stream)
             : launch_format<false>(mode, bn, x_lo != nullptr, maps, prm, grid, stream);
}

}  // namespace tx
