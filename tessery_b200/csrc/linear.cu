// Blackwell (sm_100a) tensor-core GEMM for the projections around the attention:
// out = x . w^T with x [M, K] bf16 (row-major, tokens x input channels) and w [N, K] bf16
// (row-major, output channels x input channels -- the layout of the reference's
// quantised weights, qwen3.py:70-73, once dequantised), fp32 accumulation in tensor
// memory.  It stands in for the reference's linear4* kernels (kernels.metal:32-51,
// 491-608, 658-773) and, with the gated epilogue, for gated4* plus silu_gate
// (kernels.metal:333-337, 609-733): the reference computes in fp32 on dequantised
// weights; here activations and weights are bf16 tensor-core operands.
//
// Tile 128 x 256 (M x N), K in steps of 64 through a 4-slot ring of shared memory filled
// by TMA (128-byte swizzle); one elected thread issues tcgen05.mma (M=128, N=256, K=16,
// four per K step) into 256 tensor-memory columns; four epilogue warps (one per 32-lane
// quarter of tensor memory, thread = output row) read the accumulator and apply the
// epilogue:
//   kStoreF32   out[m, n] = acc                       (fp32 [M, N])
//   kStoreBf16  out[m, n] = bf16(acc)                 (bf16 [M, N])
//   kAddF32     out[m, n] += acc                      (the residual stream, qwen3.py:151-152)
//   kGatedBf16  out[m, 128 t + j] = bf16(silu(acc[j]) * acc[128 + j]) for tile t, j < 128:
//               the weight rows are interleaved so that each 256-row block holds 128 gate
//               rows then the matching 128 up rows (interleave_gate_up on the host side).
// Rows past M are read as zeros (TMA bounds) and never stored.  Every wait is bounded; a
// wait that gives up records TX_ETIMEOUT | site << 8 in the status word and the roles
// drain what they issued before tensor memory is freed.
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

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr uint32_t kABytes = kBM * 128;  // 128 rows x 64 bf16
constexpr uint32_t kBBytes = kBN * 128;  // 256 rows x 64 bf16
constexpr int kMaxStages = 4;
// Shared-memory ring per number of products: 1 (x . w), 2 (x . w_hi + x . w_lo) or 3
// (x_hi . w_hi + x_hi . w_lo + x_lo . w_hi, the split-operand form: with v = hi + lo and
// both parts bf16, the three products carry about 16 significant bits of each operand).
template <int kPasses>
struct Ring {
  static constexpr int kStages = kPasses == 1 ? 4 : 2;
  static constexpr uint32_t kAParts = kPasses == 3 ? 2 : 1;
  static constexpr uint32_t kBParts = kPasses == 1 ? 1 : 2;
  static constexpr uint32_t kStageBytes = kAParts * kABytes + kBParts * kBBytes;
  static constexpr uint32_t kOffBars = kStages * kStageBytes;
  static constexpr uint32_t kSmemBytes = kOffBars + 256;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};
constexpr int kThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr uint32_t kTmemCols = 256;
constexpr long long kDrainCycles = 2000000000ll;
// kind::f16, A = B = bf16, D = f32, both K-major; N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) |
                            ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
enum : uint32_t { kBarFull = 0, kBarEmpty = kMaxStages, kBarAccum = 2 * kMaxStages,
                  kBarDrain = kBarAccum + 1, kNumBars = kBarDrain + 1 };
enum : int { kSiteEmpty = 1, kSiteFull = 2, kSiteAccum = 3 };

struct Params {
  uint32_t m, n, k;
  void *out;  // with more than one product, the gated epilogue writes a bf16 pair: hi [m, n/2]
              // then lo [m, n/2]
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

template <int kMode, int kPasses>
__global__ void __launch_bounds__(kThreads, 1)
    linear_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_xlo,
                  const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_wlo,
                  const __grid_constant__ Params p) {
  using R = Ring<kPasses>;
  constexpr int kStages = R::kStages;
  constexpr uint32_t kStageBytes = R::kStageBytes, kOffBars = R::kOffBars;
  // Offsets inside a stage: A hi, A lo (3 products), B hi, B lo (2 or 3 products).
  constexpr uint32_t kOffAlo = kABytes, kOffB = R::kAParts * kABytes, kOffBlo = kOffB + kBBytes;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_addr(smem);
  if (sbase & 1023u) {
    if (threadIdx.x == 0) report_status(p.status, kStatusBadArg);
    return;
  }
  const uint32_t bars = sbase + kOffBars;
  auto bar = [&](uint32_t i) { return bars + 8u * i; };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffBars + 8 * kNumBars);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + kOffBars + 8 * kNumBars + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM;
  const uint32_t nk = p.k / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kBarFull + s), 1);
      mbar_init(bar(kBarEmpty + s), 1);
    }
    mbar_init(bar(kBarAccum), 1);
    mbar_init(bar(kBarDrain), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(kTmemCols)
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
        const uint32_t dst = sbase + s * kStageBytes;
        mbar_expect_tx(bar(kBarFull + s), kStageBytes);
        const int kx = (int)(kb * kBK);
        tma_load_2d(dst, &tm_x, bar(kBarFull + s), kx, (int)m0);
        if (kPasses == 3) tma_load_2d(dst + kOffAlo, &tm_xlo, bar(kBarFull + s), kx, (int)m0);
        tma_load_2d(dst + kOffB, &tm_w, bar(kBarFull + s), kx, (int)n0);
        if (kPasses > 1) tma_load_2d(dst + kOffBlo, &tm_wlo, bar(kBarFull + s), kx, (int)n0);
        ++fills;
      }
      if (!ok) {
        // Every issued fill completes by itself: wait for the latest fill of each slot.
        for (uint32_t s = 0; s < kStages && s < fills; ++s) {
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
      for (uint32_t kb = 0; ok && kb < nk; ++kb) {
        const uint32_t s = kb % kStages;
        if (!(ok = wait_bar(bar(kBarFull + s), (kb / kStages) & 1, abort_flag, p.status,
                            kSiteFull, p.wait_cycles)))
          break;
        tc_fence_after();
        const uint32_t st = sbase + s * kStageBytes;
        const uint64_t ad = sw128_desc(st, 16, 1024), bd = sw128_desc(st + kOffB, 16, 1024);
        const uint64_t adl = sw128_desc(st + kOffAlo, 16, 1024);
        const uint64_t bdl = sw128_desc(st + kOffBlo, 16, 1024);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {  // 16 elements of K = 32 bytes inside the swizzled row
          const uint64_t o = (uint64_t)(ks * 2);
          umma(tmem, ad + o, bd + o, kIdesc, (kb > 0 || ks > 0) ? 1u : 0u);
          if (kPasses > 1) umma(tmem, ad + o, bdl + o, kIdesc, 1u);
          if (kPasses == 3) umma(tmem, adl + o, bd + o, kIdesc, 1u);
        }
        umma_commit(bar(kBarEmpty + s));
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
    const bool ok = __all_sync(0xffffffffu, wait_bar(bar(kBarAccum), 0, abort_flag, p.status,
                                                     kSiteAccum, p.wait_cycles));
    if (ok) {
      tc_fence_after();
      if (kMode == TX_LINEAR_GATED_BF16) {
        uint16_t *orow = static_cast<uint16_t *>(p.out) + (size_t)m * (p.n / 2) + n0 / 2;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {  // gate columns 32c.., up columns 128 + 32c..
          uint32_t g[32], u[32];
          tmem_ld32(tl + c * 32, g);
          tmem_ld32(tl + 128 + c * 32, u);
          tmem_ld_wait();
          if (m < p.m) {
            uint32_t w[16], wl[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) {
              const float a = silu(__uint_as_float(g[2 * t])) * __uint_as_float(u[2 * t]);
              const float b = silu(__uint_as_float(g[2 * t + 1])) * __uint_as_float(u[2 * t + 1]);
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
#pragma unroll 1
        for (int c = 0; c < kBN / 32; ++c) {
          uint32_t x[32];
          tmem_ld32(tl + c * 32, x);
          tmem_ld_wait();
          if (m >= p.m) continue;
          const size_t off = (size_t)m * p.n + n0 + c * 32;
          if (kMode == TX_LINEAR_STORE_BF16) {
            uint4 *o = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.out) + off);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              o[q] = make_uint4(pack_bf16x2(__uint_as_float(x[8 * q]), __uint_as_float(x[8 * q + 1])),
                                pack_bf16x2(__uint_as_float(x[8 * q + 2]), __uint_as_float(x[8 * q + 3])),
                                pack_bf16x2(__uint_as_float(x[8 * q + 4]), __uint_as_float(x[8 * q + 5])),
                                pack_bf16x2(__uint_as_float(x[8 * q + 6]), __uint_as_float(x[8 * q + 7])));
          } else {
            float4 *o = reinterpret_cast<float4 *>(static_cast<float *>(p.out) + off);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float4 v = make_float4(__uint_as_float(x[4 * q]), __uint_as_float(x[4 * q + 1]),
                                     __uint_as_float(x[4 * q + 2]), __uint_as_float(x[4 * q + 3]));
              if (kMode == TX_LINEAR_ADD_F32) {
                const float4 old = o[q];
                v.x += old.x;
                v.y += old.y;
                v.z += old.z;
                v.w += old.w;
              }
              o[q] = v;
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
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
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

// 2-D map over a row-major [rows, cols] bf16 matrix; a box is 64 columns x box_rows rows in
// the 128-byte swizzle.
bool make_map_2d(CUtensorMap *map, const void *base, uint32_t rows, uint32_t cols,
                 uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t elem[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides,
            box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int kMode, int kPasses>
cudaError_t launch_mode(const CUtensorMap (&maps)[4], const gemm::Params &prm, dim3 grid,
                        cudaStream_t stream) {
  constexpr uint32_t smem = gemm::Ring<kPasses>::kSmemBytes;
  cudaError_t e = cudaFuncSetAttribute(gemm::linear_kernel<kMode, kPasses>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  gemm::linear_kernel<kMode, kPasses><<<grid, gemm::kThreads, smem, stream>>>(
      maps[0], maps[1], maps[2], maps[3], prm);
  return cudaGetLastError();
}

template <int kPasses>
cudaError_t launch_passes(int mode, const CUtensorMap (&maps)[4], const gemm::Params &prm,
                          dim3 grid, cudaStream_t stream) {
  switch (mode) {
    case TX_LINEAR_STORE_F32: return launch_mode<TX_LINEAR_STORE_F32, kPasses>(maps, prm, grid, stream);
    case TX_LINEAR_STORE_BF16: return launch_mode<TX_LINEAR_STORE_BF16, kPasses>(maps, prm, grid, stream);
    case TX_LINEAR_ADD_F32: return launch_mode<TX_LINEAR_ADD_F32, kPasses>(maps, prm, grid, stream);
    default: return launch_mode<TX_LINEAR_GATED_BF16, kPasses>(maps, prm, grid, stream);
  }
}

}  // namespace

bool linear_supported(uint32_t m, uint32_t n, uint32_t k, int mode, const void *x, const void *w,
                      const void *out) {
  if (!m || !n || !k || n % gemm::kBN || k % gemm::kBK) return false;
  if (m > 0x7fffffffu || (uint64_t)(m + gemm::kBM - 1) / gemm::kBM > 65535u) return false;
  if (mode < TX_LINEAR_STORE_F32 || mode > TX_LINEAR_GATED_BF16) return false;
  return (uintptr_t)x % 16 == 0 && (uintptr_t)w % 16 == 0 && (uintptr_t)out % 16 == 0;
}

cudaError_t launch_linear(const void *x, const void *x_lo, const void *w, const void *w_lo,
                          void *out, uint32_t m, uint32_t n, uint32_t k, int mode, int *status,
                          long long wait_cycles, cudaStream_t stream) {
  if (!linear_supported(m, n, k, mode, x, w, out)) return cudaErrorInvalidValue;
  if ((x_lo && !w_lo) || (uintptr_t)x_lo % 16 || (uintptr_t)w_lo % 16) return cudaErrorInvalidValue;
  CUtensorMap maps[4];
  if (!make_map_2d(&maps[0], x, m, k, gemm::kBM) || !make_map_2d(&maps[2], w, n, k, gemm::kBN))
    return cudaErrorInvalidValue;
  maps[1] = maps[0];
  maps[3] = maps[2];
  if ((x_lo && !make_map_2d(&maps[1], x_lo, m, k, gemm::kBM)) ||
      (w_lo && !make_map_2d(&maps[3], w_lo, n, k, gemm::kBN)))
    return cudaErrorInvalidValue;
  gemm::Params prm;
  prm.m = m;
  prm.n = n;
  prm.k = k;
  prm.out = out;
  prm.status = status;
  prm.wait_cycles = wait_cycles > 0 ? wait_cycles : 2000000000ll;
  const dim3 grid(n / gemm::kBN, (m + gemm::kBM - 1) / gemm::kBM);
  if (x_lo) return launch_passes<3>(mode, maps, prm, grid, stream);
  if (w_lo) return launch_passes<2>(mode, maps, prm, grid, stream);
  return launch_passes<1>(mode, maps, prm, grid, stream);
}

}  // namespace tx
