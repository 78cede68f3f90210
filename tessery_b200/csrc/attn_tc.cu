// Blackwell (sm_100a) tensor-core attention for head_dim 128, bf16 q/k/v, fp32 softmax
// and accumulation: the Qwen3 causal GQA operator of qwen3.py:238-245 dispatched by
// MetalRuntime._attention (metal.py:532-569), with the semantics of kernels.metal:78-103
// (and of its tiled/tail variants :108-298).
//
// Work unit: (sequence, pair of query heads sharing one kv head, 128-row query tile).
// The two query heads of a pair share every K/V tile, so each K/V tile is fetched from
// HBM/L2 once per pair (GQA head sharing).  A persistent grid of one CTA per SM walks a
// host-built, longest-first list of units.
//
// Warp roles (320 threads, one CTA per SM):
//   warps 0-3  softmax for head slot 0 (thread t owns query row t of the tile)
//   warps 4-7  softmax for head slot 1
//   warp 8     TMA producer: Q tiles once per unit, then K_j, V_j through a 3-slot ring
//   warp 9     TMEM allocator and single-thread tcgen05.mma issuer
// Tensor memory (512 columns x 128 lanes, fp32):
//   [0,128) S for slot 0, [128,256) S for slot 1, [256,384) O slot 0, [384,512) O slot 1.
// Shared memory: Q0, Q1, 3 K/V slots and P0, P1, each a 128x128 bf16 tile stored as two
// 128-row x 128-byte atoms in the 128-byte-swizzled layout that TMA writes and the UMMA
// descriptors read; barriers after them.
//
// Per key tile j the issuer runs  S_h = Q_h K_j^T  (M=128, N=128, K=128, bf16 -> f32 in
// TMEM), the softmax warps turn S_h into P_h = exp2(S_h*scale*log2e - m) (bf16, shared
// memory) and the issuer accumulates O_h += P_h V_j in TMEM.  Tiles above the causal
// diagonal and beyond each sequence's length are never visited; the diagonal and the
// last tile are masked per row.  The running maximum is updated lazily: O is rescaled
// only when a tile's maximum exceeds the reference maximum by more than 8 (log2 units),
// which keeps every probability below 2^8 and gives the same normalised result.
//
// Every wait is bounded (about a second); a wait that gives up records
// TX_ETIMEOUT | site<<8 in the context status word, raises a CTA-wide abort flag, and
// all roles drain their in-flight copies and MMAs before TMEM is freed and the CTA exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace tx {
namespace tc {

constexpr int kTile = 128;                     // query rows, keys and head_dim per tile
constexpr int kStages = 3;                     // K/V ring slots
constexpr uint32_t kAtomBytes = 128 * 128;     // 128 rows x 64 bf16 (one swizzle column)
constexpr uint32_t kTileBytes = 2 * kAtomBytes;
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffKV = kOffQ + 2 * kTileBytes;
constexpr uint32_t kOffP = kOffKV + kStages * kTileBytes;
constexpr uint32_t kOffBar = kOffP + 2 * kTileBytes;
constexpr uint32_t kBarBytes = 256;
constexpr uint32_t kSmemBytes = kOffBar + kBarBytes + 1024;  // + base alignment slack
constexpr int kThreads = 320;
constexpr int kTmaWarp = 8, kMmaWarp = 9;
constexpr long long kWaitCycles = 2000000000ll;  // ~1 s at B200 clocks
constexpr float kRescaleThreshold = 8.0f;        // log2 units

// Barrier slots (uint64 each) inside the barrier area.
enum : uint32_t {
  kBarQFull = 0, kBarQEmpty = 1,
  kBarKVFull = 2,                   // + slot (3)
  kBarKVEmpty = kBarKVFull + 3,     // + slot (3)
  kBarSFull = kBarKVEmpty + 3,      // + head slot (2)
  kBarPFull = kBarSFull + 2,        // + head slot (2)
  kBarODone = kBarPFull + 2,        // + head slot (2)
  kBarDrain = kBarODone + 2,
  kNumBars = kBarDrain + 1
};
constexpr uint32_t kOffTmemSlot = kNumBars * 8;      // uint32 TMEM base address
constexpr uint32_t kOffAbort = kOffTmemSlot + 4;     // int abort flag
static_assert(kOffAbort + 4 <= kBarBytes, "barrier area overflow");

// Wait sites, reported in the status word for diagnosis.
enum : int {
  kSiteQEmpty = 1, kSiteKVEmpty = 2, kSiteQFull = 3, kSiteKVFull = 4, kSitePFull = 5,
  kSiteSFull = 6, kSiteODone = 7, kSiteDrain = 8
};

// ---- unit encoding --------------------------------------------------------------------
// bits 0..7 query tile, 8..13 head pair, 14..31 sequence.
__host__ __device__ __forceinline__ uint32_t encode_unit(uint32_t seq, uint32_t pair,
                                                         uint32_t tile) {
  return (seq << 14) | (pair << 8) | tile;
}

struct Params {
  const uint32_t *units;
  uint32_t n_units;
  const uint32_t *lengths;  // padded
  const int32_t *cu;        // varlen (NULL for padded)
  void *out;
  uint32_t seq;             // padded L (rows per sequence); varlen: unused
  uint32_t heads, group;    // query heads; heads per kv head
  int causal, out_bf16;
  float scale_log2;
  int *status;
};

struct Unit {
  uint32_t tok0;   // row index of position 0 of the sequence
  uint32_t q0;     // first query position of the tile
  uint32_t rows;   // rows of this sequence present in the layout
  uint32_t n;      // valid keys
  uint32_t head0;  // first query head of the pair
  uint32_t kvh;
  uint32_t nt;     // key tiles to visit
  bool live;       // the tile holds rows to write
};

__device__ __forceinline__ Unit decode(const Params &p, uint32_t code) {
  Unit u;
  uint32_t s = code >> 14, pair = (code >> 8) & 63u, t = code & 255u;
  if (p.cu) {
    int32_t a = p.cu[s], b = p.cu[s + 1];
    u.tok0 = (uint32_t)a;
    u.n = b > a ? (uint32_t)(b - a) : 0u;
    u.rows = u.n;
  } else {
    u.tok0 = s * p.seq;
    u.n = min(p.lengths[s], p.seq);
    u.rows = p.seq;
  }
  u.q0 = t * kTile;
  u.head0 = 2 * pair;
  u.kvh = u.head0 / p.group;
  u.live = u.q0 < u.rows;
  uint32_t kend = p.causal ? min(u.q0 + kTile, u.n) : u.n;
  u.nt = u.live ? (kend + kTile - 1) / kTile : 0u;
  return u;
}

// ---- PTX wrappers ---------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with parity `parity` of barrier `bar`.
__device__ __noinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                        int *status, int site) {
  if (mbar_test(bar, parity)) return true;
  long long t0 = clock64();
  while (true) {
    if (mbar_test(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort_flag = 1;
      report_status(status, kStatusTimeout | (site << 8));
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3fffu);
  d |= (uint64_t)((lbo >> 4) & 0x3fffu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3fffu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// K-major operand (rows = M or N, 64 bf16 of K per 128-byte row; 8-row groups 1024 B
// apart).  Step `ks` (16 elements of K) of a 128-wide K: atom ks/4, 32 B per step.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile, int ks) {
  return sw128_desc(tile + (ks >> 2) * kAtomBytes + (ks & 3) * 32, 16, 1024);
}
// MN-major operand (V as B of P.V: N = head_dim contiguous, K = keys).  The two 64-wide
// N halves are the two atoms (16 KB apart, leading byte offset); 8-key groups are
// 1024 B apart (stride byte offset); step `ks` covers keys 16ks..16ks+15.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile, int ks) {
  return sw128_desc(tile + ks * 2048, kAtomBytes, 1024);
}

// Instruction descriptor: kind::f16, A=B=bf16, D=f32, M=128, N=128.
constexpr uint32_t kIdescQK = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 3) << 17) |
                              ((128u >> 4) << 24);
constexpr uint32_t kIdescPV = kIdescQK | (1u << 16);  // B is MN-major

__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
      "[%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---- the kernel -----------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                   const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles.
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bars = sbase + kOffBar;
  uint32_t *tmem_slot = (uint32_t *)(smem + kOffBar + kOffTmemSlot);
  volatile int *abort_flag = (volatile int *)(smem + kOffBar + kOffAbort);
  auto bar = [&](uint32_t i) { return bars + 8u * i; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(bar(kBarQFull), 1);
    mbar_init(bar(kBarQEmpty), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kBarKVFull + s), 1);
      mbar_init(bar(kBarKVEmpty + s), 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(bar(kBarSFull + h), 1);
      mbar_init(bar(kBarPFull + h), 128);
      mbar_init(bar(kBarODone + h), 1);
    }
    mbar_init(bar(kBarDrain), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == kTmaWarp && lane == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kTmaWarp) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t loads = 0, units_done = 0;
      uint32_t armed[kStages] = {0, 0, 0};   // fills per slot (for the abort drain)
      bool ok = true;
      for (uint32_t ui = blockIdx.x; ok && ui < p.n_units; ui += gridDim.x) {
        Unit u = decode(p, p.units[ui]);
        if (!u.nt) continue;
        if (units_done > 0 &&
            !(ok = wait_phase(bar(kBarQEmpty), (units_done - 1) & 1, abort_flag, p.status,
                              kSiteQEmpty)))
          break;
        mbar_expect_tx(bar(kBarQFull), 2 * kTileBytes);
        for (int h = 0; h < 2; ++h)
          for (int a = 0; a < 2; ++a)
            tma_load_3d(sbase + kOffQ + h * kTileBytes + a * kAtomBytes, &tm_q, bar(kBarQFull),
                        a * 64, (int)(u.head0 + h), (int)(u.tok0 + u.q0));
        ++units_done;
        for (uint32_t j = 0; ok && j < u.nt; ++j) {
          for (int which = 0; which < 2; ++which) {  // 0: K_j, 1: V_j
            uint32_t slot = loads % kStages, round = loads / kStages;
            if (round > 0 && !(ok = wait_phase(bar(kBarKVEmpty + slot), (round - 1) & 1,
                                               abort_flag, p.status, kSiteKVEmpty)))
              break;
            uint32_t dst = sbase + kOffKV + slot * kTileBytes;
            mbar_expect_tx(bar(kBarKVFull + slot), kTileBytes);
            const CUtensorMap *map = which ? &tm_v : &tm_k;
            for (int a = 0; a < 2; ++a)
              tma_load_3d(dst + a * kAtomBytes, map, bar(kBarKVFull + slot), a * 64,
                          (int)u.kvh, (int)(u.tok0 + j * kTile));
            ++armed[slot];
            ++loads;
          }
        }
      }
      if (!ok) {
        // Drain: every armed fill completes by itself; wait for the latest of each slot
        // and for the last Q fill so no copy lands in freed shared memory.
        for (int s = 0; s < kStages; ++s)
          if (armed[s]) {
            long long t0 = clock64();
            while (!mbar_test(bar(kBarKVFull + s), (armed[s] - 1) & 1) &&
                   clock64() - t0 < kWaitCycles) {
            }
          }
        if (units_done) {
          long long t0 = clock64();
          while (!mbar_test(bar(kBarQFull), (units_done - 1) & 1) &&
                 clock64() - t0 < kWaitCycles) {
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t loads = 0, units_done = 0;
      uint32_t pcount[2] = {0, 0};  // p_full completions consumed per head slot
      bool ok = true;
      const uint32_t tS[2] = {tmem + 0, tmem + 128};
      const uint32_t tO[2] = {tmem + 256, tmem + 384};
      const uint32_t q_tile[2] = {sbase + kOffQ, sbase + kOffQ + kTileBytes};
      const uint32_t p_tile[2] = {sbase + kOffP, sbase + kOffP + kTileBytes};
      bool issued = false;
      for (uint32_t ui = blockIdx.x; ok && ui < p.n_units; ui += gridDim.x) {
        Unit u = decode(p, p.units[ui]);
        if (!u.nt) continue;
        if (!(ok = wait_phase(bar(kBarQFull), units_done & 1, abort_flag, p.status,
                              kSiteQFull)))
          break;
        ++units_done;
        // K_0
        uint32_t slotK = loads % kStages;
        if (!(ok = wait_phase(bar(kBarKVFull + slotK), (loads / kStages) & 1, abort_flag,
                              p.status, kSiteKVFull)))
          break;
        ++loads;
        tc_fence_after();
        for (int h = 0; h < 2; ++h) {
          uint32_t kt = sbase + kOffKV + slotK * kTileBytes;
          for (int ks = 0; ks < 8; ++ks)
            umma(tS[h], kmajor_desc(q_tile[h], ks), kmajor_desc(kt, ks), kIdescQK, ks > 0);
          umma_commit(bar(kBarSFull + h));
          issued = true;
        }
        umma_commit(bar(kBarKVEmpty + slotK));
        for (uint32_t j = 0; ok && j < u.nt; ++j) {
          uint32_t slotV = loads % kStages;
          if (!(ok = wait_phase(bar(kBarKVFull + slotV), (loads / kStages) & 1, abort_flag,
                                p.status, kSiteKVFull)))
            break;
          ++loads;
          const uint32_t vt = sbase + kOffKV + slotV * kTileBytes;
          const bool more = j + 1 < u.nt;
          uint32_t slotN = 0, kt = 0;
          for (int h = 0; h < 2 && ok; ++h) {
            if (!(ok = wait_phase(bar(kBarPFull + h), pcount[h] & 1, abort_flag, p.status,
                                  kSitePFull)))
              break;
            ++pcount[h];
            tc_fence_after();
            for (int ks = 0; ks < 8; ++ks)
              umma(tO[h], kmajor_desc(p_tile[h], ks), mnmajor_desc(vt, ks), kIdescPV,
                   (j > 0 || ks > 0) ? 1u : 0u);
            umma_commit(bar(kBarODone + h));
            if (more) {
              if (h == 0) {
                slotN = loads % kStages;
                if (!(ok = wait_phase(bar(kBarKVFull + slotN), (loads / kStages) & 1,
                                      abort_flag, p.status, kSiteKVFull)))
                  break;
                ++loads;
                tc_fence_after();
                kt = sbase + kOffKV + slotN * kTileBytes;
              }
              for (int ks = 0; ks < 8; ++ks)
                umma(tS[h], kmajor_desc(q_tile[h], ks), kmajor_desc(kt, ks), kIdescQK, ks > 0);
              umma_commit(bar(kBarSFull + h));
            }
          }
          if (!ok) break;
          if (more) umma_commit(bar(kBarKVEmpty + slotN));
          umma_commit(bar(kBarKVEmpty + slotV));
        }
        if (ok) umma_commit(bar(kBarQEmpty));
      }
      if (issued) {
        // Wait until every MMA this thread issued has completed (normal exit and abort).
        umma_commit(bar(kBarDrain));
        long long t0 = clock64();
        while (!mbar_test(bar(kBarDrain), 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax warpgroups ----------------
    const int hs = warp >> 2;                   // head slot
    const uint32_t r = (warp & 3) * 32 + lane;  // tile row == TMEM lane
    const uint32_t lane_base = ((uint32_t)(warp & 3) * 32u) << 16;
    const uint32_t tS = tmem + lane_base + hs * 128;
    const uint32_t tO = tmem + lane_base + 256 + hs * 128;
    uint8_t *ptile = smem + kOffP + hs * kTileBytes;
    uint32_t scount = 0, ocount = 0;
    bool ok = true;
    for (uint32_t ui = blockIdx.x; ui < p.n_units; ui += gridDim.x) {
      Unit u = decode(p, p.units[ui]);
      if (!u.live) continue;
      const uint32_t head = u.head0 + hs;
      const uint32_t qpos = u.q0 + r;
      const bool store = qpos < u.rows;
      const size_t orow = ((size_t)(u.tok0 + qpos) * p.heads + head) * kTile;
      if (!u.nt) {
        // Zero valid keys: 0/0, as the reference's running sums give.
        if (store) {
          if (p.out_bf16) {
            uint16_t *o = (uint16_t *)p.out + orow;
            for (int c = 0; c < kTile; ++c) o[c] = 0x7fc0u;
          } else {
            float *o = (float *)p.out + orow;
            for (int c = 0; c < kTile; ++c) o[c] = __int_as_float(0x7fc00000);
          }
        }
        continue;
      }
      if (!ok) break;
      const uint32_t end = p.causal ? min(qpos + 1, u.n) : u.n;
      float m_ref = -INFINITY, l = 0.f;
      for (uint32_t j = 0; j < u.nt; ++j) {
        ok = __all_sync(0xffffffffu, wait_phase(bar(kBarSFull + hs), scount & 1, abort_flag,
                                                p.status, kSiteSFull));
        if (!ok) break;
        ++scount;
        tc_fence_after();
        const int valid = (int)min(max((int)end - (int)(j * kTile), 0), kTile);
        // Pass 1: row maximum over the valid keys.
        float mx = -INFINITY;
        for (int c = 0; c < 4; ++c) {
          uint32_t x[32];
          tmem_ld32(tS + c * 32, x);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 32; ++t)
            if (c * 32 + t < valid) mx = fmaxf(mx, __uint_as_float(x[t]));
        }
        const float mt = mx * p.scale_log2;
        if (j > 0) {
          // P(j-1).V(j-1) must be complete before P and O are touched.
          ok = __all_sync(0xffffffffu, wait_phase(bar(kBarODone + hs), ocount & 1, abort_flag,
                                                  p.status, kSiteODone));
          if (!ok) break;
          ++ocount;
          tc_fence_after();
          // Rescale decision is per row; TMEM access is warp-wide (.sync.aligned), so
          // the warp rescales when any of its rows needs it (others scale by 1).
          float corr = 1.0f;
          const bool need = mt > m_ref + kRescaleThreshold;
          if (need) {
            corr = exp2f(m_ref - mt);
            l *= corr;
            m_ref = mt;
          }
          if (__any_sync(0xffffffffu, need)) {
            for (int c = 0; c < 4; ++c) {
              uint32_t x[32];
              tmem_ld32(tO + c * 32, x);
              tmem_ld_wait();
#pragma unroll
              for (int t = 0; t < 32; ++t) x[t] = __float_as_uint(__uint_as_float(x[t]) * corr);
              tmem_st32(tO + c * 32, x);
            }
            tmem_st_wait();
          }
        } else {
          m_ref = mt;
        }
        // Pass 2: probabilities -> bf16 -> P tile (128-byte swizzle, K-major).
        for (int c = 0; c < 4; ++c) {
          uint32_t x[32];
          tmem_ld32(tS + c * 32, x);
          tmem_ld_wait();
          uint32_t packed[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            const int k0 = c * 32 + 2 * t;
            float p0 = k0 < valid ? exp2f(__uint_as_float(x[2 * t]) * p.scale_log2 - m_ref) : 0.f;
            float p1 =
                k0 + 1 < valid ? exp2f(__uint_as_float(x[2 * t + 1]) * p.scale_log2 - m_ref) : 0.f;
            l += p0 + p1;
            packed[t] = pack_bf16x2(p0, p1);
          }
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const uint32_t c8 = c * 4 + g;  // 8-key group 0..15
            const uint32_t off = (c8 >> 3) * kAtomBytes + r * 128 + (((c8 & 7) ^ (r & 7)) << 4);
            *(uint4 *)(ptile + off) =
                make_uint4(packed[4 * g], packed[4 * g + 1], packed[4 * g + 2], packed[4 * g + 3]);
          }
        }
        fence_proxy_async();
        tc_fence_before();
        mbar_arrive(bar(kBarPFull + hs));
      }
      if (!ok) break;
      // Epilogue: wait for the last P.V, normalise, store.
      ok = __all_sync(0xffffffffu, wait_phase(bar(kBarODone + hs), ocount & 1, abort_flag,
                                              p.status, kSiteODone));
      if (!ok) break;
      ++ocount;
      tc_fence_after();
      const float inv = 1.0f / l;
      for (int c = 0; c < 4; ++c) {
        uint32_t x[32];
        tmem_ld32(tO + c * 32, x);
        tmem_ld_wait();
        if (!store) continue;
        if (p.out_bf16) {
          uint4 *o = (uint4 *)((uint16_t *)p.out + orow + c * 32);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              w[e] = pack_bf16x2(__uint_as_float(x[8 * g + 2 * e]) * inv,
                                 __uint_as_float(x[8 * g + 2 * e + 1]) * inv);
            o[g] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        } else {
          float4 *o = (float4 *)((float *)p.out + orow + c * 32);
#pragma unroll
          for (int g = 0; g < 8; ++g)
            o[g] = make_float4(__uint_as_float(x[4 * g]) * inv, __uint_as_float(x[4 * g + 1]) * inv,
                               __uint_as_float(x[4 * g + 2]) * inv,
                               __uint_as_float(x[4 * g + 3]) * inv);
        }
      }
      tc_fence_before();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512)
                 : "memory");
  }
}

}  // namespace tc

// ---- host side --------------------------------------------------------------------------

bool tc_attention_supported(const AttnProblem &p) {
  if (p.dim != 128 || p.in_dtype != 1) return false;
  if (!p.kv_heads || p.heads % p.kv_heads) return false;
  uint32_t group = p.heads / p.kv_heads;
  if (group % 2) return false;            // head pairs must share one kv head
  if (p.heads / 2 > 64) return false;     // pair index has 6 bits
  if ((uint64_t)p.seq > 255u * 128u) return false;  // tile index has 8 bits
  if (p.batch >= (1u << 18)) return false;
  if ((uintptr_t)p.q % 16 || (uintptr_t)p.k % 16 || (uintptr_t)p.v % 16 || (uintptr_t)p.out % 16)
    return false;
  return true;
}

uint32_t tc_max_units(const AttnProblem &p) {
  uint32_t tiles = (p.seq + tc::kTile - 1) / tc::kTile;
  return p.batch * (p.heads / 2) * tiles;
}

// Longest-first list of units.  Cost of a unit = key tiles it visits (host lengths
// known) or, without host lengths, its query-tile index (later tiles of a causal
// sequence visit more key tiles).
uint32_t tc_build_units(const AttnProblem &p, const uint32_t *lengths_host, const int32_t *cu_host,
                        uint32_t *units) {
  const uint32_t tiles = (p.seq + tc::kTile - 1) / tc::kTile;
  const uint32_t pairs = p.heads / 2;
  struct Item { uint32_t cost, code; };
  std::vector<Item> items;
  items.reserve((size_t)p.batch * pairs * tiles);
  for (uint32_t s = 0; s < p.batch; ++s) {
    uint32_t n, rows;
    bool known = false;
    if (p.cu_seqlens) {
      if (cu_host) {
        int32_t a = cu_host[s], b = cu_host[s + 1];
        n = b > a ? (uint32_t)(b - a) : 0u;
        rows = n;
        known = true;
      } else {
        n = rows = p.seq;
      }
    } else {
      rows = p.seq;
      n = lengths_host ? std::min(lengths_host[s], p.seq) : p.seq;
      known = lengths_host != nullptr;
    }
    for (uint32_t t = 0; t < tiles; ++t) {
      uint32_t q0 = t * tc::kTile;
      if (q0 >= rows) break;
      uint32_t cost;
      if (known) {
        uint32_t kend = p.causal ? std::min(q0 + (uint32_t)tc::kTile, n) : n;
        cost = (kend + tc::kTile - 1) / tc::kTile;
      } else {
        cost = p.causal ? t + 1 : tiles;
      }
      for (uint32_t hp = 0; hp < pairs; ++hp) items.push_back({cost, tc::encode_unit(s, hp, t)});
    }
  }
  std::stable_sort(items.begin(), items.end(),
                   [](const Item &a, const Item &b) { return a.cost > b.cost; });
  for (size_t i = 0; i < items.size(); ++i) units[i] = items[i].code;
  return (uint32_t)items.size();
}

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

// 3-D map over a [rows, heads, 128] bf16 tensor; box = 128 rows x 1 head x 64 columns,
// 128-byte swizzle, zero fill beyond the last row.
bool make_map(CUtensorMap *map, const void *base, uint32_t rows, uint32_t heads) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {128, heads, rows};
  cuuint64_t strides[2] = {128 * 2, (cuuint64_t)heads * 128 * 2};
  cuuint32_t box[3] = {64, 1, 128};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims,
                  strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_attention_tc(const AttnProblem &p, const uint32_t *units, uint32_t n_units,
                                int num_sms, int *status, cudaStream_t stream) {
  if (!n_units) return cudaSuccess;
  CUtensorMap mq, mk, mv;
  const uint32_t rows = p.total;
  if (!make_map(&mq, p.q, rows, p.heads) || !make_map(&mk, p.k, rows, p.kv_heads) ||
      !make_map(&mv, p.v, rows, p.kv_heads))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(tc::attn_tc_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)tc::kSmemBytes);
  if (e != cudaSuccess) return e;
  tc::Params prm;
  prm.units = units;
  prm.n_units = n_units;
  prm.lengths = p.lengths;
  prm.cu = p.cu_seqlens;
  prm.out = p.out;
  prm.seq = p.seq;
  prm.heads = p.heads;
  prm.group = p.heads / p.kv_heads;
  prm.causal = p.causal;
  prm.out_bf16 = p.out_dtype == 1;
  prm.scale_log2 = p.scale * 1.4426950408889634f;
  prm.status = status;
  uint32_t grid = std::min<uint32_t>(n_units, (uint32_t)num_sms);
  tc::attn_tc_kernel<<<grid, tc::kThreads, tc::kSmemBytes, stream>>>(mq, mk, mv, prm);
  return cudaGetLastError();
}

}  // namespace tx
