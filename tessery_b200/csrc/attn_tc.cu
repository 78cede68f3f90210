// Blackwell (sm_100a) tensor-core attention for head_dim 128, bf16 q/k/v, fp32 softmax
// and accumulation: the Qwen3 causal GQA operator of qwen3.py:238-245 dispatched by
// MetalRuntime._attention (metal.py:532-569), with the semantics of kernels.metal:78-103
// (and of its tiled/tail variants :108-298).  Optionally fused in front: the q RMSNorm +
// RoPE of qwen3.py:216-237 (kernels.metal:53-74), applied to each Q tile in shared memory.
//
// Work unit: (sequence, pair of query heads sharing one kv head, 128-row query tile).
// The two query heads of a pair share every K/V tile, so each K/V tile is fetched once
// per pair (GQA head sharing).  A persistent grid of one CTA per SM walks a host-built,
// longest-first list of units.
//
// Warp roles (320 threads, one CTA per SM):
//   warps 0-3  head slot 0: q prologue on the Q tile, softmax, epilogue (thread t = row t)
//   warps 4-7  head slot 1
//   warp 8     TMA producer: Q_h tiles (each as soon as its last QK of the previous unit
//              has run), then K_j, V_j through a 3-slot ring
//   warp 9     TMEM allocator and single-thread tcgen05.mma issuer
// Tensor memory (512 columns x 128 lanes, fp32):
//   [0,128) S slot 0, [128,256) S slot 1, [256,384) O slot 0, [384,512) O slot 1.
// Shared memory: Q0, Q1, 3 K/V slots, P0, P1: 128x128 bf16 tiles, each two 128-row x
// 128-byte atoms in the 128-byte-swizzled layout that TMA writes and UMMA reads.  After
// the last P.V of a unit, P_h is the staging buffer of the output tile, which leaves by
// TMA bulk-tensor stores.
//
// Per key tile j the issuer runs S_h = Q_h K_j^T (M=128, N=128, K=128, bf16 -> f32 in
// TMEM); the softmax warps turn S_h into P_h = exp2(S_h*scale*log2e - m) (bf16, shared
// memory); the issuer accumulates O_h += P_h V_j in TMEM.  Tiles above the causal
// diagonal and beyond each sequence's length are never visited; the diagonal and the
// last tile are masked per row.  The running maximum is updated lazily: O is rescaled
// only when a tile maximum exceeds the reference maximum by more than 8 (log2 units),
// so every probability stays below 2^8 and the normalised result is unchanged.
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
constexpr uint32_t kOffMisc = kOffP + 2 * kTileBytes;
constexpr uint32_t kMiscBytes = 768;
constexpr uint32_t kSmemBytes = kOffMisc + kMiscBytes + 1024;  // + base alignment slack
constexpr int kThreads = 320;
constexpr int kTmaWarp = 8, kMmaWarp = 9;
constexpr long long kWaitCycles = 2000000000ll;  // ~1 s at B200 clocks
constexpr float kRescaleThreshold = 8.0f;        // log2 units
constexpr uint32_t kStageBytes = 4096;           // one 32-row x 128-byte output box

// Barrier slots (uint64 each) at the start of the misc area.
enum : uint32_t {
  kBarQFull = 0,                      // + head slot: Q_h landed (TMA transaction count)
  kBarQReady = kBarQFull + 2,         // + head slot: Q_h transformed (256 arrivals)
  kBarQEmpty = kBarQReady + 2,        // + head slot: last QK_h of the unit ran
  kBarKVFull = kBarQEmpty + 2,        // + ring slot
  kBarKVEmpty = kBarKVFull + kStages,
  kBarSFull = kBarKVEmpty + kStages,  // + head slot
  kBarPFull = kBarSFull + 2,          // + head slot (128 arrivals)
  kBarODone = kBarPFull + 2,          // + head slot
  kBarXform = kBarODone + 2,          // q prologue: both row norms read (256 arrivals)
  kBarDrain = kBarXform + 1,
  kNumBars = kBarDrain + 1
};
constexpr uint32_t kOffTmemSlot = kNumBars * 8;   // uint32 TMEM base address
constexpr uint32_t kOffAbort = kOffTmemSlot + 4;  // int abort flag
constexpr uint32_t kOffQw = 256;                  // bf16 q-norm weight [128]
constexpr uint32_t kOffInvFreq = 512;             // float inverse frequencies [64]
static_assert(kOffAbort + 4 <= kOffQw, "misc area overflow");
static_assert(kSmemBytes <= 232448, "shared memory budget");

// Wait sites, reported in the status word for diagnosis.
enum : int {
  kSiteQEmpty = 1, kSiteKVEmpty = 2, kSiteQReady = 3, kSiteKVFull = 4, kSitePFull = 5,
  kSiteSFull = 6, kSiteODone = 7, kSiteQFull = 8, kSiteXform = 9
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
  uint32_t seq;             // padded L (rows per sequence)
  uint32_t heads, group;    // query heads; heads per kv head
  int causal, out_bf16;
  float scale_log2;
  int *status;
  const uint16_t *q_norm_w;  // fused q prologue when non-NULL
  float eps, theta;
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

// Bounded wait without a status report (drains after an abort).
__device__ __forceinline__ void drain_phase(uint32_t bar, uint32_t parity) {
  long long t0 = clock64();
  while (!mbar_test(bar, parity) && clock64() - t0 < kWaitCycles) {
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
// L2 prefetch of one box (no shared memory, no completion tracking).
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap *map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, uint32_t src, int x, int y,
                                             int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
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

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
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

// 2^x on the special-function unit; results below 2^-126 flush to zero (probabilities that
// small are negligible against a row sum of at least 1).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// sin and cos of a float angle: Cody-Waite reduction by 2*pi (2*pi split into a float
// head and a float tail) to [-pi, pi], then the hardware approximations, which are
// accurate to about 2^-21 absolute on that interval.
__device__ __forceinline__ void sincos_reduced(float angle, float *s, float *c) {
  const float k = rintf(angle * 0.159154943091895336f);
  float r = fmaf(k, -6.28318548202514648f, angle);
  r = fmaf(k, 1.74845553e-07f, r);
  __sincosf(r, s, c);
}

__device__ __forceinline__ uint32_t u4_at(const uint4 &v, int e) {
  return e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w;
}
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ void acc_squares(float (&ssq)[4], const uint4 &v) {
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t x = u4_at(v, e);
    ssq[e] = fmaf(bf16_lo(x), bf16_lo(x), ssq[e]);
    ssq[e] = fmaf(bf16_hi(x), bf16_hi(x), ssq[e]);
  }
}

// In-place q RMSNorm + RoPE of the two Q tiles (head slots 0 and 1) of a unit, shared
// by both warpgroups: the thread owning row r in warpgroup `part` transforms row r of
// both tiles for the rotation pairs c in [32*part, 32*part + 32), so each (position, c)
// sine and cosine is evaluated once for the two heads.  Arithmetic per element follows
// kernels.metal:53-74: x * inv * w, then the rotation of (element c, element c + 64) by
// angle pos * inv_freq[c].  Every row norm reads the whole row, half of which the other
// warpgroup rewrites, so the two passes are separated by a barrier of both warpgroups.
// Pass 1 of the q prologue: inverse RMS of row r of both Q tiles.
__device__ __forceinline__ void q_row_norms(uint32_t q_tiles, uint32_t r, float eps,
                                            float (&inv)[2]) {
  const uint32_t sw = r & 7;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t row = q_tiles + h * kTileBytes + r * 128;
    float ssq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < 16; ++c)
      acc_squares(ssq, ld_shared_v4(row + (c >> 3) * kAtomBytes + (((c & 7) ^ sw) << 4)));
    inv[h] = 1.0f / sqrtf(((ssq[0] + ssq[1]) + (ssq[2] + ssq[3])) / 128.0f + eps);
  }
}

// Pass 2: normalise and rotate this warpgroup's half of the rotation pairs of row r of
// both tiles (run only after both warpgroups finished pass 1 on the tiles).
__device__ __forceinline__ void q_rotate_pair(uint32_t q_tiles, uint32_t r, uint32_t pos,
                                              int part, const uint16_t *w,
                                              const float *inv_freq, const float (&inv)[2]) {
  const uint32_t sw = r & 7;
  const float fpos = (float)pos;
#pragma unroll 1
  for (int gg = 0; gg < 4; ++gg) {  // pass 2: own chunk groups, both heads at once
    const uint32_t g = 4 * part + gg;
    uint4 lo[2], hi[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t row = q_tiles + h * kTileBytes + r * 128;
      lo[h] = ld_shared_v4(row + ((g ^ sw) << 4));
      hi[h] = ld_shared_v4(row + kAtomBytes + ((g ^ sw) << 4));
    }
    uint32_t out_lo[2][4], out_hi[2][4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float ra[2][2], rb[2][2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {  // element within the bf16 pair
        const uint32_t c = 8 * g + 2 * e + hh;
        float s, co;
        sincos_reduced(fpos * inv_freq[c], &s, &co);
        const float wa = bf16_bits_to_f32(w[c]), wb = bf16_bits_to_f32(w[c + 64]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t A = u4_at(lo[h], e), B = u4_at(hi[h], e);
          const float a = (hh ? bf16_hi(A) : bf16_lo(A)) * inv[h] * wa;
          const float b = (hh ? bf16_hi(B) : bf16_lo(B)) * inv[h] * wb;
          ra[h][hh] = a * co - b * s;
          rb[h][hh] = a * s + b * co;
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        out_lo[h][e] = pack_bf16x2(ra[h][0], ra[h][1]);
        out_hi[h][e] = pack_bf16x2(rb[h][0], rb[h][1]);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t row = q_tiles + h * kTileBytes + r * 128;
      st_shared_v4(row + ((g ^ sw) << 4), out_lo[h][0], out_lo[h][1], out_lo[h][2], out_lo[h][3]);
      st_shared_v4(row + kAtomBytes + ((g ^ sw) << 4), out_hi[h][0], out_hi[h][1], out_hi[h][2],
                   out_hi[h][3]);
    }
  }
}

// exp2(x*sl - m) of one 32-key chunk of a row (0 for keys at or past `valid`), rounded to
// bf16 pairs and stored into the row's slots (`prow` = shared address of row r of the
// swizzled K-major P tile).  Returns the chunk's probability sum.
__device__ __forceinline__ float emit_p(const uint32_t (&x)[32], int c, int valid, float sl,
                                        float m, uint32_t prow, uint32_t r) {
  float sum[4] = {0.f, 0.f, 0.f, 0.f};
  uint32_t packed[16];
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    const int k0 = c * 32 + 2 * t;
    float p0 = k0 < valid ? ex2(fmaf(__uint_as_float(x[2 * t]), sl, -m)) : 0.f;
    float p1 = k0 + 1 < valid ? ex2(fmaf(__uint_as_float(x[2 * t + 1]), sl, -m)) : 0.f;
    sum[t & 3] += p0 + p1;
    packed[t] = pack_bf16x2(p0, p1);
  }
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint32_t c8 = c * 4 + g;  // 8-key group 0..15
    st_shared_v4(prow + (c8 >> 3) * kAtomBytes + (((c8 & 7) ^ (r & 7)) << 4), packed[4 * g],
                 packed[4 * g + 1], packed[4 * g + 2], packed[4 * g + 3]);
  }
  return (sum[0] + sum[1]) + (sum[2] + sum[3]);
}

// ---- the kernel -----------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                   const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v,
                   const __grid_constant__ CUtensorMap tm_o, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles.
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bars = sbase + kOffMisc;
  uint8_t *misc = smem + kOffMisc;
  uint32_t *tmem_slot = (uint32_t *)(misc + kOffTmemSlot);
  volatile int *abort_flag = (volatile int *)(misc + kOffAbort);
  uint16_t *qw_s = (uint16_t *)(misc + kOffQw);
  float *invf_s = (float *)(misc + kOffInvFreq);
  auto bar = [&](uint32_t i) { return bars + 8u * i; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int h = 0; h < 2; ++h) {
      mbar_init(bar(kBarQFull + h), 1);
      mbar_init(bar(kBarQReady + h), 256);
      mbar_init(bar(kBarQEmpty + h), 1);
      mbar_init(bar(kBarSFull + h), 1);
      mbar_init(bar(kBarPFull + h), 128);
      mbar_init(bar(kBarODone + h), 1);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kBarKVFull + s), 1);
      mbar_init(bar(kBarKVEmpty + s), 1);
    }
    mbar_init(bar(kBarXform), 256);
    mbar_init(bar(kBarDrain), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (p.q_norm_w) {
    for (int i = threadIdx.x; i < 128; i += kThreads) qw_s[i] = p.q_norm_w[i];
    for (int i = threadIdx.x; i < 64; i += kThreads)
      invf_s[i] = (float)pow((double)p.theta, -2.0 * (double)i / 128.0);
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
    prefetch_tmap(&tm_o);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kTmaWarp) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t loads = 0, units_done = 0;
      uint32_t armed[kStages] = {0, 0, 0};  // fills per slot (for the abort drain)
      bool ok = true;
      for (uint32_t ui = blockIdx.x; ok && ui < p.n_units; ui += gridDim.x) {
        Unit u = decode(p, p.units[ui]);
        if (!u.nt) continue;
        for (int h = 0; h < 2 && ok; ++h) {
          if (units_done > 0 &&
              !(ok = wait_phase(bar(kBarQEmpty + h), (units_done - 1) & 1, abort_flag,
                                p.status, kSiteQEmpty)))
            break;
          mbar_expect_tx(bar(kBarQFull + h), kTileBytes);
          for (int a = 0; a < 2; ++a)
            tma_load_3d(sbase + kOffQ + h * kTileBytes + a * kAtomBytes, &tm_q,
                        bar(kBarQFull + h), a * 64, (int)(u.head0 + h), (int)(u.tok0 + u.q0));
        }
        if (!ok) break;
        ++units_done;
        // Warm L2 with the next unit's tiles so that its TMA loads hit L2.
        for (uint32_t un = ui + gridDim.x; un < p.n_units; un += gridDim.x) {
          const Unit v = decode(p, p.units[un]);
          if (!v.nt) continue;
          for (int h = 0; h < 2; ++h)
            for (int a = 0; a < 2; ++a)
              tma_prefetch_3d(&tm_q, a * 64, (int)(v.head0 + h), (int)(v.tok0 + v.q0));
          for (uint32_t j = 0; j < v.nt; ++j)
            for (int a = 0; a < 2; ++a) {
              tma_prefetch_3d(&tm_k, a * 64, (int)v.kvh, (int)(v.tok0 + j * kTile));
              tma_prefetch_3d(&tm_v, a * 64, (int)v.kvh, (int)(v.tok0 + j * kTile));
            }
          break;
        }
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
        // Every armed fill completes by itself: wait for the latest of each slot and for
        // the Q fills so that no copy lands in shared memory after the CTA exits.
        for (int s = 0; s < kStages; ++s)
          if (armed[s]) drain_phase(bar(kBarKVFull + s), (armed[s] - 1) & 1);
        for (int h = 0; h < 2; ++h)
          if (units_done) drain_phase(bar(kBarQFull + h), (units_done - 1) & 1);
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
        // K_0 and both Q tiles, then S_h = Q_h K_0^T.
        uint32_t slotK = loads % kStages;
        if (!(ok = wait_phase(bar(kBarKVFull + slotK), (loads / kStages) & 1, abort_flag,
                              p.status, kSiteKVFull)))
          break;
        ++loads;
        const uint32_t kt0 = sbase + kOffKV + slotK * kTileBytes;
        for (int h = 0; h < 2 && ok; ++h) {
          if (!(ok = wait_phase(bar(kBarQReady + h), units_done & 1, abort_flag, p.status,
                                kSiteQReady)))
            break;
          tc_fence_after();
          for (int ks = 0; ks < 8; ++ks)
            umma(tS[h], kmajor_desc(q_tile[h], ks), kmajor_desc(kt0, ks), kIdescQK, ks > 0);
          umma_commit(bar(kBarSFull + h));
          if (u.nt == 1) umma_commit(bar(kBarQEmpty + h));
          issued = true;
        }
        if (!ok) break;
        ++units_done;
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
              if (j + 2 == u.nt) umma_commit(bar(kBarQEmpty + h));  // last QK_h of the unit
            }
          }
          if (!ok) break;
          if (more) umma_commit(bar(kBarKVEmpty + slotN));
          umma_commit(bar(kBarKVEmpty + slotV));
        }
      }
      if (issued) {
        // Wait until every MMA this thread issued has completed (normal exit and abort).
        umma_commit(bar(kBarDrain));
        drain_phase(bar(kBarDrain), 0);
      }
    }
    __syncwarp();
  } else {
    // ---------------- q prologue, softmax and epilogue (one warpgroup per head slot) ----
    const int hs = warp >> 2;                   // head slot
    const uint32_t wq = (uint32_t)(warp & 3);   // warp within the warpgroup
    const uint32_t r = wq * 32 + lane;          // tile row == TMEM lane
    const uint32_t lane_base = (wq * 32u) << 16;
    const uint32_t tS = tmem + lane_base + hs * 128;
    const uint32_t tO = tmem + lane_base + 256 + hs * 128;
    const uint32_t prow = sbase + kOffP + hs * kTileBytes + r * 128;  // row r of P_h
    // Output staging of this warp: the P rows it writes itself (rows 32*wq.. of each of
    // the two atoms of P_h, 4 KB each), so only this warp's bulk stores read them.
    const uint32_t stage[2] = {sbase + kOffP + hs * kTileBytes + wq * kStageBytes,
                               sbase + kOffP + hs * kTileBytes + kAtomBytes + wq * kStageBytes};
    uint32_t qcount = 0, scount = 0, ocount = 0;
    bool ok = true;
    // Q tiles of a unit: wait for both copies, apply the q prologue (both warpgroups,
    // half the rotation pairs each), hand both tiles to the issuer.
    uint32_t prepared = 0xffffffffu, xcount = 0;
    auto prepare = [&](uint32_t index, const Unit &v) {
      for (int h = 0; h < 2 && ok; ++h)
        ok = __all_sync(0xffffffffu, wait_phase(bar(kBarQFull + h), qcount & 1, abort_flag,
                                                p.status, kSiteQFull));
      if (!ok) return;
      ++qcount;
      if (p.q_norm_w) {
        float inv[2];
        q_row_norms(sbase + kOffQ, r, p.eps, inv);
        mbar_arrive(bar(kBarXform));
        ok = __all_sync(0xffffffffu, wait_phase(bar(kBarXform), xcount & 1, abort_flag, p.status,
                                                kSiteXform));
        ++xcount;
        if (!ok) return;
        q_rotate_pair(sbase + kOffQ, r, v.q0 + r, hs, qw_s, invf_s, inv);
        fence_proxy_async();
      }
      mbar_arrive(bar(kBarQReady + 0));
      mbar_arrive(bar(kBarQReady + 1));
      prepared = index;
    };
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
      if (prepared != ui) prepare(ui, u);
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
        // Row maximum over the valid keys: chunks 0-1, then 2-3 (kept for the exp pass).
        uint32_t xa[32], xb[32];
        float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        tmem_ld32(tS + 0, xa);
        tmem_ld32(tS + 32, xb);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          if (t < valid) mq[t & 1] = fmaxf(mq[t & 1], __uint_as_float(xa[t]));
          if (32 + t < valid) mq[2 + (t & 1)] = fmaxf(mq[2 + (t & 1)], __uint_as_float(xb[t]));
        }
        uint32_t xc[32], xd[32];
        tmem_ld32(tS + 64, xc);
        tmem_ld32(tS + 96, xd);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          if (64 + t < valid) mq[t & 1] = fmaxf(mq[t & 1], __uint_as_float(xc[t]));
          if (96 + t < valid) mq[2 + (t & 1)] = fmaxf(mq[2 + (t & 1)], __uint_as_float(xd[t]));
        }
        const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
        const float mt = mx * p.scale_log2;
        if (j > 0) {
          // P(j-1).V(j-1), which reads P and accumulates into O, has completed: the issuer
          // committed s_full(j) after it, and a commit tracks every earlier tcgen05 op of
          // the issuing thread.  Its o_done phase is therefore complete; count it.
          ++ocount;
          // Rescale decision is per row; TMEM access is warp-wide (.sync.aligned), so
          // the warp rescales when any of its rows needs it (others scale by 1).
          float corr = 1.0f;
          const bool need = mt > m_ref + kRescaleThreshold;
          if (need) {
            corr = ex2(m_ref - mt);
            l *= corr;
            m_ref = mt;
          }
          if (__any_sync(0xffffffffu, need)) {
            for (int c = 0; c < 4; ++c) {
              uint32_t o[32];
              tmem_ld32(tO + c * 32, o);
              tmem_ld_wait();
#pragma unroll
              for (int t = 0; t < 32; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * corr);
              tmem_st32(tO + c * 32, o);
            }
            tmem_st_wait();
          }
        } else {
          m_ref = mt;
        }
        if (j == 0) {
          // P_h was the previous unit's output staging: its bulk stores must have read it.
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
        }
        // Probabilities -> bf16 -> P tile: chunks 2-3 from registers while chunks 0-1 are
        // loaded again from TMEM.
        tmem_ld32(tS + 0, xa);
        l += emit_p(xc, 2, valid, p.scale_log2, m_ref, prow, r);
        tmem_ld32(tS + 32, xb);
        l += emit_p(xd, 3, valid, p.scale_log2, m_ref, prow, r);
        tmem_ld_wait();
        l += emit_p(xa, 0, valid, p.scale_log2, m_ref, prow, r);
        l += emit_p(xb, 1, valid, p.scale_log2, m_ref, prow, r);
        fence_proxy_async();
        tc_fence_before();
        mbar_arrive(bar(kBarPFull + hs));
      }
      if (!ok) break;
      // Hand the next unit's Q tiles to the issuer before this unit's epilogue, so the
      // tensor cores start on it while the output leaves.
      for (uint32_t un = ui + gridDim.x; un < p.n_units; un += gridDim.x) {
        const Unit v = decode(p, p.units[un]);
        if (v.live && v.nt) {
          prepare(un, v);
          break;
        }
      }
      if (!ok) break;
      // Epilogue: wait for the last P.V, normalise, store.  Warps whose 32 rows are all
      // inside the sequence stage their rows (swizzled, in the now free P tile) and send
      // them with TMA bulk-tensor stores; a warp at a ragged end stores row by row.
      ok = __all_sync(0xffffffffu, wait_phase(bar(kBarODone + hs), ocount & 1, abort_flag,
                                              p.status, kSiteODone));
      if (!ok) break;
      ++ocount;
      tc_fence_after();
      const float inv = 1.0f / l;
      const uint32_t wrow0 = u.q0 + wq * 32;
      const bool bulk = wrow0 + 32 <= u.rows;
      const uint32_t srow0 = (uint32_t)lane * 128;
      const uint32_t sw = (uint32_t)lane & 7;
      if (!p.out_bf16) {
        uint32_t ob[2][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if ((c & 1) == 0) {  // two 32-column chunks per TMEM round trip
            tmem_ld32(tO + c * 32, ob[0]);
            tmem_ld32(tO + c * 32 + 32, ob[1]);
            tmem_ld_wait();
          }
          uint32_t (&x)[32] = ob[c & 1];
#pragma unroll
          for (int t = 0; t < 32; ++t) x[t] = __float_as_uint(__uint_as_float(x[t]) * inv);
          if (bulk) {
            const uint32_t buf = stage[c & 1];
            if (c >= 2) {
              if (lane == 0) bulk_wait_read<1>();
              __syncwarp();
            }
#pragma unroll
            for (int g = 0; g < 8; ++g)
              st_shared_v4(buf + srow0 + (((uint32_t)g ^ sw) << 4), x[4 * g], x[4 * g + 1],
                           x[4 * g + 2], x[4 * g + 3]);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&tm_o, buf, c * 32, (int)head, (int)(u.tok0 + wrow0));
              bulk_commit();
            }
          } else if (store) {
            float4 *o = (float4 *)((float *)p.out + orow + c * 32);
#pragma unroll
            for (int g = 0; g < 8; ++g)
              o[g] = make_float4(__uint_as_float(x[4 * g]), __uint_as_float(x[4 * g + 1]),
                                 __uint_as_float(x[4 * g + 2]), __uint_as_float(x[4 * g + 3]));
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t w[32];
          uint32_t xa[32], xb[32];
          tmem_ld32(tO + c * 64, xa);
          tmem_ld32(tO + c * 64 + 32, xb);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            w[t] = pack_bf16x2(__uint_as_float(xa[2 * t]) * inv, __uint_as_float(xa[2 * t + 1]) * inv);
            w[16 + t] =
                pack_bf16x2(__uint_as_float(xb[2 * t]) * inv, __uint_as_float(xb[2 * t + 1]) * inv);
          }
          if (bulk) {
            const uint32_t buf = stage[c];
#pragma unroll
            for (int g = 0; g < 8; ++g)
              st_shared_v4(buf + srow0 + (((uint32_t)g ^ sw) << 4), w[4 * g], w[4 * g + 1],
                           w[4 * g + 2], w[4 * g + 3]);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&tm_o, buf, c * 64, (int)head, (int)(u.tok0 + wrow0));
              bulk_commit();
            }
          } else if (store) {
            uint4 *o = (uint4 *)((uint16_t *)p.out + orow + c * 64);
#pragma unroll
            for (int g = 0; g < 8; ++g)
              o[g] = make_uint4(w[4 * g], w[4 * g + 1], w[4 * g + 2], w[4 * g + 3]);
          }
        }
      }
      tc_fence_before();
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
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

// 3-D map over a [rows, heads, 128] tensor; a box is box_rows rows x 1 head x 128 bytes
// of elements, in the 128-byte swizzle.
bool make_map(CUtensorMap *map, const void *base, uint32_t rows, uint32_t heads, bool f32,
              uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t esz = f32 ? 4 : 2;
  cuuint64_t dims[3] = {128, heads, rows};
  cuuint64_t strides[2] = {128 * esz, (cuuint64_t)heads * 128 * esz};
  cuuint32_t box[3] = {(cuuint32_t)(128 / esz), 1, box_rows};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                  const_cast<void *>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_attention_tc(const AttnProblem &p, const uint32_t *units, uint32_t n_units,
                                int num_sms, int *status, const uint16_t *q_norm_w, float eps,
                                float theta, cudaStream_t stream) {
  if (!n_units) return cudaSuccess;
  CUtensorMap mq, mk, mv, mo;
  const uint32_t rows = p.total;
  if (!make_map(&mq, p.q, rows, p.heads, false, 128) ||
      !make_map(&mk, p.k, rows, p.kv_heads, false, 128) ||
      !make_map(&mv, p.v, rows, p.kv_heads, false, 128) ||
      !make_map(&mo, p.out, rows, p.heads, p.out_dtype == 0, 32))
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
  prm.q_norm_w = q_norm_w;
  prm.eps = eps;
  prm.theta = theta;
  uint32_t grid = std::min<uint32_t>(n_units, (uint32_t)num_sms);
  tc::attn_tc_kernel<<<grid, tc::kThreads, tc::kSmemBytes, stream>>>(mq, mk, mv, mo, prm);
  return cudaGetLastError();
}

}  // namespace tx
