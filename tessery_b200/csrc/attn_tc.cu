// Blackwell (sm_100a) tensor-core attention for head_dim 128, bf16 q/k/v, fp32 softmax
// and accumulation: the Qwen3 causal GQA operator of qwen3.py:238-245 dispatched by
// MetalRuntime._attention (metal.py:532-569), with the semantics of kernels.metal:78-103
// (and of its tiled/tail variants :108-298).  Optionally fused in front: the q RMSNorm +
// RoPE of qwen3.py:216-237 (kernels.metal:53-74), applied to each Q tile in shared memory.
//
// Work unit: (sequence, pair of query heads sharing one kv head, 128-row query tile);
// when the query heads per kv head are odd, a unit holds one head.  The heads of a unit
// share every K/V tile (GQA head sharing).  A persistent grid of one CTA per SM; each
// CTA runs its own contiguous part of a host-built work list (units assigned longest
// first to the least-loaded CTA).
//
// Warp roles (576 threads, one CTA per SM), specialised so that each serial per-unit
// step runs beside the others instead of in front of them:
//   warps 0-3   softmax of head slot 0 (thread t = query row t), and after a unit's last
//               P.V its epilogue (O from tensor memory, scaled by the row sum the thread
//               holds, staged swizzled in a per-warp 32-row chunk, sent by TMA
//               bulk-tensor stores)
//   warps 4-7   the same for head slot 1
//   warps 8-15  the q prologue of the next unit (RMSNorm + RoPE of its Q tiles in shared
//               memory, as soon as they land; warpgroup h takes rows 64h..64h+63 of both
//               heads, two lanes per row)
//   warp 16     TMA producer: Q tiles of the unit two ahead (into the buffer whose last
//               Q.K^T has run) and K and V tiles of 128 keys through a 2-slot ring, with
//               an L2 prefetch of V_{j+1} beside the load of K_{j+1} (prefetching all of
//               the next unit's tiles competed with the loads on the critical path: 3-9 %
//               slower, measured)
//   warp 17     TMEM allocator and single-thread tcgen05.mma issuer
// Tensor memory (512 columns x 128 lanes, fp32), per head slot h at column 256h:
//   [0,128) S_h, [128,256) O_h.
// P_h (bf16) is written over the first 64 columns of S_h and read from there by P.V as
// the tensor-memory A operand, so P needs no shared memory.  Shared memory: two unit
// buffers of Q tiles (2 x 128x128 bf16 each, so the next unit's Q is loaded and
// transformed while this one runs), 2 ring slots (128x128 bf16: K or V), and one output
// staging chunk per softmax warp (32 rows x 128 bytes), all in the 128-byte-swizzled
// layout that TMA and UMMA use (a 128-byte row holds 64 bf16 or 32 fp32).
//
// Key tile j of a unit (every MMA is M=128 x N=128 x K=16, issued 8 at a time): the
// issuer runs S_h = Q_h K_j^T; the softmax warps of head h take the row maximum of S_h
// (first pass over tensor memory) and write P_h = exp2(S_h*scale*log2e - m) (second
// pass); the issuer runs O_h += P_h V_j and at once
// S_h = Q_h K_{j+1}^T.  Both heads alternate, so one head's softmax overlaps the other
// head's products.  Because S_h of tile j+1 is committed after P_h.V of tile j, a
// softmax warp that sees S_h full also knows that O_h holds every earlier tile.  Tiles
// above the causal diagonal and beyond each sequence's length are never visited; the
// diagonal and the last tile are masked per row.  In a sequence's last key tile, P.V
// runs only over the 16-key steps that hold keys before the end, and the V rows past the
// end inside the last such step are set to zero on chip.  The running maximum is updated
// lazily: O is rescaled only when a tile maximum exceeds the reference maximum by more
// than 8 (log2 units), so every probability stays below 2^8 and the normalised result
// is unchanged.
//
// Every wait is bounded (a per-launch limit, about a second by default); a wait that
// gives up records TX_ETIMEOUT | site<<8 in the context status word, raises a CTA-wide
// abort flag, and all roles drain their in-flight copies and MMAs before TMEM is freed
// and the CTA exits.  The drains themselves wait for work already issued, which completes
// by itself; they are bounded by the default limit.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"


namespace tx {
namespace tc {

constexpr int kQRows = 128;                     // query rows per tile (TMEM lanes)
constexpr int kKeys = 128;                      // keys per K/V tile
constexpr int kStages = 2;                      // K/V ring slots
constexpr uint32_t kQAtom = 128 * 128;          // 128 rows x 64 bf16
constexpr uint32_t kQBytes = 2 * kQAtom;         // one head's Q tile
constexpr uint32_t kQBufBytes = 2 * kQBytes;     // a unit's Q tiles (two head slots)
constexpr uint32_t kKVAtom = kKeys * 128;       // 128 keys x 64 bf16
constexpr uint32_t kKVBytes = 2 * kKVAtom;
constexpr uint32_t kChunkBytes = 32 * 128;      // output staging: 32 rows x 128 bytes
constexpr uint32_t kStageSlots = 1;             // staging chunks per epilogue warp
constexpr uint32_t kOffQ = 0;                   // two unit buffers of Q tiles
constexpr uint32_t kOffKV = kOffQ + 2 * kQBufBytes;
constexpr uint32_t kOffStage = kOffKV + kStages * kKVBytes;
constexpr uint32_t kOffMisc = kOffStage + 8 * kStageSlots * kChunkBytes;
constexpr uint32_t kMiscBytes = 3072;
// The whole per-CTA budget; the dynamic shared-memory window must start 1024-byte
// aligned (the swizzled tiles need it), which the kernel checks.
constexpr uint32_t kSmemBytes = kOffMisc + kMiscBytes;
constexpr int kThreads = 576;
constexpr int kEpiWarp0 = 8, kTmaWarp = 16, kMmaWarp = 17;
constexpr uint32_t kTmemCols = 512;
constexpr long long kWaitCycles = 2000000000ll;  // ~1 s at B200 clocks
constexpr float kRescaleThreshold = 8.0f;        // log2 units

// Barrier slots (uint64 each) at the start of the misc area.  "h" = head slot,
// "b" = Q buffer.
enum : uint32_t {
  kBarQFull = 0,                      // + b: the unit's Q tiles landed (TMA bytes)
  kBarQReady = kBarQFull + 2,         // + b: Q tiles transformed (256 arrivals)
  kBarQEmpty = kBarQReady + 2,        // + b: every Q.K^T reading the buffer ran (commit)
  kBarKVFull = kBarQEmpty + 2,        // + ring slot
  kBarKVEmpty = kBarKVFull + kStages,
  kBarSFull = kBarKVEmpty + kStages,  // + h: S_h of the next key tile (commit)
  kBarPFull = kBarSFull + 2,          // + h: P_h written over S_h (128 arrivals)
  kBarPVDone = kBarPFull + 2,         // + h: P_h.V ran (commit)
  kBarOFree = kBarPVDone + 2,         // + h: O_h read out (128 arrivals)
  kBarDrain = kBarOFree + 2,
  kNumBars = kBarDrain + 1
};
constexpr uint32_t kOffTmemSlot = kNumBars * 8;   // uint32 TMEM base address
constexpr uint32_t kOffAbort = kOffTmemSlot + 4;  // int abort flag
constexpr uint32_t kOffQw = 512;                  // bf16 q-norm weight [128]
constexpr uint32_t kOffInvFreq = 768;             // float inverse frequencies [64]
static_assert(kOffAbort + 4 <= kOffQw, "misc area overflow");
static_assert(kOffInvFreq + 64 * 4 <= kMiscBytes, "misc area overflow");
static_assert(kSmemBytes <= 232448, "shared memory budget");
static_assert(kOffKV % 1024 == 0 && kOffStage % 1024 == 0, "swizzled tiles need 1024 B alignment");

// Wait sites, reported in the status word for diagnosis.
enum : int {
  kSiteQEmpty = 1, kSiteKVEmpty = 2, kSiteQReady = 3, kSiteKVFull = 4, kSitePFull = 5,
  kSiteSFull = 6, kSitePVDone = 7, kSiteQFull = 8, kSiteOFree = 10
};

// ---- unit encoding --------------------------------------------------------------------
// Sort key of a unit on the host: bits 0..7 query tile, 8..13 head pair (or head),
// 14..31 sequence.
__host__ __device__ __forceinline__ uint32_t encode_unit(uint32_t seq, uint32_t idx,
                                                         uint32_t tile) {
  return (seq << 14) | (idx << 8) | tile;
}
// A unit in the work list: two words.  With the lengths known on the host ("exact"):
// x = tile | head pair << 8 | valid keys << 14, y = row of position 0 of the sequence,
// so the kernel decodes a unit without reading the lengths.  Otherwise x = tile | head
// pair << 8 and y = the sequence index, and the kernel reads the device lengths.
__host__ __device__ __forceinline__ uint2 unit_words(uint32_t tile, uint32_t idx, uint32_t n,
                                                    uint32_t y) {
  return make_uint2(tile | (idx << 8) | (n << 14), y);
}

struct Params {
  const uint2 *units;       // work units, grouped by CTA
  const uint32_t *offsets;  // CTA c runs units [offsets[c], offsets[c+1])
  uint32_t n_units;
  int exact;                // units carry their valid keys and first row
  const uint32_t *lengths;  // padded
  const int32_t *cu;        // varlen (NULL for padded)
  void *out;
  uint32_t seq;             // padded L (rows per sequence)
  uint32_t heads, group;    // query heads; query heads per kv head
  uint32_t nh;              // heads per unit: 2 (pairs) or 1
  int causal;
  float scale_log2;
  int *status;
  const uint16_t *q_norm_w;  // fused q prologue when non-NULL
  const uint16_t *k_norm_w;  // weights of the k RMSNorm applied to k (NULL: none known)
  float eps;
  long long wait_cycles;     // limit of every bounded wait, in SM clock cycles
  float inv_freq[64];        // RoPE theta^(-2c/128), c < 64
};

struct Unit {
  uint32_t tok0;   // row index of position 0 of the sequence
  uint32_t q0;     // first query position of the tile
  uint32_t rows;   // rows of this sequence present in the layout
  uint32_t n;      // valid keys
  uint32_t head0;  // first query head of the unit
  uint32_t kvh;
  uint32_t nt;     // key tiles to visit
  bool live;       // the tile holds rows to write
};

__device__ __forceinline__ Unit decode(const Params &p, uint2 w) {
  Unit u;
  const uint32_t idx = (w.x >> 8) & 63u, t = w.x & 255u;
  if (p.exact) {
    u.n = w.x >> 14;
    u.tok0 = w.y;
    u.rows = p.cu ? u.n : p.seq;
  } else if (p.cu) {
    const int32_t a = p.cu[w.y], b = p.cu[w.y + 1];
    u.tok0 = (uint32_t)a;
    u.n = b > a ? (uint32_t)(b - a) : 0u;
    u.rows = u.n;
  } else {
    u.tok0 = w.y * p.seq;
    u.n = min(p.lengths[w.y], p.seq);
    u.rows = p.seq;
  }
  u.q0 = t * kQRows;
  u.head0 = idx * p.nh;
  u.kvh = u.head0 / p.group;
  u.live = u.q0 < u.rows;
  uint32_t kend = p.causal ? min(u.q0 + kQRows, u.n) : u.n;
  u.nt = u.live ? (kend + kKeys - 1) / kKeys : 0u;
  return u;
}

// The next unit of this CTA at or after index `from` that visits key tiles (n_units when
// there is none).
__device__ __forceinline__ uint32_t next_work(const Params &p, uint32_t from) {
  const uint32_t end = p.offsets[blockIdx.x + 1];
  for (uint32_t ui = from; ui < end; ++ui)
    if (decode(p, p.units[ui]).nt) return ui;
  return p.n_units;
}

// Walks this CTA's units in order with the words of the next unit loaded one unit ahead,
// so that the load's latency hides behind the current unit's work.
struct UnitCursor {
  uint32_t ui, end;
  uint2 w;
  __device__ __forceinline__ UnitCursor(const Params &p) {
    ui = p.offsets[blockIdx.x];
    end = p.offsets[blockIdx.x + 1];
    w = ui < end ? p.units[ui] : make_uint2(0u, 0u);
  }
  __device__ __forceinline__ bool more() const { return ui < end; }
  // The current unit; starts the load of the next one and advances.
  __device__ __forceinline__ Unit take(const Params &p) {
    const uint2 cur = w;
    if (ui + 1 < end) w = p.units[ui + 1];
    ++ui;
    return decode(p, cur);
  }
};

// ---- PTX wrappers (tcgen05.cuh) and attention-specific descriptors -----------------
using namespace ptx;

// Bounded wait for the phase with parity `parity` of barrier `bar`; gives up after
// `limit` SM cycles.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                        int *status, int site, long long limit) {
  if (mbar_test(bar, parity)) return true;
  long long t0 = clock64();
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

// Bounded wait without a status report (drains after an abort).
__device__ __forceinline__ void drain_phase(uint32_t bar, uint32_t parity) {
  long long t0 = clock64();
  while (!mbar_test(bar, parity) && clock64() - t0 < kWaitCycles) {
  }
}

// K-major operand: rows (M or N) of 64 bf16 of K per 128-byte row, 8-row groups 1024 B
// apart, one atom per 64 columns of K (`atom` bytes apart).  Step `ks` (16 elements of
// K): atom ks/4, 32 bytes per step inside the swizzled row.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile, int ks, uint32_t atom) {
  return sw128_desc(tile + (ks >> 2) * atom + (ks & 3) * 32, 16, 1024);
}
// MN-major operand (V as B of P.V: N = head_dim contiguous, K = keys).  The two 64-wide
// N halves are the two atoms (leading byte offset = atom size); 8-key groups are 1024 B
// apart (stride byte offset); step `ks` covers keys 16ks..16ks+15.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile, int ks) {
  return sw128_desc(tile + ks * 2048, kKVAtom, 1024);
}

// Instruction descriptors, kind::f16 with A=B=bf16, D=f32: bit 4 D format, bits 7 and 10
// A/B formats, bit 16 B MN-major, N>>3 at bit 17, M>>4 at bit 24.
constexpr uint32_t kIdescBase = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 4) << 24);
constexpr uint32_t kIdescQK = kIdescBase | ((uint32_t)(kKeys >> 3) << 17);    // N = kKeys
constexpr uint32_t kIdescPV = kIdescBase | (1u << 16) | ((128u >> 3) << 17);  // N = 128

// In-place q RMSNorm + RoPE of one half of row `row` in each of the `nh` head tiles of a
// unit's Q buffer (`qbuf`: per head 128 rows x 128 bf16, two 64-column atoms, 128-byte
// swizzle).  Half `half` covers rotation columns c in [32 half, 32 half + 32) and their
// partners c + 64; lanes 2i and 2i+1 hold the two halves of one row and add their sums
// of squares by shuffle, so the calling warp must run this with all lanes (`live` false
// for a row that belongs to no output: the lane only takes part in the shuffle).
// Per element pair this is kernels.metal:53-74 -- a = x_c * inv * w_c,
// b = x_{c+64} * inv * w_{c+64}, then (a cos - b sin, a sin + b cos) with the angle
// pos * inv_freq[c] -- regrouped as inv * (x_c (w_c cos) - x_{c+64} (w_{c+64} sin)) and
// inv * (x_c (w_c sin) + x_{c+64} (w_{c+64} cos)), so that the four weighted sines and
// cosines of a column are computed once for both heads.  `w_s` is the shared-memory
// address of the bf16 weights.
__device__ __forceinline__ void q_transform_half_row(uint32_t qbuf, uint32_t nh, uint32_t row,
                                                     uint32_t half, uint32_t pos, bool live,
                                                     uint32_t w_s, const float *inv_freq,
                                                     float eps) {
  const uint32_t sw = row & 7;
  uint64_t inv2[2];
#pragma unroll
  for (uint32_t hd = 0; hd < 2; ++hd) {
    uint64_t acc[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
    if (live && hd < nh) {
      const uint32_t ra = qbuf + hd * kQBytes + row * 128;
#pragma unroll
      for (uint32_t c = 0; c < 4; ++c) {
        const uint32_t off = ((4 * half + c) ^ sw) << 4;
        const uint4 lo = ld_shared_v4(ra + off), hi = ld_shared_v4(ra + kQAtom + off);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint64_t xl = bf16x2_f2(u4_at(lo, e)), xh = bf16x2_f2(u4_at(hi, e));
          acc[0] = fma2(xl, xl, acc[0]);
          acc[1] = fma2(xh, xh, acc[1]);
        }
      }
    }
    const float2 a0 = f2_unpack(acc[0]), a1 = f2_unpack(acc[1]);
    float sum = (a0.x + a0.y) + (a1.x + a1.y);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    const float inv = 1.0f / sqrtf(sum / 128.0f + eps);
    inv2[hd] = f2(inv, inv);
  }
  if (!live) return;
  const float fpos = (float)pos;
#pragma unroll 1
  for (uint32_t c = 0; c < 4; ++c) {  // 16-byte chunk g: columns 8g..8g+7 and 64+8g..
    const uint32_t g = 4 * half + c, off = (g ^ sw) << 4;
    float co[8], si[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) rope_sincos(fpos * inv_freq[8 * g + e], &si[e], &co[e]);
    const uint4 wa = ld_shared_v4(w_s + 16 * g), wb = ld_shared_v4(w_s + 128 + 16 * g);
    // Per column pair e (columns 8g+2e, 8g+2e+1): w_c cos, -w_p sin, w_c sin, w_p cos.
    uint64_t fa[4], fb[4], fc[4], fd[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint64_t wc = bf16x2_f2(u4_at(wa, e)), wp = bf16x2_f2(u4_at(wb, e));
      const uint64_t cs = f2(co[2 * e], co[2 * e + 1]), sn = f2(si[2 * e], si[2 * e + 1]);
      fa[e] = mul2(wc, cs);
      fb[e] = mul2(wp, f2(-si[2 * e], -si[2 * e + 1]));
      fc[e] = mul2(wc, sn);
      fd[e] = mul2(wp, cs);
    }
#pragma unroll
    for (uint32_t hd = 0; hd < 2; ++hd) {
      if (hd >= nh) break;
      const uint32_t ra = qbuf + hd * kQBytes + row * 128;
      const uint4 lo = ld_shared_v4(ra + off), hi = ld_shared_v4(ra + kQAtom + off);
      uint32_t out_lo[4], out_hi[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint64_t xc = bf16x2_f2(u4_at(lo, e)), xp = bf16x2_f2(u4_at(hi, e));
        const float2 ra2 = f2_unpack(mul2(fma2(xp, fb[e], mul2(xc, fa[e])), inv2[hd]));
        const float2 rb2 = f2_unpack(mul2(fma2(xp, fd[e], mul2(xc, fc[e])), inv2[hd]));
        out_lo[e] = pack_bf16x2(ra2.x, ra2.y);
        out_hi[e] = pack_bf16x2(rb2.x, rb2.y);
      }
      st_shared_v4(ra + off, out_lo[0], out_lo[1], out_lo[2], out_lo[3]);
      st_shared_v4(ra + kQAtom + off, out_hi[0], out_hi[1], out_hi[2], out_hi[3]);
    }
  }
}

// exp2(x*sl - m) of one 32-key chunk of a row (0 for keys at or past `valid`), as 16 bf16
// pairs; returns the chunk's sum.  One code path for full and masked chunks: the kernel's
// warp roles share each sub-partition's instruction cache, so smaller code runs faster
// than a separate unmasked copy.
__device__ __forceinline__ float exp_chunk(const uint32_t (&x)[32], int c, int valid, float sl,
                                           float m, uint32_t (&packed)[16]) {
  const uint64_t sl2 = f2(sl, sl), nm2 = f2(-m, -m);
  uint64_t sum[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    const int k0 = c * 32 + 2 * t;
    const float2 z = f2_unpack(fma2(f2_bits(x[2 * t], x[2 * t + 1]), sl2, nm2));
    float p0 = ex2(z.x), p1 = ex2(z.y);
    p0 = k0 < valid ? p0 : 0.f;
    p1 = k0 + 1 < valid ? p1 : 0.f;
    sum[t & 1] = add2(sum[t & 1], f2(p0, p1));
    packed[t] = pack_bf16x2(p0, p1);
  }
  const float2 s0 = f2_unpack(sum[0]), s1 = f2_unpack(sum[1]);
  return (s0.x + s1.x) + (s0.y + s1.y);
}

// max(a, b, c) in one instruction.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// ---- the kernel -----------------------------------------------------------------------
// 96 registers per thread: 18 warps put 5 warps on some SM sub-partition, whose 16K
// registers then allow 102 each.
// kOutBf16: bf16 output (else fp32), one instantiation each so that a launch carries
// only its own epilogue.
template <bool kOutBf16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                   const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v,
                   const __grid_constant__ CUtensorMap tm_o, const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_addr(smem);
  if (sbase & 1023u) {  // the swizzled tiles need a 1024-byte aligned window
    if (threadIdx.x == 0) report_status(p.status, kStatusBadArg);
    return;
  }
  const uint32_t bars = sbase + kOffMisc;
  uint8_t *misc = smem + kOffMisc;
  uint32_t *tmem_slot = (uint32_t *)(misc + kOffTmemSlot);
  volatile int *abort_flag = (volatile int *)(misc + kOffAbort);
  uint16_t *qw_s = (uint16_t *)(misc + kOffQw);
  float *invf_s = (float *)(misc + kOffInvFreq);
  auto bar = [&](uint32_t i) { return bars + 8u * i; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t nh = p.nh;

  if (threadIdx.x == 0) {
    for (int h = 0; h < 2; ++h) {
      mbar_init(bar(kBarQFull + h), 1);
      mbar_init(bar(kBarQReady + h), 256);  // every thread of both aux warpgroups
      mbar_init(bar(kBarQEmpty + h), 1);
      mbar_init(bar(kBarSFull + h), 1);
      mbar_init(bar(kBarPFull + h), 128);
      mbar_init(bar(kBarPVDone + h), 1);
      mbar_init(bar(kBarOFree + h), 128);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kBarKVFull + s), 1);
      mbar_init(bar(kBarKVEmpty + s), 1);
    }
    mbar_init(bar(kBarDrain), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (p.q_norm_w) {
    for (int i = threadIdx.x; i < 128; i += kThreads) qw_s[i] = p.q_norm_w[i];
    for (int i = threadIdx.x; i < 64; i += kThreads) invf_s[i] = p.inv_freq[i];
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(kTmemCols)
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
    // Q tiles of the first work unit, its first K tile, then the second unit's Q tiles
    // (so that the first unit's tiles, which everything waits for at the start, do not
    // share the memory system with them); then per work unit k: its K/V tiles in the
    // order the issuer consumes them (K_0, then V_j, K_{j+1} for j = 0..), and the Q tiles
    // of work unit k+2 into buffer k%2 once the last Q.K^T of unit k has run.
    if (lane == 0) {
      uint32_t loads = 0;
      // Per ring slot: bit s = parity of its fills so far, bit 8+s = slot ever filled;
      // per Q buffer b: bit 16+b = parity of its fills, bit 18+b = ever filled (for the
      // abort drain).
      uint32_t armed = 0;
      bool ok = true;
      auto load_kv = [&](const CUtensorMap *map, const Unit &u, uint32_t j) {
        const uint32_t slot = loads & (kStages - 1), round = loads / kStages;
        if (round > 0 && !(ok = wait_phase(bar(kBarKVEmpty + slot), (round - 1) & 1,
                                           abort_flag, p.status, kSiteKVEmpty, p.wait_cycles)))
          return;
        const uint32_t dst = sbase + kOffKV + slot * kKVBytes;
        mbar_expect_tx(bar(kBarKVFull + slot), kKVBytes);
        for (int a = 0; a < 2; ++a)
          tma_load_3d(dst + a * kKVAtom, map, bar(kBarKVFull + slot), a * 64, (int)u.kvh,
                      (int)(u.tok0 + j * kKeys));
        armed ^= 1u << slot;
        armed |= 1u << (8 + slot);
        ++loads;
      };
      auto load_q = [&](uint32_t ui, uint32_t b) {
        const Unit v = decode(p, p.units[ui]);
        mbar_expect_tx(bar(kBarQFull + b), nh * kQBytes);
        for (uint32_t h = 0; h < nh; ++h)
          for (int a = 0; a < 2; ++a)
            tma_load_3d(sbase + kOffQ + b * kQBufBytes + h * kQBytes + a * kQAtom, &tm_q,
                        bar(kBarQFull + b), a * 64, (int)(v.head0 + h), (int)(v.tok0 + v.q0));
        armed ^= 1u << (16 + b);
        armed |= 1u << (18 + b);
      };
      uint32_t cur = next_work(p, p.offsets[blockIdx.x]);
      uint32_t nxt = cur < p.n_units ? next_work(p, cur + 1) : p.n_units;
      if (cur < p.n_units) load_q(cur, 0);
      // K may be written by the kernel launched just before this one (the k prologue):
      // with a programmatic dependent launch this grid starts while that one drains, so
      // wait for it before the first K load.  Q, V, the lengths and the work list were in
      // place before the prologue started (the launch is programmatic only then).
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (uint32_t k = 0; ok && cur < p.n_units; ++k) {
        const Unit u = decode(p, p.units[cur]);
        const uint32_t ahead = nxt < p.n_units ? next_work(p, nxt + 1) : p.n_units;
        load_kv(&tm_k, u, 0);
        if (k == 0 && nxt < p.n_units) load_q(nxt, 1);
        for (uint32_t j = 0; ok && j < u.nt; ++j) {
          load_kv(&tm_v, u, j);
          if (ok && j + 1 < u.nt) {
            load_kv(&tm_k, u, j + 1);
            // V_{j+1} can only be loaded once P.V of tile j has freed its ring slot: bring
            // it into L2 now, so that the load then hits (measured 2-3 % faster; a
            // prefetch of all of the next unit's tiles was slower).
            for (int a = 0; a < 2; ++a)
              tma_prefetch_3d(&tm_v, a * 64, (int)u.kvh, (int)(u.tok0 + (j + 1) * kKeys));
          }
        }
        if (ok && ahead < p.n_units) {
          const uint32_t b = k & 1;
          if ((ok = wait_phase(bar(kBarQEmpty + b), (k >> 1) & 1, abort_flag, p.status,
                               kSiteQEmpty, p.wait_cycles)))
            load_q(ahead, b);
        }
        cur = nxt;
        nxt = ahead;
      }
      if (!ok) {
        // Every armed fill completes by itself: wait for the latest of each slot and Q
        // buffer so that no copy lands in shared memory after the CTA exits.
        for (int s = 0; s < kStages; ++s)
          if (bit(armed, 8 + s)) drain_phase(bar(kBarKVFull + s), bit(armed, s) ^ 1u);
        for (int b = 0; b < 2; ++b)
          if (bit(armed, 18 + b)) drain_phase(bar(kBarQFull + b), bit(armed, 16 + b) ^ 1u);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    // Per work unit: S_h = Q_h K_0^T for both heads; then per key tile j: for each head,
    // O_h (+)= P_h V_j and at once S_h = Q_h K_{j+1}^T into the columns P_h.V has just
    // read (tcgen05.mma of one thread run in order), so one head's softmax overlaps the
    // other head's products.  The whole warp follows the schedule (its waits are
    // warp-wide); lane 0 issues the MMAs and commits, and all lanes clear the V rows at
    // or past a sequence's end in the unit's last key tile.
    const bool leader = lane == 0;
    uint32_t loads = 0, units_done = 0;
    uint32_t pbits = 0, obits = 0;  // parities: P-full per head, O-free per head
    bool ok = true, issued = false;
    uint32_t qbuf = 0;  // Q buffer of the current unit
    auto wait_all = [&](uint32_t b, uint32_t parity, int site) -> bool {
      return __all_sync(0xffffffffu,
                        wait_phase(b, parity, abort_flag, p.status, site, p.wait_cycles));
    };
    auto commit = [&](uint32_t b) {
      if (leader) umma_commit(b);
    };
    // The next ring slot (a K or V tile, in load order): wait for it.
    auto take = [&](uint32_t *slot) -> bool {
      *slot = loads & (kStages - 1);
      if (!(ok = wait_all(bar(kBarKVFull + *slot), (loads / kStages) & 1, kSiteKVFull)))
        return false;
      ++loads;
      tc_fence_after();
      return true;
    };
    // S_h = Q_h K^T (M=128, N=128 keys, K=128) from the K tile in ring slot `slot`.
    // Descriptors of step 0; step ks adds its byte offset / 16 to the start-address
    // field (addresses stay below 256 KB, so the field never carries).
    auto qk_head = [&](uint32_t h, uint32_t slot) {
      if (leader) {
        const uint64_t kd = kmajor_desc(sbase + kOffKV + slot * kKVBytes, 0, kKVAtom);
        const uint64_t qd =
            kmajor_desc(sbase + kOffQ + qbuf * kQBufBytes + h * kQBytes, 0, kQAtom);
        const uint32_t d = tmem + h * 256;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma(d, qd + (uint64_t)((ks >> 2) * (kQAtom >> 4) + (ks & 3) * 2),
               kd + (uint64_t)((ks >> 2) * (kKVAtom >> 4) + (ks & 3) * 2), kIdescQK, ks > 0);
        umma_commit(bar(kBarSFull + h));
      }
      issued = true;
    };
    // O_h (+)= P_h V with P_h (bf16, 128 keys) in the first 64 columns of S_h, over the
    // first `steps` 16-key steps of the tile (the steps past a sequence's end hold only
    // zero probabilities and are not issued).
    auto pv_head = [&](uint32_t h, uint32_t slot, uint32_t acc, uint32_t steps) {
      if (leader) {
        const uint64_t vd = mnmajor_desc(sbase + kOffKV + slot * kKVBytes, 0);
        const uint32_t pt = tmem + h * 256, d = tmem + h * 256 + 128;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          if ((uint32_t)ks < steps)
            umma_ts(d, pt + ks * 8, vd + (uint64_t)(ks * (2048 >> 4)), kIdescPV,
                    (acc || ks > 0) ? 1u : 0u);
        umma_commit(bar(kBarPVDone + h));
      }
    };
    // Rows [first, last) of the V tile in ring slot `slot` set to zero (at most 15 rows:
    // the rest of the last 16-key step that P.V reads): those keys lie at or past the
    // sequence's end (padding, or the next packed sequence), their probabilities are zero,
    // and zero times a non-finite value would not be.  Whole 128-byte rows of both
    // 64-column atoms, so the swizzle does not matter.
    auto clear_v_rows = [&](uint32_t slot, uint32_t first, uint32_t last) {
      const uint32_t base = sbase + kOffKV + slot * kKVBytes;
      for (uint32_t i = first * 16 + lane; i < last * 16; i += 32) {
        const uint32_t row = i >> 4, atom = (i >> 3) & 1u, c = i & 7u;
        st_shared_v4(base + atom * kKVAtom + row * 128 + c * 16, 0u, 0u, 0u, 0u);
      }
      fence_proxy_async();  // generic-proxy writes seen by the tensor core's reads
      __syncwarp();
    };
    for (UnitCursor uc(p); ok && uc.more();) {
      const Unit u = uc.take(p);
      if (!u.nt) continue;
      // Work unit k uses Q buffer k % 2 (fill k / 2 of that buffer).
      qbuf = units_done & 1;
      if (!(ok = wait_all(bar(kBarQReady + qbuf), (units_done >> 1) & 1, kSiteQReady))) break;
      ++units_done;
      tc_fence_after();
      uint32_t slotK;
      if (!take(&slotK)) break;
      for (uint32_t h = 0; h < nh; ++h) qk_head(h, slotK);
      commit(bar(kBarKVEmpty + slotK));
      if (u.nt == 1) commit(bar(kBarQEmpty + qbuf));  // the unit's last Q.K^T
      for (uint32_t j = 0; ok && j < u.nt; ++j) {
        uint32_t slotV;
        if (!take(&slotV)) break;
        // Keys of this tile before the sequence's end (a visited tile holds at least one),
        // and the 16-key steps of P.V that cover them.
        const uint32_t vkeys = min(u.n - j * kKeys, (uint32_t)kKeys);
        const uint32_t vsteps = (vkeys + 15) / 16;
        if (vkeys < vsteps * 16) clear_v_rows(slotV, vkeys, vsteps * 16);
        const bool more = j + 1 < u.nt;
        for (uint32_t h = 0; h < nh && ok; ++h) {
          if (!(ok = wait_all(bar(kBarPFull + h), bit(pbits, h), kSitePFull))) break;
          pbits ^= 1u << h;
          if (j == 0 && units_done > 1) {
            // O_h still holds the previous unit until the epilogue has read it.
            if (!(ok = wait_all(bar(kBarOFree + h), bit(obits, h), kSiteOFree))) break;
            obits ^= 1u << h;
          }
          tc_fence_after();
          pv_head(h, slotV, j > 0, vsteps);
          if (more) {
            if (h == 0 && !take(&slotK)) break;
            qk_head(h, slotK);
          }
        }
        if (!ok) break;
        commit(bar(kBarKVEmpty + slotV));
        if (more) {
          commit(bar(kBarKVEmpty + slotK));
          if (j + 2 == u.nt) commit(bar(kBarQEmpty + qbuf));  // Q.K^T of the last tile
        }
      }
    }
    if (issued && leader) {
      // Wait until every MMA this thread issued has completed (normal exit and abort).
      umma_commit(bar(kBarDrain));
      drain_phase(bar(kBarDrain), 0);
    }
    __syncwarp();
  } else if (warp < kEpiWarp0) {
    // ---------------- softmax (thread = query row of head slot h) ----------------------
    const uint32_t h = (uint32_t)warp >> 2;
    const uint32_t wq = (uint32_t)warp & 3;
    const uint32_t r = wq * 32 + lane;  // tile row == TMEM lane
    const uint32_t lane_base = (wq * 32u) << 16;
    const uint32_t tS = tmem + lane_base + h * 256;
    const uint32_t tO = tS + 128;
    uint32_t tiles = 0;   // key tiles processed
    uint32_t chunks = 0;  // staging chunks this warp has sent
    bool ok = true;
    const uint32_t srow = (uint32_t)lane * 128, sw = (uint32_t)lane & 7;
    const uint32_t stage0 = sbase + kOffStage + (uint32_t)warp * kStageSlots * kChunkBytes;
    // The staging slot for this warp's next chunk, once the store that last read it is done.
    auto take_slot = [&]() -> uint32_t {
      if (lane == 0) bulk_wait_read<kStageSlots - 1>();
      __syncwarp();
      return stage0 + (chunks++ % kStageSlots) * kChunkBytes;
    };
    // Sends this warp's staged 32 rows (chunk at `slot`) to columns [x, ..) of `head`.
    auto send = [&](uint32_t slot, int x, uint32_t head, uint32_t row0) {
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(&tm_o, slot, x, (int)head, (int)row0);
        bulk_commit();
      }
    };
    // Epilogue of unit v for head slot h, once its last P.V ran: O read out of tensor
    // memory 32 columns at a time (after the last read O is released to the next unit),
    // normalised by the row sum l, stored.  Warps whose 32 rows all lie inside the
    // sequence stage each 32-row chunk in shared memory and send it with a TMA bulk-tensor
    // store; a warp at a ragged end stores row by row.
    auto epilogue = [&](const Unit &v, float l) {
      const uint32_t qpos = v.q0 + r;
      const bool store = qpos < v.rows;
      const uint32_t wrow0 = v.q0 + wq * 32;
      const bool bulk = wrow0 + 32 <= v.rows;
      const float inv = 1.0f / l;
      const uint32_t head = v.head0 + h;
      const size_t orow = ((size_t)(v.tok0 + qpos) * p.heads + head) * 128;
      if (!kOutBf16) {
        // Chunk c + 1 is read out of tensor memory and scaled while the store of chunk c
        // still reads the staging slot.
        uint32_t x[32];
        tmem_ld32(tO, x);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) x[t] = __float_as_uint(__uint_as_float(x[t]) * inv);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {  // 32 fp32 columns = one 128-byte staging row
          if (bulk) {
            const uint32_t slot = take_slot();
#pragma unroll
            for (int g = 0; g < 8; ++g)
              st_shared_v4(slot + srow + (((uint32_t)g ^ sw) << 4), x[4 * g], x[4 * g + 1],
                           x[4 * g + 2], x[4 * g + 3]);
            send(slot, c * 32, head, v.tok0 + wrow0);
          } else if (store) {
            float4 *o = (float4 *)((float *)p.out + orow + c * 32);
#pragma unroll
            for (int g = 0; g < 8; ++g)
              o[g] = make_float4(__uint_as_float(x[4 * g]), __uint_as_float(x[4 * g + 1]),
                                 __uint_as_float(x[4 * g + 2]), __uint_as_float(x[4 * g + 3]));
          }
          if (c < 3) {
            tmem_ld32(tO + (c + 1) * 32, x);
            tmem_ld_wait();
            if (c == 2) {  // O read out: released to the next unit's P.V
              tc_fence_before();
              mbar_arrive(bar(kBarOFree + h));
            }
#pragma unroll
            for (int t = 0; t < 32; ++t) x[t] = __float_as_uint(__uint_as_float(x[t]) * inv);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {  // 64 bf16 columns = one 128-byte staging row
          const uint32_t slot = bulk ? take_slot() : 0u;
#pragma unroll 1
          for (int half = 0; half < 2; ++half) {  // 32 columns = 4 16-byte units
            uint32_t x[32], w[16];
            tmem_ld32(tO + c * 64 + half * 32, x);
            tmem_ld_wait();
            if (c == 1 && half == 1) {
              tc_fence_before();
              mbar_arrive(bar(kBarOFree + h));
            }
#pragma unroll
            for (int t = 0; t < 16; ++t)
              w[t] = pack_bf16x2(__uint_as_float(x[2 * t]) * inv,
                                 __uint_as_float(x[2 * t + 1]) * inv);
            if (bulk) {
#pragma unroll
              for (int g = 0; g < 4; ++g)
                st_shared_v4(slot + srow + (((uint32_t)(4 * half + g) ^ sw) << 4), w[4 * g],
                             w[4 * g + 1], w[4 * g + 2], w[4 * g + 3]);
            } else if (store) {
              uint4 *o = (uint4 *)((uint16_t *)p.out + orow + c * 64 + half * 32);
#pragma unroll
              for (int g = 0; g < 4; ++g)
                o[g] = make_uint4(w[4 * g], w[4 * g + 1], w[4 * g + 2], w[4 * g + 3]);
            }
          }
          if (bulk) send(slot, c * 64, head, v.tok0 + wrow0);
        }
      }
    };
    // With the weights of both RMSNorms known, every score is bounded: an RMSNorm output
    // over 128 columns has norm <= max|w| sqrt(128) (the rotation keeps it), so
    // |q.k| scale log2(e) <= 128 max|w_q| max|w_k| scale log2(e), with 2^-6 of slack for
    // the bf16 roundings.  Up to 64, exp2 of a score with the fixed reference 0 lies in
    // [2^-64, 2^64]: one pass over each tile, no row maximum, no rescaling.
    bool single = false;
    if (p.q_norm_w && p.k_norm_w) {
      float wq = 0.f, wk = 0.f;
      for (int i = lane; i < 128; i += 32) {
        wq = fmaxf(wq, fabsf(__uint_as_float((uint32_t)qw_s[i] << 16)));
        wk = fmaxf(wk, fabsf(__uint_as_float((uint32_t)p.k_norm_w[i] << 16)));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        wq = fmaxf(wq, __shfl_xor_sync(0xffffffffu, wq, o));
        wk = fmaxf(wk, __shfl_xor_sync(0xffffffffu, wk, o));
      }
      single = 128.0f * wq * wk * p.scale_log2 * 1.0157f <= 64.0f;
    }
    for (UnitCursor uc(p); ok && h < nh && uc.more();) {
      const Unit u = uc.take(p);
      if (!u.nt) continue;
      const uint32_t qpos = u.q0 + r;
      const uint32_t end = p.causal ? min(qpos + 1, u.n) : u.n;
      // A warp whose 32 rows all lie past the end of a packed sequence produces no output:
      // it leaves S in place of P (those rows of O are never stored) and only keeps the
      // barriers in step.
      const bool warp_live = __any_sync(0xffffffffu, qpos < u.rows);
      float m_ref = -INFINITY, l = 0.f;
      for (uint32_t j = 0; j < u.nt; ++j, ++tiles) {
        ok = __all_sync(0xffffffffu, wait_phase(bar(kBarSFull + h), tiles & 1, abort_flag,
                                                p.status, kSiteSFull, p.wait_cycles));
        if (!ok) break;
        tc_fence_after();
        if (!warp_live) {
          tc_fence_before();
          mbar_arrive(bar(kBarPFull + h));
          continue;
        }
        const int valid = (int)min(max((int)end - (int)(j * kKeys), 0), kKeys);
        if (single) {
          m_ref = 0.f;
        } else {
          // Pass 1: the tile's row maximum (64 columns in registers at a time).
          float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            // Keys masked for every row of the warp (causal diagonal, ragged end) are skipped.
            if (__all_sync(0xffffffffu, half * 64 >= valid)) break;
            uint32_t xa[32], xb[32];
            tmem_ld32(tS + half * 64, xa);
            tmem_ld32(tS + half * 64 + 32, xb);
            tmem_ld_wait();
            const float ninf = -INFINITY;
#pragma unroll
            for (int t = 0; t < 32; t += 2) {  // keys at or past `valid` do not count
              const int ka = half * 64 + t, kb = ka + 32;
              mq[t & 2 ? 1 : 0] = fmax3(mq[t & 2 ? 1 : 0],
                                        ka < valid ? __uint_as_float(xa[t]) : ninf,
                                        ka + 1 < valid ? __uint_as_float(xa[t + 1]) : ninf);
              mq[t & 2 ? 3 : 2] = fmax3(mq[t & 2 ? 3 : 2],
                                        kb < valid ? __uint_as_float(xb[t]) : ninf,
                                        kb + 1 < valid ? __uint_as_float(xb[t + 1]) : ninf);
            }
          }
          const float mt = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * p.scale_log2;
          if (j > 0) {
            // Rescale decision is per row; TMEM access is warp-wide (.sync.aligned), so the
            // warp rescales when any of its rows needs it (others scale by 1).  S of this
            // tile was committed after P.V of the previous one, so O_h is complete.
            float corr = 1.0f;
            const bool need = mt > m_ref + kRescaleThreshold;
            if (need) {
              corr = ex2(m_ref - mt);
              l *= corr;
              m_ref = mt;
            }
            if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
              for (int c = 0; c < 8; ++c) {  // 16 columns at a time
                uint32_t o[16];
                tmem_ld16(tO + c * 16, o);
                tmem_ld_wait();
#pragma unroll
                for (int t = 0; t < 16; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * corr);
                tmem_st16(tO + c * 16, o);
              }
              tmem_st_wait();
            }
          } else {
            m_ref = mt;
          }
        }
        // Pass 2: P = exp2(S*scale*log2e - m) as bf16 pairs over the first 64 columns
        // (keys 32c..32c+31 in columns 16c..16c+15; each chunk is read before the chunk
        // it overlaps is written).
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t x[32], packed[16];
          if (__all_sync(0xffffffffu, c * 32 >= valid)) {  // masked for every row of the warp
#pragma unroll
            for (int t = 0; t < 16; ++t) packed[t] = 0u;
            tmem_st16(tS + c * 16, packed);
            continue;
          }
          tmem_ld32(tS + c * 32, x);
          tmem_ld_wait();
          l += exp_chunk(x, c, valid, p.scale_log2, m_ref, packed);
          tmem_st16(tS + c * 16, packed);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(bar(kBarPFull + h));
      }
      if (!ok) break;
      // The unit's last P.V ran: O_h out of tensor memory, normalised, stored.
      ok = __all_sync(0xffffffffu, wait_phase(bar(kBarPVDone + h), (tiles - 1) & 1, abort_flag,
                                              p.status, kSitePVDone, p.wait_cycles));
      if (!ok) break;
      tc_fence_after();
      epilogue(u, l);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  } else {
    // ---------------- q prologue ---------------------------------------------------------
    // Warpgroup h transforms rows [64h, 64h + 64) of every head tile of the next unit (two
    // lanes per row), as soon as its tiles land; the warpgroup of head slot h also writes
    // the NaN rows of units without valid keys.
    const uint32_t h = (uint32_t)(warp - kEpiWarp0) >> 2;
    const uint32_t wq = (uint32_t)warp & 3;
    const uint32_t r = wq * 32 + lane;
    const uint32_t xrow = 64 * h + (r >> 1), xhalf = r & 1;  // this thread's transform share
    bool ok = true;
    // Wait for fill `phase` of buffer b, apply the q prologue to this thread's share of
    // the unit's tiles, hand them to the issuer (which waits for all 256 threads).
    auto prepare = [&](uint32_t ui, uint32_t b, uint32_t phase) {
      ok = __all_sync(0xffffffffu, wait_phase(bar(kBarQFull + b), phase & 1, abort_flag,
                                              p.status, kSiteQFull, p.wait_cycles));
      if (!ok) return;
      if (p.q_norm_w) {
        // Rows past the end of a packed sequence belong to no output: left as loaded.
        const Unit v = decode(p, p.units[ui]);
        q_transform_half_row(sbase + kOffQ + b * kQBufBytes, nh, xrow, xhalf, v.q0 + xrow,
                             v.q0 + xrow < v.rows, smem_addr(qw_s), invf_s, p.eps);
        fence_proxy_async();
      }
      mbar_arrive(bar(kBarQReady + b));
    };
    // The q prologue of work unit 0, then per work unit k the q prologue of work unit k+1
    // (whose tiles the producer loads once unit k-1's last Q.K^T has run).  Both
    // warpgroups transform every unit.
    const bool epi = h < nh;
    uint32_t next = next_work(p, p.offsets[blockIdx.x]);
    if (next < p.n_units) prepare(next, 0, 0);
    next = next < p.n_units ? next_work(p, next + 1) : p.n_units;
    uint32_t k = 0;  // work units done
    for (UnitCursor uc(p); ok && uc.more();) {
      const Unit u = uc.take(p);
      if (!u.live) continue;
      if (!u.nt) {
        if (!epi) continue;
        // Zero valid keys: 0/0, as the reference's running sums give.
        const uint32_t qpos = u.q0 + r;
        if (qpos < u.rows) {
          const size_t orow = ((size_t)(u.tok0 + qpos) * p.heads + u.head0 + h) * 128;
          if (kOutBf16) {
            uint16_t *o = (uint16_t *)p.out + orow;
            for (int c = 0; c < 128; ++c) o[c] = 0x7fc0u;
          } else {
            float *o = (float *)p.out + orow;
            for (int c = 0; c < 128; ++c) o[c] = __int_as_float(0x7fc00000);
          }
        }
        continue;
      }
      if (next < p.n_units) {
        prepare(next, (k + 1) & 1, (k + 1) >> 1);
        if (!ok) break;
        next = next_work(p, next + 1);
      }
      ++k;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace tc

// ---- host side --------------------------------------------------------------------------

bool tc_attention_supported(const AttnProblem &p) {
  if (p.dim != 128 || p.in_dtype != 1) return false;
  if (!p.kv_heads || p.heads % p.kv_heads) return false;
  if (p.heads > 64) return false;                   // head (pair) index has 6 bits
  if ((uint64_t)p.seq > 255u * 128u) return false;  // tile index has 8 bits
  if (p.batch >= (1u << 18)) return false;
  if ((uintptr_t)p.q % 16 || (uintptr_t)p.k % 16 || (uintptr_t)p.v % 16 || (uintptr_t)p.out % 16)
    return false;
  return true;
}

namespace {
// Query heads per unit: pairs when the heads per kv head are even (both heads of a
// pair read the same K/V), else one.
uint32_t heads_per_unit(const AttnProblem &p) {
  return (p.heads / p.kv_heads) % 2 == 0 ? 2u : 1u;
}
}  // namespace

uint32_t tc_max_units(const AttnProblem &p) {
  uint32_t tiles = (p.seq + tc::kQRows - 1) / tc::kQRows;
  return p.batch * (p.heads / heads_per_unit(p)) * tiles;
}

uint32_t tc_grid(uint32_t n_units, int num_sms) {
  return std::min<uint32_t>(n_units, (uint32_t)std::max(num_sms, 1));
}

uint32_t tc_work_words(const AttnProblem &p, int num_sms) {
  // Two words per unit, then the offsets; rounded to 16 bytes so that consecutive lists
  // (one per chunk of a host-buffer call) keep their units 8-byte aligned.
  const uint32_t w = 2 * tc_max_units(p) + (uint32_t)std::max(num_sms, 1) + 1;
  return (w + 3) & ~3u;
}

namespace {

// Key tiles a unit (sequence s, query tile t) visits, 0..511.  Without host lengths the
// cost is an estimate from the query-tile index (later tiles of a causal sequence visit
// more key tiles).
uint32_t unit_tiles(const AttnProblem &p, const uint32_t *lengths_host, const int32_t *cu_host,
                    uint32_t s, uint32_t t, uint32_t *rows_out) {
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
  *rows_out = rows;
  const uint32_t q0 = t * tc::kQRows;
  uint32_t kend;
  if (known) kend = p.causal ? std::min(q0 + (uint32_t)tc::kQRows, n) : n;
  else kend = p.causal ? std::min(q0 + (uint32_t)tc::kQRows, p.seq) : p.seq;
  return std::min((kend + tc::kKeys - 1) / tc::kKeys, 511u);
}

// Relative cost of a unit for the load balance.  Traced on B200 at the padded Qwen
// benchmark shape, a unit's time on the softmax warps is ~8k / 16k / 27k / 38k cycles for
// 1 / 2 / 3 / 4 key tiles; costs closer to that (tiles, 5 tiles - 1) and with a larger
// fixed part (tiles + 2, tiles + 3, 2 tiles + 3) balanced no better than this one.
uint32_t unit_cost(uint32_t tiles) { return 2 * tiles + 1; }

// Min-heap of (load << 16 | cta) keys over the CTAs (grid <= 65535).
struct LoadHeap {
  uint64_t *h;
  uint32_t n;
  void push_all(uint32_t grid) {
    n = grid;
    for (uint32_t c = 0; c < grid; ++c) h[c] = c;  // load 0, ordered by CTA
  }
  // Adds `cost` to the least-loaded CTA and returns it.
  uint32_t take(uint32_t cost) {
    const uint32_t cta = (uint32_t)(h[0] & 0xffffu);
    h[0] += (uint64_t)cost << 16;
    for (uint32_t i = 0;;) {  // sift down
      uint32_t l = 2 * i + 1, r = l + 1, m = i;
      if (l < n && h[l] < h[m]) m = l;
      if (r < n && h[r] < h[m]) m = r;
      if (m == i) break;
      std::swap(h[i], h[m]);
      i = m;
    }
    return cta;
  }
};

}  // namespace

// The work list, built without allocating: the units sorted by cost, longest first (a
// counting sort on the key tiles, stable, so the units of one (sequence, query tile) --
// whose heads share K/V tiles through their kv head -- stay adjacent), then assigned in
// that order to the least-loaded CTA (longest-processing-time scheduling) and written
// grouped by CTA as two words each (unit_words), followed by the grid+1 offsets of the
// groups.
uint32_t tc_build_units(const AttnProblem &p, const uint32_t *lengths_host, const int32_t *cu_host,
                        int num_sms, uint32_t *sorted, uint32_t *work) {
  constexpr uint32_t kMaxTiles = 511;
  const uint32_t tiles = (p.seq + tc::kQRows - 1) / tc::kQRows;
  const uint32_t per_tile = p.heads / heads_per_unit(p);
  uint32_t count[kMaxTiles + 1] = {};
  for (uint32_t s = 0; s < p.batch; ++s)
    for (uint32_t t = 0; t < tiles; ++t) {
      uint32_t rows;
      const uint32_t c = unit_tiles(p, lengths_host, cu_host, s, t, &rows);
      if (t * tc::kQRows >= rows) break;
      count[c] += per_tile;
    }
  uint32_t start[kMaxTiles + 1];
  uint32_t total = 0;
  for (int c = (int)kMaxTiles; c >= 0; --c) {  // highest cost first
    start[c] = total;
    total += count[c];
  }
  for (uint32_t s = 0; s < p.batch; ++s)
    for (uint32_t t = 0; t < tiles; ++t) {
      uint32_t rows;
      const uint32_t c = unit_tiles(p, lengths_host, cu_host, s, t, &rows);
      if (t * tc::kQRows >= rows) break;
      for (uint32_t i = 0; i < per_tile; ++i) sorted[start[c]++] = tc::encode_unit(s, i, t);
    }
  const uint32_t grid = tc_grid(total, num_sms);
  uint32_t *offsets = work + 2 * total;
  // The words of unit `code` (see unit_words): valid keys and first row when the lengths
  // are known here, else the sequence index for the kernel to look up.
  const bool exact = p.cu_seqlens ? cu_host != nullptr : lengths_host != nullptr;
  auto words = [&](uint32_t code) -> uint2 {
    const uint32_t s = code >> 14, idx = (code >> 8) & 63u, t = code & 255u;
    if (!exact) return tc::unit_words(t, idx, 0u, s);
    uint32_t n, tok0;
    if (p.cu_seqlens) {
      const int32_t a = cu_host[s], b = cu_host[s + 1];
      n = b > a ? (uint32_t)(b - a) : 0u;
      tok0 = (uint32_t)a;
    } else {
      n = std::min(lengths_host[s], p.seq);
      tok0 = s * p.seq;
    }
    return tc::unit_words(t, idx, n, tok0);
  };
  if (!total) {
    offsets[0] = 0;
    return 0;
  }
  // Two identical greedy passes: the first counts each CTA's units, the second places
  // them (no per-unit assignment array needed).
  uint64_t heap_mem[1024];
  uint32_t cursor[1024];
  const uint32_t g = std::min<uint32_t>(grid, 1024u);
  LoadHeap heap{heap_mem, 0};
  for (int pass = 0; pass < 2; ++pass) {
    heap.push_all(g);
    if (pass == 0)
      for (uint32_t c = 0; c < g; ++c) cursor[c] = 0;
    for (uint32_t i = 0; i < total; ++i) {
      const uint32_t code = sorted[i];
      uint32_t rows;
      const uint32_t cost =
          unit_cost(unit_tiles(p, lengths_host, cu_host, code >> 14, code & 255u, &rows));
      const uint32_t cta = heap.take(cost);
      if (pass == 0) {
        ++cursor[cta];
      } else {
        const uint2 w = words(code);
        work[2 * cursor[cta]] = w.x;
        work[2 * cursor[cta] + 1] = w.y;
        ++cursor[cta];
      }
    }
    if (pass == 0) {
      uint32_t acc = 0;
      for (uint32_t c = 0; c < g; ++c) {
        offsets[c] = acc;
        acc += cursor[c];
        cursor[c] = offsets[c];
      }
      offsets[g] = acc;
    }
  }
  return total;
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

// 3-D map over a [rows, heads, 128] tensor of bf16 (or fp32); a box is box_rows rows x
// 1 head x 128 bytes of elements, in the 128-byte swizzle.
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

cudaError_t tc_preload() {
  cudaFuncAttributes attr;
  cudaError_t e = cudaFuncGetAttributes(&attr, tc::attn_tc_kernel<false>);
  return e == cudaSuccess ? cudaFuncGetAttributes(&attr, tc::attn_tc_kernel<true>) : e;
}

cudaError_t launch_attention_tc(const AttnProblem &p, const uint32_t *units, uint32_t n_units,
                                int num_sms, int *status, const uint16_t *q_norm_w, float eps,
                                float theta, cudaStream_t stream, bool after_prologue,
                                long long wait_cycles, bool exact_units,
                                const uint16_t *k_norm_w) {
  if (!n_units) return cudaSuccess;
  CUtensorMap mq, mk, mv, mo;
  const uint32_t rows = p.total;
  if (!make_map(&mq, p.q, rows, p.heads, false, tc::kQRows) ||
      !make_map(&mk, p.k, rows, p.kv_heads, false, tc::kKeys) ||
      !make_map(&mv, p.v, rows, p.kv_heads, false, tc::kKeys) ||
      !make_map(&mo, p.out, rows, p.heads, p.out_dtype == 0, 32))
    return cudaErrorInvalidValue;
  const bool out_bf16 = p.out_dtype == 1;
  auto kernel = out_bf16 ? tc::attn_tc_kernel<true> : tc::attn_tc_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)tc::kSmemBytes);
  if (e != cudaSuccess) return e;
  tc::Params prm;
  prm.units = reinterpret_cast<const uint2 *>(units);
  prm.offsets = units + 2 * n_units;
  prm.n_units = n_units;
  prm.exact = exact_units ? 1 : 0;
  prm.lengths = p.lengths;
  prm.cu = p.cu_seqlens;
  prm.out = p.out;
  prm.seq = p.seq;
  prm.heads = p.heads;
  prm.group = p.heads / p.kv_heads;
  prm.nh = heads_per_unit(p);
  prm.causal = p.causal;
  prm.scale_log2 = p.scale * 1.4426950408889634f;
  prm.status = status;
  prm.q_norm_w = q_norm_w;
  prm.k_norm_w = q_norm_w ? k_norm_w : nullptr;
  prm.eps = eps;
  prm.wait_cycles = wait_cycles > 0 ? wait_cycles : tc::kWaitCycles;
  for (int i = 0; i < 64; ++i)
    prm.inv_freq[i] = (float)std::pow((double)theta, -2.0 * (double)i / 128.0);
  const uint32_t grid = std::min(tc_grid(n_units, num_sms), 1024u);
  // Programmatic dependent launch, only right after this library's k prologue: the CTAs
  // may then start (barrier set-up, tensor-memory allocation, Q loads and the q prologue)
  // while the prologue finishes, and the producer waits for it before reading K
  // (griddepcontrol.wait).  Everything else the kernel reads was written before the
  // prologue started.  After any other kernel (a caller's kernel that may have just
  // written q or the lengths) the launch is an ordinary stream-ordered one.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(tc::kThreads);
  cfg.dynamicSmemBytes = tc::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = after_prologue ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, kernel, mq, mk, mv, mo, prm);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace tx
