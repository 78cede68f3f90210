// tx_attention_padded_noalloc: the bf16 tensor-core attention without any device-memory
// allocation, for callers that may not allocate.
//
// Who needs it: hosts that reserve all device memory up front (a serving process whose
// memory is carved out of one arena at start-up, an embedded runtime with a fixed
// memory budget) and treat any later allocation as an error, because cudaMalloc can
// fail when memory is full or fragmented and cudaMalloc/cudaFree can stall the whole
// device while they run.  Such callers cannot create a libtessattn context either
// (tx_create allocates its status word), so this entry point takes no context.
//
// How: the only scratch the kernel needs besides its inputs and outputs is the work
// list (one uint32 per unit of work).  It lives in the file-scope array below, which the
// CUDA runtime places in device memory when the module is loaded; every GPU that loads
// the library holds it until the process exits.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/tessattn.h"
#include "kernels.h"

namespace {

// Capacity of the work list: units = batch * heads/2 * ceil(seq / 128) (heads, not
// pairs, when the query heads per kv head are odd); two words per unit.
constexpr uint32_t kNoAllocMaxUnits = 16384;
// The work list also holds one offset per CTA of the grid, plus one.
constexpr uint32_t kNoAllocMaxOffsets = 1025;
// Words 0..63 are unused (they keep the work list 256-byte aligned after the header of
// earlier versions); words 64..: the work list (units grouped by CTA, then the offsets).
constexpr uint32_t kHeaderWords = 64;

static __device__ __align__(256) uint32_t
    g_noalloc_scratch[kHeaderWords + 2 * kNoAllocMaxUnits + kNoAllocMaxOffsets + 3];

// Device address of g_noalloc_scratch per device, looked up once with that device
// current.  In host code the array's name is only a host-side stand-in, not a device
// address, so the kernel must be given the looked-up address.
std::mutex g_noalloc_mu;
uint32_t *g_noalloc_ptr[64] = {};
int g_noalloc_sms[64] = {};
// Host work space for building the work list (under the mutex).
uint32_t g_host_sorted[kNoAllocMaxUnits];
uint32_t g_host_work[2 * kNoAllocMaxUnits + kNoAllocMaxOffsets + 3];

}  // namespace

extern "C" int tx_attention_padded_noalloc(const void *q, const void *k, const void *v,
                                           const uint32_t *lengths, const uint32_t *lengths_host,
                                           void *out, uint32_t batch, uint32_t seq,
                                           uint32_t heads, uint32_t kv_heads, int out_dtype,
                                           int causal, float scale, const uint16_t *q_norm_w,
                                           float eps, float theta, int *status, void *stream) {
  // The status word is required: a bounded wait that gives up is reported only there.
  if (!q || !k || !v || !lengths || !lengths_host || !out || !status) return TX_EINVAL;
  if (out_dtype != TX_F32 && out_dtype != TX_BF16) return TX_EINVAL;
  if (!batch || !seq || !(scale > 0.f) || !(scale < 1e30f)) return TX_EINVAL;
  if ((uint64_t)batch * seq > 0xffffffffull) return TX_EINVAL;
  for (uint32_t b = 0; b < batch; ++b)
    if (lengths_host[b] > seq) return TX_EINVAL;
  tx::AttnProblem p{};
  p.q = q; p.k = k; p.v = v; p.out = out; p.lengths = lengths; p.cu_seqlens = nullptr;
  p.batch = batch; p.seq = seq; p.total = batch * seq; p.heads = heads; p.kv_heads = kv_heads;
  p.dim = 128; p.in_dtype = TX_BF16; p.out_dtype = out_dtype; p.causal = causal ? 1 : 0;
  p.scale = scale;
  if (!tx::tc_attention_supported(p)) return TX_EINVAL;
  if (tx::tc_max_units(p) > kNoAllocMaxUnits) return TX_EINVAL;  // beyond the static list

  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return TX_ECUDA;
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    // One-time set-up for this device (the caller's current device).
    void *ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return TX_ECUDA;
    // Loads the kernel's module now (with lazy module loading its code would otherwise be
    // placed in device memory at the first launch, a later allocation).
    if (tx::tc_preload() != cudaSuccess) return TX_ECUDA;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
      return TX_ECUDA;
    g_noalloc_sms[device] = sms;
    g_noalloc_ptr[device] = (uint32_t *)ptr;
  }
  uint32_t *scratch = g_noalloc_ptr[device];
  cudaStream_t s = (cudaStream_t)stream;
  // The work list is copied from a static host array that the next call overwrites: a
  // captured copy would replay another call's list, so a capturing stream is refused.
  cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &capturing) != cudaSuccess) return TX_ECUDA;
  if (capturing != cudaStreamCaptureStatusNone) return TX_EINVAL;
  int *st = status;
  const int sms = g_noalloc_sms[device];
  if (sms < 1 || tx::tc_grid(tx::tc_max_units(p), sms) + 1 > kNoAllocMaxOffsets) return TX_EINVAL;
  // tc_build_units sorts and balances with fixed-size arrays on the stack and the static
  // host arrays above: no allocation.
  const uint32_t n = tx::tc_build_units(p, lengths_host, nullptr, sms, g_host_sorted, g_host_work);
  const uint32_t words = 2 * n + tx::tc_grid(n, sms) + 1;
  // The array keeps the previous call's contents: the status word must start at zero.
  if (cudaMemsetAsync(st, 0, sizeof(int), s) != cudaSuccess) return TX_ECUDA;
  if (n && cudaMemcpyAsync(scratch + kHeaderWords, g_host_work, words * sizeof(uint32_t),
                           cudaMemcpyHostToDevice, s) != cudaSuccess)
    return TX_ECUDA;
  cudaError_t e = tx::launch_attention_tc(p, scratch + kHeaderWords, n, sms, st, q_norm_w, eps,
                                          theta, s, /*after_prologue=*/false, /*wait_cycles=*/0,
                                          /*exact_units=*/true);
  return e == cudaSuccess ? TX_OK : TX_ECUDA;
}
