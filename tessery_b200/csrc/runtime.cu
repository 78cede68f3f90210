// C ABI of libtessattn.so: the CUDA counterpart of the reference's Objective-C++ Metal
// runtime (src/metal_inference/native/runtime.mm) for the attention hot path.
//
// A context owns one CUDA stream on one device, a device status word written by
// kernels whose bounded waits give up, and scratch memory (prologue outputs, the
// tensor-core work list).  Commands (tx_begin .. tx_finish) bracket dispatches with CUDA
// events the way mi_begin/mi_finish bracket a Metal command buffer.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <condition_variable>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <vector>

#include "../../include/tessattn.h"
#include "kernels.h"

namespace {

constexpr uint32_t kAbiVersion = 10;
constexpr uint32_t kHostChunks = 8;              // most chunks of a host-buffer call
constexpr size_t kHostChunkBytes = 16u << 20;     // bytes moved per chunk, at least
// Padded layout, host-buffer calls: the valid k/v rows of consecutive sequences are
// copied as one span, padded rows between them included, while the padding between two
// sequences is at most this many bytes (fewer copies against more bytes: at the Qwen
// padded benchmark shape 256 KB measured best of 0, 256 KB and 1 MB, by ~3 %); the
// padded rows copied are never attended.
constexpr size_t kMergeGapBytes = 256u << 10;

struct Ctx;

// Host memcpy over a few worker threads and the calling thread, for the staging of
// pageable host arrays through page-locked memory (one thread copies ~15 GB/s on the
// B200 hosts measured; four reach the ~50 GB/s the host gives).  copy() hands out 1 MB
// pieces of its segments and returns once every piece has been copied.
class CopyPool {
 public:
  struct Seg {
    uint8_t *dst;
    const uint8_t *src;
    size_t bytes;
  };
  explicit CopyPool(unsigned workers) {
    for (unsigned i = 0; i < workers; ++i) threads_.emplace_back([this] { loop(); });
  }
  ~CopyPool() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
    }
    wake_.notify_all();
    for (std::thread &t : threads_) t.join();
  }
  void copy(const std::vector<Seg> &segs) {
    std::vector<Seg> pieces;
    for (const Seg &sg : segs)
      for (size_t o = 0; o < sg.bytes; o += kPiece)
        pieces.push_back({sg.dst + o, sg.src + o, std::min(kPiece, sg.bytes - o)});
    if (pieces.empty()) return;
    {
      std::lock_guard<std::mutex> g(mu_);
      jobs_ = &pieces;
      next_ = 0;
      left_ = pieces.size();
      ++gen_;
    }
    wake_.notify_all();
    work();
    std::unique_lock<std::mutex> lk(mu_);
    done_.wait(lk, [&] { return left_ == 0; });
    jobs_ = nullptr;
  }

 private:
  static constexpr size_t kPiece = 1u << 20;
  void work() {
    for (;;) {
      Seg sg;
      {
        std::lock_guard<std::mutex> g(mu_);
        if (!jobs_ || next_ >= jobs_->size()) return;
        sg = (*jobs_)[next_++];
      }
      std::memcpy(sg.dst, sg.src, sg.bytes);
      std::lock_guard<std::mutex> g(mu_);
      if (--left_ == 0) done_.notify_all();
    }
  }
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(mu_);
        wake_.wait(lk, [&] { return stop_ || gen_ != seen; });
        if (stop_) return;
        seen = gen_;
      }
      work();
    }
  }
  std::vector<std::thread> threads_;
  std::mutex mu_;
  std::condition_variable wake_, done_;
  const std::vector<Seg> *jobs_ = nullptr;
  size_t next_ = 0, left_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

struct Buf {
  Ctx *ctx;
  void *dev;
  uint64_t size;
};

struct Ctx {
  int device = 0;
  int sms = 0;
  cudaStream_t stream = nullptr;
  std::recursive_mutex mu;
  std::string err;
  // command state
  bool open = false;
  cudaEvent_t ev_begin = nullptr, ev_end = nullptr;
  double last_gpu = -1.0;
  // per-dispatch profiling
  bool profile = false;
  std::vector<cudaEvent_t> prof_events;  // pairs
  size_t prof_used = 0;
  std::vector<double> prof_seconds;
  // per-kernel timing of the typed entry points: an event pair around each launch of
  // the last call (at most kKernelMarks / 2 launches)
  bool ktime = false;
  cudaEvent_t kt_ev[8] = {};
  int kt_n = 0;
  // device status word
  int *status = nullptr;
  // scratch
  void *qk_scratch = nullptr;
  size_t qk_bytes = 0;
  uint32_t *units = nullptr;
  size_t units_cap = 0;
  std::vector<uint32_t> units_host;
  uint32_t *hp_units = nullptr;  // page-locked work lists of one host-buffer call
  size_t hp_units_cap = 0;
  uint64_t units_key = 0;
  uint32_t units_count = 0;
  cudaEvent_t scratch_done = nullptr;  // last launch that read scratch
  std::set<Buf *> buffers;
  // Accounting of the buffers above: bytes live now, the most ever live at once, and
  // the number and bytes of every allocation made.
  uint64_t mem_live = 0, mem_peak = 0, mem_allocs = 0, mem_alloc_bytes = 0;
  const char *last_kernel = "";
  uint64_t launches = 0;  // kernels this context has launched
  long long wait_cycles = 0;  // bounded-wait limit of the tensor-core kernel (0: default)
  // host-buffer entry points: device copies of the caller's arrays, a copy-in and a
  // copy-out stream beside `stream`, and an event pair per chunk
  void *hp_mem = nullptr;
  size_t hp_bytes = 0;
  cudaStream_t hp_up = nullptr, hp_down = nullptr;
  cudaEvent_t hp_ev[2 * kHostChunks] = {};
  std::vector<int32_t> hp_cu;  // per-chunk cu_seqlens, rebased to each chunk's first row
  uint64_t hp_h2d = 0, hp_d2h = 0;  // bytes the last host-buffer call copied each way
  // pageable host arrays: page-locked staging (the device copies' layout), the copy
  // threads, and per chunk an event after its copy out
  uint8_t *st_mem = nullptr;
  size_t st_bytes = 0;
  std::unique_ptr<CopyPool> st_pool;
  cudaEvent_t hp_out_ev[kHostChunks] = {};
};

std::mutex g_create_mu;
std::string g_create_err;

int fail(Ctx *c, int code, const char *msg) {
  if (c) c->err = msg;
  return code;
}

int cuda_fail(Ctx *c, cudaError_t e, const char *what) {
  if (c) {
    c->err = std::string(what) + ": " + cudaGetErrorName(e);
  }
  return TX_ECUDA;
}

// Makes `stream` wait for the previous user of the context's scratch memory.
cudaError_t scratch_acquire(Ctx *c, cudaStream_t stream) {
  return cudaStreamWaitEvent(stream, c->scratch_done, 0);
}
cudaError_t scratch_release(Ctx *c, cudaStream_t stream) {
  return cudaEventRecord(c->scratch_done, stream);
}

cudaError_t ensure_qk_scratch(Ctx *c, size_t bytes) {
  if (c->qk_bytes >= bytes) return cudaSuccess;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  if (c->qk_scratch) cudaFree(c->qk_scratch);
  c->qk_scratch = nullptr;
  c->qk_bytes = 0;
  e = cudaMalloc(&c->qk_scratch, bytes);
  if (e != cudaSuccess) return e;
  c->qk_bytes = bytes;
  return cudaSuccess;
}

cudaError_t ensure_units(Ctx *c, size_t count) {
  if (c->units_cap >= count) return cudaSuccess;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  if (c->units) cudaFree(c->units);
  c->units = nullptr;
  c->units_cap = 0;
  c->units_key = 0;
  e = cudaMalloc(&c->units, count * sizeof(uint32_t));
  if (e != cudaSuccess) return e;
  c->units_cap = count;
  return cudaSuccess;
}

uint64_t fnv1a(uint64_t h, const void *data, size_t n) {
  const uint8_t *p = (const uint8_t *)data;
  for (size_t i = 0; i < n; ++i) { h ^= p[i]; h *= 1099511628211ull; }
  return h;
}

// Reads and clears the device status word after the stream has drained.
int check_status(Ctx *c) {
  int st = 0;
  cudaError_t e = cudaMemcpy(&st, c->status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(c, e, "status read");
  if (st) {
    cudaMemsetAsync(c->status, 0, sizeof(int), c->stream);  // before the next launch
    cudaStreamSynchronize(c->stream);
    char msg[128];
    if ((st & 0xff) == TX_ETIMEOUT) {
      snprintf(msg, sizeof msg, "device wait timed out (site %d)", (st >> 8) & 0xffff);
      return fail(c, TX_ETIMEOUT, msg);
    }
    if ((st & 0xff) == TX_EINVAL)
      return fail(c, TX_EINVAL, "a kernel rejected its arguments on the device");
    snprintf(msg, sizeof msg, "device reported status %d", st);
    return fail(c, TX_ECUDA, msg);
  }
  return TX_OK;
}

bool buf_ok(Buf *b, Ctx *c) { return b && b->ctx == c && c->buffers.count(b); }

struct Params64 {
  uint32_t n, rows, cols, k, heads, kv_heads, seq, batch, dim, group, u0, u1;
  float eps, theta, scale, reserved;
};
static_assert(sizeof(Params64) == 64, "Params block is 64 bytes");

constexpr int kKernelMarks = 8;
// Event marks around one kernel launch of a typed call, when kernel timing is on.
void kt_mark(Ctx *c, cudaStream_t stream) {
  if (!c->ktime || c->kt_n >= kKernelMarks) return;
  if (!c->kt_ev[c->kt_n] && cudaEventCreate(&c->kt_ev[c->kt_n]) != cudaSuccess) return;
  cudaEventRecord(c->kt_ev[c->kt_n++], stream);
}

// Core of the typed entry points (padded when cu == nullptr).
// `units_dev` / `units_n`: a work list already on the device (host-buffer calls upload
// every chunk's list in one copy ahead of the data); NULL builds and uploads it here.
int run_attention(Ctx *c, tx::AttnProblem p, const uint32_t *lengths_host,
                  const int32_t *cu_host, const uint16_t *q_w, const uint16_t *k_w, float eps,
                  float theta, cudaStream_t stream, const uint32_t *units_dev = nullptr,
                  uint32_t units_n = 0) {
  if (!p.q || !p.k || !p.v || !p.out) return fail(c, TX_EINVAL, "null tensor pointer");
  if (p.cu_seqlens == nullptr && p.lengths == nullptr)
    return fail(c, TX_EINVAL, "lengths or cu_seqlens required");
  if (!p.heads || !p.kv_heads || p.heads % p.kv_heads)
    return fail(c, TX_EINVAL, "heads must be a positive multiple of kv_heads");
  if (!p.dim || p.dim > 256) return fail(c, TX_EINVAL, "head_dim must be in 1..256");
  if (p.in_dtype != TX_F32 && p.in_dtype != TX_BF16) return fail(c, TX_EINVAL, "bad in_dtype");
  if (p.out_dtype != TX_F32 && p.out_dtype != TX_BF16) return fail(c, TX_EINVAL, "bad out_dtype");
  if (!std::isfinite(p.scale)) return fail(c, TX_EINVAL, "scale must be finite");
  const bool prologue = q_w != nullptr || k_w != nullptr;
  if (prologue && !(p.dim == 32 || p.dim == 64 || p.dim == 128 || p.dim == 256))
    return fail(c, TX_EINVAL, "prologue supports head_dim 32, 64, 128, 256");
  if (prologue && !(eps >= 0.f && std::isfinite(eps) && std::isfinite(theta) && theta > 0.f))
    return fail(c, TX_EINVAL, "bad eps/theta");
  if (p.cu_seqlens) {
    if (!p.batch) return fail(c, TX_EINVAL, "nseq must be positive");
    if (cu_host) {
      if (cu_host[0] != 0) return fail(c, TX_EINVAL, "cu_seqlens[0] must be 0");
      for (uint32_t s = 0; s < p.batch; ++s) {
        if (cu_host[s + 1] < cu_host[s]) return fail(c, TX_EINVAL, "cu_seqlens must not decrease");
        if ((uint32_t)(cu_host[s + 1] - cu_host[s]) > p.seq)
          return fail(c, TX_EINVAL, "sequence longer than max_len");
      }
      if ((uint32_t)cu_host[p.batch] != p.total) return fail(c, TX_EINVAL, "cu_seqlens[nseq] != total");
    }
  } else {
    if (!p.batch || !p.seq) return fail(c, TX_EINVAL, "batch and seq must be positive");
    if (lengths_host)
      for (uint32_t b = 0; b < p.batch; ++b)
        if (lengths_host[b] > p.seq) return fail(c, TX_EINVAL, "length exceeds seq");
    p.total = p.batch * p.seq;
  }
  c->kt_n = 0;
  if (!p.total) return TX_OK;
  if ((uint64_t)p.total * p.heads * p.dim >= (1ull << 40))
    return fail(c, TX_EINVAL, "problem too large");

  // Short sequences: one launch with the q/k prologue fused, no scratch or work list.
  if (p.in_dtype == TX_BF16 && tx::short_attention_supported(p)) {
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return cuda_fail(c, e, "cudaSetDevice");
    kt_mark(c, stream);
    if ((e = tx::launch_attention_short(p, q_w, k_w, eps, theta, c->status, stream)) !=
        cudaSuccess)
      return cuda_fail(c, e, "attention launch");
    kt_mark(c, stream);
    c->last_kernel = "short_d128";
    ++c->launches;
    return TX_OK;
  }
  const bool tc_path = p.in_dtype == TX_BF16 && p.scale > 0.f && tx::tc_attention_supported(p);
  // head_dim 32, fp32: both products on the tensor cores (three-product TF32 splits).
  const bool d32tc_path = !tc_path && tx::d32_tc_supported(p);
  const bool d32_path = !tc_path && !d32tc_path && p.dim == 32 &&
                        p.batch <= 65535u && p.heads <= 65535u &&
                        (uintptr_t)p.q % 16 == 0 && (uintptr_t)p.k % 16 == 0 &&
                        (uintptr_t)p.v % 16 == 0 && (uintptr_t)p.out % 16 == 0;
  const bool f32tc_path = !tc_path && !d32tc_path && !d32_path && tx::f32_tc_supported(p);
  cudaError_t e = cudaSetDevice(c->device);
  if (e != cudaSuccess) return cuda_fail(c, e, "cudaSetDevice");
  bool uses_scratch = prologue || tc_path;
  if (uses_scratch && (e = scratch_acquire(c, stream)) != cudaSuccess)
    return cuda_fail(c, e, "scratch wait");

  // Work list of the tensor-core kernel, uploaded before the prologue launch: the
  // attention kernel is launched as a programmatic dependent of the prologue and may
  // start while the prologue runs, so everything it reads besides k must already be in
  // place in stream order.
  if (tc_path && !units_dev) {
    const uint32_t cap = tx::tc_max_units(p), words = tx::tc_work_words(p, c->sms);
    uint64_t key = 1469598103934665603ull;
    uint32_t hdr[8] = {p.batch, p.seq, p.heads, p.kv_heads, (uint32_t)p.causal,
                       p.cu_seqlens ? 1u : 0u, lengths_host || cu_host ? 1u : 0u, p.total};
    key = fnv1a(key, hdr, sizeof hdr);
    if (lengths_host) key = fnv1a(key, lengths_host, sizeof(uint32_t) * p.batch);
    if (cu_host) key = fnv1a(key, cu_host, sizeof(int32_t) * (p.batch + 1));
    if (key != c->units_key) {
      if ((e = ensure_units(c, words)) != cudaSuccess) return cuda_fail(c, e, "work list allocation");
      c->units_host.resize((size_t)cap + words);
      uint32_t *work = c->units_host.data() + cap;
      c->units_count = tx::tc_build_units(p, lengths_host, cu_host, c->sms, c->units_host.data(),
                                          work);
      const uint32_t upload = 2 * c->units_count + tx::tc_grid(c->units_count, c->sms) + 1;
      // Pageable source: the call returns once the data is staged, so the host vector
      // can be rebuilt by the next call.
      if (c->units_count &&
          (e = cudaMemcpyAsync(c->units, work, upload * sizeof(uint32_t),
                               cudaMemcpyHostToDevice, stream)) != cudaSuccess)
        return cuda_fail(c, e, "work list upload");
      c->units_key = key;
    }
  }

  // The tensor-core kernel applies the q prologue to each Q tile in shared memory; k
  // (read by several query tiles) is normalised once into scratch, valid rows only.
  const uint16_t *tc_q_w = tc_path ? q_w : nullptr;
  const bool pro_q = q_w != nullptr && !tc_path, pro_k = k_w != nullptr;
  if (pro_q || pro_k) {
    const int mid = p.in_dtype;  // normalised q/k keep the attention kernel's input type
    const size_t esz = mid == TX_BF16 ? 2 : 4;
    const size_t qn = pro_q ? (size_t)p.total * p.heads * p.dim : 0;
    const size_t kn = pro_k ? (size_t)p.total * p.kv_heads * p.dim : 0;
    if ((e = ensure_qk_scratch(c, (qn + kn) * esz + 256)) != cudaSuccess)
      return cuda_fail(c, e, "scratch allocation");
    void *qs = c->qk_scratch;
    void *ks = (uint8_t *)c->qk_scratch + ((qn * esz + 255) & ~(size_t)255);
    tx::PrologueProblem pp{};
    pp.q = pro_q ? p.q : nullptr;
    pp.k = pro_k ? p.k : nullptr;
    pp.q_out = qs; pp.k_out = ks;
    pp.tokens = p.total; pp.seq = p.seq;
    pp.cu_seqlens = p.cu_seqlens; pp.nseq = p.batch;
    pp.heads = p.heads; pp.kv_heads = p.kv_heads; pp.dim = p.dim;
    pp.in_dtype = p.in_dtype; pp.out_dtype = mid;
    pp.q_w = q_w; pp.k_w = k_w; pp.eps = eps; pp.theta = theta;
    pp.lengths = tc_path && !p.cu_seqlens ? p.lengths : nullptr;
    kt_mark(c, stream);
    if ((e = tx::launch_qk_norm_rope(pp, stream)) != cudaSuccess)
      return cuda_fail(c, e, "prologue launch");
    kt_mark(c, stream);
    ++c->launches;
    if (pro_q) p.q = qs;
    if (pro_k) p.k = ks;
  }

  kt_mark(c, stream);
  if (tc_path) {
    // pro_k: the k prologue was the launch just before on this stream.
    if ((e = tx::launch_attention_tc(p, units_dev ? units_dev : c->units,
                                     units_dev ? units_n : c->units_count, c->sms, c->status,
                                     tc_q_w, eps, theta, stream, pro_k, c->wait_cycles,
                                     tx::tc_units_exact(p, lengths_host, cu_host),
                                     pro_k ? k_w : nullptr)) !=
        cudaSuccess)
      return cuda_fail(c, e, "attention launch");
    c->last_kernel = "tc_bf16_d128";
    ++c->launches;
  } else if (d32tc_path) {
    if ((e = tx::launch_attention_d32_tc(p, c->status, stream, c->sms)) != cudaSuccess)
      return cuda_fail(c, e, "attention launch");
    c->last_kernel = "d32_tc";
    ++c->launches;
  } else if (f32tc_path) {
    if ((e = tx::launch_attention_f32_tc(p, c->status, stream)) != cudaSuccess)
      return cuda_fail(c, e, "attention launch");
    c->last_kernel = "f32_tc";
    ++c->launches;
  } else if (d32_path) {
    if ((e = tx::launch_attention_d32(p, stream)) != cudaSuccess)
      return cuda_fail(c, e, "attention launch");
    c->last_kernel = "d32";
    ++c->launches;
  } else {
    if ((e = tx::launch_attention_simt(p, stream)) != cudaSuccess)
      return cuda_fail(c, e, "attention launch");
    c->last_kernel = "simt";
    ++c->launches;
  }
  kt_mark(c, stream);
  if (uses_scratch && (e = scratch_release(c, stream)) != cudaSuccess)
    return cuda_fail(c, e, "scratch event");
  return TX_OK;
}

// Host-buffer attention: q/k/v/out (and lengths or cu_seqlens) in host memory.  The
// sequences are split into up to kHostChunks chunks of whole sequences; chunk i's rows are
// copied in on one stream, its kernels run on the context's stream once they have
// landed, and its output rows are copied out on a third stream, so copies in, kernels and
// copies out of different chunks overlap (with page-locked host memory the two copy
// directions run at once).  Returns after the last output row is in host memory.
int run_attention_host(Ctx *c, tx::AttnProblem p, const uint32_t *lengths, const int32_t *cu,
                       const uint16_t *q_w, const uint16_t *k_w, float eps, float theta) {
  if (!p.q || !p.k || !p.v || !p.out) return fail(c, TX_EINVAL, "null tensor pointer");
  if (!lengths && !cu) return fail(c, TX_EINVAL, "lengths or cu_seqlens required");
  if (p.in_dtype != TX_F32 && p.in_dtype != TX_BF16) return fail(c, TX_EINVAL, "bad in_dtype");
  if (p.out_dtype != TX_F32 && p.out_dtype != TX_BF16) return fail(c, TX_EINVAL, "bad out_dtype");
  if (!p.heads || !p.kv_heads || !p.dim || p.dim > 256 || !p.batch)
    return fail(c, TX_EINVAL, "bad shape");
  const uint32_t nseq = p.batch;
  if (cu) {
    if (cu[0] != 0) return fail(c, TX_EINVAL, "cu_seqlens[0] must be 0");
    for (uint32_t s = 0; s < nseq; ++s)
      if (cu[s + 1] < cu[s]) return fail(c, TX_EINVAL, "cu_seqlens must not decrease");
    if ((uint32_t)cu[nseq] != p.total) return fail(c, TX_EINVAL, "cu_seqlens[nseq] != total");
  } else {
    if (!p.seq) return fail(c, TX_EINVAL, "batch and seq must be positive");
    if ((uint64_t)nseq * p.seq > 0xffffffffull) return fail(c, TX_EINVAL, "too many tokens");
    p.total = nseq * p.seq;
  }
  const size_t ein = p.in_dtype == TX_BF16 ? 2 : 4, eout = p.out_dtype == TX_BF16 ? 2 : 4;
  const size_t qrow = (size_t)p.heads * p.dim * ein, kvrow = (size_t)p.kv_heads * p.dim * ein;
  const size_t orow = (size_t)p.heads * p.dim * eout, rows = p.total;
  if (!rows) return TX_OK;
  // Chunks: first[i] = first sequence of chunk i, balanced by rows.
  const size_t moved = rows * (qrow + 2 * kvrow + orow);
  uint32_t nch = (uint32_t)std::min<size_t>({(moved + kHostChunkBytes - 1) / kHostChunkBytes,
                                             (size_t)kHostChunks, (size_t)nseq});
  nch = std::max(nch, 1u);
  auto row_of = [&](uint32_t s) -> size_t { return cu ? (size_t)cu[s] : (size_t)s * p.seq; };
  uint32_t first[kHostChunks + 1];
  first[0] = 0;
  uint32_t used = 1;
  for (uint32_t i = 1; i < nch; ++i) {
    const size_t target = rows * i / nch;
    uint32_t s = first[used - 1] + 1;
    while (s < nseq && row_of(s) < target) ++s;
    if (s >= nseq) break;
    first[used++] = s;
  }
  first[used] = nseq;
  nch = used;
  if (cu) {  // each chunk's cu_seqlens, rebased to the chunk's first row
    c->hp_cu.resize(nseq + nch);
    for (uint32_t i = 0; i < nch; ++i)
      for (uint32_t s = first[i]; s <= first[i + 1]; ++s)
        c->hp_cu[first[i] + i + (s - first[i])] = cu[s] - cu[first[i]];
  }
  // Chunk i as a problem on device pointers (base = the device copy buffers).
  auto up256 = [](size_t b) { return (b + 255) & ~(size_t)255; };
  const size_t oq = 0, ok = oq + up256(rows * qrow), ov = ok + up256(rows * kvrow);
  const size_t oo = ov + up256(rows * kvrow), om = oo + up256(rows * orow);
  const size_t meta = cu ? (size_t)(nseq + nch) * 4 : (size_t)nseq * 4;
  const size_t ow = om + up256(meta), ou = ow + 2 * up256((size_t)p.dim * 2);
  auto chunk_problem = [&](uint32_t i, uint8_t *dev) -> tx::AttnProblem {
    const size_t r0 = row_of(first[i]), r1 = row_of(first[i + 1]);
    tx::AttnProblem pc = p;
    pc.q = dev + oq + r0 * qrow;
    pc.k = dev + ok + r0 * kvrow;
    pc.v = dev + ov + r0 * kvrow;
    pc.out = dev + oo + r0 * orow;
    pc.batch = first[i + 1] - first[i];
    if (cu) {
      const int32_t *cc = c->hp_cu.data() + first[i] + i;
      pc.cu_seqlens = (const int32_t *)(dev + om) + first[i] + i;
      pc.lengths = nullptr;
      pc.total = (uint32_t)(r1 - r0);
      uint32_t mx = 0;
      for (uint32_t s = 0; s < pc.batch; ++s) mx = std::max<uint32_t>(mx, cc[s + 1] - cc[s]);
      pc.seq = std::max(mx, 1u);
    } else {
      pc.lengths = (const uint32_t *)(dev + om) + first[i];
      pc.cu_seqlens = nullptr;
    }
    return pc;
  };
  // Device memory: q, k, v, out, lengths or the rebased cu_seqlens, the weights, then the
  // tensor-core work lists of the chunks (bounded by their shapes).
  size_t wl_words = 0;
  for (uint32_t i = 0; i < nch; ++i) wl_words += tx::tc_work_words(chunk_problem(i, nullptr), c->sms);
  const size_t need = ou + up256(wl_words * 4);
  cudaError_t e = cudaSetDevice(c->device);
  if (e != cudaSuccess) return cuda_fail(c, e, "cudaSetDevice");
  if (c->hp_bytes < need) {
    if ((e = cudaDeviceSynchronize()) != cudaSuccess) return cuda_fail(c, e, "synchronize");
    if (c->hp_mem) cudaFree(c->hp_mem);
    c->hp_mem = nullptr;
    c->hp_bytes = 0;
    if ((e = cudaMalloc(&c->hp_mem, need)) != cudaSuccess) return cuda_fail(c, e, "host-path buffers");
    c->hp_bytes = need;
  }
  if (c->hp_units_cap < wl_words) {  // every earlier call has drained: nothing reads it
    if (c->hp_units) cudaFreeHost(c->hp_units);
    c->hp_units = nullptr;
    c->hp_units_cap = 0;
    if (wl_words &&
        (e = cudaHostAlloc((void **)&c->hp_units, wl_words * 4, cudaHostAllocDefault)) != cudaSuccess)
      return cuda_fail(c, e, "work list staging");
    c->hp_units_cap = wl_words;
  }
  if (!c->hp_up) {
    if ((e = cudaStreamCreateWithFlags(&c->hp_up, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaStreamCreateWithFlags(&c->hp_down, cudaStreamNonBlocking)) != cudaSuccess)
      return cuda_fail(c, e, "copy streams");
    for (cudaEvent_t &ev : c->hp_ev)
      if ((e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming)) != cudaSuccess)
        return cuda_fail(c, e, "copy events");
    for (cudaEvent_t &ev : c->hp_out_ev)
      if ((e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming)) != cudaSuccess)
        return cuda_fail(c, e, "copy events");
  }
  uint8_t *dev = (uint8_t *)c->hp_mem;
  // Work lists of the chunks that take the tensor-core kernel, built here and uploaded in
  // one copy ahead of the data: a small copy queued on the compute stream would wait in
  // the copy engine behind the bulk copies of every chunk queued before it.
  size_t wl_off[kHostChunks];
  uint32_t wl_n[kHostChunks];
  bool wl_tc[kHostChunks];
  size_t wl_used = 0;
  for (uint32_t i = 0; i < nch; ++i) {
    const tx::AttnProblem pc = chunk_problem(i, dev);
    wl_tc[i] = pc.in_dtype == TX_BF16 && !tx::short_attention_supported(pc) && pc.scale > 0.f &&
               tx::tc_attention_supported(pc);
    wl_off[i] = wl_used;
    wl_n[i] = 0;
    if (!wl_tc[i]) continue;
    c->units_host.resize(tx::tc_max_units(pc));
    wl_n[i] = tx::tc_build_units(pc, cu ? nullptr : lengths + first[i],
                                 cu ? c->hp_cu.data() + first[i] + i : nullptr, c->sms,
                                 c->units_host.data(), c->hp_units + wl_used);
    wl_used += tx::tc_work_words(pc, c->sms);
  }
  // Pageable host arrays go through page-locked staging laid out like the device copies
  // (a DMA from pageable memory is staged by the driver a piece at a time at a fraction
  // of the link's speed): chunk i's input rows are copied into the staging by the copy
  // threads before its copies in are queued, and its output rows out of it once its copy
  // out has landed, while the device works on the neighbouring chunks.
  auto pageable = [](const void *ptr) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
      cudaGetLastError();
      return true;
    }
    return a.type == cudaMemoryTypeUnregistered;
  };
  const bool sq = pageable(p.q), sk = pageable(p.k), sv = pageable(p.v), so = pageable(p.out);
  if (sq || sk || sv || so) {
    if (c->st_bytes < om) {  // every earlier call has drained: nothing reads it
      if (c->st_mem) cudaFreeHost(c->st_mem);
      c->st_mem = nullptr;
      c->st_bytes = 0;
      if ((e = cudaHostAlloc((void **)&c->st_mem, om, cudaHostAllocDefault)) != cudaSuccess)
        return cuda_fail(c, e, "page-locked staging");
      c->st_bytes = om;
    }
    if (!c->st_pool) {
      const unsigned hw = std::thread::hardware_concurrency();
      c->st_pool.reset(new CopyPool(std::max(1u, std::min(4u, hw / 2))));
    }
  }
  uint8_t *st = c->st_mem;
  const uint8_t *hq = (const uint8_t *)p.q, *hk = (const uint8_t *)p.k, *hv = (const uint8_t *)p.v;
  uint8_t *ho = (uint8_t *)p.out;
  // Sources of the copies in and destination of the copies out.
  const uint8_t *cq = sq ? st + oq : hq, *ck = sk ? st + ok : hk, *cv = sv ? st + ov : hv;
  uint8_t *co = so ? st + oo : ho;
  // Drains every stream of this call (no copy may touch the caller's memory after return).
  auto drain = [&]() {
    cudaStreamSynchronize(c->hp_up);
    cudaStreamSynchronize(c->stream);
    cudaStreamSynchronize(c->hp_down);
  };
  // Nothing of an earlier call may still read these buffers.
  if ((e = cudaStreamWaitEvent(c->hp_up, c->scratch_done, 0)) != cudaSuccess)
    return cuda_fail(c, e, "stream wait");
  c->hp_h2d = meta + (q_w ? (size_t)p.dim * 2 : 0) + (k_w ? (size_t)p.dim * 2 : 0) +
              wl_used * 4;
  c->hp_d2h = 0;
  if (cu)
    e = cudaMemcpyAsync(dev + om, c->hp_cu.data(), meta, cudaMemcpyHostToDevice, c->hp_up);
  else
    e = cudaMemcpyAsync(dev + om, lengths, meta, cudaMemcpyHostToDevice, c->hp_up);
  if (e == cudaSuccess && q_w)
    e = cudaMemcpyAsync(dev + ow, q_w, (size_t)p.dim * 2, cudaMemcpyHostToDevice, c->hp_up);
  if (e == cudaSuccess && k_w)
    e = cudaMemcpyAsync(dev + ow + up256((size_t)p.dim * 2), k_w, (size_t)p.dim * 2,
                        cudaMemcpyHostToDevice, c->hp_up);
  if (e == cudaSuccess && wl_used)
    e = cudaMemcpyAsync(dev + ou, c->hp_units, wl_used * 4, cudaMemcpyHostToDevice, c->hp_up);
  if (e != cudaSuccess) {
    drain();
    return cuda_fail(c, e, "copy in");
  }
  const uint16_t *dqw = q_w ? (const uint16_t *)(dev + ow) : nullptr;
  const uint16_t *dkw = k_w ? (const uint16_t *)(dev + ow + up256((size_t)p.dim * 2)) : nullptr;
  // k and v rows of chunk i as (first byte, bytes) spans of the k (or v) array.  Padded
  // layout: each sequence's valid rows cross the link, in spans over consecutive sequences
  // that take the padded rows between them along while a gap is at most kMergeGapBytes
  // (fewer, larger copies); rows at or past a length are never attended, and every kernel
  // either skips them or clears them on chip, so the device rows there may hold anything
  // (an earlier call's rows, or the caller's padding copied along).
  std::vector<std::pair<size_t, size_t>> kv_spans;
  auto spans_of = [&](uint32_t i) {
    kv_spans.clear();
    const size_t r0 = row_of(first[i]), r1 = row_of(first[i + 1]);
    if (cu) {
      kv_spans.push_back({r0 * kvrow, (r1 - r0) * kvrow});
      return;
    }
    for (uint32_t b = first[i]; b < first[i + 1];) {
      const size_t s0 = (size_t)b * p.seq;
      size_t end = s0 + std::min(lengths[b], p.seq);  // rows [s0, end) are copied
      uint32_t b1 = b;
      while (b1 + 1 < first[i + 1] &&
             ((size_t)(b1 + 1) * p.seq - end) * kvrow <= kMergeGapBytes) {
        ++b1;
        end = (size_t)b1 * p.seq + std::min(lengths[b1], p.seq);
      }
      if (end > s0) kv_spans.push_back({s0 * kvrow, (end - s0) * kvrow});
      b = b1 + 1;
    }
  };
  // Output rows of chunk j from the staging into the caller's array, once they landed.
  auto unstage_out = [&](uint32_t j) -> cudaError_t {
    const size_t r0 = row_of(first[j]), n = row_of(first[j + 1]) - r0;
    const cudaError_t err = cudaEventSynchronize(c->hp_out_ev[j]);
    if (err == cudaSuccess) c->st_pool->copy({{ho + r0 * orow, co + r0 * orow, n * orow}});
    return err;
  };
  for (uint32_t i = 0; i < nch; ++i) {
    const size_t r0 = row_of(first[i]), r1 = row_of(first[i + 1]), n = r1 - r0;
    spans_of(i);
    if (sq || sk || sv) {
      std::vector<CopyPool::Seg> segs;
      if (sq) segs.push_back({st + oq + r0 * qrow, hq + r0 * qrow, n * qrow});
      for (const auto &sp : kv_spans) {
        if (sk) segs.push_back({st + ok + sp.first, hk + sp.first, sp.second});
        if (sv) segs.push_back({st + ov + sp.first, hv + sp.first, sp.second});
      }
      c->st_pool->copy(segs);
    }
    c->hp_h2d += n * qrow;
    e = cudaMemcpyAsync(dev + oq + r0 * qrow, cq + r0 * qrow, n * qrow, cudaMemcpyHostToDevice,
                        c->hp_up);
    for (const auto &sp : kv_spans) {
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(dev + ok + sp.first, ck + sp.first, sp.second,
                            cudaMemcpyHostToDevice, c->hp_up);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(dev + ov + sp.first, cv + sp.first, sp.second,
                            cudaMemcpyHostToDevice, c->hp_up);
      c->hp_h2d += 2 * sp.second;
    }
    if (e != cudaSuccess ||
        (e = cudaEventRecord(c->hp_ev[2 * i], c->hp_up)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(c->stream, c->hp_ev[2 * i], 0)) != cudaSuccess) {
      drain();
      return cuda_fail(c, e, "copy in");
    }
    const tx::AttnProblem pc = chunk_problem(i, dev);
    const int rc = run_attention(c, pc, cu ? nullptr : lengths + first[i],
                                 cu ? c->hp_cu.data() + first[i] + i : nullptr, dqw, dkw, eps,
                                 theta, c->stream,
                                 wl_tc[i] ? (const uint32_t *)(dev + ou) + wl_off[i] : nullptr,
                                 wl_n[i]);
    if (rc != TX_OK) {
      drain();
      return rc;
    }
    if ((e = cudaEventRecord(c->hp_ev[2 * i + 1], c->stream)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(c->hp_down, c->hp_ev[2 * i + 1], 0)) != cudaSuccess ||
        (e = cudaMemcpyAsync(co + r0 * orow, dev + oo + r0 * orow, n * orow,
                             cudaMemcpyDeviceToHost, c->hp_down)) != cudaSuccess ||
        (e = cudaEventRecord(c->hp_out_ev[i], c->hp_down)) != cudaSuccess ||
        (so && i > 0 && (e = unstage_out(i - 1)) != cudaSuccess)) {
      drain();
      return cuda_fail(c, e, "copy out");
    }
    c->hp_d2h += n * orow;
  }
  if (so && (e = unstage_out(nch - 1)) != cudaSuccess) {
    drain();
    return cuda_fail(c, e, "copy out");
  }
  // The next call's copies in wait for this one's kernels and copies out.
  if ((e = cudaEventRecord(c->scratch_done, c->hp_down)) != cudaSuccess) {
    drain();
    return cuda_fail(c, e, "event");
  }
  drain();
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(c, e, "host-buffer attention");
  return check_status(c);
}

// Profiling hooks around one dispatch of an open command.
void prof_begin(Ctx *c) {
  if (!c->profile) return;
  if (c->prof_used + 2 > c->prof_events.size()) {
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    c->prof_events.push_back(a);
    c->prof_events.push_back(b);
  }
  cudaEventRecord(c->prof_events[c->prof_used], c->stream);
}
void prof_end(Ctx *c) {
  if (!c->profile) return;
  cudaEventRecord(c->prof_events[c->prof_used + 1], c->stream);
  c->prof_used += 2;
}

}  // namespace

namespace tx {
int ctx_fail(void *ctx, int code, const char *msg) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return code;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  return fail(c, code, msg);
}
}  // namespace tx

extern "C" {

uint32_t tx_abi_version(void) { return kAbiVersion; }

void *tx_create(int device) {
  std::lock_guard<std::mutex> g(g_create_mu);
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    g_create_err = std::string("no CUDA device: ") + cudaGetErrorName(e);
    return nullptr;
  }
  if (device < 0 || device >= count) {
    g_create_err = "device index out of range";
    return nullptr;
  }
  cudaDeviceProp prop;
  if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) {
    g_create_err = std::string("device query: ") + cudaGetErrorName(e);
    return nullptr;
  }
  if (prop.major != 10) {
    g_create_err = "device is not sm_100 (this library is built for sm_100a only)";
    return nullptr;
  }
  if ((e = cudaSetDevice(device)) != cudaSuccess) {
    g_create_err = std::string("cudaSetDevice: ") + cudaGetErrorName(e);
    return nullptr;
  }
  Ctx *c = new Ctx();
  c->device = device;
  c->sms = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreate(&c->ev_begin) != cudaSuccess || cudaEventCreate(&c->ev_end) != cudaSuccess ||
      cudaEventCreateWithFlags(&c->scratch_done, cudaEventDisableTiming) != cudaSuccess ||
      cudaMalloc(&c->status, sizeof(int)) != cudaSuccess ||
      cudaMemsetAsync(c->status, 0, sizeof(int), c->stream) != cudaSuccess) {
    g_create_err = "context resources";
    tx_destroy(c);
    return nullptr;
  }
  cudaEventRecord(c->scratch_done, c->stream);
  cudaStreamSynchronize(c->stream);
  return c;
}

void tx_destroy(void *ctx) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return;
  {
    std::lock_guard<std::recursive_mutex> g(c->mu);
    cudaSetDevice(c->device);
    cudaDeviceSynchronize();
    for (Buf *b : c->buffers) {
      cudaFree(b->dev);
      delete b;
    }
    c->buffers.clear();
    if (c->qk_scratch) cudaFree(c->qk_scratch);
    if (c->units) cudaFree(c->units);
    if (c->status) cudaFree(c->status);
    for (cudaEvent_t ev : c->prof_events) cudaEventDestroy(ev);
    for (cudaEvent_t ev : c->kt_ev)
      if (ev) cudaEventDestroy(ev);
    if (c->ev_begin) cudaEventDestroy(c->ev_begin);
    if (c->ev_end) cudaEventDestroy(c->ev_end);
    if (c->scratch_done) cudaEventDestroy(c->scratch_done);
    if (c->hp_mem) cudaFree(c->hp_mem);
    if (c->hp_units) cudaFreeHost(c->hp_units);
    for (cudaEvent_t ev : c->hp_ev)
      if (ev) cudaEventDestroy(ev);
    for (cudaEvent_t ev : c->hp_out_ev)
      if (ev) cudaEventDestroy(ev);
    if (c->st_mem) cudaFreeHost(c->st_mem);
    c->st_pool.reset();
    if (c->hp_up) cudaStreamDestroy(c->hp_up);
    if (c->hp_down) cudaStreamDestroy(c->hp_down);
    if (c->stream) cudaStreamDestroy(c->stream);
  }
  delete c;
}

const char *tx_last_error(void *ctx) {
  if (!ctx) return g_create_err.c_str();
  return ((Ctx *)ctx)->err.c_str();
}

int tx_device_sms(void *ctx) { return ctx ? ((Ctx *)ctx)->sms : 0; }

int tx_set_wait_limit(void *ctx, int64_t cycles) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (cycles < 0) return fail(c, TX_EINVAL, "wait limit must be >= 0");
  c->wait_cycles = (long long)cycles;
  return TX_OK;
}

const char *tx_last_kernel(void *ctx) { return ctx ? ((Ctx *)ctx)->last_kernel : ""; }

uint64_t tx_launch_count(void *ctx) { return ctx ? ((Ctx *)ctx)->launches : 0; }

void *tx_buffer(void *ctx, const void *host, uint64_t size) {
  Ctx *c = (Ctx *)ctx;
  if (!c || !size || size > (1ull << 40)) {
    if (c) c->err = "bad buffer size";
    return nullptr;
  }
  std::lock_guard<std::recursive_mutex> g(c->mu);
  cudaSetDevice(c->device);
  void *d = nullptr;
  cudaError_t e = cudaMalloc(&d, size);
  if (e != cudaSuccess) {
    cuda_fail(c, e, "cudaMalloc");
    cudaGetLastError();
    return nullptr;
  }
  // The fill runs on the context's stream, which does not wait for the legacy default
  // stream (a plain cudaMemset or pageable cudaMemcpy there could land after kernels this
  // context queues next), and is complete before the buffer is handed out.
  e = host ? cudaMemcpyAsync(d, host, size, cudaMemcpyHostToDevice, c->stream)
           : cudaMemsetAsync(d, 0, size, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) {
    cuda_fail(c, e, "buffer init");
    cudaFree(d);
    return nullptr;
  }
  Buf *b = new Buf{c, d, size};
  c->buffers.insert(b);
  c->mem_live += size;
  c->mem_peak = std::max(c->mem_peak, c->mem_live);
  ++c->mem_allocs;
  c->mem_alloc_bytes += size;
  return b;
}

void tx_free(void *buffer) {
  Buf *b = (Buf *)buffer;
  if (!b) return;
  Ctx *c = b->ctx;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!c->buffers.count(b)) return;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  cudaFree(b->dev);
  c->buffers.erase(b);
  c->mem_live -= b->size;
  delete b;
}

int tx_memory_stats(void *ctx, uint64_t *out) {
  Ctx *c = (Ctx *)ctx;
  if (!c || !out) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  out[0] = c->mem_live;
  out[1] = c->mem_peak;
  out[2] = c->mem_allocs;
  out[3] = c->mem_alloc_bytes;
  return TX_OK;
}

int tx_host_copy_bytes(void *ctx, uint64_t *out) {
  Ctx *c = (Ctx *)ctx;
  if (!c || !out) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  out[0] = c->hp_h2d;
  out[1] = c->hp_d2h;
  return TX_OK;
}

int tx_read(void *buffer, void *out, uint64_t bytes) {
  Buf *b = (Buf *)buffer;
  if (!b || !out) return TX_EINVAL;
  Ctx *c = b->ctx;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!buf_ok(b, c)) return TX_EINVAL;
  if (bytes > b->size) return fail(c, TX_EINVAL, "read beyond buffer");
  cudaSetDevice(c->device);
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e == cudaSuccess) e = cudaMemcpy(out, b->dev, bytes, cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? TX_OK : cuda_fail(c, e, "read");
}

int tx_write(void *buffer, const void *src, uint64_t bytes) {
  Buf *b = (Buf *)buffer;
  if (!b || !src) return TX_EINVAL;
  Ctx *c = b->ctx;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!buf_ok(b, c)) return TX_EINVAL;
  if (bytes > b->size) return fail(c, TX_EINVAL, "write beyond buffer");
  cudaSetDevice(c->device);
  // Ordered after the context's queued work and complete before returning (a pageable
  // cudaMemcpy may return before its DMA lands).
  cudaError_t e = cudaMemcpyAsync(b->dev, src, bytes, cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  return e == cudaSuccess ? TX_OK : cuda_fail(c, e, "write");
}

void *tx_buffer_device_ptr(void *buffer) { return buffer ? ((Buf *)buffer)->dev : nullptr; }
uint64_t tx_buffer_size(void *buffer) { return buffer ? ((Buf *)buffer)->size : 0; }

void *tx_host_alloc(uint64_t size) {
  void *p = nullptr;
  if (!size || cudaHostAlloc(&p, size, cudaHostAllocDefault) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return p;
}

void tx_host_free(void *ptr) {
  if (ptr) cudaFreeHost(ptr);
}

int tx_begin(void *ctx) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (c->open) return fail(c, TX_EINVAL, "command already open");
  cudaSetDevice(c->device);
  c->prof_used = 0;
  c->prof_seconds.clear();
  cudaError_t e = cudaEventRecord(c->ev_begin, c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "begin");
  c->open = true;
  return TX_OK;
}

int tx_dispatch(void *ctx, const char *name, void **buffers, uint32_t count, const void *params,
                uint32_t size, uint64_t threads, uint32_t group) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!c->open) return fail(c, TX_EINVAL, "no open command");
  if (!name || !params || size != 64 || count > 8 || !threads || !group)
    return fail(c, TX_EINVAL, "bad dispatch arguments");
  Buf *b[8] = {};
  for (uint32_t i = 0; i < count; ++i) {
    b[i] = (Buf *)buffers[i];
    if (!buf_ok(b[i], c)) return fail(c, TX_EINVAL, "foreign or freed buffer");
  }
  Params64 pr;
  memcpy(&pr, params, 64);
  cudaSetDevice(c->device);
  cudaError_t e = cudaSuccess;
  const std::string n(name);

  if (n == "rms_norm") {
    // threads = rows * group (one threadgroup per row, kernels.metal:53-56)
    if (count != 3 || threads % group) return fail(c, TX_EINVAL, "rms_norm: bad arguments");
    uint64_t rows = threads / group;
    if (!pr.cols || rows * pr.cols * 4 > b[0]->size || rows * pr.cols * 4 > b[2]->size ||
        (uint64_t)pr.cols * 2 > b[1]->size)
      return fail(c, TX_EINVAL, "rms_norm: buffer too small");
    prof_begin(c);
    e = tx::launch_rms_norm((const float *)b[0]->dev, (const uint16_t *)b[1]->dev,
                            (float *)b[2]->dev, (uint32_t)rows, pr.cols, pr.eps, c->stream);
    if (e == cudaSuccess) ++c->launches;
    prof_end(c);
  } else if (n == "rope") {
    // one thread per rotated pair, i < n (kernels.metal:65-67)
    if (count != 1 || !pr.dim || pr.dim % 2 || !pr.heads || !pr.seq)
      return fail(c, TX_EINVAL, "rope: bad arguments");
    uint64_t rows = ((uint64_t)pr.n + pr.dim / 2 - 1) / (pr.dim / 2);
    if (rows * pr.dim * 4 > b[0]->size) return fail(c, TX_EINVAL, "rope: buffer too small");
    prof_begin(c);
    e = tx::launch_rope((float *)b[0]->dev, pr.n, pr.heads, pr.seq, pr.dim, pr.theta, c->stream);
    if (e == cudaSuccess) ++c->launches;
    prof_end(c);
  } else if (n == "attention" || n == "attention_tiled" || n == "attention_tail_32" ||
             n == "attention_tail_128" || n == "attention_d32") {
    if (count != 5) return fail(c, TX_EINVAL, "attention: five buffers expected");
    if (!pr.heads || !pr.kv_heads || pr.heads % pr.kv_heads || !pr.dim || pr.dim > 256 || !pr.seq)
      return fail(c, TX_EINVAL, "attention: bad shape");
    // Token count from the reference grid (metal.py:543-569).
    uint64_t tokens;
    if (n == "attention" || n == "attention_d32") {
      if (threads % ((uint64_t)pr.heads * 32)) return fail(c, TX_EINVAL, "attention: bad grid");
      tokens = threads / 32 / pr.heads;
    } else if (n == "attention_tiled") {
      if (threads % ((uint64_t)pr.heads * 128)) return fail(c, TX_EINVAL, "attention: bad grid");
      tokens = threads / 128 / pr.heads * 8;
    } else {
      uint64_t per = (uint64_t)pr.heads * 128 * ((pr.seq + 7) / 8);
      if (threads % per) return fail(c, TX_EINVAL, "attention: bad grid");
      tokens = threads / per * pr.seq;
    }
    if (!tokens || tokens % pr.seq) return fail(c, TX_EINVAL, "attention: tokens not a multiple of seq");
    uint64_t batch = tokens / pr.seq;
    uint64_t qbytes = tokens * pr.heads * pr.dim * 4, kbytes = tokens * pr.kv_heads * pr.dim * 4;
    if (b[0]->size < qbytes || b[1]->size < kbytes || b[2]->size < kbytes ||
        b[3]->size < batch * 4 || b[4]->size < qbytes)
      return fail(c, TX_EINVAL, "attention: buffer too small");
    tx::AttnProblem p{};
    p.q = b[0]->dev; p.k = b[1]->dev; p.v = b[2]->dev; p.out = b[4]->dev;
    p.lengths = (const uint32_t *)b[3]->dev;
    p.batch = (uint32_t)batch; p.seq = pr.seq; p.total = (uint32_t)tokens;
    p.heads = pr.heads; p.kv_heads = pr.kv_heads; p.dim = pr.dim;
    p.in_dtype = TX_F32; p.out_dtype = TX_F32;
    p.causal = pr.u0 ? 0 : 1;
    p.scale = pr.scale;
    prof_begin(c);
    int rc = run_attention(c, p, nullptr, nullptr, nullptr, nullptr, 0.f, 0.f, c->stream);
    prof_end(c);
    if (rc) return rc;
  } else if (n == "pool_project") {
    // buffers [x, lengths, out]; one 32-thread group per sequence (kernels.metal:339-349)
    if (count != 3 || threads % 32 || !pr.seq || !pr.cols || !pr.dim || pr.dim > pr.cols)
      return fail(c, TX_EINVAL, "pool_project: bad arguments");
    uint64_t batch = threads / 32;
    if (batch * pr.seq * pr.cols * 4 > b[0]->size || batch * 4 > b[1]->size ||
        batch * pr.dim * 4 > b[2]->size)
      return fail(c, TX_EINVAL, "pool_project: buffer too small");
    tx::PoolProblem pp{};
    pp.x = b[0]->dev; pp.in_dtype = TX_F32; pp.lengths = (const uint32_t *)b[1]->dev;
    pp.out = (float *)b[2]->dev; pp.batch = (uint32_t)batch; pp.seq = pr.seq;
    pp.cols = pr.cols; pp.dim = pr.dim; pp.first_token = pr.u1 ? 1 : 0;
    prof_begin(c);
    e = tx::launch_pool_project(pp, c->stream);
    if (e == cudaSuccess) {
      ++c->launches;
      c->last_kernel = "pool_project";
    }
    prof_end(c);
  } else if (n == "embedding4") {
    // buffers [ids, packed, scales, biases, out]; n = tokens * cols (kernels.metal:21-28)
    const uint32_t cols = pr.cols;
    if (count != 5 || !cols || cols % 64 || pr.n % cols)
      return fail(c, TX_EINVAL, "embedding4: bad arguments");
    const uint64_t tokens = pr.n / cols, vocab = b[1]->size / ((uint64_t)cols / 2);
    if (b[0]->size < tokens * 4 || b[2]->size < vocab * (cols / 64) * 2 ||
        b[3]->size < vocab * (cols / 64) * 2 || b[4]->size < (uint64_t)pr.n * 4 || !vocab)
      return fail(c, TX_EINVAL, "embedding4: buffer too small");
    prof_begin(c);
    e = tx::launch_embedding4((const uint32_t *)b[0]->dev, (uint32_t)tokens,
                              (const uint32_t *)b[1]->dev, (const uint16_t *)b[2]->dev,
                              (const uint16_t *)b[3]->dev, (float *)b[4]->dev, cols,
                              (uint32_t)vocab, c->status, c->stream);
    if (e == cudaSuccess) ++c->launches;
    prof_end(c);
  } else if (n.rfind("linear4", 0) == 0) {
    // buffers [x, packed, scales, biases, out], fp32 (kernels.metal:32-51 and the tiled
    // variants :491-608, 658-773, routed by metal.py:416-483); the rows each variant covers
    // follow from its grid: [n, ...) for the 8-row tiles and tails, [0, ...) for the
    // 16- and 32-row tiles.
    const uint32_t rows = pr.rows, cols = pr.cols, k = pr.k;
    if (count != 5 || !rows || !cols || !k || k % 64) return fail(c, TX_EINVAL, "linear4: bad arguments");
    const uint64_t tiles32 = (uint64_t)(cols / 32);
    uint64_t t0 = 0, t1 = rows;
    if (n == "linear4") {
      t0 = pr.n;
      t1 = std::min<uint64_t>(rows, t0 + 4 * (threads / 32 / cols));
    } else if (n == "linear4_tiled") {
      if (!tiles32) return fail(c, TX_EINVAL, "linear4: bad grid");
      t0 = pr.n;
      t1 = std::min<uint64_t>(rows, t0 + 8 * (threads / (tiles32 * 128)));
    } else if (n == "linear4_tail") {
      t0 = pr.n;
    } else if (n == "linear4_16x32_k64" || n == "linear4_32x32_k64") {
      if (!tiles32) return fail(c, TX_EINVAL, "linear4: bad grid");
      const uint64_t tile = n == "linear4_16x32_k64" ? 16 : 32;
      t1 = std::min<uint64_t>(rows, tile * (threads / (tiles32 * 256)));
    } else if (n != "linear4_small3") {
      return fail(c, TX_EINVAL, "unknown kernel name");
    }
    if (b[0]->size < (uint64_t)rows * k * 4 || b[1]->size < (uint64_t)cols * (k / 8) * 4 ||
        b[2]->size < (uint64_t)cols * (k / 64) * 2 || b[3]->size < (uint64_t)cols * (k / 64) * 2 ||
        b[4]->size < (uint64_t)rows * cols * 4)
      return fail(c, TX_EINVAL, "linear4: buffer too small");
    prof_begin(c);
    e = tx::launch_linear4_f32((const float *)b[0]->dev, (const uint32_t *)b[1]->dev,
                               (const uint16_t *)b[2]->dev, (const uint16_t *)b[3]->dev,
                               (float *)b[4]->dev, (uint32_t)std::min<uint64_t>(t0, rows),
                               (uint32_t)t1, cols, k, c->stream);
    if (e == cudaSuccess) ++c->launches;
    prof_end(c);
  } else if (n == "silu_gate" || n == "add") {
    // silu_gate [gate, up] in place (kernels.metal:333-337); add [a, b, out] (:300-304)
    const bool silu = n == "silu_gate";
    if (count != (silu ? 2u : 3u)) return fail(c, TX_EINVAL, "elementwise: bad arguments");
    for (uint32_t i = 0; i < count; ++i)
      if (b[i]->size < (uint64_t)pr.n * 4) return fail(c, TX_EINVAL, "elementwise: buffer too small");
    prof_begin(c);
    e = silu ? tx::launch_silu_gate((float *)b[0]->dev, (const float *)b[1]->dev, pr.n, c->stream)
             : tx::launch_add((const float *)b[0]->dev, (const float *)b[1]->dev,
                              (float *)b[2]->dev, pr.n, c->stream);
    if (e == cudaSuccess) ++c->launches;
    prof_end(c);
  } else if (n == "layer_norm") {
    // [x, w, bias, out], one threadgroup of `group` threads per row (kernels.metal:362-373)
    if (count != 4 || threads % group) return fail(c, TX_EINVAL, "layer_norm: bad arguments");
    const uint64_t rows = threads / group, bytes = rows * pr.cols * 4;
    if (!tx::bert_cols_ok(pr.cols))
      return fail(c, TX_EINVAL, "layer_norm: cols at most 1024");
    if (b[0]->size < bytes || b[3]->size < bytes || b[1]->size < pr.cols * 4u ||
        b[2]->size < pr.cols * 4u)
      return fail(c, TX_EINVAL, "layer_norm: buffer too small");
    prof_begin(c);
    e = tx::launch_layer_norm_rows((const float *)b[0]->dev, (const float *)b[1]->dev,
                                   (const float *)b[2]->dev, (float *)b[3]->dev, nullptr, TX_F32,
                                   (uint32_t)rows, pr.cols, pr.eps, c->stream);
    if (e == cudaSuccess) ++c->launches;
    prof_end(c);
  } else if (n == "embedding_position") {
    // [ids, words, positions, types, out], n = tokens * cols (kernels.metal:353-361)
    if (count != 5 || !pr.cols || !pr.seq || pr.n % pr.cols)
      return fail(c, TX_EINVAL, "embedding_position: bad arguments");
    const uint64_t tokens = pr.n / pr.cols;
    if (b[0]->size < tokens * 4 || b[4]->size < (uint64_t)pr.n * 4 ||
        b[2]->size < (uint64_t)std::min<uint64_t>(tokens, pr.seq) * pr.cols * 4 ||
        b[3]->size < pr.cols * 4u)
      return fail(c, TX_EINVAL, "embedding_position: buffer too small");
    prof_begin(c);
    e = tx::launch_embedding_position((const uint32_t *)b[0]->dev, (const float *)b[1]->dev,
                                      (const float *)b[2]->dev, (const float *)b[3]->dev,
                                      (float *)b[4]->dev, pr.n, pr.cols, pr.seq, c->stream);
    if (e == cudaSuccess) ++c->launches;
    prof_end(c);
  } else if (n == "gelu_f32" || n == "add_bias" || n == "silu_f32") {
    // gelu_f32 [x] in place (:381-391), add_bias [x, bias] (:376-379), silu_f32 [x, out]
    // (:328-331); n elements
    const uint32_t want = n == "gelu_f32" ? 1u : 2u;
    if (count != want || (n == "add_bias" && !pr.cols))
      return fail(c, TX_EINVAL, "elementwise: bad arguments");
    if (b[0]->size < (uint64_t)pr.n * 4 || (n == "silu_f32" && b[1]->size < (uint64_t)pr.n * 4) ||
        (n == "add_bias" && b[1]->size < pr.cols * 4u))
      return fail(c, TX_EINVAL, "elementwise: buffer too small");
    prof_begin(c);
    if (n == "gelu_f32")
      e = tx::launch_gelu((float *)b[0]->dev, pr.n, c->stream);
    else if (n == "add_bias")
      e = tx::launch_add_bias((float *)b[0]->dev, (const float *)b[1]->dev, pr.n, pr.cols,
                              c->stream);
    else
      e = tx::launch_silu((const float *)b[0]->dev, (float *)b[1]->dev, pr.n, c->stream);
    if (e == cudaSuccess) ++c->launches;
    prof_end(c);
  } else if (n == "transpose_f32") {
    // [x, out], x [rows, cols] (kernels.metal:323-326)
    const uint64_t bytes = (uint64_t)pr.rows * pr.cols * 4;
    if (count != 2 || b[0]->size < bytes || b[1]->size < bytes)
      return fail(c, TX_EINVAL, "transpose_f32: bad arguments");
    prof_begin(c);
    e = tx::launch_transpose((const float *)b[0]->dev, (float *)b[1]->dev, pr.rows, pr.cols,
                             c->stream);
    if (e == cudaSuccess) ++c->launches;
    prof_end(c);
  } else if (n.rfind("matmul", 0) == 0) {
    // [a, bt, out(, bias)]: out[r, c] = a[r, :] . bt[c, :] (+ bias[c]) (kernels.metal:306-321,
    // 392-487).  The rows each name covers follow from its grid as in the reference:
    // matmul_f32 / matmul_bias_f32 take 4 rows per threadgroup per output column starting at
    // row n; the tiled and chunk32 forms take 8 rows per threadgroup per 32 columns from 0.
    const bool bias = n == "matmul_bias_f32" || n == "matmul_bias_f32_chunk32";
    const bool tiles = n == "matmul_f32_tiled" || n == "matmul_f32_chunk32" ||
                       n == "matmul_bias_f32_chunk32";
    if (!bias && !tiles && n != "matmul_f32") return fail(c, TX_EINVAL, "unknown kernel name");
    if (count != (bias ? 4u : 3u) || !pr.rows || !pr.cols || !pr.k || threads % group)
      return fail(c, TX_EINVAL, "matmul: bad arguments");
    const uint64_t groups = threads / group;
    uint64_t row0 = 0, row_end = 0;
    if (tiles) {
      if (pr.cols % 32) return fail(c, TX_EINVAL, "matmul: tiled forms need cols % 32 == 0");
      const uint64_t per = pr.cols / 32;
      row_end = std::min<uint64_t>(pr.rows, 8 * ((groups + per - 1) / per));
    } else {
      row0 = pr.n;
      row_end = std::min<uint64_t>(pr.rows, row0 + 4 * ((groups + pr.cols - 1) / pr.cols));
    }
    if (b[0]->size < (uint64_t)pr.rows * pr.k * 4 || b[1]->size < (uint64_t)pr.cols * pr.k * 4 ||
        b[2]->size < (uint64_t)pr.rows * pr.cols * 4 || (bias && b[3]->size < pr.cols * 4u))
      return fail(c, TX_EINVAL, "matmul: buffer too small");
    prof_begin(c);
    e = tx::launch_matmul_f32((const float *)b[0]->dev, (const float *)b[1]->dev,
                              bias ? (const float *)b[3]->dev : nullptr, (float *)b[2]->dev,
                              (uint32_t)row0, (uint32_t)row_end, pr.cols, pr.k, c->stream);
    if (e == cudaSuccess) ++c->launches;
    prof_end(c);
  } else if (n == "qk_norm_rope") {
    // buffers: q, k (f32, in place), q_norm weight, k_norm weight (bf16); n = tokens
    if (count != 4 || !pr.heads || !pr.kv_heads || !pr.seq)
      return fail(c, TX_EINVAL, "qk_norm_rope: bad arguments");
    if (!(pr.dim == 32 || pr.dim == 64 || pr.dim == 128 || pr.dim == 256))
      return fail(c, TX_EINVAL, "qk_norm_rope: head_dim 32, 64, 128 or 256");
    uint64_t qbytes = (uint64_t)pr.n * pr.heads * pr.dim * 4;
    uint64_t kbytes = (uint64_t)pr.n * pr.kv_heads * pr.dim * 4;
    if (b[0]->size < qbytes || b[1]->size < kbytes || b[2]->size < pr.dim * 2u ||
        b[3]->size < pr.dim * 2u)
      return fail(c, TX_EINVAL, "qk_norm_rope: buffer too small");
    tx::PrologueProblem pp{};
    pp.q = b[0]->dev; pp.k = b[1]->dev; pp.q_out = b[0]->dev; pp.k_out = b[1]->dev;
    pp.tokens = pr.n; pp.seq = pr.seq; pp.heads = pr.heads; pp.kv_heads = pr.kv_heads;
    pp.dim = pr.dim; pp.in_dtype = TX_F32; pp.out_dtype = TX_F32;
    pp.q_w = (const uint16_t *)b[2]->dev; pp.k_w = (const uint16_t *)b[3]->dev;
    pp.eps = pr.eps; pp.theta = pr.theta;
    prof_begin(c);
    e = tx::launch_qk_norm_rope(pp, c->stream);
    if (e == cudaSuccess) ++c->launches;
    prof_end(c);
  } else {
    return fail(c, TX_EINVAL, "unknown kernel name");
  }
  if (e != cudaSuccess) return cuda_fail(c, e, "launch");
  return TX_OK;
}

int tx_finish(void *ctx) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!c->open) return fail(c, TX_EINVAL, "no open command");
  cudaSetDevice(c->device);
  c->open = false;
  c->last_gpu = -1.0;
  cudaError_t e = cudaEventRecord(c->ev_end, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(c, e, "command");
  int rc = check_status(c);
  if (rc) return rc;
  float ms = 0.f;
  if (cudaEventElapsedTime(&ms, c->ev_begin, c->ev_end) == cudaSuccess) c->last_gpu = ms * 1e-3;
  if (c->profile) {
    for (size_t i = 0; i + 1 < c->prof_used; i += 2) {
      float t = 0.f;
      if (cudaEventElapsedTime(&t, c->prof_events[i], c->prof_events[i + 1]) != cudaSuccess) {
        c->prof_seconds.clear();
        return fail(c, TX_ECUDA, "profile timing");
      }
      c->prof_seconds.push_back(t * 1e-3);
    }
  }
  return TX_OK;
}

void tx_abort(void *ctx) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  cudaGetLastError();
  c->open = false;
  c->prof_used = 0;
}

double tx_gpu_seconds(void *ctx) { return ctx ? ((Ctx *)ctx)->last_gpu : -1.0; }

int tx_profile_enable(void *ctx, int enabled) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (c->open) return fail(c, TX_EINVAL, "command open");
  c->profile = enabled != 0;
  c->prof_used = 0;
  c->prof_seconds.clear();
  return TX_OK;
}

int tx_kernel_timing(void *ctx, int enabled) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  c->ktime = enabled != 0;
  c->kt_n = 0;
  return TX_OK;
}

int tx_kernel_times(void *ctx, double *seconds, uint32_t cap, uint32_t *count) {
  Ctx *c = (Ctx *)ctx;
  if (!c || !count) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  const uint32_t n = (uint32_t)c->kt_n / 2;
  *count = n;
  if (n > cap || (n && !seconds)) return fail(c, TX_EINVAL, "kernel times: capacity");
  if (!n) return TX_OK;
  cudaError_t e = cudaEventSynchronize(c->kt_ev[2 * n - 1]);
  if (e != cudaSuccess) return cuda_fail(c, e, "kernel times");
  for (uint32_t i = 0; i < n; ++i) {
    float ms = 0.f;
    if ((e = cudaEventElapsedTime(&ms, c->kt_ev[2 * i], c->kt_ev[2 * i + 1])) != cudaSuccess)
      return cuda_fail(c, e, "kernel times");
    seconds[i] = ms * 1e-3;
  }
  return TX_OK;
}

int tx_profile_read(void *ctx, double *seconds, uint32_t count) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (c->open || count != c->prof_seconds.size()) return fail(c, TX_EINVAL, "profile count");
  if (count) memcpy(seconds, c->prof_seconds.data(), count * sizeof(double));
  return TX_OK;
}

int tx_attention_padded(void *ctx, const void *q, const void *k, const void *v,
                        const uint32_t *lengths, const uint32_t *lengths_host, void *out,
                        uint32_t batch, uint32_t seq, uint32_t heads, uint32_t kv_heads,
                        uint32_t dim, int in_dtype, int out_dtype, int causal, float scale,
                        const uint16_t *q_norm_w, const uint16_t *k_norm_w, float eps,
                        float theta, void *stream) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  tx::AttnProblem p{};
  p.q = q; p.k = k; p.v = v; p.out = out; p.lengths = lengths; p.cu_seqlens = nullptr;
  p.batch = batch; p.seq = seq; p.heads = heads; p.kv_heads = kv_heads; p.dim = dim;
  p.in_dtype = in_dtype; p.out_dtype = out_dtype; p.causal = causal ? 1 : 0; p.scale = scale;
  if (!lengths) return fail(c, TX_EINVAL, "lengths required");
  if ((uint64_t)batch * seq > 0xffffffffull) return fail(c, TX_EINVAL, "too many tokens");
  return run_attention(c, p, lengths_host, nullptr, q_norm_w, k_norm_w, eps, theta,
                       stream ? (cudaStream_t)stream : c->stream);
}

int tx_attention_varlen(void *ctx, const void *q, const void *k, const void *v,
                        const int32_t *cu_seqlens, const int32_t *cu_seqlens_host, uint32_t nseq,
                        uint32_t total, uint32_t max_len, void *out, uint32_t heads,
                        uint32_t kv_heads, uint32_t dim, int in_dtype, int out_dtype, int causal,
                        float scale, const uint16_t *q_norm_w, const uint16_t *k_norm_w, float eps,
                        float theta, void *stream) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!cu_seqlens) return fail(c, TX_EINVAL, "cu_seqlens required");
  if (!max_len) return fail(c, TX_EINVAL, "max_len must be positive");
  tx::AttnProblem p{};
  p.q = q; p.k = k; p.v = v; p.out = out; p.lengths = nullptr; p.cu_seqlens = cu_seqlens;
  p.batch = nseq; p.seq = max_len; p.total = total; p.heads = heads; p.kv_heads = kv_heads;
  p.dim = dim; p.in_dtype = in_dtype; p.out_dtype = out_dtype; p.causal = causal ? 1 : 0;
  p.scale = scale;
  return run_attention(c, p, nullptr, cu_seqlens_host, q_norm_w, k_norm_w, eps, theta,
                       stream ? (cudaStream_t)stream : c->stream);
}

int tx_attention_padded_host(void *ctx, const void *q, const void *k, const void *v,
                             const uint32_t *lengths, void *out, uint32_t batch, uint32_t seq,
                             uint32_t heads, uint32_t kv_heads, uint32_t dim, int in_dtype,
                             int out_dtype, int causal, float scale, const uint16_t *q_norm_w,
                             const uint16_t *k_norm_w, float eps, float theta) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (c->open) return fail(c, TX_EINVAL, "a command is open");
  tx::AttnProblem p{};
  p.q = q; p.k = k; p.v = v; p.out = out;
  p.batch = batch; p.seq = seq; p.heads = heads; p.kv_heads = kv_heads; p.dim = dim;
  p.in_dtype = in_dtype; p.out_dtype = out_dtype; p.causal = causal ? 1 : 0; p.scale = scale;
  if (!lengths) return fail(c, TX_EINVAL, "lengths required");
  for (uint32_t b = 0; b < batch; ++b)
    if (lengths[b] > seq) return fail(c, TX_EINVAL, "length exceeds seq");
  return run_attention_host(c, p, lengths, nullptr, q_norm_w, k_norm_w, eps, theta);
}

int tx_attention_varlen_host(void *ctx, const void *q, const void *k, const void *v,
                             const int32_t *cu_seqlens, uint32_t nseq, uint32_t total, void *out,
                             uint32_t heads, uint32_t kv_heads, uint32_t dim, int in_dtype,
                             int out_dtype, int causal, float scale, const uint16_t *q_norm_w,
                             const uint16_t *k_norm_w, float eps, float theta) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (c->open) return fail(c, TX_EINVAL, "a command is open");
  if (!cu_seqlens) return fail(c, TX_EINVAL, "cu_seqlens required");
  tx::AttnProblem p{};
  p.q = q; p.k = k; p.v = v; p.out = out;
  p.batch = nseq; p.total = total; p.heads = heads; p.kv_heads = kv_heads; p.dim = dim;
  p.in_dtype = in_dtype; p.out_dtype = out_dtype; p.causal = causal ? 1 : 0; p.scale = scale;
  return run_attention_host(c, p, nullptr, cu_seqlens, q_norm_w, k_norm_w, eps, theta);
}

int tx_qk_norm_rope(void *ctx, const void *q, const void *k, void *q_out, void *k_out,
                    uint32_t tokens, uint32_t seq, const int32_t *cu_seqlens, uint32_t nseq,
                    const uint32_t *lengths, uint32_t heads, uint32_t kv_heads, uint32_t dim,
                    int in_dtype, int out_dtype, const uint16_t *q_norm_w,
                    const uint16_t *k_norm_w, float eps, float theta, void *stream) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!q && !k) return fail(c, TX_EINVAL, "q or k required");
  if ((q && (!q_out || !q_norm_w)) || (k && (!k_out || !k_norm_w)))
    return fail(c, TX_EINVAL, "null pointer");
  if (!(dim == 32 || dim == 64 || dim == 128 || dim == 256))
    return fail(c, TX_EINVAL, "head_dim 32, 64, 128 or 256");
  if (!heads || !kv_heads) return fail(c, TX_EINVAL, "heads must be positive");
  if (!cu_seqlens && !seq) return fail(c, TX_EINVAL, "seq must be positive");
  if (cu_seqlens && !nseq) return fail(c, TX_EINVAL, "nseq must be positive");
  if (cu_seqlens && lengths) return fail(c, TX_EINVAL, "lengths apply to the padded layout");
  if ((in_dtype != TX_F32 && in_dtype != TX_BF16) || (out_dtype != TX_F32 && out_dtype != TX_BF16))
    return fail(c, TX_EINVAL, "bad dtype");
  if (in_dtype != out_dtype && ((q && q == q_out) || (k && k == k_out)))
    return fail(c, TX_EINVAL, "in-place prologue needs equal dtypes");
  tx::PrologueProblem pp{};
  pp.q = q; pp.k = k; pp.q_out = q_out; pp.k_out = k_out; pp.tokens = tokens; pp.seq = seq;
  pp.cu_seqlens = cu_seqlens; pp.nseq = nseq; pp.heads = heads; pp.kv_heads = kv_heads;
  pp.dim = dim; pp.in_dtype = in_dtype; pp.out_dtype = out_dtype; pp.q_w = q_norm_w;
  pp.k_w = k_norm_w; pp.eps = eps; pp.theta = theta; pp.lengths = lengths;
  cudaSetDevice(c->device);

  cudaError_t e = tx::launch_qk_norm_rope(pp, stream ? (cudaStream_t)stream : c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "prologue launch");
  ++c->launches;
  return TX_OK;
}

int tx_pool_project(void *ctx, const void *x, int in_dtype, const uint32_t *lengths,
                    const int32_t *cu_seqlens, float *out, uint32_t batch, uint32_t seq,
                    uint32_t cols, uint32_t dim, int first_token, const uint16_t *norm_w,
                    float eps, void *stream) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!x || !out) return fail(c, TX_EINVAL, "null pointer");
  if (!lengths == !cu_seqlens) return fail(c, TX_EINVAL, "exactly one of lengths, cu_seqlens");
  if (in_dtype != TX_F32 && in_dtype != TX_BF16) return fail(c, TX_EINVAL, "bad dtype");
  if (!dim || dim > cols) return fail(c, TX_EINVAL, "need 0 < dim <= cols");
  if (lengths && !seq) return fail(c, TX_EINVAL, "seq must be positive");
  if (!(eps >= 0.f)) return fail(c, TX_EINVAL, "eps must be >= 0");
  if (!batch) return TX_OK;
  tx::PoolProblem p{};
  p.x = x; p.in_dtype = in_dtype; p.lengths = lengths; p.cu_seqlens = cu_seqlens; p.out = out;
  p.batch = batch; p.seq = seq; p.cols = cols; p.dim = dim; p.first_token = first_token ? 1 : 0;
  p.norm_w = norm_w; p.eps = eps;
  cudaSetDevice(c->device);
  cudaError_t e = tx::launch_pool_project(p, stream ? (cudaStream_t)stream : c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "pool launch");
  c->last_kernel = "pool_project";
  ++c->launches;
  return TX_OK;
}

int tx_dequant4(void *ctx, const uint32_t *packed, const uint16_t *scales,
                const uint16_t *biases, uint16_t *out, uint16_t *out_lo, uint32_t rows,
                uint32_t cols, void *stream) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!packed || !scales || !biases || !out) return fail(c, TX_EINVAL, "null pointer");
  if (!rows || !cols || cols % 64 || (uintptr_t)out % 16 || (uintptr_t)out_lo % 16 ||
      (uintptr_t)packed % 4)
    return fail(c, TX_EINVAL, "dequant4: cols % 64 == 0, aligned pointers");
  cudaSetDevice(c->device);
  cudaError_t e = tx::launch_dequant4(packed, scales, biases, out, out_lo, rows, cols,
                                      stream ? (cudaStream_t)stream : c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "dequant4 launch");
  ++c->launches;
  return TX_OK;
}

int tx_split_bf16(void *ctx, const float *x, uint16_t *out, uint64_t n, void *stream) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!x || !out) return fail(c, TX_EINVAL, "null pointer");
  cudaSetDevice(c->device);
  cudaError_t e = tx::launch_split_bf16(x, out, n, stream ? (cudaStream_t)stream : c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "split launch");
  ++c->launches;
  return TX_OK;
}

int tx_embedding4(void *ctx, const uint32_t *ids, uint32_t tokens, const uint32_t *packed,
                  const uint16_t *scales, const uint16_t *biases, float *out, uint32_t cols,
                  uint32_t vocab, void *stream) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!ids || !packed || !scales || !biases || !out) return fail(c, TX_EINVAL, "null pointer");
  if (!cols || cols % 64 || !vocab || (uintptr_t)out % 16)
    return fail(c, TX_EINVAL, "embedding4: cols % 64 == 0, vocab > 0");
  cudaSetDevice(c->device);
  cudaError_t e = tx::launch_embedding4(ids, tokens, packed, scales, biases, out, cols, vocab,
                                        c->status, stream ? (cudaStream_t)stream : c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "embedding4 launch");
  ++c->launches;
  return TX_OK;
}

int tx_rms_norm_rows(void *ctx, const float *x, const uint16_t *w, void *out, int out_dtype,
                     uint32_t rows, uint32_t cols, float eps, void *stream) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!x || !w || !out) return fail(c, TX_EINVAL, "null pointer");
  if (out_dtype != TX_F32 && out_dtype != TX_BF16 && out_dtype != TX_BF16X2)
    return fail(c, TX_EINVAL, "bad out_dtype");
  if (!cols || cols % 4 || (uintptr_t)x % 16 || (uintptr_t)out % 16 || (uintptr_t)w % 8 ||
      !(eps >= 0.f))
    return fail(c, TX_EINVAL, "rms_norm_rows: cols % 4 == 0, aligned pointers");
  cudaSetDevice(c->device);
  const int kind = out_dtype == TX_F32 ? 0 : out_dtype == TX_BF16 ? 1 : 2;
  cudaError_t e = tx::launch_rms_norm_rows(x, w, out, kind, rows, cols, eps,
                                           stream ? (cudaStream_t)stream : c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "rms_norm_rows launch");
  ++c->launches;
  return TX_OK;
}

int tx_linear(void *ctx, const void *x, const void *x_lo, const void *w, const void *w_lo,
              const float *bias, void *out, uint32_t m, uint32_t n, uint32_t k, int mode,
              int fmt, uint32_t part, void *stream) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!x || !w || !out) return fail(c, TX_EINVAL, "null pointer");
  if (!x_lo != !w_lo) return fail(c, TX_EINVAL, "linear: x_lo and w_lo go together");
  if (!m) return TX_OK;
  if (!tx::linear_supported(m, n, k, mode, fmt, part, x, w, out) || (uintptr_t)x_lo % 16 ||
      (uintptr_t)w_lo % 16 || (uintptr_t)bias % 16 || (bias && mode == TX_LINEAR_GATED_BF16))
    return fail(c, TX_EINVAL,
                "linear: n, part % 128 == 0, k % 64 (bf16) or 32 (f32), aligned pointers, mode");
  cudaSetDevice(c->device);
  cudaError_t e = tx::launch_linear(x, x_lo, w, w_lo, bias, out, m, n, k, mode, fmt, part,
                                    c->status, c->wait_cycles,
                                    stream ? (cudaStream_t)stream : c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "linear launch");
  c->last_kernel = fmt == TX_F32 ? "linear_tf32" : "linear";
  ++c->launches;
  return TX_OK;
}

int tx_split_tf32(void *ctx, const float *x, float *out, uint64_t n, void *stream) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!x || !out) return fail(c, TX_EINVAL, "null pointer");
  if (n % 4 || (uintptr_t)x % 16 || (uintptr_t)out % 16)
    return fail(c, TX_EINVAL, "split_tf32: n % 4 == 0, 16-byte aligned pointers");
  cudaSetDevice(c->device);
  cudaError_t e = tx::launch_split_tf32(x, out, n, stream ? (cudaStream_t)stream : c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "split_tf32 launch");
  ++c->launches;
  return TX_OK;
}

int tx_layer_norm_rows(void *ctx, const float *x, const float *w, const float *b, float *out,
                       void *pair, int split, uint32_t rows, uint32_t cols, float eps,
                       void *stream) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!x || !w || !b || !out) return fail(c, TX_EINVAL, "null pointer");
  if (!tx::bert_cols_ok(cols) || (pair && split != TX_F32 && split != TX_BF16X2) ||
      !(eps >= 0.f))
    return fail(c, TX_EINVAL, "layer_norm_rows: cols at most 1024, split format");
  cudaSetDevice(c->device);
  cudaError_t e = tx::launch_layer_norm_rows(x, w, b, out, pair, split, rows, cols, eps,
                                             stream ? (cudaStream_t)stream : c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "layer_norm_rows launch");
  ++c->launches;
  return TX_OK;
}

int tx_bert_embed(void *ctx, const uint32_t *ids, const int32_t *cu_seqlens, uint32_t nseq,
                  uint32_t seq, uint32_t tokens, const float *words, const float *positions,
                  const float *types, uint32_t vocab, uint32_t max_pos, const float *ln_w,
                  const float *ln_b, float eps, float *out, void *pair, int split, uint32_t cols,
                  void *stream) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  if (!ids || !words || !positions || !types || !ln_w || !ln_b || !out)
    return fail(c, TX_EINVAL, "null pointer");
  if (!tx::bert_cols_ok(cols) || !vocab || !max_pos || (cu_seqlens ? !nseq : !seq) ||
      (pair && split != TX_F32 && split != TX_BF16X2) || !(eps >= 0.f))
    return fail(c, TX_EINVAL, "bert_embed: bad arguments");
  tx::BertEmbedProblem p{};
  p.ids = ids; p.cu = cu_seqlens; p.nseq = nseq; p.seq = seq; p.tokens = tokens; p.cols = cols;
  p.vocab = vocab; p.max_pos = max_pos; p.words = words; p.positions = positions;
  p.types = types; p.ln_w = ln_w; p.ln_b = ln_b; p.eps = eps; p.out = out; p.pair = pair;
  p.split = split; p.status = c->status;
  cudaSetDevice(c->device);
  cudaError_t e = tx::launch_bert_embed(p, stream ? (cudaStream_t)stream : c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "bert_embed launch");
  ++c->launches;
  return TX_OK;
}

int tx_device_count(void) {
  int n = 0;
  return cudaGetDeviceCount(&n) == cudaSuccess && n > 0 ? n : 0;
}

int tx_sync(void *ctx, void *stream) {
  Ctx *c = (Ctx *)ctx;
  if (!c) return TX_EINVAL;
  std::lock_guard<std::recursive_mutex> g(c->mu);
  cudaSetDevice(c->device);
  cudaError_t e = cudaStreamSynchronize(stream ? (cudaStream_t)stream : c->stream);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(c, e, "sync");
  return check_status(c);
}

}  // extern "C"
