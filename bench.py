#!/usr/bin/env python
"""Benchmark of the encoder-attention hot path on B200 (one process per GPU).

One step = one pass of the hot path over one batch of synthetic input.  Workloads
(--workload), each restating one of the benchmark configurations with seeded data:

  qwen_padded  (default) Qwen3-Embedding-0.6B attention layer: 32 sequences per GPU,
               right-padded to L=512, lengths ~ U[32, 512], 16 query / 8 kv heads,
               head_dim 128, causal, q/k RMSNorm (eps 1e-6, bf16 weights 1+N(0,0.02)) +
               RoPE (theta 1e6), bf16 N(0,1) inputs, fp32 softmax/accumulation, fp32 out.
               Step = the k prologue kernel (RMSNorm + RoPE of the valid k rows) + the
               tcgen05 attention kernel, which applies the q RMSNorm + RoPE to each Q tile
               in shared memory.  Weak scaling: 32*N sequences over N GPUs.
  qwen_f32     the qwen_padded batch with float32 q/k/v (the reference adapter's float
               buffers, qwen3.py:238-245): step = one q/k RMSNorm + RoPE launch (fp32, into
               scratch) + the fp32 head_dim-128 attention (tensor-core TF32 split-operand
               scores, FP32-pipe softmax and P.V).
  qwen_varlen  the same layer on 256 sequences packed by cu_seqlens (no padding), lengths
               log-normal (median 96, sigma 0.8) clipped to [2, 512].  The 256 sequences
               are split across the N GPUs: strong scaling.
  bge          BGE-small attention block: batch 4, L=128, 12 heads x 32, bidirectional,
               fp32 N(0,1)/sqrt(32), lengths ~ U[16, 128] (3 MB: a latency figure).
  bge_scaled   the same distribution at batch 4096 per GPU (2.5 GB of contract bytes), the
               bandwidth figure of the head_dim-32 kernel.
  tails_qwen / tails_bge
               short-sequence tails: 32 sequences of length U[2, 32], packed, bf16 N(0,1),
               Qwen shape (with the q/k prologue) or BGE shape (bidirectional).  The Qwen
               step is one launch of the short-sequence kernel, q/k prologue included.
  pool_qwen    the step after the last layer: final hidden states [32, 512, 1024] fp32 per
               GPU, lengths ~ U[32, 512]; the final RMSNorm of the last valid token of
               each sequence fused with last-token pooling and L2 normalisation
               (metric: sequences/s; a latency figure, 32 rows of 4 KB).
  qwen_forward the whole Qwen3-0.6B embedding forward around the attention: 28 layers,
               uint4 random weights (seed 9; scales N(0,0.02), biases N(0,0.01)), 32 texts
               per GPU of U[32, 512] random token ids (seed 5), packed, last-token pooling,
               1024-d L2-normalised output (metric: texts/s; weak scaling, 32 per GPU).
  bge_forward  the whole BGE-small (BERT) fp32 embedding forward around the head_dim-32
               attention: 12 layers, random fp32 weights (seed 11), 256 texts per GPU of
               U[16, 128] random token ids (seed 1), packed, CLS pooling, 384-d output;
               projections on TF32 tensor cores with split operands (fp32 accuracy).

Multi-GPU (torchrun, N ranks): sequences are assigned to ranks longest-first; shards are
independent, so there is no collective on the data path (torch.distributed is used only
for the barrier and the max-over-ranks of the timings).

Timing: W untimed warm-up steps, then K steps bracketed by barrier + synchronize; each
step is timed with CUDA events on the launching stream and L2 is flushed (256 MiB
write) between steps, outside the events.  value = valid tokens of all ranks / max over
ranks of the summed step times.  e2e = the same metric through the public NumPy API
(tessery_b200.attention) with page-locked host inputs: H2D copies, kernels and the D2H
read of the output inside the timed region.

--impl reference: the reference's own CPU formula for this path (its float32 NumPy
attention, restated with the q/k prologue in oracle/), timed on the host cores; rank 0
only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "attention tokens/s at Qwen3-0.6B shape & % of bf16 TC peak, 1/2/4/8 B200"
WORKLOADS = ("qwen_padded", "qwen_f32", "qwen_varlen", "bge", "bge_scaled", "tails_qwen", "tails_bge",
             "pool_qwen", "qwen_forward", "bge_forward")
# FP32 FMA throughput of the SIMT cores: 148 SMs x 128 lanes x 2 flops x 1.965 GHz
# (nominal; packed f32x2 FMA doubles it).  Used for the head_dim-32 compute floor.
FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=WORKLOADS, default="qwen_padded")
    p.add_argument("--batch", type=int, default=4096,
                   help="per-GPU batch of bge_scaled (smaller for profiler captures)")
    p.add_argument("--e2e-steps", type=int, default=10)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--one-process", action="store_true",
                   help="drive --gpus devices from this one process through the sharded "
                        "entry points (tessery_b200.sharded) and report their e2e figure")
    p.add_argument("--soak-seconds", type=float, default=1.5,
                   help="step loop run under the clock sampler right before the timed region")
    return p.parse_args()


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def profile_traffic(workload: str) -> dict:
    """DRAM bytes per launch from ncu captures (profiles/traffic.json), per workload."""
    path = ROOT / "profiles" / "traffic.json"
    if path.exists():
        return json.loads(path.read_text()).get(workload, {})
    return {}


# ---- workloads ----------------------------------------------------------------------------
def make_workload(name: str, rank: int, world: int, scaled_batch: int = 4096):
    from tessery_b200 import workloads

    return workloads.benchmark_workload(name, rank, world, scaled_batch)


def scaling_of(name: str) -> str:
    return "strong" if name == "qwen_varlen" else "weak"


def metric_of(name: str) -> str:
    if name == "qwen_padded":
        return METRIC
    shape = "BGE-small d32" if "bge" in name else "Qwen3-0.6B"
    return f"attention tokens/s, {name} ({shape} shape)"


def config_block(name: str, w, world: int) -> dict:
    per_gpu = {"qwen_padded": 32, "qwen_f32": 32, "bge": 4, "bge_scaled": w.batch, "tails_qwen": 32,
               "tails_bge": 32}
    glob = 256 if name == "qwen_varlen" else per_gpu[name] * world
    cfg = {"workload": name, "global_batch": glob, "heads": w.heads, "kv_heads": w.kv_heads,
           "head_dim": w.dim, "causal": w.causal, "layout": w.layout,
           "input_dtype": w.in_dtype, "output_dtype": "f32",
           "parallelism": f"sequence shards x{world} (longest first), no collective"}
    if w.layout == "padded":
        cfg["seq_len"] = w.seq
    else:
        cfg["max_len"] = w.seq
    cfg["lengths"] = {"qwen_padded": "U[32,512] seed 2", "qwen_f32": "U[32,512] seed 2",
                      "qwen_varlen":
                      "lognormal(ln 96, 0.8) clip [2,512] seed 3", "bge": "U[16,128] seed 1",
                      "bge_scaled": "U[16,128] seed 1", "tails_qwen": "U[2,32] seed 4",
                      "tails_bge": "U[2,32] seed 4"}[name]
    if w.q_norm_weight is not None:
        cfg["prologue"] = "q/k RMSNorm eps 1e-6 + RoPE theta 1e6"
    contract = w.q.nbytes + w.k.nbytes + w.v.nbytes + w.q.size * 4
    cfg["l2"] = (f"flushed between timed steps (256 MiB write); contract bytes "
                 f"{contract / 1e6:.1f} MB per GPU")
    return cfg


# ---- clocks ------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9], strict=False):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "power_w_max": max(power), "samples": len(sm), "reasons": sorted(reasons)}


def physical_gpu(local_rank: int) -> int:
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        ids = [x.strip() for x in visible.split(",") if x.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


# ---- CPU formula (reference arm and cpu_baseline) ------------------------------------------
def cpu_formula(w, n_seqs: int):
    """The reference's float32 NumPy formula (q/k RMSNorm + RoPE when the workload has
    them, then attention) on the first n_seqs sequences of the workload; returns
    (seconds, valid tokens)."""
    import oracle
    from tessery_b200.workloads import from_bf16_bits

    widen = from_bf16_bits if w.in_dtype == "bf16" else (lambda a: a)
    n_seqs = min(n_seqs, w.batch)
    if w.layout == "padded":
        q, k, v = (widen(a[:n_seqs]) for a in (w.q, w.k, w.v))
        lengths = w.lengths[:n_seqs]
        tokens = int(np.minimum(lengths, w.seq).sum())
        start = time.perf_counter()
        if w.q_norm_weight is not None:
            pos = np.broadcast_to(np.arange(w.seq), (q.shape[0], w.seq))
            q, k = oracle.qk_norm_rope(q, k, w.q_norm_weight, w.k_norm_weight, w.eps, w.theta,
                                       pos, dtype=np.float32)
        oracle.attention_padded(q, k, v, lengths, w.causal, w.scale, dtype=np.float32)
    else:
        cu = w.cu_seqlens[: n_seqs + 1]
        end = int(cu[-1])
        q, k, v = (widen(a[:end]) for a in (w.q, w.k, w.v))
        tokens = end
        start = time.perf_counter()
        if w.q_norm_weight is not None:
            pos = np.concatenate([np.arange(cu[i + 1] - cu[i]) for i in range(n_seqs)])
            q, k = oracle.qk_norm_rope(q, k, w.q_norm_weight, w.k_norm_weight, w.eps, w.theta,
                                       pos, dtype=np.float32)
        oracle.attention_varlen(q, k, v, cu, w.causal, w.scale, dtype=np.float32)
    return time.perf_counter() - start, tokens


def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        counts = [i.get("num_threads", 0) for i in threadpool_info()]
        return max(counts) if counts else os.cpu_count() or 1
    except Exception:
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def sample_size(w, target_seconds: float) -> int:
    """Sequences of the workload that take about target_seconds through cpu_formula."""
    n0 = min(2, w.batch)
    seconds, _ = cpu_formula(w, n0)  # also warms BLAS
    return int(max(1, min(w.batch, target_seconds / max(seconds / n0, 1e-6))))


def one_core(run, target_seconds: float) -> dict:
    """`run(seconds) -> (value, sample)` with every BLAS pool limited to one thread."""
    try:
        from threadpoolctl import threadpool_limits
    except ImportError:
        return {"value": None, "cores": 1, "sample": "threadpoolctl missing"}
    with threadpool_limits(limits=1):
        value, sample = run(target_seconds)
    return {"value": value, "cores": 1, "sample": sample}


def host_cores() -> dict:
    try:
        affinity = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        affinity = None
    return {"os_cpu_count": os.cpu_count(), "affinity_cpus": affinity}


def cpu_baseline_run(w, target_seconds: float = 6.0) -> dict:
    n = sample_size(w, target_seconds)
    times = []
    for _ in range(2):
        seconds, tokens = cpu_formula(w, n)
        times.append(seconds)
    sec = min(times)
    prologue = ", q/k prologue included" if w.q_norm_weight is not None else ""

    def single(seconds_target):
        n1 = sample_size(w, seconds_target)
        s1, t1 = cpu_formula(w, n1)
        return t1 / s1, f"first {n1} sequences (valid tokens {t1}), one run"

    return {"value": tokens / sec, "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
            "sample": f"first {n} of {w.batch} sequences of the workload (valid tokens {tokens}),"
                      f" float32 NumPy{prologue}, best of 2",
            "cpu_model": cpu_model(), **host_cores(),
            "one_core": one_core(single, target_seconds / 2)}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    w = make_workload(args.workload, 0, world, args.batch)
    # Size each step so the run stays within a few minutes.
    n = sample_size(w, 1.0)
    for _ in range(args.warmup):
        cpu_formula(w, n)
    total, tokens = 0.0, 0
    for _ in range(args.steps):
        s, t = cpu_formula(w, n)
        total += s
        tokens += t
    value = tokens / total
    line = {"metric": metric_of(args.workload), "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
            "scaling": scaling_of(args.workload), "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": config_block(args.workload, w, world),
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cpu_threads(),
                             "kind": "port",
                             "sample": f"first {n} of {w.batch} sequences per step, float32 "
                                       "NumPy restatement of the reference formula",
                             "cpu_model": cpu_model()},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- GPU arm ------------------------------------------------------------------------------
def run_ours(args):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    from tessery_b200 import TX_BF16, TX_F32, CudaRuntime, attention
    from tessery_b200.host import pinned_copy, pinned_empty

    rt = CudaRuntime(local)
    name = args.workload
    w = make_workload(name, rank, world, args.batch)
    H, KV, D = w.heads, w.kv_heads, w.dim
    in_code = TX_BF16 if w.in_dtype == "bf16" else TX_F32
    dev = torch.device("cuda", local)

    def to_dev(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    q, k, v = to_dev(w.q), to_dev(w.k), to_dev(w.v)
    prologue = w.q_norm_weight is not None
    # fp32 inputs: the library normalises and rotates q and k in one launch of the general
    # prologue (into scratch), then runs the attention kernel on the results.
    f32_prologue = prologue and in_code == TX_F32
    if prologue:
        qw, kw = to_dev(w.q_norm_weight), to_dev(w.k_norm_weight)
    out = torch.empty(w.q.shape, dtype=torch.float32, device=dev)
    if w.layout == "padded":
        lengths = to_dev(w.lengths.astype(np.uint32).view(np.int32))
        lengths_host = w.lengths.astype(np.uint32)
        B, L = w.q.shape[:2]
    else:
        cu = to_dev(w.cu_seqlens.astype(np.int32))
        cu_host = w.cu_seqlens.astype(np.int32)
        nseq, total = w.batch, int(cu_host[-1])
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    # A dedicated stream: the legacy default stream has handle 0, which the library reads
    # as "use the context's own stream".
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream
    assert sptr != 0
    def attend():
        extra = {}
        if prologue:
            extra = dict(eps=w.eps, theta=w.theta, q_norm_weight=qw.data_ptr(),
                         k_norm_weight=kw.data_ptr())
        if w.layout == "padded":
            rt.attention_padded_device(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                       lengths.data_ptr(), out.data_ptr(), batch=B, seq=L,
                                       heads=H, kv_heads=KV, dim=D, in_dtype=in_code,
                                       out_dtype=TX_F32, causal=w.causal, scale=w.scale,
                                       lengths_host=lengths_host, stream=sptr, **extra)
        else:
            rt.attention_varlen_device(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                       cu.data_ptr(), out.data_ptr(), nseq=nseq, total=total,
                                       max_len=w.seq, heads=H, kv_heads=KV, dim=D,
                                       in_dtype=in_code, out_dtype=TX_F32, causal=w.causal,
                                       scale=w.scale, cu_seqlens_host=cu_host, stream=sptr,
                                       **extra)

    def step():
        # One library call: with both norm weights the library normalises and rotates the
        # valid k rows (one launch) and runs the attention kernel, which applies the q
        # prologue to each Q tile in shared memory, as a programmatic dependent of it
        # (sequences of at most 32 tokens: one launch of the short-sequence kernel with
        # the q and k prologue inside; fp32: one q/k prologue launch, then the attention).
        attend()

    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    kernel = rt.last_kernel()

    # Clock sampler: soak loop of the same step, then the timed region.
    sampler = ClockSampler(physical_gpu(local))
    sampler.start()
    t_end = time.perf_counter() + args.soak_seconds
    while time.perf_counter() < t_end:
        for _ in range(20):
            flush.zero_()
            step()
        torch.cuda.synchronize()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = rt.launch_count()
    wall0 = time.perf_counter()
    # The timed steps carry no event between the prologue and the attention launch: the
    # attention kernel is a programmatic dependent of the prologue and may start while it
    # drains, which an event in between would prevent.
    for i in range(args.steps):
        flush.zero_()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    if dist:
        dist.barrier()
    launches = rt.launch_count() - launches0
    clocks = sampler.stop()
    rt.sync(sptr)  # device status word (bounded-wait timeouts) must be clean

    # Per-kernel device times of the same call, from separate untimed steps with the
    # library's kernel timing on (an event pair around each launch, which also keeps the
    # attention kernel from starting before the prologue ends): the per-kernel rooflines,
    # not `value`.
    rt.kernel_timing(True)
    pro_ms, att_ms = [], []
    for i in range(args.steps):
        flush.zero_()
        step()
        times = rt.kernel_times()
        att_ms.append(times[-1] * 1e3)
        if len(times) > 1:
            pro_ms.append(times[0] * 1e3)
    rt.kernel_timing(False)
    torch.cuda.synchronize()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends, strict=True)]
    total_s = sum(step_ms) * 1e-3
    tokens = w.valid_tokens() * args.steps
    flops = w.useful_flops()
    local_stats = torch.tensor([total_s, float(tokens), float(flops)], dtype=torch.float64,
                               device=dev)
    if dist:
        mx = local_stats.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = local_stats.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        total_max, tokens_all = float(mx[0]), float(sm[1])
    else:
        total_max, tokens_all = total_s, float(tokens)
    value = tokens_all / total_max

    # e2e through the public NumPy API with page-locked host buffers.
    hq, hk, hv = pinned_copy(w.q), pinned_copy(w.k), pinned_copy(w.v)
    hout = pinned_empty(w.q.shape, np.float32)
    if w.layout == "padded":
        hsel = {"lengths": pinned_copy(w.lengths.astype(np.uint32))}
    else:
        hsel = {"cu_seqlens": pinned_copy(w.cu_seqlens.astype(np.int32))}
    hpro = {}
    if prologue:
        hpro = {"q_norm_weight": pinned_copy(w.q_norm_weight),
                "k_norm_weight": pinned_copy(w.k_norm_weight), "eps": w.eps, "theta": w.theta}

    def e2e_step():
        return attention(hq, hk, hv, causal=w.causal, scale=w.scale, runtime=rt, out=hout,
                         **hsel, **hpro)

    e2e_step()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        result = e2e_step()
    e2e_s = time.perf_counter() - t0
    # Bytes the library's copies moved in the last call (per step), both directions.
    h2d, d2h = rt.host_copy_bytes()
    first = int(w.seq_lengths[0])
    check = result[0, :first] if w.layout == "padded" else result[:first]
    assert np.isfinite(check).all()
    e2e_stats = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(e2e_stats, op=dist.ReduceOp.MAX)
    e2e_tokens_all = tokens_all / args.steps * args.e2e_steps
    e2e_value = e2e_tokens_all / float(e2e_stats[0])
    # The same calls with the workload's own (pageable) NumPy arrays and a library-owned
    # output, as a plain NumPy caller makes them.
    def pageable_step():
        return attention(w.q, w.k, w.v, causal=w.causal, scale=w.scale, runtime=rt, **{
            k_: np.asarray(v_) for k_, v_ in hsel.items()}, **hpro)

    pageable_step()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        pageable_step()
    pageable = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(pageable, op=dist.ReduceOp.MAX)
    pageable_value = e2e_tokens_all / float(pageable[0])

    roof, prologue_roof = rooflines(w, name, kernel, statistics.mean(att_ms) * 1e-3,
                                    statistics.mean(pro_ms) * 1e-3 if pro_ms else None,
                                    pro_qk=f32_prologue)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_run(w)

    if rank == 0:
        peaks = measured_peaks()
        line = {"metric": metric_of(name), "value": value, "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": 1e3 * total_max / args.steps, "higher_is_better": True,
                "scaling": scaling_of(name), "vs_baseline": None, "dtype": w.in_dtype,
                "data": f"synthetic (seeded, {w.in_dtype} inputs; lengths "
                        f"{config_block(name, w, world)['lengths']})",
                "config": config_block(name, w, world), "roofline": roof,
                "attention_ms": statistics.mean(att_ms),
                "useful_tflops_attention": flops / (statistics.mean(att_ms) * 1e-3) / 1e12,
                "tc_frac_of_dense_peak_incl_prologue": flops / (total_s / args.steps) / 1e12
                / peaks["bf16_tflops"],
                "route": kernel, "cpu_baseline": cpu,
                "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h, "steps": args.e2e_steps,
                        "path": "tessery_b200.attention (NumPy in/out, pinned host buffers)"},
                "e2e_pageable": {"value": pageable_value, "unit": "tokens/s",
                                 "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                                 "steps": args.e2e_steps,
                                 "path": "tessery_b200.attention (the workload's pageable "
                                         "NumPy arrays, library-owned output)"},
                "gpu_launches": launches, "wall_s_timed_region": wall, "clocks": clocks}
        if prologue_roof:
            line["prologue_roofline"] = prologue_roof
            line["prologue_ms"] = statistics.mean(pro_ms)
        line["kernel_timing"] = ("per-kernel times from separate steps of the same call with "
                                 "the library's kernel timing on (tx_kernel_times)")
        print(json.dumps(line), flush=True)
    rt.close()
    if dist:
        dist.destroy_process_group()


def rooflines(w, name: str, kernel: str, att_s: float, pro_s: float | None,
              pro_qk: bool = False):
    """Roofline of the attention launch and, when present, of the prologue launch (the
    k rows; pro_qk: every q and k row, the fp32 route).

    Algorithmic bytes of the attention launch (contract I/O): every q row (padded rows
    produce outputs too), the valid k and v rows, the fp32 output of every q row, the q
    norm weight when the q prologue is fused.  FLOPs: 4 * head_dim * heads per useful
    (query, key) pair of valid query rows.  The fp32 head_dim-128 kernel (f32_tc) does
    half of them (Q.K^T) on the tensor cores as three TF32 products and the other half
    (P.V) on the FP32 pipe: its compute floor is the larger of the two pipes' times.
    """
    peaks = measured_peaks()
    traffic = profile_traffic(name)
    esz = 2 if w.in_dtype == "bf16" else 4
    valid = w.valid_tokens()
    kv_valid_bytes = valid * w.kv_heads * w.dim * esz  # one of k or v
    fused_w = w.q_norm_weight.nbytes if w.q_norm_weight is not None else 0
    att_bytes = w.q.nbytes + 2 * kv_valid_bytes + w.q.size * 4 + fused_w
    flops = w.useful_flops()
    t_hbm = att_bytes / (peaks["hbm_gbs"] * 1e9)
    hbm = {"achieved": att_bytes / att_s / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
           "frac": att_bytes / att_s / 1e9 / peaks["hbm_gbs"],
           "algorithmic_bytes_per_launch": att_bytes}
    kname = {"tc_bf16_d128": "attn_tc_kernel", "d32": "attention_d32_kernel",
             "d32_tc": "attn_d32_tc_kernel", "simt": "attention_simt_kernel",
             "short_d128": "attn_short_kernel", "f32_tc": "attn_f32_tc_kernel"}.get(kernel,
                                                                                 kernel)
    if kernel == "f32_tc":
        tf32 = peaks["bf16_tflops"] / 2
        t_pv = flops / 2 / (FP32_NOMINAL_TFLOPS * 1e12)
        t_qk = 3 * flops / 2 / (tf32 * 1e12)
        t_c = max(t_pv, t_qk)
        comp = {"achieved": flops / 2 / att_s / 1e12, "peak": FP32_NOMINAL_TFLOPS,
                "unit": "TFLOP/s", "frac": t_pv / att_s,
                "algorithmic_flops_per_launch": flops / 2, "work": "P.V on the FP32 pipe",
                "peak_source": "nominal FP32 FMA, 148 SMs x 128 lanes x 2 x 1.965 GHz",
                "scores_floor_us": 1e6 * t_qk,
                "scores_peak": f"TF32 = measured bf16 burst / 2 ({tf32:.0f} TFLOP/s), "
                               "3 products"}
        comp_bound, comp_key = "fp32", "fp32"
        main = hbm if t_hbm >= t_c else comp
    elif kernel in ("tc_bf16_d128", "short_d128"):  # bf16 tensor-core contractions
        t_c = flops / (peaks["bf16_tflops"] * 1e12)
        comp = {"achieved": flops / att_s / 1e12, "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": flops / att_s / 1e12 / peaks["bf16_tflops"],
                "algorithmic_flops_per_launch": flops}
        comp_bound, comp_key = "tensor", "tensor"
    else:
        t_c = flops / (FP32_NOMINAL_TFLOPS * 1e12)
        comp = {"achieved": flops / att_s / 1e12, "peak": FP32_NOMINAL_TFLOPS,
                "unit": "TFLOP/s", "frac": flops / att_s / 1e12 / FP32_NOMINAL_TFLOPS,
                "algorithmic_flops_per_launch": flops,
                "peak_source": "nominal FP32 FMA, 148 SMs x 128 lanes x 2 x 1.965 GHz"}
        comp_bound, comp_key = "fp32", "fp32"
    if kernel != "f32_tc":
        main = hbm if t_hbm >= t_c or comp_bound == "fp32" else comp
    bound = "hbm" if main is hbm else comp_bound
    roof = {"bound": bound, "kernel": kname, "achieved": main["achieved"],
            "peak": main["peak"], "unit": main["unit"], "frac": main["frac"],
            "peak_source": f"{peaks['source']} (kernel timed alone: burst figures)",
            "traffic": traffic.get(kname), "hbm": hbm, comp_key: comp,
            "floor_us": {"hbm": 1e6 * t_hbm, comp_key: 1e6 * t_c},
            "launch_us": 1e6 * att_s}
    pro = None
    if pro_s is not None and pro_qk:
        pro_bytes = 2 * (w.q.nbytes + w.k.nbytes) + w.q_norm_weight.nbytes + w.k_norm_weight.nbytes
        pro = {"bound": "hbm", "kernel": "qk_norm_rope_kernel (every q and k row)",
               "achieved": pro_bytes / pro_s / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
               "frac": pro_bytes / pro_s / 1e9 / peaks["hbm_gbs"],
               "algorithmic_bytes_per_launch": pro_bytes,
               "traffic": traffic.get("qk_norm_rope_kernel"), "launch_us": 1e6 * pro_s}
    elif pro_s is not None:
        pro_bytes = 2 * kv_valid_bytes + w.k_norm_weight.nbytes
        pro = {"bound": "hbm", "kernel": "norm_rope_rows_bf16_kernel (k rows)",
               "achieved": pro_bytes / pro_s / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
               "frac": pro_bytes / pro_s / 1e9 / peaks["hbm_gbs"],
               "algorithmic_bytes_per_launch": pro_bytes,
               "traffic": traffic.get("norm_rope_rows_bf16_kernel"), "launch_us": 1e6 * pro_s}
    return roof, pro


# ---- pooling (the step after the last layer) --------------------------------------------
def pool_workload(rank: int):
    from tessery_b200.workloads import to_bf16_bits

    rng = np.random.default_rng(5 + 1000 * rank)
    b, seq, cols = 32, 512, 1024
    lengths = rng.integers(32, seq + 1, size=b).astype(np.uint32)
    x = rng.standard_normal(size=(b, seq, cols), dtype=np.float32)
    w = to_bf16_bits(1.0 + 0.02 * rng.standard_normal(cols).astype(np.float32))
    return x, lengths, w


def pool_config(world: int) -> dict:
    return {"workload": "pool_qwen", "global_batch": 32 * world, "seq_len": 512, "cols": 1024,
            "dim": 1024, "pooling": "last token", "final_norm": "RMSNorm eps 1e-6 fused",
            "lengths": "U[32,512] seed 5", "input_dtype": "f32",
            "parallelism": f"sequence shards x{world}, no collective",
            "l2": "flushed between timed steps (256 MiB write)"}


def pool_cpu(x, lengths, w, n: int):
    """The reference's order: rms_norm over every token (qwen3.py:281), then
    pool_project (kernels.metal:339-349), float32 NumPy; returns seconds."""
    import oracle

    start = time.perf_counter()
    normed = oracle.rms_norm(x[:n], w, 1e-6, dtype=np.float32)
    oracle.pool_project(normed, lengths[:n], x.shape[2], False, dtype=np.float32)
    return time.perf_counter() - start


def run_pool_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    x, lengths, w = pool_workload(0)
    n = x.shape[0]
    for _ in range(args.warmup):
        pool_cpu(x, lengths, w, n)
    total = sum(pool_cpu(x, lengths, w, n) for _ in range(args.steps))
    value = n * args.steps / total
    line = {"metric": "pooled embeddings/s (final RMSNorm + last-token pool + L2)",
            "value": value, "unit": "sequences/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": pool_config(1), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "sequences/s", "cores": cpu_threads(),
                             "kind": "port",
                             "sample": f"all {n} sequences per step: rms_norm of every token "
                                       "then pool_project, float32 NumPy",
                             "cpu_model": cpu_model()},
            "e2e": {"value": value, "unit": "sequences/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_pool(args):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    from tessery_b200 import CudaRuntime, pool_project
    from tessery_b200.host import pinned_copy, pinned_empty

    rt = CudaRuntime(local)
    x, lengths, w = pool_workload(rank)
    b, seq, cols = x.shape
    dev = torch.device("cuda", local)
    xd = torch.from_numpy(x).to(dev)
    ld = torch.from_numpy(lengths.view(np.int32)).to(dev)
    wd = torch.from_numpy(w.view(np.int16)).to(dev)
    out = torch.empty((b, cols), dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream
    assert sptr != 0

    def step():
        rt.pool_project_device(xd.data_ptr(), out.data_ptr(), batch=b, cols=cols, dim=cols,
                               seq=seq, lengths=ld.data_ptr(), norm_weight=wd.data_ptr(),
                               eps=1e-6, stream=sptr)

    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(physical_gpu(local))
    sampler.start()
    t_end = time.perf_counter() + args.soak_seconds
    while time.perf_counter() < t_end:
        for _ in range(20):
            flush.zero_()
            step()
        torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = rt.launch_count()
    for i in range(args.steps):
        flush.zero_()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    launches = rt.launch_count() - launches0
    clocks = sampler.stop()
    rt.sync(sptr)
    ms = [s.elapsed_time(e) for s, e in zip(starts, ends, strict=True)]
    total_s = sum(ms) * 1e-3
    stats = torch.tensor([total_s], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    value = b * world * args.steps / float(stats[0])

    hx, hl, hw = pinned_copy(x), pinned_copy(lengths), pinned_copy(w)
    hout = pinned_empty((b, cols), np.float32)

    def e2e_step():
        return pool_project(hx, lengths=hl, norm_weight=hw, eps=1e-6, runtime=rt, out=hout)

    e2e_step()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        result = e2e_step()
    e2e = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(e2e, op=dist.ReduceOp.MAX)
    assert np.isfinite(result).all()
    e2e_value = b * world * args.e2e_steps / float(e2e[0])

    peaks = measured_peaks()
    mean_s = statistics.mean(ms) * 1e-3
    nbytes = b * cols * 4 + w.nbytes + b * 4 + b * cols * 4  # picked rows, weight, lengths, out
    roof = {"bound": "hbm", "kernel": "pool_project_kernel",
            "achieved": nbytes / mean_s / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": nbytes / mean_s / 1e9 / peaks["hbm_gbs"],
            "algorithmic_bytes_per_launch": nbytes, "launch_us": 1e6 * mean_s,
            "peak_source": f"{peaks['source']} (kernel timed alone: burst figures)",
            "traffic": profile_traffic("pool_qwen").get("pool_project_kernel"),
            "note": "latency-bound: 32 rows of 4 KB per launch"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        times = [pool_cpu(x, lengths, w, b) for _ in range(3)]
        cpu = {"value": b / min(times), "unit": "sequences/s", "cores": cpu_threads(),
               "kind": "port", "sample": f"all {b} sequences: rms_norm of every token then "
                                        "pool_project, float32 NumPy, best of 3",
               "cpu_model": cpu_model()}
    if rank == 0:
        line = {"metric": "pooled embeddings/s (final RMSNorm + last-token pool + L2)",
                "value": value, "unit": "sequences/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": 1e3 * float(stats[0]) / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic (seeded N(0,1) fp32 hidden states)",
                "config": pool_config(world), "roofline": roof, "route": "pool_project",
                "cpu_baseline": cpu,
                "e2e": {"value": e2e_value, "unit": "sequences/s",
                        "h2d_bytes_per_step": hx.nbytes + hl.nbytes + hw.nbytes,
                        "d2h_bytes_per_step": result.nbytes, "steps": args.e2e_steps,
                        "path": "tessery_b200.pool_project (NumPy in/out, pinned host buffers)"},
                "gpu_launches": launches, "clocks": clocks}
        print(json.dumps(line), flush=True)
    rt.close()
    if dist:
        dist.destroy_process_group()


# ---- whole embedding forwards around the attention (Qwen3 and BGE-small) -----------------
FORWARD_METRIC = "Qwen3-0.6B embedding forward texts/s (28 layers, uint4 weights)"
BGE_FORWARD_METRIC = "BGE-small embedding forward texts/s (12 layers, fp32)"


class ForwardSpec:
    """One whole-forward benchmark: its texts, weights, model, CPU baseline and config."""

    def __init__(self, workload: str):
        self.workload = workload
        self.qwen = workload == "qwen_forward"
        self.metric = FORWARD_METRIC if self.qwen else BGE_FORWARD_METRIC
        self.per_rank = 32 if self.qwen else 256
        self.weight_seed = 9 if self.qwen else 11

    def cfg(self):
        if self.qwen:
            from tessery_b200.qwen3 import Qwen3Config

            return Qwen3Config()
        from tessery_b200.bert import BertConfig

        return BertConfig()

    def texts(self, rank: int, world: int):
        """per_rank texts per rank, assigned longest first over per_rank * world texts;
        Qwen: lengths U[32, 512] (seed 5); BGE: U[16, 128] (seed 1, the BGE attention
        configuration's distribution).  Random token ids (seed + 1000 * rank)."""
        from tessery_b200 import shard_sequences

        cfg = self.cfg()
        seed, lo, hi = (5, 32, 512) if self.qwen else (1, 16, 128)
        lengths = np.random.default_rng(seed).integers(lo, hi + 1, size=self.per_rank * world)
        owned = lengths[shard_sequences(lengths, world, causal=self.qwen)[rank]]
        rng = np.random.default_rng(seed + 1000 * rank)
        ids = rng.integers(0, cfg.vocab, size=(owned.size, int(owned.max())), dtype=np.int64)
        return cfg, ids, owned

    def weights(self, cfg):
        if self.qwen:
            from tessery_b200.qwen3 import random_weights
        else:
            from tessery_b200.bert import random_weights
        return random_weights(cfg, seed=self.weight_seed)

    def model(self, weights, cfg, rt):
        if self.qwen:
            from tessery_b200.qwen3 import Qwen3Encoder

            return Qwen3Encoder(weights, cfg, runtime=rt)
        from tessery_b200.bert import BertEncoder

        return BertEncoder(weights, cfg, runtime=rt)

    def enqueue(self, model, ids, cu, cu_host, pooled, stream):
        if self.qwen:
            model.enqueue(ids, cu, cu_host, pooled, model.cfg.hidden, stream=stream)
        else:
            model.enqueue(ids, cu, cu_host, pooled, stream=stream)

    def forward(self, model, ids, lengths):
        if self.qwen:
            return model.forward(ids, lengths, dimensions=model.cfg.hidden)
        return model.forward(ids, lengths)

    def cpu(self, weights, cfg, ids, lengths, n: int) -> float:
        """The reference's float32 forward restated (oracle/) on the first n texts; s."""
        import oracle.bert as ob
        import oracle.qwen3 as oq

        start = time.perf_counter()
        for i in range(n):
            one, ln = ids[i:i + 1, :lengths[i]], lengths[i:i + 1]
            if self.qwen:
                oq.qwen3_forward(weights, cfg, one, ln, cfg.hidden, dtype=np.float32)
            else:
                ob.bert_forward(weights, cfg, one, ln, dtype=np.float32)
        return time.perf_counter() - start

    def cpu_source(self) -> str:
        return ("float32 NumPy restatement of qwen3.py:112-296" if self.qwen
                else "float32 NumPy restatement of bert.py:104-235")

    def config(self, world: int) -> dict:
        if self.qwen:
            return {"workload": "qwen_forward", "global_batch": 32 * world,
                    "seq_len": "U[32,512]", "layers": 28, "hidden": 1024, "heads": 16,
                    "kv_heads": 8, "head_dim": 128, "intermediate": 3072, "vocab": 151669,
                    "weights": "uint4 random (seed 9)",
                    "pooling": "last token, L2-normalised 1024-d",
                    "layout": "packed (cu_seqlens)",
                    "parallelism": f"text shards x{world} (longest first), no collective",
                    "l2": "not flushed: per-step activations and weights exceed L2 (126 MB)"}
        return {"workload": "bge_forward", "global_batch": 256 * world, "seq_len": "U[16,128]",
                "layers": 12, "hidden": 384, "heads": 12, "head_dim": 32,
                "intermediate": 1536, "vocab": 30522,
                "weights": "fp32 random (seed 11; N(0, 0.02^2), LayerNorm 1 + N(0, 0.02^2))",
                "pooling": "CLS, L2-normalised 384-d", "layout": "packed (cu_seqlens)",
                "precision": "fp32 path: TF32 split operands, three products, chunked sums",
                "parallelism": f"text shards x{world} (longest first), no collective",
                "l2": "not flushed: per-step activations exceed L2 (126 MB)"}

    def roofline(self, flops: float, seconds: float) -> dict:
        peaks = measured_peaks()
        bf16 = peaks["bf16_tflops_sustained"] or peaks["bf16_tflops"]
        achieved = flops / seconds / 1e12
        if self.qwen:
            return {"bound": "tensor", "kernel": "whole forward (linear_kernel dominant)",
                    "achieved": achieved, "peak": bf16, "unit": "TFLOP/s",
                    "frac": achieved / bf16, "algorithmic_flops_per_step": flops,
                    "peak_source": f"{peaks['source']} sustained bf16 (a long multi-kernel "
                                   "step)", "traffic": None}
        # fp32 work on TF32 tensor cores: half the bf16 rate, three products per product.
        peak = bf16 / 2 / 3
        return {"bound": "tensor", "kernel": "whole forward (TF32 linear_kernel dominant)",
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "algorithmic_flops_per_step": flops,
                "peak_source": f"{peaks['source']} sustained bf16 / 2 (TF32 rate) / 3 (split "
                               "operands)", "traffic": None}


def run_forward_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    spec = ForwardSpec(args.workload)
    cfg, ids, lengths = spec.texts(0, world)
    weights = spec.weights(cfg)
    spec.cpu(weights, cfg, ids, lengths, 1)  # warm-up (BLAS threads, page-in)
    n = 2 if spec.qwen else 8  # texts per step: a bounded sample of the workload
    total = sum(spec.cpu(weights, cfg, ids, lengths, n) for _ in range(args.steps))
    value = n * args.steps / total
    sample = [int(v) for v in lengths[:n]]
    line = {"metric": spec.metric, "value": value, "unit": "texts/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": spec.config(world), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "texts/s", "cores": cpu_threads(),
                             **host_cores(), "kind": "port",
                             "sample": f"first {n} texts per step (lengths {sample}), "
                                       + spec.cpu_source(),
                             "cpu_model": cpu_model()},
            "e2e": {"value": value, "unit": "texts/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_forward(args):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    from tessery_b200 import CudaRuntime

    spec = ForwardSpec(args.workload)
    rt = CudaRuntime(local)
    cfg, ids, lengths = spec.texts(rank, world)
    weights = spec.weights(cfg)
    model = spec.model(weights, cfg, rt)
    dev = torch.device("cuda", local)
    cu_host = np.zeros(lengths.size + 1, np.int32)
    cu_host[1:] = np.cumsum(lengths)
    tokens = np.concatenate([ids[b, :lengths[b]] for b in range(lengths.size)]).astype(np.uint32)
    ids_d = torch.from_numpy(tokens.view(np.int32)).to(dev)
    cu_d = torch.from_numpy(cu_host).to(dev)
    pooled = torch.empty((lengths.size, cfg.hidden), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream

    def step():
        spec.enqueue(model, ids_d.data_ptr(), cu_d.data_ptr(), cu_host, pooled.data_ptr(), sptr)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(physical_gpu(local))
    sampler.start()
    t_end = time.perf_counter() + args.soak_seconds
    while time.perf_counter() < t_end:
        step()
        torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = rt.launch_count()
    for i in range(args.steps):
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    launches = rt.launch_count() - launches0
    clocks = sampler.stop()
    rt.sync(sptr)
    ms = [s.elapsed_time(e) for s, e in zip(starts, ends, strict=True)]
    stats = torch.tensor([sum(ms) * 1e-3], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    total_s = float(stats[0])
    value = lengths.size * world * args.steps / total_s

    # e2e through the encoder's forward: host token ids in, pooled rows back.
    spec.forward(model, ids, lengths)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        result = spec.forward(model, ids, lengths)
    e2e_stats = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(e2e_stats, op=dist.ReduceOp.MAX)
    e2e_value = lengths.size * world * args.e2e_steps / float(e2e_stats[0])
    assert np.allclose(np.linalg.norm(result, axis=1), 1.0, atol=1e-4)

    flops = model.flops(lengths)
    roof = spec.roofline(flops, statistics.mean(ms) * 1e-3)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        spec.cpu(weights, cfg, ids, lengths, 1)
        n = 4 if spec.qwen else 16
        sec = spec.cpu(weights, cfg, ids, lengths, n)
        sample = [int(v) for v in lengths[:n]]
        cpu = {"value": n / sec, "unit": "texts/s", "cores": cpu_threads(), **host_cores(),
               "kind": "port",
               "sample": f"first {n} of {lengths.size} texts (lengths {sample}), "
                         + spec.cpu_source(),
               "cpu_model": cpu_model()}
    if rank == 0:
        line = {"metric": spec.metric, "value": value, "unit": "texts/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": 1e3 * total_s / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16" if spec.qwen else "f32 (TF32 split operands)",
                "data": "synthetic (seeded random weights and token ids)",
                "config": spec.config(world), "roofline": roof,
                "tokens_per_s": int(lengths.sum()) * world * args.steps / total_s,
                "route": "linear_kernel + attn_tc_kernel + row kernels" if spec.qwen
                         else "linear_kernel (TF32) + attn_d32_tc_kernel + row kernels",
                "cpu_baseline": cpu,
                "e2e": {"value": e2e_value, "unit": "texts/s",
                        "h2d_bytes_per_step": int(lengths.sum()) * 4 + (lengths.size + 1) * 4,
                        "d2h_bytes_per_step": int(result.nbytes), "steps": args.e2e_steps,
                        "path": f"tessery_b200 {type(model).__name__}.forward (token ids in, "
                                "pooled rows out)"},
                "gpu_launches": launches, "clocks": clocks}
        print(json.dumps(line), flush=True)
    model.close()
    rt.close()
    if dist:
        dist.destroy_process_group()


def run_one_process(args):
    """The whole job of a workload through the one-process multi-GPU entry points: host
    arrays in, host results out, wall clock around synchronous calls (each call returns
    after its results are on the host).  qwen_padded: 32 sequences per device; qwen_varlen:
    the 256 sequences; qwen_forward: 32 texts per device, bge_forward: 256 texts per
    device, pooled rows back."""
    from tessery_b200.sharded import DeviceGroup, ShardedQwen3Encoder, attention_sharded
    from tessery_b200.workloads import benchmark_workload, qwen_padded

    n = args.gpus
    group = DeviceGroup(range(n))
    extra = {}
    if args.workload in ("qwen_forward", "bge_forward"):
        from tessery_b200.sharded import ShardedBertEncoder

        spec = ForwardSpec(args.workload)
        cfg = spec.cfg()
        seed, lo, hi = (5, 32, 512) if spec.qwen else (1, 16, 128)
        lengths = np.random.default_rng(seed).integers(lo, hi + 1, size=spec.per_rank * n)
        ids = np.random.default_rng(seed).integers(0, cfg.vocab, size=(lengths.size, hi))
        sharded = ShardedQwen3Encoder if spec.qwen else ShardedBertEncoder
        model = sharded(spec.weights(cfg), cfg, group=group)

        def step():
            return model.forward(ids, lengths)

        units, unit, metric = lengths.size, "texts/s", spec.metric
        h2d = int(lengths.sum()) * 4
        config = spec.config(n)
        extra["tokens"] = int(lengths.sum())
    elif args.workload in ("qwen_padded", "qwen_varlen"):
        if args.workload == "qwen_padded":
            lengths = np.random.default_rng(2).integers(32, 513, size=32 * n)
            w = qwen_padded(batch=lengths.size, seq=512, seed=2, lengths=lengths)
            sel = {"lengths": w.lengths}
        else:
            w = benchmark_workload("qwen_varlen", 0, 1)
            sel = {"cu_seqlens": w.cu_seqlens}
        model = None
        from tessery_b200.host import pinned_copy, pinned_empty

        # Page-locked inputs and output, as for the one-device e2e figure.
        hq, hk, hv = pinned_copy(w.q), pinned_copy(w.k), pinned_copy(w.v)
        hout = pinned_empty(w.q.shape, np.float32)
        kw = dict(group=group, causal=w.causal, scale=w.scale, q_norm_weight=w.q_norm_weight,
                  k_norm_weight=w.k_norm_weight, eps=w.eps, theta=w.theta, **sel)

        def step():
            return attention_sharded(hq, hk, hv, out=hout, **kw)

        def pageable_step():
            return attention_sharded(w.q, w.k, w.v, **kw)

        extra["pageable"] = pageable_step

        units, unit, metric = w.valid_tokens(), "tokens/s", metric_of(args.workload)
        h2d = 0  # counted by the library after the timed calls
        config = config_block(args.workload, w, n)
    else:
        raise SystemExit("--one-process takes qwen_padded, qwen_varlen, qwen_forward or "
                         "bge_forward")
    for _ in range(max(args.warmup, 3)):
        result = step()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        result = step()
    seconds = time.perf_counter() - t0
    value = units * args.e2e_steps / seconds
    if model is None:  # attention: the bytes every device's copies moved in the last step
        h2d = sum(rt_.host_copy_bytes()[0] for rt_ in group.runtimes)
    pageable = extra.pop("pageable", None)
    if pageable is not None:
        pageable()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            pageable()
        extra["e2e_pageable"] = {"value": units * args.e2e_steps / (time.perf_counter() - t0),
                                 "unit": unit, "path": "the workload's pageable NumPy arrays"}
    config = {**config, "parallelism": f"one process, {n} devices, shards longest first"}
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": n,
            "steps": args.e2e_steps, "warmup": max(args.warmup, 3),
            "ms_per_step": 1e3 * seconds / args.e2e_steps, "higher_is_better": True,
            "scaling": "weak" if args.workload.endswith("_forward") else scaling_of(args.workload),
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
            "config": config, "impl": "ours-one-process",
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": int(result.nbytes), "steps": args.e2e_steps,
                    "path": "tessery_b200.sharded (host arrays in, host results out; "
                            "page-locked for the attention workloads)"},
            "host_gbs": {"h2d": h2d / (seconds / args.e2e_steps) / 1e9,
                         "d2h": result.nbytes / (seconds / args.e2e_steps) / 1e9},
            **extra}
    print(json.dumps(line), flush=True)
    if model is not None:
        model.close()
    group.close()


def main():
    args = parse_args()
    if args.one_process:
        run_one_process(args)
        return
    if args.workload == "pool_qwen":
        run_pool_reference(args) if args.impl == "reference" else run_pool(args)
        return
    if args.workload in ("qwen_forward", "bge_forward"):
        run_forward_reference(args) if args.impl == "reference" else run_forward(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
