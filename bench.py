#!/usr/bin/env python
"""Benchmark of the encoder-attention hot path on B200 (one process per GPU).

Default workload (one step = one pass of the hot path over one batch):
  Qwen3-Embedding-0.6B attention layer: 32 sequences per GPU,
  right-padded to L=512, lengths ~ U[32, 512] (seeded), 16 query / 8 kv heads,
  head_dim 128, causal, q/k RMSNorm (eps 1e-6, bf16 weights 1+N(0,0.02)) + RoPE
  (theta 1e6), bf16 N(0,1) inputs, fp32 softmax/accumulation, fp32 output.
  One step = the k prologue kernel (RMSNorm + RoPE of the valid k rows) + the tcgen05
  attention kernel, which applies the q RMSNorm + RoPE to each Q tile in shared memory.

Multi-GPU (torchrun, N ranks): a global batch of 32*N sequences is split across ranks
by sequence (longest-processing-time first); shards are independent, so there is no
collective on the data path (torch.distributed is used only for the barrier and the
max-over-ranks of the timings).  Per-GPU work is fixed as N grows: scaling "weak".

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
SEQS_PER_GPU = 32
SEQ_LEN = 512
LENGTH_SEED = 2


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--e2e-steps", type=int, default=10)
    p.add_argument("--no-cpu-baseline", action="store_true")
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


def profile_traffic() -> dict | None:
    path = ROOT / "profiles" / "traffic.json"
    if path.exists():
        return json.loads(path.read_text())
    return None


def global_lengths(world: int) -> np.ndarray:
    rng = np.random.default_rng(LENGTH_SEED)
    return rng.integers(32, SEQ_LEN + 1, size=SEQS_PER_GPU * world)


def rank_workload(rank: int, world: int):
    from tessery_b200 import shard_sequences, workloads

    lengths = global_lengths(world)
    owned = shard_sequences(lengths, world, causal=True)[rank]
    return workloads.qwen_padded(batch=len(owned), seq=SEQ_LEN, seed=LENGTH_SEED + 1000 * rank,
                                 lengths=lengths[owned])


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
    """The reference's float32 NumPy formula (q/k RMSNorm + RoPE, then attention) on the
    first n_seqs sequences of the workload; returns (seconds, valid tokens)."""
    import oracle
    from tessery_b200.workloads import from_bf16_bits

    sel = slice(0, n_seqs)
    q, k, v = (from_bf16_bits(a[sel]) for a in (w.q, w.k, w.v))
    lengths = w.lengths[sel]
    start = time.perf_counter()
    pos = np.broadcast_to(np.arange(w.seq), (q.shape[0], w.seq))
    qn, kn = oracle.qk_norm_rope(q, k, w.q_norm_weight, w.k_norm_weight, w.eps, w.theta, pos,
                                 dtype=np.float32)
    oracle.attention_padded(qn, kn, v, lengths, True, w.scale, dtype=np.float32)
    return time.perf_counter() - start, int(np.minimum(lengths, w.seq).sum())


def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        counts = [i.get("num_threads", 0) for i in threadpool_info()]
        return max(counts) if counts else os.cpu_count() or 1
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline_run(w, target_seconds: float = 12.0) -> dict:
    seconds, tokens = cpu_formula(w, 2)  # warm BLAS, estimate
    per_seq = seconds / 2
    n = int(max(2, min(w.batch, target_seconds / max(per_seq, 1e-6) / 2)))
    times = []
    for _ in range(2):
        seconds, tokens = cpu_formula(w, n)
        times.append(seconds)
    sec = min(times)
    return {"value": tokens / sec, "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
            "sample": f"first {n} of {w.batch} sequences of the workload (valid tokens {tokens}),"
                      f" float32 NumPy, q/k prologue included, best of 2",
            "cpu_model": cpu_model()}


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def config_block(world: int) -> dict:
    return {"workload": "qwen3_0.6b_attention_padded_b32_l512", "global_batch": SEQS_PER_GPU * world,
            "seq_len": SEQ_LEN, "heads": 16, "kv_heads": 8, "head_dim": 128, "causal": True,
            "prologue": "q/k RMSNorm eps 1e-6 + RoPE theta 1e6",
            "lengths": "U[32,512] seeded", "parallelism": f"sequence shards x{world} (LPT), no collective",
            "l2": "flushed between timed steps (256 MiB write); inputs 134 MB > L2"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    w = rank_workload(0, 1)
    # Size each step so the run stays within a few minutes.
    sec2, _ = cpu_formula(w, 2)
    n = int(max(1, min(w.batch, 1.0 / max(sec2 / 2, 1e-6))))
    for _ in range(args.warmup):
        cpu_formula(w, n)
    total, tokens = 0.0, 0
    for _ in range(args.steps):
        s, t = cpu_formula(w, n)
        total += s
        tokens += t
    value = tokens / total
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": config_block(1), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cpu_threads(),
                             "kind": "port",
                             "sample": f"first {n} of 32 sequences per step, float32 NumPy "
                                       "restatement of the reference formula with q/k prologue",
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
    w = rank_workload(rank, world)
    B, L, H, KV, D = w.batch, w.seq, w.heads, w.kv_heads, w.dim
    dev = torch.device("cuda", local)

    def to_dev(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    q, k, v = to_dev(w.q), to_dev(w.k), to_dev(w.v)
    lengths = to_dev(w.lengths.astype(np.uint32).view(np.int32))
    qw, kw = to_dev(w.q_norm_weight), to_dev(w.k_norm_weight)
    kn = torch.empty_like(k)
    out = torch.empty((B, L, H, D), dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    # A dedicated stream: the legacy default stream has handle 0, which the library reads
    # as "use the context's own stream".
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream
    assert sptr != 0
    lengths_host = w.lengths.astype(np.uint32)

    def step():
        # k: RMSNorm + RoPE of the valid rows into kn (bf16); q: fused into the attention
        # kernel, which normalises and rotates each Q tile in shared memory.
        rt.qk_norm_rope_device(None, k.data_ptr(), None, kn.data_ptr(), tokens=B * L, seq=L,
                               heads=H, kv_heads=KV, dim=D, q_norm_weight=None,
                               k_norm_weight=kw.data_ptr(), lengths=lengths.data_ptr(),
                               in_dtype=TX_BF16, out_dtype=TX_BF16, eps=w.eps, theta=w.theta,
                               stream=sptr)
        mid.record(stream)
        rt.attention_padded_device(q.data_ptr(), kn.data_ptr(), v.data_ptr(),
                                   lengths.data_ptr(), out.data_ptr(), batch=B, seq=L, heads=H,
                                   kv_heads=KV, dim=D, in_dtype=TX_BF16, out_dtype=TX_F32,
                                   causal=True, scale=w.scale, lengths_host=lengths_host,
                                   q_norm_weight=qw.data_ptr(), eps=w.eps, theta=w.theta,
                                   stream=sptr)

    mid = torch.cuda.Event(enable_timing=True)
    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        step()
    torch.cuda.synchronize()

    # Clock sampler: soak loop of the same step, then the timed region.
    sampler = ClockSampler(physical_gpu(local))
    sampler.start()
    t_end = time.perf_counter() + args.soak_seconds
    while time.perf_counter() < t_end:
        for _ in range(20):
            step()
        torch.cuda.synchronize()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    mids = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = rt.launch_count()
    wall0 = time.perf_counter()
    for i in range(args.steps):
        flush.zero_()
        starts[i].record(stream)
        mid = mids[i]
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    if dist:
        dist.barrier()
    launches = rt.launch_count() - launches0
    clocks = sampler.stop()
    rt.sync(sptr)  # device status word (bounded-wait timeouts) must be clean

    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends, strict=True)]
    pro_ms = [s.elapsed_time(m) for s, m in zip(starts, mids, strict=True)]
    att_ms = [m.elapsed_time(e) for m, e in zip(mids, ends, strict=True)]
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
    hl = pinned_copy(w.lengths.astype(np.uint32))
    hqw, hkw = pinned_copy(w.q_norm_weight), pinned_copy(w.k_norm_weight)
    hout = pinned_empty(w.q.shape, np.float32)

    def e2e_step():
        return attention(hq, hk, hv, lengths=hl, causal=True, q_norm_weight=hqw,
                         k_norm_weight=hkw, eps=w.eps, theta=w.theta, runtime=rt, out=hout)

    e2e_step()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        result = e2e_step()
    e2e_s = time.perf_counter() - t0
    assert np.isfinite(result[0, : int(w.lengths[0])]).all()
    e2e_stats = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(e2e_stats, op=dist.ReduceOp.MAX)
    e2e_tokens_all = tokens_all / args.steps * args.e2e_steps
    e2e_value = e2e_tokens_all / float(e2e_stats[0])
    h2d = hq.nbytes + hk.nbytes + hv.nbytes + hl.nbytes + hqw.nbytes + hkw.nbytes
    d2h = result.nbytes

    peaks = measured_peaks()
    att_mean = statistics.mean(att_ms) * 1e-3
    pro_mean = statistics.mean(pro_ms) * 1e-3
    traffic = profile_traffic()
    valid = w.valid_tokens()
    kv_valid_bytes = valid * KV * D * 2  # one of k or v, valid rows, bf16
    # Contract I/O of the attention launch: every q row (padded rows are outputs too),
    # the valid k/v rows, the fp32 output of every row.
    att_bytes = w.q.nbytes + 2 * kv_valid_bytes + out.numel() * 4 + w.q_norm_weight.nbytes
    t_hbm = att_bytes / (peaks["hbm_gbs"] * 1e9)
    t_tc = flops / (peaks["bf16_tflops"] * 1e12)
    tensor = {"achieved": flops / att_mean / 1e12, "peak": peaks["bf16_tflops"],
              "unit": "TFLOP/s", "frac": flops / att_mean / 1e12 / peaks["bf16_tflops"],
              "algorithmic_flops_per_launch": flops}
    hbm = {"achieved": att_bytes / att_mean / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
           "frac": att_bytes / att_mean / 1e9 / peaks["hbm_gbs"],
           "algorithmic_bytes_per_launch": att_bytes}
    bound = "hbm" if t_hbm >= t_tc else "tensor"
    main = hbm if bound == "hbm" else tensor
    roof = {"bound": bound, "kernel": "attn_tc_kernel", "achieved": main["achieved"],
            "peak": main["peak"], "unit": main["unit"], "frac": main["frac"],
            "peak_source": f"{peaks['source']} (kernel timed alone: burst figures)",
            "traffic": traffic.get("attn_tc_kernel_bytes_per_launch") if traffic else None,
            "hbm": hbm, "tensor": tensor,
            "floor_us": {"hbm": 1e6 * t_hbm, "tensor": 1e6 * t_tc}}
    pro_bytes = 2 * kv_valid_bytes + w.k_norm_weight.nbytes
    prologue_roof = {"bound": "hbm", "kernel": "qk_norm_rope_kernel (k rows)",
                     "achieved": pro_bytes / pro_mean / 1e9, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": pro_bytes / pro_mean / 1e9 / peaks["hbm_gbs"],
                     "algorithmic_bytes_per_launch": pro_bytes,
                     "traffic": traffic.get("qk_norm_rope_bytes_per_launch") if traffic else None}
    achieved = tensor["achieved"]

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_run(w)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": 1e3 * total_max / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded N(0,1) bf16 q/k/v, lengths U[32,512])",
                "config": config_block(world), "roofline": roof, "prologue_roofline": prologue_roof,
                "attention_ms": 1e3 * att_mean, "prologue_ms": 1e3 * pro_mean,
                "useful_tflops_attention": achieved,
                "tc_frac_of_dense_peak_incl_prologue": flops / (total_s / args.steps) / 1e12
                / peaks["bf16_tflops"],
                "cpu_baseline": cpu,
                "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h, "steps": args.e2e_steps,
                        "path": "tessery_b200.attention (NumPy in/out, pinned host buffers)"},
                "gpu_launches": launches, "wall_s_timed_region": wall, "clocks": clocks}
        print(json.dumps(line), flush=True)
    rt.close()
    if dist:
        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
