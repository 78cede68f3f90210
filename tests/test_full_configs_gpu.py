"""Every sequence of each benchmark configuration against the float64 oracle (needs a B200).

The inputs are exactly the ones bench.py times (tessery_b200.workloads.benchmark_workload,
rank 0 of 1): the padded Qwen batch (32 x 512, seed 2), the 256 packed log-normal
sequences (seed 3), the same padded batch in float32, the BGE batch (4 x 128, seed 1) and both short-tail batches (seed 4).
Each test prints the maximum and the 99.9th percentile of the absolute error, so the
margin to the gate is on record.

Gates: bf16 in / fp32 accumulate <= 2e-2 max abs against a float64 oracle fed the same
bf16 inputs (q/k RMSNorm + RoPE in float64); float32 <= 1e-4 max abs and the reference's
atol 2e-6 / rtol 2e-5.
"""

import numpy as np
import pytest

import oracle
from tessery_b200 import attention, workloads
from tessery_b200.workloads import from_bf16_bits

pytestmark = pytest.mark.gpu

BF16_GATE = 2e-2
F32_GATE, F32_ATOL, F32_RTOL = 1e-4, 2e-6, 2e-5


def oracle_of(w):
    q, k, v = (from_bf16_bits(a) if w.in_dtype == "bf16" else a for a in (w.q, w.k, w.v))
    if w.layout == "padded":
        b, L = q.shape[:2]
        pos = np.broadcast_to(np.arange(L), (b, L))
    else:
        cu = w.cu_seqlens
        pos = np.concatenate([np.arange(cu[i + 1] - cu[i]) for i in range(len(cu) - 1)])
    if w.q_norm_weight is not None:
        q, k = oracle.qk_norm_rope(q, k, w.q_norm_weight, w.k_norm_weight, w.eps, w.theta, pos)
    if w.layout == "padded":
        return oracle.attention_padded(q, k, v, w.lengths, w.causal, w.scale)
    return oracle.attention_varlen(q, k, v, w.cu_seqlens, w.causal, w.scale)


def run(rt, w):
    kw = dict(causal=w.causal, scale=w.scale, runtime=rt)
    if w.q_norm_weight is not None:
        kw.update(q_norm_weight=w.q_norm_weight, k_norm_weight=w.k_norm_weight, eps=w.eps,
                  theta=w.theta)
    if w.layout == "padded":
        return attention(w.q, w.k, w.v, lengths=w.lengths, **kw)
    return attention(w.q, w.k, w.v, cu_seqlens=w.cu_seqlens, **kw)


def report(name, got, want):
    err = np.abs(got.astype(np.float64) - want)
    mx, p999 = float(err.max()), float(np.quantile(err, 0.999))
    print(f"\nFULLCONFIG {name}: rows {got.shape[0] * (got.shape[1] if got.ndim == 4 else 1)}"
          f" max_abs {mx:.4g} p99.9 {p999:.4g}")
    return mx


@pytest.mark.parametrize("name,route", [("qwen_padded", "tc_bf16_d128"),
                                        ("qwen_varlen", "tc_bf16_d128"),
                                        ("tails_qwen", "short_d128")])
def test_qwen_benchmark_config_every_sequence(runtime, name, route):
    w = workloads.benchmark_workload(name)
    got = run(runtime, w)
    assert runtime.last_kernel() == route
    assert np.isfinite(got).all()
    assert report(name, got, oracle_of(w)) <= BF16_GATE


def test_qwen_f32_config_every_sequence(runtime):
    """The padded Qwen batch with float32 q/k/v (the reference adapter's float buffers):
    the fp32 prologue and the fp32 head_dim-128 kernel, every row against float64."""
    w = workloads.benchmark_workload("qwen_f32")
    got = run(runtime, w)
    assert runtime.last_kernel() == "f32_tc"
    assert np.isfinite(got).all()
    assert report("qwen_f32", got, oracle_of(w)) <= F32_GATE


@pytest.mark.parametrize("name", ["bge", "tails_bge"])
def test_bge_benchmark_config_every_sequence(runtime, name):
    w = workloads.benchmark_workload(name)
    got = run(runtime, w)
    # fp32 inputs take the tensor-core scores kernel, bf16 inputs the FP32-pipe one.
    assert runtime.last_kernel() == ("d32_tc" if w.in_dtype == "f32" else "d32")
    want = oracle_of(w)
    gate = F32_GATE if w.in_dtype == "f32" else BF16_GATE
    assert report(name, got, want) <= gate
    if w.in_dtype == "f32":
        np.testing.assert_allclose(got, want, atol=F32_ATOL, rtol=F32_RTOL)
