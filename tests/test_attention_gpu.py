"""CUDA attention vs the oracle and the reference's golden vectors (needs a B200).

Tolerances (written here, per path):
  float32 kernels        : the reference's own gate, atol 2e-6 / rtol 2e-5 vs float64,
                           and <= 1e-4 max abs at the benchmark sizes.
  bf16 in / fp32 accum   : <= 2e-2 max abs vs a float64 oracle fed the same
                           bf16-rounded inputs (prologue computed in float64).
"""

import numpy as np
import pytest

import oracle
from golden_cases import compare, inputs_match, load_cases, regenerate
from tessery_b200 import (
    TX_BF16,
    TX_F32,
    InvalidInputError,
    attention,
    workloads,
)
from tessery_b200.workloads import from_bf16_bits, to_bf16_bits

pytestmark = pytest.mark.gpu

F32_ATOL, F32_RTOL = 2e-6, 2e-5
BF16_GATE = 2e-2
# Pooling and the BERT kernels (LayerNorm, embeddings, GELU, bias, f32 matmul) have their
# own golden tests (test_pool_gpu.py, test_bert_gpu.py).
CASES = [c for c in load_cases() if c.kernel not in (
    "pool_project", "layer_norm", "embedding_position", "gelu_f32", "add_bias", "matmul_f32")]


def run_reference_kernel(rt, case, inputs):
    """Runs a golden case through CudaRuntime._dispatch with the reference's kernel name
    and parameters, exactly as the reference test drives MetalRuntime."""
    arrays = [np.ascontiguousarray(a) for a in inputs.values()]
    buffers = [rt.buffer(a.nbytes, a) for a in arrays]
    try:
        if case.kernel == "rope":
            out = buffers[0]
        else:
            out = rt.buffer(int(np.prod(case.shape)) * 4)
            buffers.append(out)
        params = dict(case.dispatch)
        with rt.command():
            rt._dispatch(case.kernel, buffers, **params)
        return rt.read(out, case.shape)
    finally:
        for b in buffers:
            b.close()


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.id)
def test_reference_golden_case(runtime, case):
    inputs = regenerate(case)
    assert inputs_match(case, inputs)
    result = run_reference_kernel(runtime, case, inputs)
    # The reference's expected values at the recorded sample positions ...
    compare(case, result, rtol=F32_RTOL, atol=F32_ATOL)
    # ... and the full array against the oracle.
    from test_oracle_golden import run_oracle

    expected = run_oracle(case, inputs)
    np.testing.assert_allclose(result, expected, rtol=F32_RTOL, atol=F32_ATOL)


def test_attention_route_follows_head_dim(runtime):
    rng = np.random.default_rng(5)
    for dim, route in ((32, "d32_tc"), (64, "simt"), (128, "f32_tc")):
        q = rng.normal(size=(2, 40, 4, dim)).astype(np.float32)
        k = rng.normal(size=(2, 40, 2, dim)).astype(np.float32)
        v = rng.normal(size=k.shape).astype(np.float32)
        lengths = np.array([40, 17], np.uint32)
        bufs = [runtime.buffer(a.nbytes, a) for a in (q, k, v, lengths)]
        out = runtime.buffer(q.nbytes)
        with runtime.command():
            runtime._attention(bufs + [out], tokens=80, seq=40, heads=4, kv_heads=2, dim=dim,
                               bidirectional=1)
        assert runtime.last_kernel() == route
        got = runtime.read(out, q.shape)
        want = oracle.attention_padded(q, k, v, lengths, False, dim**-0.5)
        np.testing.assert_allclose(got, want, atol=F32_ATOL, rtol=F32_RTOL)
        for b in bufs + [out]:
            b.close()


# ---- BGE d32 fp32 ---------------------------------------------------------------------
def d32_route(runtime, batch, seq, heads=12):
    """fp32 head_dim 32: the tensor-core kernel (both products, TF32 splits) at any size."""
    return "d32_tc"


@pytest.mark.parametrize("batch,seq", [(4, 128), (3, 200), (2, 520), (30, 128)])
def test_bge_d32_fp32_device_route(runtime, batch, seq):
    """Device pointers: one launch, routed by its number of CTAs (d32_route)."""
    w = workloads.bge(batch=batch, seq=seq, seed=13, min_len=1)
    got = _padded_device_call(runtime, w.q, w.k, w.v, w.lengths, in_dtype=TX_F32,
                              causal=False, scale=w.scale)
    assert runtime.last_kernel() == d32_route(runtime, batch, seq)
    want = oracle.attention_padded(w.q, w.k, w.v, w.lengths, False, w.scale)
    np.testing.assert_allclose(got, want, atol=F32_ATOL, rtol=F32_RTOL)


@pytest.mark.parametrize("batch,seq", [(4, 128), (3, 200), (2, 520), (30, 128)])
def test_bge_d32_fp32_matches_oracle(runtime, batch, seq):
    w = workloads.bge(batch=batch, seq=seq, seed=11, min_len=1)
    w.lengths[0] = 1
    w.lengths[-1] = seq
    got = attention(w.q, w.k, w.v, lengths=w.lengths, causal=False, runtime=runtime)
    # Host arrays go through in chunks of whole sequences, routed chunk by chunk.
    assert runtime.last_kernel() in ("d32_tc", "d32")
    want = oracle.attention_padded(w.q, w.k, w.v, w.lengths, False, w.scale)
    np.testing.assert_allclose(got, want, atol=F32_ATOL, rtol=F32_RTOL)
    assert np.max(np.abs(got - want)) <= 1e-4


def test_bge_d32_causal_and_varlen(runtime):
    rng = np.random.default_rng(12)
    lengths = np.array([1, 5, 128, 129, 300], np.int64)
    cu = np.zeros(6, np.int32)
    cu[1:] = np.cumsum(lengths)
    total = int(cu[-1])
    q, k, v = [rng.normal(size=(total, 12, 32)).astype(np.float32) / np.float32(32**0.5)
               for _ in range(3)]
    for causal in (False, True):
        got = attention(q, k, v, cu_seqlens=cu, causal=causal, runtime=runtime)
        assert runtime.last_kernel() == "d32_tc"
        want = oracle.attention_varlen(q, k, v, cu, causal, 32**-0.5)
        np.testing.assert_allclose(got, want, atol=F32_ATOL, rtol=F32_RTOL)


# ---- head_dim 128 fp32 (tensor-core scores, TF32 split operands) ---------------------------
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("heads,kv_heads,seq,lengths", [
    (4, 2, 40, [40, 17]),
    (16, 8, 300, [300, 129, 1, 64, 0]),
    (6, 2, 257, [257, 256, 65, 16]),
    (2, 1, 700, [700, 333]),
])
def test_f32_d128_padded_matches_oracle(runtime, causal, heads, kv_heads, seq, lengths):
    """fp32 in and out, head_dim 128 (the Qwen3 adapter's float buffers): one launch of
    the tensor-core scores kernel; lengths that are not multiples of the 64-key tile or
    the 16-key chunk, query blocks past a sequence's end, GQA groups of 2 and 3, and a
    zero length (NaN rows, as the reference's sums give)."""
    rng = np.random.default_rng(seq + heads)
    B = len(lengths)
    lengths = np.array(lengths, np.uint32)
    q = rng.normal(size=(B, seq, heads, 128)).astype(np.float32)
    k, v = (rng.normal(size=(B, seq, kv_heads, 128)).astype(np.float32) for _ in range(2))
    got = _padded_device_call(runtime, q, k, v, lengths, in_dtype=TX_F32, causal=causal,
                              scale=128**-0.5)
    assert runtime.last_kernel() == "f32_tc"
    want = oracle.attention_padded(q, k, v, lengths, causal, 128**-0.5)
    empty = lengths == 0
    assert np.isnan(got[empty]).all()
    np.testing.assert_allclose(got[~empty], want[~empty], atol=F32_ATOL, rtol=F32_RTOL)


def test_f32_d128_varlen_and_large_logits(runtime):
    """Packed sequences, causal and not, with logits up to ~25 in size (the lazy rescale
    moves the reference maximum several times within a row).  At this size the fixed gate
    is beyond float32 arithmetic itself (the reference's formula evaluated in float32
    misses atol 2e-6 / rtol 2e-5 by 3x on ~450 elements), so the gate is that evaluation's
    own largest error: the kernel is at least as close to float64 as it."""
    rng = np.random.default_rng(81)
    lengths = np.array([1, 63, 64, 65, 200, 511], np.int64)
    cu = np.zeros(len(lengths) + 1, np.int32)
    cu[1:] = np.cumsum(lengths)
    total = int(cu[-1])
    q = rng.normal(size=(total, 8, 128)).astype(np.float32)
    k, v = (rng.normal(size=(total, 4, 128)).astype(np.float32) for _ in range(2))
    q *= np.linspace(0.2, 6.0, total, dtype=np.float32)[:, None, None]
    for causal in (False, True):
        got = attention(q, k, v, cu_seqlens=cu, causal=causal, runtime=runtime)
        assert runtime.last_kernel() == "f32_tc"
        want = oracle.attention_varlen(q, k, v, cu, causal, 128**-0.5)
        fp32 = oracle.attention_varlen(q, k, v, cu, causal, 128**-0.5, dtype=np.float32)
        assert np.max(np.abs(got - want)) <= np.max(np.abs(fp32 - want))


# ---- Qwen d128 bf16 (tensor cores) -------------------------------------------------------
def qwen_oracle(w, dtype=np.float64):
    q, k, v = (from_bf16_bits(a) for a in (w.q, w.k, w.v))
    if w.layout == "padded":
        b, L = q.shape[:2]
        pos = np.broadcast_to(np.arange(L), (b, L))
    else:
        cu = w.cu_seqlens
        pos = np.concatenate([np.arange(cu[i + 1] - cu[i]) for i in range(len(cu) - 1)])
    if w.q_norm_weight is not None:
        q, k = oracle.qk_norm_rope(q, k, w.q_norm_weight, w.k_norm_weight, w.eps, w.theta, pos,
                                   dtype)
    if w.layout == "padded":
        return oracle.attention_padded(q, k, v, w.lengths, w.causal, w.scale, dtype)
    return oracle.attention_varlen(q, k, v, w.cu_seqlens, w.causal, w.scale, dtype)


def run_workload(rt, w, out_dtype="float32", prologue=True):
    kw = dict(causal=w.causal, scale=w.scale, out_dtype=out_dtype, runtime=rt)
    if prologue and w.q_norm_weight is not None:
        kw.update(q_norm_weight=w.q_norm_weight, k_norm_weight=w.k_norm_weight, eps=w.eps,
                  theta=w.theta)
    if w.layout == "padded":
        return attention(w.q, w.k, w.v, lengths=w.lengths, **kw)
    return attention(w.q, w.k, w.v, cu_seqlens=w.cu_seqlens, **kw)


@pytest.mark.parametrize(
    "lengths,seq",
    [
        ([1, 127, 128, 129, 255, 256, 300, 512], 512),
        ([200, 1, 77, 130], 200),
        ([5, 64, 33], 64),
        ([700, 385], 700),
    ],
)
def test_qwen_padded_bf16_tensor_core(runtime, lengths, seq):
    w = workloads.qwen_padded(batch=len(lengths), seq=seq, seed=21, lengths=np.array(lengths))
    got = run_workload(runtime, w)
    assert runtime.last_kernel() == "tc_bf16_d128"
    want = qwen_oracle(w)
    err = np.max(np.abs(got - want))
    assert np.isfinite(got).all()
    assert err <= BF16_GATE, err


@pytest.mark.parametrize("weight", [1.0, 1.8, 2.1])
def test_qwen_norm_weights_around_the_score_bound(runtime, weight):
    """With both RMSNorm weights the kernel bounds every score by 128 max|w_q| max|w_k|
    scale log2(e) and, up to 64, takes one pass over each score tile with the fixed
    reference 0 (no row maximum); above it (weights of 1.9 and more here) the two-pass softmax
    with the lazily rescaled row maximum.  Both sides of the bound against the oracle, and
    the same inputs through the two-pass path (k normalised by a separate call, q weight
    only) agreeing with the one-pass result."""
    w = workloads.qwen_padded(batch=4, seq=384, seed=23, lengths=np.array([384, 200, 129, 7]))
    scale = np.float32(weight)
    w.q_norm_weight = to_bf16_bits(from_bf16_bits(w.q_norm_weight) * scale)
    w.k_norm_weight = to_bf16_bits(from_bf16_bits(w.k_norm_weight) * scale)
    got = run_workload(runtime, w)
    assert runtime.last_kernel() == "tc_bf16_d128"
    want = qwen_oracle(w)
    # Logits grow with the weights squared, and so do the effects of the bf16 roundings of
    # q, k and P: the gate scales with them.
    gate = BF16_GATE * max(1.0, weight) ** 2
    assert np.isfinite(got).all()
    assert np.max(np.abs(got - want)) <= gate
    # Two-pass route on the same numbers: k normalised and rotated first, then the
    # attention with the q weight only.
    kn = _padded_device_call_two_pass(runtime, w)
    assert np.max(np.abs(kn - want)) <= gate
    assert np.max(np.abs(kn - got)) <= gate


def _padded_device_call_two_pass(rt, w):
    B, L, H, D = w.q.shape
    bufs = {n: rt.buffer(a.nbytes, np.ascontiguousarray(a)) for n, a in
            (("q", w.q), ("k", w.k), ("v", w.v), ("len", w.lengths.astype(np.uint32)),
             ("qw", w.q_norm_weight), ("kw", w.k_norm_weight))}
    kn, out = rt.buffer(w.k.nbytes), rt.buffer(w.q.size * 4)
    try:
        rt.qk_norm_rope_device(None, bufs["k"].device_ptr, None, kn.device_ptr, tokens=B * L,
                               seq=L, heads=H, kv_heads=w.kv_heads, dim=D, q_norm_weight=None,
                               k_norm_weight=bufs["kw"].device_ptr, in_dtype=TX_BF16,
                               out_dtype=TX_BF16)
        rt.attention_padded_device(bufs["q"].device_ptr, kn.device_ptr, bufs["v"].device_ptr,
                                   bufs["len"].device_ptr, out.device_ptr, batch=B, seq=L,
                                   heads=H, kv_heads=w.kv_heads, dim=D, in_dtype=TX_BF16,
                                   out_dtype=TX_F32, causal=True, lengths_host=w.lengths,
                                   q_norm_weight=bufs["qw"].device_ptr)
        rt.sync()
        assert rt.last_kernel() == "tc_bf16_d128"
        return rt.read(out, w.q.shape)
    finally:
        for b in [*bufs.values(), kn, out]:
            b.close()


def test_kernel_times_follow_the_launches(runtime):
    """tx_kernel_times: one positive device time per kernel of the last typed call, in
    launch order (k prologue, then attention), none while timing is off."""
    w = workloads.qwen_padded(batch=2, seq=256, seed=27, lengths=np.array([256, 90]))
    B, L, H, D = w.q.shape
    rt = runtime
    bufs = {n: rt.buffer(a.nbytes, np.ascontiguousarray(a)) for n, a in
            (("q", w.q), ("k", w.k), ("v", w.v), ("len", w.lengths.astype(np.uint32)),
             ("qw", w.q_norm_weight), ("kw", w.k_norm_weight))}
    out = rt.buffer(w.q.size * 4)

    def call(**weights):
        rt.attention_padded_device(bufs["q"].device_ptr, bufs["k"].device_ptr,
                                   bufs["v"].device_ptr, bufs["len"].device_ptr, out.device_ptr,
                                   batch=B, seq=L, heads=H, kv_heads=w.kv_heads, dim=D,
                                   in_dtype=TX_BF16, out_dtype=TX_F32, causal=True,
                                   lengths_host=w.lengths, **weights)

    try:
        rt.kernel_timing(True)
        call(q_norm_weight=bufs["qw"].device_ptr, k_norm_weight=bufs["kw"].device_ptr)
        times = rt.kernel_times()
        assert len(times) == 2 and all(t > 0 for t in times)
        call()
        times = rt.kernel_times()
        assert len(times) == 1 and times[0] > 0
        rt.kernel_timing(False)
        call()
        rt.sync()
        assert rt.kernel_times() == []
    finally:
        rt.kernel_timing(False)
        for b in [*bufs.values(), out]:
            b.close()


def test_qwen_padded_bf16_out_and_no_prologue(runtime):
    w = workloads.qwen_padded(batch=3, seq=300, seed=22, lengths=np.array([300, 150, 9]))
    w.q_norm_weight = w.k_norm_weight = None  # attention only, no q/k prologue
    got = from_bf16_bits(run_workload(runtime, w, out_dtype="bf16"))
    assert runtime.last_kernel() == "tc_bf16_d128"
    assert np.max(np.abs(got - qwen_oracle(w))) <= BF16_GATE


@pytest.mark.parametrize("nseq,seed", [(7, 31), (40, 32)])
def test_qwen_varlen_bf16_tensor_core(runtime, nseq, seed):
    lengths = workloads.varlen_lengths(nseq, seed)
    lengths[0] = 1
    lengths[-1] = 512
    w = workloads.qwen_varlen(seed=seed, lengths=lengths)
    got = run_workload(runtime, w)
    assert runtime.last_kernel() == "tc_bf16_d128"
    want = qwen_oracle(w)
    assert np.max(np.abs(got - want)) <= BF16_GATE


def test_short_tails_both_shapes(runtime):
    for kind, route in (("qwen", "short_d128"), ("bge", "d32")):
        w = workloads.short_tails(kind, batch=32, seed=41)
        got = run_workload(runtime, w)
        assert runtime.last_kernel() == route
        want = qwen_oracle(w)
        assert np.max(np.abs(got - want)) <= BF16_GATE, kind


def _short_oracle(q, k, v, lengths, causal, qw, kw, eps=1e-6, theta=1e6):
    qf, kf, vf = (from_bf16_bits(a) for a in (q, k, v))
    if qw is not None:
        b, L = qf.shape[:2]
        pos = np.broadcast_to(np.arange(L), (b, L))
        qf, kf = oracle.qk_norm_rope(qf, kf, qw, kw, eps, theta, pos)
    return oracle.attention_padded(qf, kf, vf, lengths, causal, 128**-0.5)


@pytest.mark.parametrize("group", [1, 2, 4])
def test_short_sequence_kernel_padded(runtime, group):
    """Sequences of at most 32 tokens: the one-launch kernel with the q/k prologue inside,
    GQA groups 1/2/4, empty / single-token / full sequences and padded query rows, causal
    and bidirectional, with and without the prologue, fp32 and bf16 output.  A sequence
    with no valid key gives NaN rows (0/0), as the reference's running sums do."""
    rng = np.random.default_rng(60 + group)
    kv, L = 2, 32
    heads = kv * group
    lengths = np.array([0, 1, 2, 17, 31, 32], np.uint32)
    B = len(lengths)
    q = to_bf16_bits(rng.normal(size=(B, L, heads, 128)).astype(np.float32))
    k = to_bf16_bits(rng.normal(size=(B, L, kv, 128)).astype(np.float32))
    v = to_bf16_bits(rng.normal(size=(B, L, kv, 128)).astype(np.float32))
    qw = to_bf16_bits(1 + 0.02 * rng.normal(size=128).astype(np.float32))
    kw = to_bf16_bits(1 + 0.02 * rng.normal(size=128).astype(np.float32))
    for causal in (True, False):
        for pro in (True, False):
            extra = dict(q_norm_weight=qw, k_norm_weight=kw, eps=1e-6, theta=1e6) if pro else {}
            want = _short_oracle(q, k, v, lengths, causal, qw if pro else None, kw)
            for out_dtype in ("float32", "bf16"):
                got = attention(q, k, v, lengths=lengths, causal=causal, out_dtype=out_dtype,
                                runtime=runtime, **extra)
                assert runtime.last_kernel() == "short_d128"
                if out_dtype == "bf16":
                    got = from_bf16_bits(got)
                assert np.isnan(got[0]).all() and np.isfinite(got[1:]).all()
                assert np.max(np.abs(got[1:] - want[1:])) <= BF16_GATE, (causal, pro, out_dtype)


def test_short_sequence_kernel_varlen_matches_tensor_core(runtime):
    """Packed short sequences through the short kernel and, with one sequence made longer
    than 32, through the tensor-core kernel: the rows of the common sequences agree."""
    w = workloads.short_tails("qwen", batch=24, seed=43)
    got = run_workload(runtime, w)
    assert runtime.last_kernel() == "short_d128"
    assert np.max(np.abs(got - qwen_oracle(w))) <= BF16_GATE
    lengths = np.diff(w.cu_seqlens).astype(np.int64)
    long = workloads.short_tails("qwen", batch=24, seed=43)
    extra = 40
    cu = np.concatenate([[0], np.cumsum(np.append(lengths, extra))]).astype(np.int32)
    rng = np.random.default_rng(7)
    pad = lambda a: np.concatenate([a, to_bf16_bits(rng.normal(size=(extra,) + a.shape[1:])
                                                    .astype(np.float32))])
    long.q, long.k, long.v = pad(w.q), pad(w.k), pad(w.v)
    long.cu_seqlens, long.seq = cu, extra
    got_tc = run_workload(runtime, long)
    assert runtime.last_kernel() == "tc_bf16_d128"
    assert np.max(np.abs(got_tc[: got.shape[0]] - got)) <= BF16_GATE


def test_short_sequence_kernel_rejects_long_sequence_on_device(runtime):
    """max_len claims 32 but the device offsets hold a 40-token sequence and no host copy
    was given: the kernel's own check reports an invalid argument at the next sync (the
    over-long sequence is not touched), and the context stays usable."""
    rng = np.random.default_rng(9)
    total, heads, kv = 50, 4, 2
    cu = np.array([0, 10, 50], np.int32)
    arrays = {n: to_bf16_bits(rng.normal(size=(total, h, 128)).astype(np.float32))
              for n, h in (("q", heads), ("k", kv), ("v", kv))}
    bufs = {n: runtime.buffer(a.nbytes, np.ascontiguousarray(a)) for n, a in arrays.items()}
    cub = runtime.buffer(cu.nbytes, cu)
    out = runtime.buffer(total * heads * 128 * 4)
    try:
        runtime.attention_varlen_device(bufs["q"].device_ptr, bufs["k"].device_ptr,
                                        bufs["v"].device_ptr, cub.device_ptr, out.device_ptr,
                                        nseq=2, total=total, max_len=32, heads=heads, kv_heads=kv,
                                        dim=128, in_dtype=TX_BF16, out_dtype=TX_F32, causal=True)
        assert runtime.last_kernel() == "short_d128"
        with pytest.raises(InvalidInputError):
            runtime.sync()
        runtime.sync()  # cleared: the next call starts clean
    finally:
        for b in [*bufs.values(), cub, out]:
            b.close()


@pytest.mark.parametrize("out_dtype", ["float32", "bf16"])
def test_bge_d32_bf16_inputs(runtime, out_dtype):
    """bf16 inputs on the head_dim-32 kernel: rows are widened to fp32 as they are staged,
    so against the oracle on the same (bf16-valued) inputs only fp32 rounding remains for
    fp32 output; bf16 output adds one rounding of the result."""
    w = workloads.bge(batch=3, seq=200, seed=13, min_len=1)
    w.lengths[:] = [1, 200, 77]
    q, k, v = (to_bf16_bits(a) for a in (w.q, w.k, w.v))
    got = attention(q, k, v, lengths=w.lengths, causal=False, out_dtype=out_dtype,
                    runtime=runtime)
    assert runtime.last_kernel() == "d32"
    want = oracle.attention_padded(*(from_bf16_bits(a) for a in (q, k, v)), w.lengths, False,
                                   w.scale)
    if out_dtype == "bf16":
        got = from_bf16_bits(got)
        np.testing.assert_allclose(got, want, atol=1e-2, rtol=1e-2)
    else:
        np.testing.assert_allclose(got, want, atol=F32_ATOL, rtol=F32_RTOL)


def test_bidirectional_bf16_tensor_core(runtime):
    w = workloads.qwen_padded(batch=3, seq=260, seed=23, lengths=np.array([260, 100, 1]))
    w.causal = False
    got = run_workload(runtime, w)
    assert runtime.last_kernel() == "tc_bf16_d128"
    assert np.max(np.abs(got - qwen_oracle(w))) <= BF16_GATE


def test_extreme_logits_bf16_tensor_core(runtime):
    """The reference's extreme-logit patterns (+-1131 logits, masked 1e10 values) on
    the bf16 tensor-core path."""
    for case in [c for c in CASES if c.test.startswith("test_tiled_attention_extreme")]:
        inp = regenerate(case)
        k, v = inp["k"], inp["v"]
        causal = not case.dispatch["bidirectional"]
        # The reference's 2 heads / 2 kv heads, and 4 query heads over the same 2 kv heads
        # (GQA group 2).
        for q2 in (inp["q"], np.concatenate([inp["q"], inp["q"]], axis=2)):
            got = attention(to_bf16_bits(q2), to_bf16_bits(k), to_bf16_bits(v),
                            lengths=inp["lengths"], causal=causal, runtime=runtime)
            assert runtime.last_kernel() == "tc_bf16_d128"
            want = oracle.attention_padded(q2, from_bf16_bits(to_bf16_bits(k)),
                                           from_bf16_bits(to_bf16_bits(v)), inp["lengths"],
                                           causal, 128**-0.5)
            # No overflow at +-1131 logits, and the masked 1e10 values never leak.
            assert np.max(np.abs(got - want)) <= BF16_GATE, case.id


@pytest.mark.parametrize("heads,kv_heads", [(6, 2), (3, 3), (16, 1)])
def test_tensor_core_any_gqa_group(runtime, heads, kv_heads):
    """Query heads per kv head of 3 (odd), 1 (MHA) and 16 on the tensor-core kernel."""
    rng = np.random.default_rng(heads * 10 + kv_heads)
    lengths = np.array([1, 130, 64, 200], np.uint32)
    B, L, D = 4, 200, 128
    q = to_bf16_bits(rng.normal(size=(B, L, heads, D)).astype(np.float32))
    k = to_bf16_bits(rng.normal(size=(B, L, kv_heads, D)).astype(np.float32))
    v = to_bf16_bits(rng.normal(size=(B, L, kv_heads, D)).astype(np.float32))
    for causal in (True, False):
        got = attention(q, k, v, lengths=lengths, causal=causal, runtime=runtime)
        assert runtime.last_kernel() == "tc_bf16_d128"
        want = oracle.attention_padded(from_bf16_bits(q), from_bf16_bits(k), from_bf16_bits(v),
                                       lengths, causal, D**-0.5)
        assert np.max(np.abs(got - want)) <= BF16_GATE


def test_full_size_qwen_properties(runtime):
    """The padded Qwen benchmark shape at full size (32 x 512): size-independent
    properties (padded == varlen on valid rows, determinism) and spot sequences against
    the oracle (every sequence is checked in test_full_configs_gpu.py)."""
    w = workloads.qwen_padded(seed=2)
    got = run_workload(runtime, w)
    again = run_workload(runtime, w)
    assert np.array_equal(got, again)  # deterministic
    assert np.isfinite(got).all()
    sel = [0, 7, 31]
    sub = workloads.Workload(**{**w.__dict__, "q": w.q[sel], "k": w.k[sel], "v": w.v[sel],
                                "lengths": w.lengths[sel]})
    assert np.max(np.abs(got[sel] - qwen_oracle(sub))) <= BF16_GATE
    # Same sequences packed: valid rows must be identical bit for bit.
    lens = w.lengths.astype(np.int64)
    cu = np.zeros(lens.size + 1, np.int32)
    cu[1:] = np.cumsum(lens)
    pack = lambda a: np.concatenate([a[b, :lens[b]] for b in range(lens.size)])  # noqa: E731
    packed = attention(pack(w.q), pack(w.k), pack(w.v), cu_seqlens=cu, causal=True,
                       q_norm_weight=w.q_norm_weight, k_norm_weight=w.k_norm_weight,
                       runtime=runtime)
    assert np.array_equal(packed, pack(got))


def test_zero_length_gives_nan_rows(runtime):
    w = workloads.qwen_padded(batch=2, seq=128, seed=24, lengths=np.array([0, 50]))
    got = run_workload(runtime, w)
    assert np.isnan(got[0]).all()
    assert np.isfinite(got[1]).all()


def test_invalid_arguments_are_rejected(runtime):
    w = workloads.qwen_padded(batch=2, seq=64, seed=25, lengths=np.array([64, 3]))
    with pytest.raises(InvalidInputError):
        attention(w.q, w.k, w.v, lengths=np.array([65, 3]), runtime=runtime)
    with pytest.raises(InvalidInputError):
        attention(w.q, w.k[:, :, :3], w.v[:, :, :3], lengths=w.lengths, runtime=runtime)
    bad = np.array([0, 5, 3], np.int32)
    q = w.q.reshape(-1, 16, 128)[:5]
    k = w.k.reshape(-1, 8, 128)[:5]
    with pytest.raises(InvalidInputError):
        attention(q, k, k, cu_seqlens=bad, runtime=runtime)
    # the context is still usable afterwards
    got = run_workload(runtime, w)
    assert np.isfinite(got).all()


def test_prologue_matches_oracle(runtime):
    from tessery_b200 import qk_norm_rope

    rng = np.random.default_rng(51)
    tokens, seq = 6 * 64, 64
    q = rng.normal(size=(tokens, 16, 128)).astype(np.float32)
    k = rng.normal(size=(tokens, 8, 128)).astype(np.float32)
    qw = to_bf16_bits(1 + 0.02 * rng.normal(size=128).astype(np.float32))
    kw = to_bf16_bits(1 + 0.02 * rng.normal(size=128).astype(np.float32))
    pos = np.arange(tokens) % seq
    want_q, want_k = oracle.qk_norm_rope(q, k, qw, kw, 1e-6, 1e6, pos)
    got_q, got_k = qk_norm_rope(q, k, qw, kw, seq=seq, runtime=runtime)
    np.testing.assert_allclose(got_q, want_q, atol=2e-5, rtol=2e-5)
    np.testing.assert_allclose(got_k, want_k, atol=2e-5, rtol=2e-5)
    bq, bk = qk_norm_rope(to_bf16_bits(q), to_bf16_bits(k), qw, kw, seq=seq, runtime=runtime)
    wq, wk = oracle.qk_norm_rope(from_bf16_bits(to_bf16_bits(q)), from_bf16_bits(to_bf16_bits(k)),
                                 qw, kw, 1e-6, 1e6, pos)
    # bf16 output: within one bf16 rounding of the float64 result.
    np.testing.assert_allclose(from_bf16_bits(bq), wq, rtol=2 ** -8, atol=1e-6)
    np.testing.assert_allclose(from_bf16_bits(bk), wk, rtol=2 ** -8, atol=1e-6)


def test_prologue_at_long_positions_matches_oracle(runtime):
    """RoPE angles up to ~3e4 radians (one sequence of 30000 tokens): the FMA-pipe sine and
    cosine after the quadrant reduction stay within the float32 gate."""
    from tessery_b200 import qk_norm_rope

    rng = np.random.default_rng(52)
    tokens = 30000
    q = rng.normal(size=(tokens, 2, 128)).astype(np.float32)
    k = rng.normal(size=(tokens, 1, 128)).astype(np.float32)
    qw = to_bf16_bits(1 + 0.02 * rng.normal(size=128).astype(np.float32))
    kw = to_bf16_bits(1 + 0.02 * rng.normal(size=128).astype(np.float32))
    for theta in (1e4, 1e6):
        want_q, want_k = oracle.qk_norm_rope(q, k, qw, kw, 1e-6, theta, np.arange(tokens))
        got_q, got_k = qk_norm_rope(q, k, qw, kw, seq=tokens, theta=theta, runtime=runtime)
        np.testing.assert_allclose(got_q, want_q, atol=2e-5, rtol=2e-5)
        np.testing.assert_allclose(got_k, want_k, atol=2e-5, rtol=2e-5)


def test_typed_dtype_codes():
    assert (TX_F32, TX_BF16) == (0, 1)


def _device_path(rt, w):
    """The same workload through the device-pointer entry point, one call, one launch set."""
    arrays = {n: np.ascontiguousarray(a) for n, a in (("q", w.q), ("k", w.k), ("v", w.v),
                                                        ("qw", w.q_norm_weight),
                                                        ("kw", w.k_norm_weight))}
    if w.layout == "padded":
        arrays["sel"] = w.lengths.astype(np.uint32)
    else:
        arrays["sel"] = w.cu_seqlens.astype(np.int32)
    bufs = {n: rt.buffer(a.nbytes, a) for n, a in arrays.items()}
    out = rt.buffer(w.q.size * 4)
    try:
        D = w.dim
        kw = dict(in_dtype=TX_BF16, out_dtype=TX_F32, causal=w.causal,
                  q_norm_weight=bufs["qw"].device_ptr, k_norm_weight=bufs["kw"].device_ptr)
        if w.layout == "padded":
            B, L, H = w.q.shape[:3]
            rt.attention_padded_device(bufs["q"].device_ptr, bufs["k"].device_ptr,
                                       bufs["v"].device_ptr, bufs["sel"].device_ptr,
                                       out.device_ptr, batch=B, seq=L, heads=H,
                                       kv_heads=w.kv_heads, dim=D, lengths_host=arrays["sel"], **kw)
        else:
            T, H = w.q.shape[:2]
            cu = arrays["sel"]
            rt.attention_varlen_device(bufs["q"].device_ptr, bufs["k"].device_ptr,
                                       bufs["v"].device_ptr, bufs["sel"].device_ptr,
                                       out.device_ptr, nseq=cu.size - 1, total=T,
                                       max_len=int(np.max(np.diff(cu))), heads=H,
                                       kv_heads=w.kv_heads, dim=D, cu_seqlens_host=cu, **kw)
        rt.sync()
        return rt.read(out, w.q.shape)
    finally:
        for b in [*bufs.values(), out]:
            b.close()


def test_host_buffer_entry_points_match_device_path(runtime):
    """The NumPy call goes through the host-buffer entry points, which split the sequences
    into chunks (8 here: 134 MB / 100 MB moved) and overlap copies with kernels; every row
    equals the single device-pointer call bit for bit, padded and packed, and with
    page-locked arrays as with pageable ones."""
    from tessery_b200.host import pinned_copy, pinned_empty

    padded = workloads.qwen_padded(batch=16, seq=512, seed=27)
    packed = workloads.qwen_varlen(seed=28, lengths=workloads.varlen_lengths(64, 28))
    for w in (padded, packed):
        want = _device_path(runtime, w)
        got = run_workload(runtime, w)
        assert np.array_equal(got, want), w.layout
        sel = ({"lengths": pinned_copy(w.lengths.astype(np.uint32))} if w.layout == "padded"
               else {"cu_seqlens": pinned_copy(w.cu_seqlens.astype(np.int32))})
        hout = pinned_empty(w.q.shape, np.float32)
        attention(pinned_copy(w.q), pinned_copy(w.k), pinned_copy(w.v), causal=w.causal,
                  scale=w.scale, q_norm_weight=w.q_norm_weight, k_norm_weight=w.k_norm_weight,
                  eps=w.eps, theta=w.theta, runtime=runtime, out=hout, **sel)
        assert np.array_equal(hout, want), w.layout


def test_host_buffer_copies_padding_spans_and_counts_bytes(runtime):
    """The padded host-buffer call copies each chunk's valid k/v rows in spans that take
    short padding gaps along; the caller's padded rows (NaN k, Inf v here) then reach the
    device and are still never attended: every row equals the device call on clean
    padding bit for bit.  tx_host_copy_bytes reports what crossed the link: at least the
    q rows and the valid k/v rows, at most the whole arrays, and the output rows back."""
    w = workloads.qwen_padded(batch=16, seq=512, seed=31)
    want = _device_path(runtime, w)
    k = _poison_padding(w.k, w.lengths, np.uint16(0x7FC0))  # bf16 NaN
    v = _poison_padding(w.v, w.lengths, np.uint16(0x7F80))  # bf16 +Inf
    got = attention(w.q, k, v, lengths=w.lengths, causal=w.causal, scale=w.scale,
                    q_norm_weight=w.q_norm_weight, k_norm_weight=w.k_norm_weight, eps=w.eps,
                    theta=w.theta, runtime=runtime)
    assert np.array_equal(got, want)
    h2d, d2h = runtime.host_copy_bytes()
    valid_kv = 2 * int(np.sum(w.lengths)) * w.kv_heads * w.dim * 2
    assert w.q.nbytes + valid_kv <= h2d <= w.q.nbytes + k.nbytes + v.nbytes + (1 << 20)
    assert d2h == got.nbytes


def test_host_buffer_mixed_pageable_and_page_locked_arrays(runtime):
    """Each host array is staged through page-locked memory only when it is pageable:
    page-locked inputs with a pageable `out`, pageable inputs with a page-locked `out`,
    and everything pageable all give the device call's rows bit for bit (the output
    rows of a pageable `out` are copied out of the staging chunk by chunk)."""
    from tessery_b200.host import pinned_copy, pinned_empty

    padded = workloads.qwen_padded(batch=12, seq=512, seed=33)
    packed = workloads.qwen_varlen(seed=34, lengths=workloads.varlen_lengths(48, 34))
    for w in (padded, packed):
        want = _device_path(runtime, w)
        sel = ({"lengths": w.lengths.astype(np.uint32)} if w.layout == "padded"
               else {"cu_seqlens": w.cu_seqlens.astype(np.int32)})
        kw = dict(causal=w.causal, scale=w.scale, q_norm_weight=w.q_norm_weight,
                  k_norm_weight=w.k_norm_weight, eps=w.eps, theta=w.theta, runtime=runtime,
                  **sel)
        pinned_in = [pinned_copy(a) for a in (w.q, w.k, w.v)]
        for inputs, out in ((pinned_in, np.empty(w.q.shape, np.float32)),
                            ((w.q, w.k, w.v), pinned_empty(w.q.shape, np.float32)),
                            ((w.q, w.k, w.v), np.empty(w.q.shape, np.float32))):
            out[...] = np.nan
            attention(*inputs, out=out, **kw)
            assert np.array_equal(out, want), w.layout


def test_composed_prologue_matches_one_call(runtime):
    """k-only prologue over the valid rows (tx_qk_norm_rope with device lengths), then
    attention with only the q weight, against the one-call path.  The one call knows both
    norm weights and so a bound on every score: it takes one softmax pass per tile with a
    fixed reference, the composed call the two-pass softmax with the row maximum, so P
    rounds to bf16 from differently shifted exponents and the results agree to the bf16
    gate, not bit for bit; both against the oracle."""
    from tessery_b200 import TX_BF16, TX_F32

    w = workloads.qwen_padded(batch=4, seq=384, seed=26, lengths=np.array([384, 200, 1, 129]))
    one_call = run_workload(runtime, w)
    rt = runtime
    bufs = {n: rt.buffer(a.nbytes, np.ascontiguousarray(a)) for n, a in
            (("q", w.q), ("k", w.k), ("v", w.v), ("len", w.lengths.astype(np.uint32)),
             ("qw", w.q_norm_weight), ("kw", w.k_norm_weight))}
    kn = rt.buffer(w.k.nbytes)
    out = rt.buffer(w.q.size * 4)
    B, L, H, D = w.q.shape
    rt.qk_norm_rope_device(None, bufs["k"].device_ptr, None, kn.device_ptr, tokens=B * L, seq=L,
                           heads=H, kv_heads=8, dim=D, q_norm_weight=None,
                           k_norm_weight=bufs["kw"].device_ptr, lengths=bufs["len"].device_ptr,
                           in_dtype=TX_BF16, out_dtype=TX_BF16)
    rt.attention_padded_device(bufs["q"].device_ptr, kn.device_ptr, bufs["v"].device_ptr,
                               bufs["len"].device_ptr, out.device_ptr, batch=B, seq=L, heads=H,
                               kv_heads=8, dim=D, in_dtype=TX_BF16, out_dtype=TX_F32,
                               causal=True, lengths_host=w.lengths,
                               q_norm_weight=bufs["qw"].device_ptr)
    rt.sync()
    got = rt.read(out, w.q.shape)
    want = qwen_oracle(w)
    assert np.max(np.abs(got - want)) <= BF16_GATE
    assert np.max(np.abs(one_call - want)) <= BF16_GATE
    assert np.max(np.abs(got - one_call)) <= BF16_GATE
    for b in list(bufs.values()) + [kn, out]:
        b.close()


# ---- padded k/v rows hold anything ---------------------------------------------------------
def _poison_padding(a, lengths, value):
    """Sets rows at positions >= length of a padded [B, L, H, d] array to `value`."""
    a = a.copy()
    for b, n in enumerate(lengths):
        a[b, int(n):] = value
    return a


def _padded_device_call(rt, q, k, v, lengths, *, in_dtype, causal, scale, qw=None, kw=None):
    B, L, H, D = q.shape
    arrays = [np.ascontiguousarray(a) for a in (q, k, v, lengths.astype(np.uint32))]
    bufs = [rt.buffer(a.nbytes, a) for a in arrays]
    wbufs = [rt.buffer(w.nbytes, np.ascontiguousarray(w)) for w in (qw, kw) if w is not None]
    out = rt.buffer(q.size * 4)
    try:
        extra = {}
        if qw is not None:
            extra = dict(q_norm_weight=wbufs[0].device_ptr, k_norm_weight=wbufs[1].device_ptr)
        rt.attention_padded_device(*(b.device_ptr for b in bufs), out.device_ptr, batch=B,
                                   seq=L, heads=H, kv_heads=k.shape[2], dim=D,
                                   in_dtype=in_dtype, out_dtype=TX_F32, causal=causal,
                                   scale=scale, lengths_host=arrays[3], **extra)
        rt.sync()
        return rt.read(out, q.shape)
    finally:
        for b in [*bufs, *wbufs, out]:
            b.close()


@pytest.mark.parametrize("route", ["tc_bf16_d128", "short_d128", "d32_tc", "d32", "f32_tc",
                                   "simt"])
def test_padded_kv_rows_may_hold_nan_or_inf(runtime, route):
    """k/v rows at or past a sequence's length hold NaN (k) and Inf (v): every route
    returns the oracle's rows, all finite, as the reference, which never reads those rows
    (kernels.metal:89-99)."""
    rng = np.random.default_rng(71)
    if route in ("tc_bf16_d128", "short_d128"):
        L = 300 if route == "tc_bf16_d128" else 32
        lengths = np.array([L, 129, 1, 200] if L == 300 else [32, 5, 17, 1])
        w = workloads.qwen_padded(batch=4, seq=L, seed=72, lengths=lengths)
        k = _poison_padding(w.k, lengths, np.uint16(0x7FC0))  # bf16 NaN
        v = _poison_padding(w.v, lengths, np.uint16(0x7F80))  # bf16 +Inf
        got = _padded_device_call(runtime, w.q, k, v, lengths, in_dtype=TX_BF16, causal=True,
                                  scale=w.scale, qw=w.q_norm_weight, kw=w.k_norm_weight)
        want = qwen_oracle(w)
        gate = BF16_GATE
    else:
        D = {"simt": 64, "f32_tc": 128}.get(route, 32)
        lengths = np.array([128, 1, 70])
        q, k, v = (rng.normal(size=(3, 128, 4, D)).astype(np.float32) for _ in range(3))
        if route == "d32":  # bf16 inputs take the FP32-pipe head_dim-32 kernel
            q, k, v = (from_bf16_bits(to_bf16_bits(a)) for a in (q, k, v))
        k = _poison_padding(k, lengths, np.float32(np.nan))
        v = _poison_padding(v, lengths, np.float32(np.inf))
        if route == "d32":
            got = _padded_device_call(runtime, *(to_bf16_bits(a) for a in (q, k, v)), lengths,
                                      in_dtype=TX_BF16, causal=False, scale=D**-0.5)
        else:
            got = _padded_device_call(runtime, q, k, v, lengths, in_dtype=TX_F32,
                                      causal=False, scale=D**-0.5)
        want = oracle.attention_padded(q, k, v, lengths, False, D**-0.5)
        gate = 1e-4
    assert runtime.last_kernel() == route
    assert np.isfinite(got).all()
    assert np.max(np.abs(got - want)) <= gate


def test_attention_reads_q_written_by_the_kernel_just_before(runtime):
    """A kernel writes q (here the library's own prologue, into a fresh buffer) and the
    attention call that reads it follows at once on the same stream, with no k prologue
    in between: the attention kernel is then launched in plain stream order and sees q."""
    w = workloads.qwen_padded(batch=3, seq=384, seed=73, lengths=np.array([384, 130, 2]))
    rt = runtime
    B, L, H, D = w.q.shape
    bufs = {n: rt.buffer(a.nbytes, np.ascontiguousarray(a)) for n, a in
            (("q", w.q), ("k", w.k), ("v", w.v), ("len", w.lengths.astype(np.uint32)),
             ("qw", w.q_norm_weight), ("kw", w.k_norm_weight))}
    qn, kn = rt.buffer(w.q.nbytes), rt.buffer(w.k.nbytes)
    out = rt.buffer(w.q.size * 4)
    try:
        rt.qk_norm_rope_device(None, bufs["k"].device_ptr, None, kn.device_ptr, tokens=B * L,
                               seq=L, heads=H, kv_heads=8, dim=D, q_norm_weight=None,
                               k_norm_weight=bufs["kw"].device_ptr, in_dtype=TX_BF16,
                               out_dtype=TX_BF16)
        for _ in range(3):
            rt.qk_norm_rope_device(bufs["q"].device_ptr, None, qn.device_ptr, None,
                                   tokens=B * L, seq=L, heads=H, kv_heads=8, dim=D,
                                   q_norm_weight=bufs["qw"].device_ptr, k_norm_weight=None,
                                   in_dtype=TX_BF16, out_dtype=TX_BF16)
            rt.attention_padded_device(qn.device_ptr, kn.device_ptr, bufs["v"].device_ptr,
                                       bufs["len"].device_ptr, out.device_ptr, batch=B, seq=L,
                                       heads=H, kv_heads=8, dim=D, in_dtype=TX_BF16,
                                       out_dtype=TX_F32, causal=True, lengths_host=w.lengths)
            rt.sync()
            assert rt.last_kernel() == "tc_bf16_d128"
            got = rt.read(out, w.q.shape)
            assert np.max(np.abs(got - qwen_oracle(w))) <= BF16_GATE
            rt.qk_norm_rope_device(bufs["v"].device_ptr, None, qn.device_ptr, None,
                                   tokens=B * L, seq=L, heads=H, kv_heads=8, dim=D,
                                   q_norm_weight=bufs["qw"].device_ptr, k_norm_weight=None,
                                   in_dtype=TX_BF16, out_dtype=TX_BF16)  # scribble over q
            rt.sync()
    finally:
        for b in [*bufs.values(), qn, kn, out]:
            b.close()


def test_device_wait_timeout_is_reported_and_context_recovers(runtime):
    """With the bounded-wait limit set to one cycle, the first wait of the tensor-core
    kernel that is not already satisfied gives up: the kernel drains its copies and
    products and returns, the host sees DeviceTimeoutError, and the same context then
    computes the right result with the default limit (counterpart of the status check of
    mi_finish, runtime.mm:217-253)."""
    from tessery_b200 import DeviceTimeoutError

    w = workloads.qwen_padded(batch=2, seq=256, seed=74, lengths=np.array([256, 100]))
    runtime.set_wait_limit(1)
    try:
        with pytest.raises(DeviceTimeoutError):
            _device_path(runtime, w)
        assert "timed out" in runtime.last_error()
    finally:
        runtime.set_wait_limit(0)
    got = _device_path(runtime, w)
    assert runtime.last_kernel() == "tc_bf16_d128"
    assert np.max(np.abs(got - qwen_oracle(w))) <= BF16_GATE
