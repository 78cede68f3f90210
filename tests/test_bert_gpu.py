"""The BERT fp32 forward around the head_dim-32 attention (needs a B200): the reference's
BERT kernels through tx_dispatch and the TF32 tensor-core GEMM against the golden vectors
recorded from the reference's own tests, the row kernels against the oracle, then the
whole forward against oracle/bert.py.

Gates: the reference's own tolerances for every golden case (matmul atol 5e-5 / rtol 5e-5
vs float64, the cancellation pattern included; LayerNorm atol 1e-6 / rtol 1e-5; GELU atol
2e-6 / rtol 1e-6); row kernels atol 1e-5; pooled CLS embeddings of the forward at cosine
>= 0.9999 against the float64 (2 layers) and float32 (12 layers) oracle.
"""

import numpy as np
import pytest

import oracle.bert as ob
from golden_cases import compare, inputs_match, load_cases, regenerate
from tessery_b200 import native
from tessery_b200.bert import BertConfig, BertEncoder, random_weights

pytestmark = pytest.mark.gpu

CASES = load_cases()
BERT_KERNELS = ("layer_norm", "embedding_position", "gelu_f32", "add_bias")


def _dev(rt, a):
    a = np.ascontiguousarray(a)
    return rt.buffer(a.nbytes, a)


@pytest.mark.parametrize("case", [c for c in CASES if c.kernel in BERT_KERNELS],
                         ids=lambda c: c.id)
def test_bert_dispatch_kernels_match_golden(runtime, case):
    """The reference's dispatch of each kernel, on this runtime (CudaRuntime._dispatch)."""
    inputs = regenerate(case)
    assert inputs_match(case, inputs)
    d = dict(case.dispatch)
    bufs = [_dev(runtime, a) for a in inputs.values()]
    try:
        if case.kernel in ("gelu_f32", "add_bias"):  # in place on the first buffer
            with runtime.command():
                runtime._dispatch(case.kernel, bufs, **d)
            got = runtime.read(bufs[0], case.shape)
        else:
            out = runtime.buffer(int(np.prod(case.shape)) * 4)
            bufs.append(out)
            with runtime.command():
                runtime._dispatch(case.kernel, bufs, **d)
            got = runtime.read(out, case.shape)
    finally:
        for b in bufs:
            b.close()
    compare(case, got)


MATMUL = [c for c in CASES if c.kernel == "matmul_f32"]


@pytest.mark.parametrize("case", MATMUL, ids=lambda c: c.id)
def test_matmul_dispatch_matches_golden(runtime, case):
    """CudaRuntime.matmul (the reference's MetalRuntime.matmul call) at the reference's
    tolerance."""
    inputs = regenerate(case)
    assert inputs_match(case, inputs)
    got = runtime.matmul(inputs["a"], np.ascontiguousarray(inputs["bt"].T))
    compare(case, got)


def _tf32_linear(rt, x, w, *, bias=None, mode=native.TX_LINEAR_STORE_F32, part=None,
                 precise=True):
    """x [m, k] . w [n, k]^T (+ bias) on the TF32 tensor-core path with split operands."""
    m, k = x.shape
    n = w.shape[0]
    xb, wb = _dev(rt, x.astype(np.float32)), _dev(rt, w.astype(np.float32))
    xs, ws = rt.buffer(2 * x.size * 4), rt.buffer(2 * w.size * 4)
    bb = _dev(rt, bias.astype(np.float32)) if bias is not None else None
    pair_out = mode == native.TX_LINEAR_GELU_SPLIT
    out = rt.buffer((2 if pair_out else 1) * m * n * 4)
    try:
        rt.split_tf32_device(xb.device_ptr, xs.device_ptr, n=x.size)
        rt.split_tf32_device(wb.device_ptr, ws.device_ptr, n=w.size)
        rt.linear_device(xs.device_ptr, ws.device_ptr, out.device_ptr, m=m, n=n, k=k, mode=mode,
                         x_lo=xs.device_ptr + x.size * 4 if precise else None,
                         w_lo=ws.device_ptr + w.size * 4 if precise else None,
                         bias=bb.device_ptr if bb else None, fmt=native.TX_F32, part=part)
        rt.sync()
        got = rt.read(out, (2, m, n) if pair_out else (m, n))
    finally:
        for b in (xb, wb, xs, ws, out) + ((bb,) if bb else ()):
            b.close()
    return got


@pytest.mark.parametrize("case", [c for c in MATMUL if c.shape[1] % 128 == 0 and
                                  c.dispatch["k"] % 32 == 0], ids=lambda c: c.id)
def test_tf32_tensor_core_gemm_matches_golden(runtime, case):
    """The reference's f32 projection cases (BGE shapes, random and cancellation
    patterns) on the three-product TF32 tensor-core GEMM, at the reference's own 5e-5."""
    inputs = regenerate(case)
    assert inputs_match(case, inputs)
    got = _tf32_linear(runtime, inputs["a"], inputs["bt"])
    compare(case, got)


def test_tf32_gemm_bias_split_columns_and_gelu(runtime):
    rng = np.random.default_rng(61)
    m, k, hid = 300, 384, 384
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (0.05 * rng.standard_normal((3 * hid, k))).astype(np.float32)
    b = rng.standard_normal(3 * hid).astype(np.float32)
    want = x.astype(np.float64) @ w.astype(np.float64).T + b
    # Fused q/k/v: three [m, hid] matrices one after the other.
    got = _tf32_linear(runtime, x, w, bias=b, part=hid)
    split = got.reshape(-1)[: 3 * m * hid].reshape(3, m, hid)
    for p in range(3):
        np.testing.assert_allclose(split[p], want[:, p * hid:(p + 1) * hid], atol=5e-5,
                                   rtol=5e-5)
    # GELU epilogue written as a TF32 operand pair: hi + lo is the fp32 value.
    wi = (0.05 * rng.standard_normal((1536, k))).astype(np.float32)
    bi = rng.standard_normal(1536).astype(np.float32)
    pair = _tf32_linear(runtime, x, wi, bias=bi, mode=native.TX_LINEAR_GELU_SPLIT)
    hi, lo = pair[0].astype(np.float64), pair[1].astype(np.float64)
    np.testing.assert_array_equal(pair[0].view(np.uint32) & 0x1FFF, 0)  # hi is TF32
    np.testing.assert_allclose(hi + lo, ob.gelu(x.astype(np.float64) @ wi.T + bi), atol=5e-5,
                               rtol=5e-5)


def test_layer_norm_rows_and_embedding_match_oracle(runtime):
    rng = np.random.default_rng(62)
    rows, cols = 77, 384
    x = (3 * rng.standard_normal((rows, cols))).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    b = (0.1 * rng.standard_normal(cols)).astype(np.float32)
    bufs = [_dev(runtime, a) for a in (x, w, b)]
    out, pair = runtime.buffer(x.nbytes), runtime.buffer(2 * x.nbytes)
    # Embeddings of three packed sequences.
    words = rng.standard_normal((50, cols)).astype(np.float32)
    positions = rng.standard_normal((40, cols)).astype(np.float32)
    types = rng.standard_normal((2, cols)).astype(np.float32)
    lengths = np.array([5, 31, 1])
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    ids = rng.integers(0, 50, size=int(cu[-1])).astype(np.uint32)
    eb = [_dev(runtime, a) for a in (words, positions, types, ids, cu)]
    emb = runtime.buffer(ids.size * cols * 4)
    try:
        runtime.layer_norm_rows_device(bufs[0].device_ptr, bufs[1].device_ptr, bufs[2].device_ptr,
                                       out.device_ptr, rows=rows, cols=cols, eps=1e-12,
                                       pair=pair.device_ptr)
        runtime.bert_embed_device(eb[3].device_ptr, emb.device_ptr, tokens=ids.size, cols=cols,
                                  words=eb[0].device_ptr, positions=eb[1].device_ptr,
                                  types=eb[2].device_ptr, vocab=50, max_pos=40,
                                  ln_w=bufs[1].device_ptr, ln_b=bufs[2].device_ptr, eps=1e-12,
                                  cu_seqlens=eb[4].device_ptr, nseq=3)
        runtime.sync()
        got = runtime.read(out, (rows, cols))
        got_pair = runtime.read(pair, (2, rows, cols))
        got_emb = runtime.read(emb, (ids.size, cols))
    finally:
        for t in (*bufs, out, pair, *eb, emb):
            t.close()
    want = ob.layer_norm(x, w, b, 1e-12)
    np.testing.assert_allclose(got, want, atol=1e-5, rtol=1e-5)
    np.testing.assert_array_equal(got_pair[0] + got_pair[1], got)
    pos = np.concatenate([np.arange(n) for n in lengths])
    want_emb = ob.layer_norm((words[ids].astype(np.float64) + types[0]) + positions[pos], w, b,
                             1e-12)
    np.testing.assert_allclose(got_emb, want_emb, atol=1e-5, rtol=1e-5)


def _cosines(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.sum(a * b, axis=1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


@pytest.mark.parametrize("layers,lengths,dtype,precise,gate", [
    (2, [2, 17, 128, 77], np.float64, True, 0.9999),
    (2, [2, 17, 128, 77], np.float64, False, 0.999),
    (12, [128, 16, 93, 64, 127, 40], np.float32, True, 0.9999),
])
def test_bert_forward_matches_oracle(runtime, layers, lengths, dtype, precise, gate):
    """The whole forward on seeded random weights: CLS embeddings against the NumPy
    restatement of bert.py:104-235 (float64 for 2 layers, the reference's float32 for 12)."""
    cfg = BertConfig(layers=layers, vocab=30522 if layers == 12 else 2000)
    weights = random_weights(cfg, seed=200 + layers)
    rng = np.random.default_rng(8)
    lengths = np.array(lengths)
    ids = rng.integers(0, cfg.vocab, size=(lengths.size, int(lengths.max())))
    model = BertEncoder(weights, cfg, runtime=runtime, precise=precise)
    try:
        got = model.forward(ids, lengths)
    finally:
        model.close()
    want = ob.bert_forward(weights, cfg, ids, lengths, dtype=dtype)
    cos = _cosines(got, want)
    print(f"\nBERT_FORWARD layers {layers} precise {precise}: cosine min {cos.min():.8f} "
          f"max abs {np.max(np.abs(got - want)):.3g}")
    assert cos.min() >= gate
    if precise:
        np.testing.assert_allclose(got, want, atol=1e-4)
