"""The Qwen3 embedding forward around the attention (needs a B200): the tensor-core GEMM
and its epilogues, uint4 dequantisation, the uint4 embedding and the row RMSNorm against
NumPy / the oracle, then the whole forward against oracle/qwen3.py.

Gates: GEMM with fp32 output vs float64 of the same bf16 operands, rtol 1e-5 of the
row scale; bf16 outputs within one bf16 rounding (2^-8 relative) plus that; dequantised
bf16 weights within one bf16 ulp of the exact value; embedding and RMSNorm fp32 at
atol 1e-5 / rtol 1e-5; pooled embeddings of the forward against the oracle (the
reference's fp32 forward restated) at cosine >= 0.9999 in precise mode (bf16-pair
projection operands, fp32 attention) and at the cosine the bf16 fast mode reaches.
"""

import numpy as np
import pytest

import oracle
import oracle.qwen3 as oq
from tessery_b200 import native
from tessery_b200.qwen3 import Qwen3Config, Qwen3Encoder, random_weights
from tessery_b200.workloads import from_bf16_bits, to_bf16_bits

pytestmark = pytest.mark.gpu


def _dev(rt, a):
    a = np.ascontiguousarray(a)
    return rt.buffer(a.nbytes, a)


@pytest.mark.parametrize("mode", ["f32", "bf16", "add", "gated"])
@pytest.mark.parametrize("m", [1, 300, 1024])
def test_linear_epilogues_match_numpy(runtime, mode, m):
    rng = np.random.default_rng(90 + m)
    n, k = 512, 1024
    x = to_bf16_bits(rng.standard_normal((m, k), dtype=np.float32))
    w = to_bf16_bits(0.05 * rng.standard_normal((n, k), dtype=np.float32))
    acc = from_bf16_bits(x).astype(np.float64) @ from_bf16_bits(w).astype(np.float64).T
    scale = np.sqrt(k) * 0.05
    code = {"f32": native.TX_LINEAR_STORE_F32, "bf16": native.TX_LINEAR_STORE_BF16,
            "add": native.TX_LINEAR_ADD_F32, "gated": native.TX_LINEAR_GATED_BF16}[mode]
    if mode == "gated":
        out_shape, out_dtype, nbytes = (m, n // 2), np.uint16, m * (n // 2) * 2
        gate = acc.reshape(m, n // 256, 2, 128)[:, :, 0].reshape(m, n // 2)
        up = acc.reshape(m, n // 256, 2, 128)[:, :, 1].reshape(m, n // 2)
        want = oq.silu_gate(gate, up)
    elif mode == "bf16":
        out_shape, out_dtype, nbytes, want = (m, n), np.uint16, m * n * 2, acc
    else:
        out_shape, out_dtype, nbytes, want = (m, n), np.float32, m * n * 4, acc
    init = rng.standard_normal(out_shape).astype(np.float32) if mode == "add" else None
    xb, wb = _dev(runtime, x), _dev(runtime, w)
    ob = runtime.buffer(nbytes, init)
    try:
        runtime.linear_device(xb.device_ptr, wb.device_ptr, ob.device_ptr, m=m, n=n, k=k, mode=code)
        runtime.sync()
        got = runtime.read(ob, out_shape, dtype=out_dtype)
    finally:
        for b in (xb, wb, ob):
            b.close()
    if mode == "add":
        want = want + init
    if out_dtype == np.uint16:
        got = from_bf16_bits(got)
        np.testing.assert_allclose(got, want, rtol=2**-8, atol=1e-5 * scale * 8)
    else:
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5 * scale)


def test_linear_rejects_unsupported_shapes(runtime):
    from tessery_b200 import InvalidInputError

    buf = runtime.buffer(1 << 20)
    try:
        with pytest.raises(InvalidInputError):  # n not a multiple of 256
            runtime.linear_device(buf.device_ptr, buf.device_ptr, buf.device_ptr, m=4, n=200,
                                  k=64, mode=native.TX_LINEAR_STORE_F32)
        with pytest.raises(InvalidInputError):  # k not a multiple of 64
            runtime.linear_device(buf.device_ptr, buf.device_ptr, buf.device_ptr, m=4, n=256,
                                  k=100, mode=native.TX_LINEAR_STORE_F32)
    finally:
        buf.close()


def test_dequant4_embedding4_and_row_norm_match_oracle(runtime):
    rng = np.random.default_rng(91)
    rows, cols = 300, 1024
    packed = rng.integers(0, 2**32, size=(rows, cols // 8), dtype=np.uint32)
    scales = to_bf16_bits(0.02 * rng.standard_normal((rows, cols // 64), dtype=np.float32))
    biases = to_bf16_bits(0.01 * rng.standard_normal((rows, cols // 64), dtype=np.float32))
    exact = oq.dequant4(packed, scales, biases)
    bufs = [_dev(runtime, a) for a in (packed, scales, biases)]
    out = runtime.buffer(rows * cols * 2)
    ids = np.array([0, 299, 7, 7, 150], np.uint32)
    idb = _dev(runtime, ids)
    emb = runtime.buffer(ids.size * cols * 4)
    x = (50 * rng.standard_normal((37, cols))).astype(np.float32)
    w = to_bf16_bits(1 + 0.02 * rng.standard_normal(cols).astype(np.float32))
    xb, wb = _dev(runtime, x), _dev(runtime, w)
    nb16, nb32 = runtime.buffer(x.size * 2), runtime.buffer(x.size * 4)
    try:
        runtime.dequant4_device(*(b.device_ptr for b in bufs), out.device_ptr, rows=rows, cols=cols)
        runtime.embedding4_device(idb.device_ptr, emb.device_ptr, tokens=ids.size,
                                  packed=bufs[0].device_ptr, scales=bufs[1].device_ptr,
                                  biases=bufs[2].device_ptr, cols=cols, vocab=rows)
        runtime.rms_norm_rows_device(xb.device_ptr, wb.device_ptr, nb16.device_ptr, rows=37,
                                     cols=cols, eps=1e-6, out_dtype=native.TX_BF16)
        runtime.rms_norm_rows_device(xb.device_ptr, wb.device_ptr, nb32.device_ptr, rows=37,
                                     cols=cols, eps=1e-6, out_dtype=native.TX_F32)
        runtime.sync()
        deq = from_bf16_bits(runtime.read(out, (rows, cols), dtype=np.uint16))
        got_emb = runtime.read(emb, (ids.size, cols))
        got16 = from_bf16_bits(runtime.read(nb16, x.shape, dtype=np.uint16))
        got32 = runtime.read(nb32, x.shape)
    finally:
        for b in (*bufs, out, idb, emb, xb, wb, nb16, nb32):
            b.close()
    # Within one bf16 ulp of the exact dequantised value.
    ulp = np.abs(exact) * 2**-7 + 1e-30
    assert np.all(np.abs(deq - exact) <= ulp)
    np.testing.assert_allclose(got_emb, exact[ids], atol=1e-6, rtol=1e-6)
    want = oracle.rms_norm(x, w, 1e-6)
    np.testing.assert_allclose(got32, want, atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(got16, want, rtol=2**-8, atol=1e-6)


def test_embedding4_id_out_of_range_is_reported(runtime):
    from tessery_b200 import InvalidInputError

    packed = np.zeros((4, 8), np.uint32)
    sb = np.zeros((4, 1), np.uint16)
    bufs = [_dev(runtime, a) for a in (packed, sb, sb, np.array([1, 4], np.uint32))]
    out = runtime.buffer(2 * 64 * 4)
    try:
        runtime.embedding4_device(bufs[3].device_ptr, out.device_ptr, tokens=2,
                                  packed=bufs[0].device_ptr, scales=bufs[1].device_ptr,
                                  biases=bufs[2].device_ptr, cols=64, vocab=4)
        with pytest.raises(InvalidInputError):
            runtime.sync()
        got = runtime.read(out, (2, 64))
        assert np.all(got[0] == 0) and np.isnan(got[1]).all()
    finally:
        for b in (*bufs, out):
            b.close()


def _cosines(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.sum(a * b, axis=1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


# Pooled-embedding cosine reached on these random weights by the fast mode (bf16
# projection operands, bf16 tensor-core attention): the roundings compound over the layers
# (a float64 restatement with the same bf16 roundings injected lands at 0.9985 at 28
# layers), so the fast mode is held to the cosine it reaches, the precise mode to 0.9999.
FAST_GATE = {2: 0.9999, 28: 0.995}


@pytest.mark.parametrize("layers,lengths,dtype,precise", [
    (2, [1, 77, 200], np.float64, False),
    (2, [1, 77, 200], np.float64, True),
    (28, [37, 256, 130, 511], np.float32, False),
    (28, [37, 256, 130, 511], np.float32, True),
])
def test_forward_matches_oracle(runtime, layers, lengths, dtype, precise):
    """The whole forward on seeded random uint4 weights: pooled embeddings against the
    NumPy restatement of qwen3.py:112-296 (float64 for 2 layers; the reference's own
    float32 for the full 28 layers, to keep the oracle within seconds)."""
    cfg = Qwen3Config(layers=layers, vocab=151669 if layers == 28 else 5000)
    weights = random_weights(cfg, seed=100 + layers)
    rng = np.random.default_rng(7)
    lengths = np.array(lengths)
    ids = rng.integers(0, cfg.vocab, size=(lengths.size, int(lengths.max())))
    model = Qwen3Encoder(weights, cfg, runtime=runtime, precise=precise)
    try:
        got = model.forward(ids, lengths, dimensions=cfg.hidden)
        got_short = model.forward(ids, lengths, dimensions=256)
    finally:
        model.close()
    want = oq.qwen3_forward(weights, cfg, ids, lengths, cfg.hidden, dtype=dtype)
    cos = _cosines(got, want)
    print(f"\nQWEN_FORWARD layers {layers} precise {precise}: cosine min {cos.min():.7f} "
          f"max abs {np.max(np.abs(got - want)):.3g}")
    assert cos.min() >= (0.9999 if precise else FAST_GATE[layers])
    # Matryoshka-style truncation: the first 256 columns, normalised on their own.
    head = got[:, :256] / np.linalg.norm(got[:, :256], axis=1, keepdims=True)
    np.testing.assert_allclose(got_short, head, atol=1e-5)
