"""Golden cases recorded by tests/golden/make_golden.py from the reference's own kernel
tests (tests/real_metal/test_kernels.py in the reference).

`regenerate(case)` rebuilds a case's inputs from the seed and shapes the reference test
uses; the SHA-256 of every regenerated array must equal the one recorded from the
reference run, so the inputs are provably the reference test's inputs.
"""

from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

FIXTURE = Path(__file__).resolve().parent / "golden" / "reference_kernels.npz"
PATH_KERNELS = {"attention", "attention_tiled", "attention_tail_32", "attention_tail_128",
                "rope", "rms_norm", "pool_project", "embedding4", "linear4", "layer_norm",
                "embedding_position", "gelu_f32", "add_bias", "matmul_f32"}


def sha(a: np.ndarray) -> str:
    a = np.ascontiguousarray(a)
    return hashlib.sha256(str(a.dtype).encode() + str(a.shape).encode() + a.tobytes()).hexdigest()


@dataclass
class Case:
    test: str
    params: dict
    check: int
    kernel: str
    dispatch: dict
    input_sha256: list
    shape: tuple
    rtol: float
    atol: float
    oracle_max_abs: float
    sum: float
    sumsq: float
    index: np.ndarray
    value: np.ndarray

    @property
    def id(self) -> str:
        p = ",".join(f"{k}={v}" for k, v in self.params.items())
        return f"{self.test.removeprefix('test_')}[{p}]#{self.check}"


def load_cases() -> list[Case]:
    data = np.load(FIXTURE)
    meta = json.loads(str(data["meta"]))
    cases = []
    for i, m in enumerate(meta):
        if m["kernel"] not in PATH_KERNELS:
            continue  # e.g. silu_gate, run by the reference's RoPE test but off the path
        cases.append(Case(**{**m, "shape": tuple(m["shape"])}, index=data[f"index_{i}"],
                          value=data[f"value_{i}"]))
    return cases


def _bf16_truncate(array) -> np.ndarray:
    # The reference test's helper keeps the upper 16 bits.
    return (np.asarray(array, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def regenerate(case: Case) -> dict:
    """Inputs of the reference test behind `case` (the arrays it uploads, in order)."""
    t, p = case.test, case.params
    if t == "test_attention_against_independent_numpy":
        rng = np.random.default_rng(17)
        b, s, h, kv, d = 2, 5, 4, 2, 64
        q = rng.normal(size=(b, s, h, d)).astype(np.float32)
        k = rng.normal(size=(b, s, kv, d)).astype(np.float32)
        v = rng.normal(size=k.shape).astype(np.float32)
        return {"q": q, "k": k, "v": v, "lengths": np.array([5, 2], np.uint32)}
    if t == "test_tiled_attention_ragged_f64":
        rng = np.random.default_rng(393)
        seq, dim, heads, kv = p["seq"], p["dim"], 4, 2
        q = rng.normal(size=(2, seq, heads, dim)).astype(np.float32)
        k, v = [rng.normal(size=(2, seq, kv, dim)).astype(np.float32) for _ in range(2)]
        return {"q": q, "k": k, "v": v, "lengths": np.array(p["length_pair"], np.uint32)}
    if t == "test_tiled_attention_extreme_logits_and_masked_blocks":
        rng = np.random.default_rng(718)
        seq, heads, dim = p["seq"], 2, 128
        q = np.full((1, seq, heads, dim), 10, np.float32)
        k = q.copy()
        k[:, 1::2] *= -1
        if p["pattern"] == "later_maximum":
            k[:] = -10
            k[:, 32:64] = 10
        elif p["pattern"] == "uniform":
            k[:] = 0
        v = rng.normal(size=q.shape).astype(np.float32)
        length = 65 if p["pattern"] == "later_maximum" else 33
        v[:, length:] = 1e10
        return {"q": q, "k": k, "v": v, "lengths": np.array([length], np.uint32)}
    if t == "test_rope_and_silu":
        rng = np.random.default_rng(8)
        return {"x": rng.normal(size=(2, 3, 4, 64)).astype(np.float32)}
    if t == "test_rms_and_pool":
        rng = np.random.default_rng(4)
        x = rng.normal(size=(2, 3, 64)).astype(np.float32)
        if case.check == 0:
            return {"x": x, "w": _bf16_truncate(np.ones(64))}
        return {"x": x, "lengths": np.array([1, 3], np.uint32)}
    if t == "test_bidirectional_attention_and_cls_pool":
        rng = np.random.default_rng(83)
        batch, seq, heads, dim = 2, 5, 3, 8
        q, k, v = [rng.normal(size=(batch, seq, heads, dim)).astype(np.float32) for _ in range(3)]
        lengths = np.array([5, 2], np.uint32)
        if case.check == 0:
            return {"q": q, "k": k, "v": v, "lengths": lengths}
        return {"x": q.reshape(batch, seq, heads * dim), "lengths": lengths}
    if t == "test_quantized_embedding_and_linear":
        rng = np.random.default_rng(1)
        code = rng.integers(0, 16, size=(8, 128), dtype=np.uint32)
        packed = np.bitwise_or.reduce(
            code.reshape(8, 16, 8) << np.arange(0, 32, 4, dtype=np.uint32), axis=-1)
        scales = _bf16_truncate(np.full((8, 2), 0.125))
        biases = _bf16_truncate(np.full((8, 2), -0.5))
        ids = np.array([7, 1, 3], np.uint32)
        if case.check == 0:
            return {"ids": ids, "packed": packed, "scales": scales, "biases": biases}
        x = rng.normal(size=(3, 128)).astype(np.float32)
        return {"x": x, "packed": packed, "scales": scales, "biases": biases}
    if t == "test_layer_norm_and_absolute_embedding":
        rng = np.random.default_rng(37)
        x = rng.normal(size=(3, 67)).astype(np.float32)
        scale = rng.normal(size=67).astype(np.float32)
        bias = rng.normal(size=67).astype(np.float32)
        if case.check == 0:
            return {"x": x, "w": scale, "b": bias}
        words = rng.normal(size=(17, 67)).astype(np.float32)
        positions = rng.normal(size=(4, 67)).astype(np.float32)
        types = rng.normal(size=(2, 67)).astype(np.float32)
        ids = np.array([[1, 3, 0, 0], [5, 6, 7, 8]], np.uint32)
        return {"ids": ids, "words": words, "positions": positions, "types": types}
    if t == "test_gelu_erf_form_and_bias":
        if case.check == 0:
            return {"x": np.linspace(-12, 12, 10001, dtype=np.float32)}
        return {"x": np.arange(12, dtype=np.float32).reshape(3, 4),
                "bias": np.array([-2, -1, 1, 2], np.float32)}
    if t in ("test_general_matmul", "test_tiled_matmul_and_unaligned_fallback"):
        m, k, n = p["shape"]
        rng = np.random.default_rng(7 if t == "test_general_matmul" else 33)
        a = rng.normal(size=(m, k)).astype(np.float32)
        b = rng.normal(size=(k, n)).astype(np.float32)
        return {"a": a, "bt": np.ascontiguousarray(b.T)}
    if t == "test_f32_chunked_projections_and_bounded_tail":
        m, n, k = p["m"], p["n"], p["k"]
        rng = np.random.default_rng(2026 + m)
        x = rng.normal(size=(m, k)).astype(np.float32)
        w = rng.normal(size=(n, k)).astype(np.float32)
        if p["pattern"] == "cancellation":
            x[:, 1::2] = -x[:, ::2]
            w[:, 1::2] = w[:, ::2] + np.float32(2**-16)
        return {"a": x, "bt": w}
    raise KeyError(t)


def inputs_match(case: Case, inputs: dict) -> bool:
    return [sha(a) for a in inputs.values()] == case.input_sha256


def compare(case: Case, result: np.ndarray, rtol=None, atol=None) -> float:
    """Checks `result` at the recorded sample positions against the reference's
    expected values; returns the max abs deviation there."""
    rtol = case.rtol if rtol is None else rtol
    atol = case.atol if atol is None else atol
    got = np.asarray(result, dtype=np.float64).reshape(-1)[case.index]
    np.testing.assert_allclose(got, case.value, rtol=rtol, atol=atol)
    return float(np.max(np.abs(got - case.value))) if got.size else 0.0
