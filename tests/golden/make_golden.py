"""Generates the golden fixtures that pin the CPU oracle to the reference.

Runs where the reference project's source tree is available; its root directory is
given as the first argument or in the TESSERY_REFERENCE environment variable.  It
imports the reference's own kernel test module (tests/real_metal/test_kernels.py) and
calls its attention, RoPE, RMSNorm, pooling, uint4 embedding/projection, LayerNorm,
absolute-embedding, GELU, bias and f32 matmul tests, unmodified and with their own seeds,
grids and tolerances,
against a fake runtime whose kernels are computed by ``oracle``.  Every
``numpy.testing.assert_allclose`` the reference tests make is intercepted to record the
reference's expected array (its own NumPy formula) and the verdict, then forwarded to
NumPy, so a failing comparison fails this script (assert_array_equal checks are
recorded the same way, with zero tolerance).

Output: tests/golden/reference_kernels.npz with, per case, the kernel name and
parameters, SHA-256 of every input array, a deterministic sample of the reference's
expected values (flat indices + float64 values), their moments, and the oracle's max
abs deviation.  The GPU tests regenerate the inputs, check the hashes, and compare the
CUDA output with these samples and with the oracle.

Usage: python tests/golden/make_golden.py <reference project root>
"""

from __future__ import annotations

import contextlib
import hashlib
import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

import oracle  # noqa: E402
import oracle.bert  # noqa: E402
from oracle.qwen3 import dequant4  # noqa: E402

def reference_root() -> Path:
    """The reference project's root: argv[1], else $TESSERY_REFERENCE."""
    given = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TESSERY_REFERENCE")
    if not given:
        sys.exit("usage: make_golden.py <reference project root> (or set TESSERY_REFERENCE)")
    return Path(given)

OUT = Path(__file__).resolve().parent / "reference_kernels.npz"
SAMPLES = 512

KERNEL_TESTS = [
    "test_attention_against_independent_numpy",
    "test_tiled_attention_ragged_f64",
    "test_tiled_attention_extreme_logits_and_masked_blocks",
    "test_rope_and_silu",
    "test_rms_and_pool",
    "test_bidirectional_attention_and_cls_pool",
    "test_quantized_embedding_and_linear",
    "test_layer_norm_and_absolute_embedding",
    "test_gelu_erf_form_and_bias",
    "test_general_matmul",
    "test_tiled_matmul_and_unaligned_fallback",
    "test_f32_chunked_projections_and_bounded_tail",
]


def sha(a: np.ndarray) -> str:
    a = np.ascontiguousarray(a)
    return hashlib.sha256(str(a.dtype).encode() + str(a.shape).encode() + a.tobytes()).hexdigest()


class FakeBuffer:
    def __init__(self, size: int, data: np.ndarray | None):
        self.size = size
        self.bytes = bytearray(size) if data is None else bytearray(np.ascontiguousarray(data).tobytes())
        self.data = data
        self.pointer = 1

    def view(self, dtype) -> np.ndarray:
        return np.frombuffer(self.bytes, dtype=dtype)

    def write(self, array: np.ndarray) -> None:
        self.bytes[:] = np.ascontiguousarray(array).tobytes()

    def close(self) -> None:
        self.pointer = None


class OracleEngine:
    """The slice of MetalRuntime the reference kernel tests use, computed by the oracle."""

    active_bytes = 0

    def __init__(self, log: list):
        self.log = log
        self.dispatches: dict[str, int] = {}

    def diagnostics(self):
        return {"dispatches": dict(self.dispatches)}

    def matmul(self, a, b):
        """MetalRuntime.matmul (metal.py:750-780): validation, the dispatch names its
        routing (metal.py:664-700) would record, and the float64 product."""
        from metal_inference.errors import InferenceError

        if (a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0] or a.dtype != np.float32
                or b.dtype != np.float32 or not a.size or not b.size):
            raise InferenceError()
        m, k = a.shape
        n = b.shape[1]
        if m >= 8 and (n, k) in ((384, 384), (1536, 384), (384, 1536)):
            names = ["matmul_f32_chunk32"] + (["matmul_f32"] if m % 8 else [])
        else:
            tiled = m >= 8 and m % 8 == 0 and n % 32 == 0 and k % 8 == 0 and k <= 512
            names = ["matmul_f32_tiled" if tiled else "matmul_f32"]
        for name in names:
            self.dispatches[name] = self.dispatches.get(name, 0) + 1
        self.log.append({"kernel": "matmul_f32", "params": {"rows": m, "cols": n, "k": k},
                         "inputs": [sha(np.ascontiguousarray(a)), sha(np.ascontiguousarray(b.T))]})
        return (a.astype(np.float64) @ b.astype(np.float64)).astype(np.float32)

    def buffer(self, size, data=None):
        return FakeBuffer(size, data)

    @contextlib.contextmanager
    def command(self):
        yield

    def read(self, buffer, shape):
        return buffer.view(np.float32).reshape(shape).copy()

    def _dispatch(self, name, buffers, **kw):
        entry = {"kernel": name, "params": {k: (float(v) if isinstance(v, float) else int(v))
                                            for k, v in kw.items()},
                 "inputs": [sha(b.data) for b in buffers if b.data is not None]}
        if name in ("attention", "attention_tiled", "attention_tail_32", "attention_tail_128"):
            seq, heads, kv, dim = kw["seq"], kw["heads"], kw["kv_heads"], kw["dim"]
            q = buffers[0].view(np.float32)
            tokens = q.size // (heads * dim)
            batch = tokens // seq
            q = q.reshape(batch, seq, heads, dim)
            k = buffers[1].view(np.float32).reshape(batch, seq, kv, dim)
            v = buffers[2].view(np.float32).reshape(batch, seq, kv, dim)
            lengths = buffers[3].view(np.uint32)
            out = oracle.attention_padded(q, k, v, lengths, not kw.get("bidirectional", 0),
                                          kw.get("scale", 1.0))
            buffers[4].write(out.astype(np.float32))
        elif name == "rope":
            dim, heads, seq = kw["dim"], kw["heads"], kw["seq"]
            x = buffers[0].view(np.float32).reshape(-1, heads, dim)
            pos = np.arange(x.shape[0]) % seq
            buffers[0].write(oracle.rope(x, pos, kw["theta"]).astype(np.float32))
        elif name == "rms_norm":
            cols = kw["cols"]
            x = buffers[0].view(np.float32).reshape(-1, cols)
            w = buffers[1].view(np.uint16)
            buffers[2].write(oracle.rms_norm(x, w, kw.get("eps", 1e-6)).astype(np.float32))
        elif name == "pool_project":
            seq, cols, dim = kw["seq"], kw["cols"], kw["dim"]
            x = buffers[0].view(np.float32).reshape(-1, seq, cols)
            lengths = buffers[1].view(np.uint32)
            out = oracle.pool_project(x, lengths, dim, bool(kw.get("first_token", 0)))
            buffers[2].write(out.astype(np.float32))
        elif name == "embedding4":
            cols = kw["cols"]
            ids = buffers[0].view(np.uint32)
            packed = buffers[1].view(np.uint32).reshape(-1, cols // 8)
            groups = (-1, cols // 64)
            table = dequant4(packed, buffers[2].view(np.uint16).reshape(groups),
                             buffers[3].view(np.uint16).reshape(groups))
            buffers[4].write(table[ids].astype(np.float32))
        elif name == "linear4":
            rows, cols, k = kw["rows"], kw["cols"], kw["k"]
            x = buffers[0].view(np.float32).reshape(rows, k).astype(np.float64)
            w = dequant4(buffers[1].view(np.uint32).reshape(cols, k // 8),
                         buffers[2].view(np.uint16).reshape(cols, k // 64),
                         buffers[3].view(np.uint16).reshape(cols, k // 64))
            buffers[4].write((x @ w.T).astype(np.float32))
        elif name == "layer_norm":
            cols = kw["cols"]
            x = buffers[0].view(np.float32).reshape(-1, cols)
            out = oracle.bert.layer_norm(x, buffers[1].view(np.float32),
                                         buffers[2].view(np.float32), kw["eps"])
            buffers[3].write(out.astype(np.float32))
        elif name == "embedding_position":
            cols, seq = kw["cols"], kw["seq"]
            ids = buffers[0].view(np.uint32).reshape(-1, seq)
            out = oracle.bert.embedding_position(
                ids, buffers[1].view(np.float32).reshape(-1, cols),
                buffers[2].view(np.float32).reshape(-1, cols),
                buffers[3].view(np.float32).reshape(-1, cols))
            buffers[4].write(out.astype(np.float32))
        elif name == "gelu_f32":
            buffers[0].write(oracle.bert.gelu(buffers[0].view(np.float32)).astype(np.float32))
        elif name == "add_bias":
            cols = kw["cols"]
            x = buffers[0].view(np.float32).reshape(-1, cols).astype(np.float64)
            buffers[0].write((x + buffers[1].view(np.float32)).astype(np.float32))
        elif name == "silu_gate":  # harness only: the RoPE test also exercises silu_gate
            a = buffers[0].view(np.float32).astype(np.float64)
            b = buffers[1].view(np.float32).astype(np.float64)
            buffers[0].write((a / (1 + np.exp(-a)) * b).astype(np.float32))
        else:
            raise NotImplementedError(name)
        self.log.append(entry)


def load_reference_tests():
    root = reference_root()
    sys.path.insert(0, str(root / "src"))
    path = root / "tests" / "real_metal" / "test_kernels.py"
    spec = importlib.util.spec_from_file_location("reference_test_kernels", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def grid(function):
    """Cartesian product of the function's pytest.mark.parametrize marks."""
    cases = [dict()]
    for mark in getattr(function, "pytestmark", []):
        if mark.name != "parametrize":
            continue
        names = [n.strip() for n in mark.args[0].split(",")]
        values = mark.args[1]
        new = []
        for base in cases:
            for value in values:
                row = dict(base)
                if len(names) == 1:
                    row[names[0]] = value
                else:
                    row.update(dict(zip(names, value, strict=True)))
                new.append(row)
        cases = new
    return cases


def main() -> None:
    module = load_reference_tests()
    rng = np.random.default_rng(20260909)
    records = []
    original = np.testing.assert_allclose
    for test_name in KERNEL_TESTS:
        function = getattr(module, test_name)
        for params in grid(function):
            log: list = []
            checks: list = []

            def capture(actual, desired, rtol=1e-7, atol=0, **kw):
                actual = np.asarray(actual)
                desired = np.asarray(desired)
                checks.append((actual.copy(), desired.astype(np.float64).copy(), rtol, atol))
                return original(actual, desired, rtol=rtol, atol=atol, **kw)

            def capture_equal(actual, desired, **kw):
                capture(actual, desired, rtol=0.0, atol=0.0)

            original_equal = np.testing.assert_array_equal
            np.testing.assert_allclose = capture
            np.testing.assert_array_equal = capture_equal
            try:
                function(OracleEngine(log), **params)
            finally:
                np.testing.assert_allclose = original
                np.testing.assert_array_equal = original_equal
            for index, (actual, desired, rtol, atol) in enumerate(checks):
                flat = desired.reshape(-1)
                count = min(SAMPLES, flat.size)
                idx = np.sort(rng.choice(flat.size, size=count, replace=False)).astype(np.int64)
                dispatch = log[index] if index < len(log) else log[-1]
                records.append({
                    "test": test_name,
                    "params": {k: (list(v) if isinstance(v, tuple) else v) for k, v in params.items()},
                    "check": index,
                    "kernel": dispatch["kernel"],
                    "dispatch": dispatch["params"],
                    "input_sha256": dispatch["inputs"],
                    "shape": list(desired.shape),
                    "rtol": float(rtol),
                    "atol": float(atol),
                    "oracle_max_abs": float(np.max(np.abs(actual.astype(np.float64) - desired))),
                    "sum": float(desired.sum()),
                    "sumsq": float((desired * desired).sum()),
                    "index": idx,
                    "value": flat[idx],
                })
            print(f"{test_name} {params}: {len(checks)} checks passed", flush=True)
    meta = [{k: v for k, v in r.items() if k not in ("index", "value")} for r in records]
    arrays = {}
    for i, r in enumerate(records):
        arrays[f"index_{i}"] = r["index"]
        arrays[f"value_{i}"] = r["value"]
    np.savez_compressed(OUT, meta=np.array(json.dumps(meta)), **arrays)
    print(f"wrote {OUT} ({len(records)} checks)")


if __name__ == "__main__":
    main()
