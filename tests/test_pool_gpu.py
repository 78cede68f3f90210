"""Embedding pooling (pool_project, kernels.metal:339-349, with the final rms_norm of
qwen3.py:281-290 optionally fused) on a B200 against the oracle and the reference's
golden vectors.

Tolerance: the reference's own gate for pool_project, atol 1e-6 on unit-norm rows
(test_kernels.py:113-122), for fp32 inputs; bf16 inputs are compared with the oracle
fed the same bf16 values, so the same gate applies.
"""

import numpy as np
import pytest

import oracle
from golden_cases import compare, load_cases, regenerate
from tessery_b200 import InvalidInputError, pool_project
from tessery_b200.workloads import from_bf16_bits, to_bf16_bits

pytestmark = pytest.mark.gpu

ATOL = 1e-6
POOL_CASES = [c for c in load_cases() if c.kernel == "pool_project"]


@pytest.mark.parametrize("case", POOL_CASES, ids=lambda c: c.id)
def test_reference_golden_pool_case(runtime, case):
    """Through CudaRuntime._dispatch with the reference's kernel name and parameters."""
    inputs = regenerate(case)
    arrays = [np.ascontiguousarray(a) for a in inputs.values()]
    buffers = [runtime.buffer(a.nbytes, a) for a in arrays]
    out = runtime.buffer(int(np.prod(case.shape)) * 4)
    try:
        with runtime.command():
            runtime._dispatch("pool_project", buffers + [out], **case.dispatch)
        assert runtime.last_kernel() == "pool_project"
        got = runtime.read(out, case.shape)
    finally:
        for b in buffers + [out]:
            b.close()
    compare(case, got, rtol=0, atol=ATOL)
    d = case.dispatch
    want = oracle.pool_project(inputs["x"], inputs["lengths"], d["dim"],
                               bool(d.get("first_token", 0)))
    np.testing.assert_allclose(got, want, atol=ATOL, rtol=0)


@pytest.mark.parametrize("cols,dim", [(1024, 1024), (1024, 512), (384, 384), (130, 67)])
@pytest.mark.parametrize("first_token", [False, True])
def test_pool_padded_fp32(runtime, cols, dim, first_token):
    rng = np.random.default_rng(cols + dim + first_token)
    b, seq = 9, 37
    x = rng.normal(size=(b, seq, cols)).astype(np.float32)
    lengths = rng.integers(1, seq + 1, size=b).astype(np.uint32)
    lengths[0], lengths[-1] = 1, seq
    got = pool_project(x, lengths=lengths, dim=dim, first_token=first_token, runtime=runtime)
    assert runtime.last_kernel() == "pool_project"
    want = oracle.pool_project(x, lengths, dim, first_token)
    np.testing.assert_allclose(got, want, atol=ATOL, rtol=0)


@pytest.mark.parametrize("cols,dim", [(1024, 1024), (1024, 256), (100, 90)])
def test_pool_with_fused_final_norm(runtime, cols, dim):
    """RMSNorm of the pooled row with the final norm weight, then L2 normalisation: the
    same result as normalising every token (qwen3.py:281) and pooling afterwards."""
    rng = np.random.default_rng(7 + cols)
    b, seq, eps = 6, 20, 1e-6
    x = (3 * rng.normal(size=(b, seq, cols))).astype(np.float32)
    w = to_bf16_bits(1.0 + 0.02 * rng.normal(size=cols).astype(np.float32))
    lengths = np.array([1, 20, 7, 13, 2, 19], np.uint32)
    got = pool_project(x, lengths=lengths, dim=dim, norm_weight=w, eps=eps, runtime=runtime)
    normed = oracle.rms_norm(x, w, eps)
    want = oracle.pool_project(normed, lengths, dim, False)
    np.testing.assert_allclose(got, want, atol=ATOL, rtol=0)


@pytest.mark.parametrize("first_token", [False, True])
def test_pool_packed_bf16(runtime, first_token):
    rng = np.random.default_rng(21)
    lengths = np.array([1, 5, 300, 2, 77])
    cu = np.zeros(lengths.size + 1, np.int32)
    cu[1:] = np.cumsum(lengths)
    x = to_bf16_bits(rng.normal(size=(int(cu[-1]), 1024)).astype(np.float32))
    w = to_bf16_bits(1.0 + 0.02 * rng.normal(size=1024).astype(np.float32))
    got = pool_project(x, cu_seqlens=cu, first_token=first_token, norm_weight=w,
                       runtime=runtime)
    xf = from_bf16_bits(x)
    want = oracle.pool_project_packed(oracle.rms_norm(xf, w, 1e-6), cu, 1024, first_token)
    np.testing.assert_allclose(got, want, atol=ATOL, rtol=0)
    # Unit rows, as the reference's callers check (qwen3.py:293-297).
    np.testing.assert_allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)


def test_pool_rows_without_a_valid_token_are_nan(runtime):
    rng = np.random.default_rng(3)
    x = rng.normal(size=(3, 8, 64)).astype(np.float32)
    got = pool_project(x, lengths=np.array([0, 8, 9], np.uint32), runtime=runtime)
    assert np.isnan(got[0]).all() and np.isnan(got[2]).all()
    np.testing.assert_allclose(got[1], oracle.pool_project(x[1:2], [8], 64, False)[0],
                               atol=ATOL, rtol=0)
    cu = np.array([0, 0, 8, 8], np.int32)
    got = pool_project(x.reshape(24, 64), cu_seqlens=cu, runtime=runtime)
    assert np.isnan(got[0]).all() and np.isnan(got[2]).all()
    assert np.isfinite(got[1]).all()


def test_pool_invalid_arguments(runtime):
    x = np.zeros((2, 4, 16), np.float32)
    with pytest.raises(InvalidInputError):
        pool_project(x, lengths=np.array([1, 1], np.uint32), dim=17, runtime=runtime)
    with pytest.raises(InvalidInputError):
        pool_project(x, runtime=runtime)
    with pytest.raises(InvalidInputError):
        pool_project(x.astype(np.float64), lengths=np.array([1, 1]), runtime=runtime)
