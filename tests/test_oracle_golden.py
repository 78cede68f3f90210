"""The CPU oracle against the golden vectors recorded from the reference's own tests."""

import numpy as np
import pytest

import oracle
import oracle.bert
import oracle.qwen3
from golden_cases import compare, inputs_match, load_cases, regenerate

CASES = load_cases()


def run_oracle(case, inputs):
    d = case.dispatch
    if case.kernel.startswith("attention"):
        return oracle.attention_padded(inputs["q"], inputs["k"], inputs["v"], inputs["lengths"],
                                       not d.get("bidirectional", 0), d["scale"])
    if case.kernel == "rope":
        x = inputs["x"].reshape(-1, d["heads"], d["dim"])
        pos = np.arange(x.shape[0]) % d["seq"]
        return oracle.rope(x, pos, d["theta"]).reshape(inputs["x"].shape)
    if case.kernel == "rms_norm":
        x = inputs["x"].reshape(-1, d["cols"])
        return oracle.rms_norm(x, inputs["w"], d["eps"]).reshape(inputs["x"].shape)
    if case.kernel == "pool_project":
        return oracle.pool_project(inputs["x"], inputs["lengths"], d["dim"],
                                   bool(d.get("first_token", 0)))
    if case.kernel == "layer_norm":
        return oracle.bert.layer_norm(inputs["x"], inputs["w"], inputs["b"], d["eps"])
    if case.kernel == "embedding_position":
        return oracle.bert.embedding_position(inputs["ids"], inputs["words"],
                                              inputs["positions"], inputs["types"])
    if case.kernel == "gelu_f32":
        return oracle.bert.gelu(inputs["x"])
    if case.kernel == "add_bias":
        return inputs["x"].astype(np.float64) + inputs["bias"]
    if case.kernel == "matmul_f32":
        return inputs["a"].astype(np.float64) @ inputs["bt"].astype(np.float64).T
    if case.kernel in ("embedding4", "linear4"):
        table = oracle.qwen3.dequant4(inputs["packed"], inputs["scales"], inputs["biases"])
        if case.kernel == "embedding4":
            return table[inputs["ids"]]
        return inputs["x"].astype(np.float64) @ table.T
    raise KeyError(case.kernel)


def test_fixture_covers_reference_grids():
    tests = {c.test for c in CASES}
    assert "test_tiled_attention_ragged_f64" in tests
    ragged = [c for c in CASES if c.test == "test_tiled_attention_ragged_f64"]
    assert len(ragged) == 44  # 2 dims x 2 directions x 11 (seq, lengths) rows
    extreme = [c for c in CASES if c.test.startswith("test_tiled_attention_extreme")]
    assert len(extreme) == 24
    assert all(c.oracle_max_abs <= c.atol + c.rtol * 1e10 for c in CASES)


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.id)
def test_oracle_matches_reference_expectations(case):
    inputs = regenerate(case)
    assert inputs_match(case, inputs), "regenerated inputs differ from the reference run"
    result = run_oracle(case, inputs)
    assert tuple(result.shape) == case.shape
    compare(case, result)
    # Whole-array moments recorded from the reference's expected array (which some
    # reference tests compute in float32: the element tolerance, summed, bounds the gap).
    np.testing.assert_allclose(np.sum(result, dtype=np.float64), case.sum, rtol=1e-9,
                               atol=1e-6 * max(1.0, abs(case.sum))
                               + case.atol * np.sqrt(result.size))


def test_gelu_restatements_agree():
    """The reference's float32 Abramowitz-Stegun evaluation of gelu_f32 and the math.erf
    form agree within the approximation's 1.5e-7 (plus float32 rounding)."""
    x = np.linspace(-12, 12, 10001, dtype=np.float32)
    np.testing.assert_allclose(oracle.bert.gelu_as(x), oracle.bert.gelu(x), atol=2e-6,
                               rtol=1e-6)


def test_packed_pool_matches_padded_pool():
    """The packed-row pooling restatement picks the same rows as the padded one."""
    rng = np.random.default_rng(9)
    x = rng.normal(size=(4, 10, 48))
    lengths = np.array([1, 10, 4, 7])
    cu = np.zeros(5, np.int64)
    cu[1:] = np.cumsum(lengths)
    packed = np.concatenate([x[b, :n] for b, n in enumerate(lengths)])
    for first in (False, True):
        np.testing.assert_array_equal(oracle.pool_project_packed(packed, cu, 40, first),
                                      oracle.pool_project(x, lengths, 40, first))
