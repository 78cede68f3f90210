"""The one-process multi-GPU entry points on every visible device (needs a B200): results
of the sharded calls equal the one-device call's results bit for bit, since every
sequence goes through the same kernels with the same inputs wherever it lands."""

import numpy as np
import pytest

from tessery_b200 import attention
from tessery_b200.qwen3 import Qwen3Config, Qwen3Encoder, random_weights
from tessery_b200.sharded import DeviceGroup, ShardedQwen3Encoder, attention_sharded, device_count
from tessery_b200.workloads import qwen_padded, qwen_varlen, varlen_lengths

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def group():
    g = DeviceGroup()
    yield g
    g.close()


def test_device_count_matches_group(group):
    assert device_count() == len(group) >= 1


def test_sharded_varlen_attention_equals_one_device(group):
    w = qwen_varlen(seed=31, lengths=varlen_lengths(96, 31))
    kw = dict(causal=True, scale=w.scale, q_norm_weight=w.q_norm_weight,
              k_norm_weight=w.k_norm_weight, eps=w.eps, theta=w.theta)
    got = attention_sharded(w.q, w.k, w.v, group=group, cu_seqlens=w.cu_seqlens, **kw)
    want = attention(w.q, w.k, w.v, cu_seqlens=w.cu_seqlens, runtime=group.runtimes[0], **kw)
    np.testing.assert_array_equal(got, want)


def test_sharded_padded_attention_equals_one_device(group):
    w = qwen_padded(batch=24, seq=256, seed=32)
    kw = dict(causal=True, scale=w.scale, q_norm_weight=w.q_norm_weight,
              k_norm_weight=w.k_norm_weight, eps=w.eps, theta=w.theta)
    got = attention_sharded(w.q, w.k, w.v, group=group, lengths=w.lengths, **kw)
    want = attention(w.q, w.k, w.v, lengths=w.lengths, runtime=group.runtimes[0], **kw)
    valid = np.arange(w.seq)[None, :] < w.lengths[:, None]
    np.testing.assert_array_equal(got[valid], want[valid])


def test_sharded_forward_equals_one_device(group):
    cfg = Qwen3Config(layers=2, vocab=3000)
    weights = random_weights(cfg, seed=33)
    rng = np.random.default_rng(33)
    lengths = rng.integers(1, 300, size=11)
    ids = rng.integers(0, cfg.vocab, size=(lengths.size, int(lengths.max())))
    sharded = ShardedQwen3Encoder(weights, cfg, group=group)
    single = Qwen3Encoder(weights, cfg, runtime=group.runtimes[0])
    try:
        got = sharded.forward(ids, lengths)
        want = single.forward(ids, lengths)
    finally:
        sharded.close()
        single.close()
    np.testing.assert_array_equal(got, want)


def test_sharded_bert_forward_equals_one_device(group):
    from tessery_b200.bert import BertConfig, BertEncoder
    from tessery_b200.bert import random_weights as bert_weights
    from tessery_b200.sharded import ShardedBertEncoder

    cfg = BertConfig(layers=2, vocab=1000)
    weights = bert_weights(cfg, seed=34)
    rng = np.random.default_rng(34)
    lengths = rng.integers(1, 128, size=13)
    ids = rng.integers(0, cfg.vocab, size=(lengths.size, int(lengths.max())))
    sharded = ShardedBertEncoder(weights, cfg, group=group)
    single = BertEncoder(weights, cfg, runtime=group.runtimes[0])
    try:
        got = sharded.forward(ids, lengths)
        want = single.forward(ids, lengths)
    finally:
        sharded.close()
        single.close()
    np.testing.assert_array_equal(got, want)
