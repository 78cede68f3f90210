"""Host logic of the one-process multi-GPU entry points (tessery_b200/sharded.py) on CPU:
the device calls are replaced by the NumPy oracle, so what is checked is the split of a
batch into longest-first shards, the gather of each shard's rows, the scatter of the
results back into batch order, empty shards, and error propagation."""

from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import oracle
from tessery_b200 import sharded
from tessery_b200.partition import pack, shard_by_cost, shard_ranges


class FakeRuntime:
    def __init__(self, device):
        self.device = device
        self.calls = []

    def close(self):
        pass


def fake_group(n):
    group = sharded.DeviceGroup.__new__(sharded.DeviceGroup)
    group.devices = list(range(n))
    group.runtimes = [FakeRuntime(d) for d in range(n)]
    group._pool = ThreadPoolExecutor(max_workers=n)
    return group


@pytest.fixture
def cpu_attention(monkeypatch):
    """sharded.attention replaced by the float64 oracle."""

    def attention(q, k, v, *, lengths=None, cu_seqlens=None, causal=True, scale=None,
                  runtime=None, out=None, **_):
        scale = q.shape[-1] ** -0.5 if scale is None else scale
        if lengths is not None:
            r = oracle.attention_padded(q, k, v, lengths, causal, scale)
            runtime.calls.append(len(lengths))
        else:
            r = oracle.attention_varlen(q, k, v, cu_seqlens, causal, scale)
            runtime.calls.append(len(cu_seqlens) - 1)
        out[...] = r
        return out

    monkeypatch.setattr(sharded, "attention", attention)


@pytest.mark.parametrize("devices", [1, 2, 3, 8])
@pytest.mark.parametrize("causal", [True, False])
def test_padded_shards_match_the_whole_batch(cpu_attention, devices, causal):
    rng = np.random.default_rng(devices)
    b, seq, h, kv, d = 6, 40, 4, 2, 32
    lengths = rng.integers(1, seq + 1, size=b)
    q = rng.standard_normal((b, seq, h, d)).astype(np.float32)
    k = rng.standard_normal((b, seq, kv, d)).astype(np.float32)
    v = rng.standard_normal((b, seq, kv, d)).astype(np.float32)
    group = fake_group(devices)
    got = sharded.attention_sharded(q, k, v, group=group, lengths=lengths, causal=causal)
    want = oracle.attention_padded(q, k, v, lengths, causal, d**-0.5)
    valid = np.arange(seq)[None, :] < lengths[:, None]
    np.testing.assert_allclose(got[valid], want[valid], rtol=1e-6, atol=1e-6)
    # Every sequence went to exactly one device.
    calls = [sum(rt.calls) for rt in group.runtimes]
    assert sum(calls) == b
    assert sum(1 for c in calls if c) <= min(devices, b)
    group.close()


@pytest.mark.parametrize("devices", [1, 2, 4])
def test_packed_shards_match_the_whole_batch(cpu_attention, devices):
    rng = np.random.default_rng(10 + devices)
    lengths = rng.integers(1, 70, size=9)
    cu = pack(lengths)
    t, h, kv, d = int(cu[-1]), 4, 2, 32
    q = rng.standard_normal((t, h, d)).astype(np.float32)
    k = rng.standard_normal((t, kv, d)).astype(np.float32)
    v = rng.standard_normal((t, kv, d)).astype(np.float32)
    group = fake_group(devices)
    got = sharded.attention_sharded(q, k, v, group=group, cu_seqlens=cu, causal=True)
    want = oracle.attention_varlen(q, k, v, cu, True, d**-0.5)
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)
    group.close()


@pytest.mark.parametrize("world", [1, 2, 3, 8, 20])
def test_contiguous_ranges_cover_and_balance(world):
    rng = np.random.default_rng(world)
    cost = rng.integers(1, 1000, size=50)
    ranges = shard_ranges(cost, world)
    assert ranges[0][0] == 0 and ranges[-1][1] == cost.size
    assert all(a <= b for a, b in ranges)
    assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
    loads = [int(cost[a:b].sum()) for a, b in ranges]
    if world <= cost.size:
        assert max(loads) <= cost.sum() / world + cost.max()


def test_shards_balance_cost_longest_first():
    cost = np.array([100, 1, 60, 50, 5, 40])
    owned = shard_by_cost(cost, 2)
    loads = sorted(int(cost[o].sum()) for o in owned)
    assert loads == [116, 140]  # 100+40 | 60+50+5+1
    assert sorted(np.concatenate(owned).tolist()) == list(range(cost.size))


def test_an_error_on_one_device_is_raised_after_all_finish(monkeypatch):
    finished = []

    def attention(q, k, v, *, runtime=None, out=None, **_):
        if runtime.device == 1:
            raise RuntimeError("device 1 failed")
        finished.append(runtime.device)
        return out

    monkeypatch.setattr(sharded, "attention", attention)
    q = np.zeros((4, 8, 2, 32), np.float32)
    k = np.zeros((4, 8, 1, 32), np.float32)
    group = fake_group(3)
    with pytest.raises(RuntimeError, match="device 1"):
        sharded.attention_sharded(q, k, k, group=group, lengths=np.array([8, 7, 6, 5]))
    assert sorted(finished) == [0, 2]
    group.close()


def test_sharded_forward_scatters_pooled_rows(monkeypatch):
    """ShardedQwen3Encoder: every text's pooled row comes back at its batch position."""
    import tessery_b200.qwen3 as q3

    class FakeEncoder:
        def __init__(self, weights, cfg, runtime=None, precise=False):
            self.rt = runtime
            self.cfg = cfg

        def flops(self, lengths):
            n = np.asarray(lengths, dtype=np.int64)
            return int((1000 * n + n * n).sum())

        def forward(self, ids, lengths, dimensions=None):
            self.rt.calls.append(len(lengths))
            # Row = (first id, length, device) so placement can be checked.
            rows = np.zeros((len(lengths), dimensions), np.float32)
            rows[:, 0] = ids[:, 0]
            rows[:, 1] = lengths
            rows[:, 2] = self.rt.device
            return rows

        def close(self):
            pass

    monkeypatch.setattr(q3, "Qwen3Encoder", FakeEncoder)
    group = fake_group(3)
    model = sharded.ShardedQwen3Encoder({}, q3.Qwen3Config(layers=1), group=group)
    rng = np.random.default_rng(3)
    lengths = rng.integers(1, 50, size=10)
    ids = rng.integers(0, 1000, size=(10, 50))
    got = model.forward(ids, lengths, dimensions=8)
    np.testing.assert_array_equal(got[:, 0], ids[:, 0])
    np.testing.assert_array_equal(got[:, 1], lengths)
    assert sorted(sum(rt.calls) for rt in group.runtimes) == sorted(
        int(o.size) for o in shard_by_cost(1000 * lengths + lengths**2, 3))
    model.close()
    group.close()
