"""Host-side logic that needs no GPU: kernel routing, the Params block, sharding,
varlen packing, workload statistics and error mapping."""

import struct
from types import SimpleNamespace

import numpy as np
import pytest

from tessery_b200 import batching, partition, workloads
from tessery_b200.errors import DeviceTimeoutError, InferenceError, InvalidInputError
from tessery_b200.runtime import CudaRuntime, _raise_for


@pytest.mark.parametrize(
    "seq,dim,expected",
    [(32, 32, "attention_d32"), (64, 128, "attention"), (65, 128, "attention"),
     (128, 32, "attention_d32"), (511, 128, "attention"), (128, 64, "attention"),
     (513, 32, "attention_d32"), (1024, 128, "attention")],
)
def test_attention_route_and_grid(seq, dim, expected):
    calls = []
    fake = SimpleNamespace(_dispatch=lambda *a, **kw: calls.append((a, kw)))
    CudaRuntime._attention(fake, [], tokens=2 * seq, seq=seq, heads=4, kv_heads=2, dim=dim,
                           bidirectional=1)
    (args, kw), = calls
    assert args[0] == expected
    # One 32-thread group per (token, head), the grid of the reference's scalar kernel,
    # from which the library derives tokens = threads / 32 / heads.
    assert kw["threads"] == 2 * seq * 4 * 32 and kw["group_size"] == 32
    assert kw["scale"] == pytest.approx(dim**-0.5)
    assert kw["bidirectional"] == 1


def test_params_block_layout_matches_reference():
    # metal.py:596-614 packs "<12I4f"; the runtime builds the same 64 bytes field by field.
    import ctypes as ct

    from tessery_b200.runtime import _Params

    block = struct.pack("<12I4f", 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 1, 0, 1e-6, 1e6, 0.125, 0.0)
    assert len(block) == 64
    fields = struct.unpack("<12I4f", block)
    assert fields[4:7] == (5, 6, 7) and fields[10] == 1
    assert fields[14] == pytest.approx(0.125)
    ours = _Params(n=1, rows=2, cols=3, k=4, heads=5, kv_heads=6, seq=7, batch=8, dim=9,
                   group=10, bidirectional=1, first_token=0, eps=1e-6, theta=1e6, scale=0.125)
    assert ct.sizeof(ours) == 64
    assert bytes(ours) == block


def test_status_codes_map_to_stable_errors():
    _raise_for(0)
    with pytest.raises(InvalidInputError):
        _raise_for(1)
    with pytest.raises(InferenceError):
        _raise_for(2)
    with pytest.raises(DeviceTimeoutError):
        _raise_for(3)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_lpt_shards_cover_every_sequence_once_and_balance(world):
    lengths = workloads.varlen_lengths(256, 3)
    shards = partition.shard_sequences(lengths, world, causal=True)
    allidx = np.sort(np.concatenate(shards))
    assert np.array_equal(allidx, np.arange(lengths.size))
    cost = partition.sequence_cost(lengths, True)
    loads = np.array([cost[s].sum() for s in shards])
    # LPT bound: max load <= mean + largest single cost
    assert loads.max() <= loads.mean() + cost.max()


def test_gather_shard_and_pack_roundtrip():
    lengths = np.array([3, 1, 4, 2])
    cu = partition.pack(lengths)
    rows = np.arange(cu[-1] * 2).reshape(-1, 2)
    part, cu_part = partition.gather_shard(rows, cu, np.array([2, 0]))
    assert np.array_equal(cu_part, [0, 4, 7])
    assert np.array_equal(part[:4], rows[4:8]) and np.array_equal(part[4:], rows[0:3])


def test_varlen_batches_respect_budget_and_order():
    lengths = np.array([5, 600, 3, 3, 3, 100])
    groups = list(batching.varlen_batches(lengths, max_tokens=512, max_sequences=3))
    rows = np.concatenate([r for r, _ in groups])
    assert np.array_equal(rows, np.arange(lengths.size))
    for r, cu in groups:
        assert cu[-1] == lengths[r].sum()
        assert len(r) <= 3
        assert cu[-1] <= 512 or len(r) == 1
    with pytest.raises(ValueError):
        list(batching.varlen_batches(np.array([0, 2]), 10))


def test_pack_unpack_rows_roundtrip():
    rng = np.random.default_rng(0)
    ids = rng.integers(0, 100, size=(4, 9))
    lengths = np.array([9, 1, 4, 7])
    packed, cu = batching.pack_rows(ids, lengths)
    back = batching.unpack_rows(packed, cu, 9, fill=-1)
    for b in range(4):
        assert np.array_equal(back[b, : lengths[b]], ids[b, : lengths[b]])
        assert (back[b, lengths[b]:] == -1).all()


def test_workload_shapes_and_statistics():
    w = workloads.qwen_padded(batch=4, seq=64, seed=1)
    assert w.q.shape == (4, 64, 16, 128) and w.q.dtype == np.uint16
    assert w.k.shape == (4, 64, 8, 128)
    assert ((w.lengths >= 32) & (w.lengths <= 64)).all()
    n = w.lengths.astype(np.int64)
    assert w.useful_pairs() == int((n * (n + 1) // 2).sum())
    assert w.useful_flops() == 4 * 128 * 16 * w.useful_pairs()
    b = workloads.bge(batch=2, seq=16, seed=1)
    assert b.q.dtype == np.float32 and b.useful_pairs() == int((b.lengths.astype(int) ** 2).sum())
    v = workloads.qwen_varlen(nseq=50, seed=3)
    d = np.diff(v.cu_seqlens)
    assert d.min() >= 2 and d.max() <= 512 and v.q.shape[0] == v.cu_seqlens[-1]
    t = workloads.short_tails("bge", batch=8, seed=4)
    assert t.dim == 32 and not t.causal and np.diff(t.cu_seqlens).max() <= 32


def test_bf16_conversion_rounds_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38], np.float32)
    bits = workloads.to_bf16_bits(x)
    back = workloads.from_bf16_bits(bits)
    assert back[0] == 1.0
    assert back[1] == 1.0  # tie (1 + 2^-8) rounds to even
    assert back[2] == np.float32(1.015625)
    assert back[3] == -2.5
    import oracle

    assert np.array_equal(oracle.bf16_bits(x), bits)


def test_gate_up_interleave_blocks():
    from tessery_b200.qwen3 import interleave_gate_up

    g = np.arange(256 * 3).reshape(256, 3)
    u = -g
    fused = interleave_gate_up(g, u)
    assert np.array_equal(fused[:128], g[:128]) and np.array_equal(fused[128:256], u[:128])
    assert np.array_equal(fused[256:384], g[128:]) and np.array_equal(fused[384:], u[128:])
