"""The N>1 path on CPU: two gloo ranks shard one varlen batch by sequence (LPT), each
computes its own shard with no data-path collective, and the union of the shards equals
the single-process result.  A rank that fails is detected by its peer as an error (short
process-group timeout), never a hang.  The per-rank compute here is the CPU oracle, a
stand-in for the per-GPU kernel; only the host logic is under test."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from tessery_b200 import gather_shard, shard_sequences, workloads
from tessery_b200.workloads import from_bf16_bits


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def small_batch():
    lengths = workloads.varlen_lengths(12, 9, median=20, hi=64)
    w = workloads.qwen_varlen(seed=9, lengths=lengths)
    return w


def rank_main(rank, world, port, out_dir, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        w = small_batch()
        lengths = np.diff(w.cu_seqlens)
        owned = shard_sequences(lengths, world, causal=True)[rank]
        q, cu = gather_shard(from_bf16_bits(w.q), w.cu_seqlens, owned)
        k, _ = gather_shard(from_bf16_bits(w.k), w.cu_seqlens, owned)
        v, _ = gather_shard(from_bf16_bits(w.v), w.cu_seqlens, owned)
        if rank == fail_rank:
            raise RuntimeError("injected rank failure")
        out = oracle.attention_varlen(q, k, v, cu, True, w.scale)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), owned=owned, cu=cu, out=out)
        dist.barrier()  # host-side completion only; no tensor crosses ranks
    except RuntimeError as e:
        with open(os.path.join(out_dir, f"rank{rank}.err"), "w") as f:
            f.write(str(e))
    finally:
        dist.destroy_process_group()


def run(world, fail_rank, tmp_path):
    port = free_port()
    mp.start_processes(rank_main, args=(world, port, str(tmp_path), fail_rank), nprocs=world,
                       join=True, start_method="spawn")


def test_two_ranks_reproduce_single_process(tmp_path):
    run(2, -1, tmp_path)
    w = small_batch()
    full = oracle.attention_varlen(from_bf16_bits(w.q), from_bf16_bits(w.k), from_bf16_bits(w.v),
                                   w.cu_seqlens, True, w.scale)
    seen = []
    for r in range(2):
        d = np.load(tmp_path / f"rank{r}.npz")
        for j, s in enumerate(d["owned"]):
            a, b = w.cu_seqlens[s], w.cu_seqlens[s + 1]
            np.testing.assert_array_equal(d["out"][d["cu"][j]:d["cu"][j + 1]], full[a:b])
            seen.append(int(s))
    assert sorted(seen) == list(range(len(w.cu_seqlens) - 1))


def test_failed_rank_is_reported_not_hung(tmp_path):
    run(2, 1, tmp_path)
    assert (tmp_path / "rank1.err").read_text() == "injected rank failure"
    # The surviving rank's barrier ended with an error instead of waiting forever.
    assert (tmp_path / "rank0.err").exists()
    assert not (tmp_path / "rank1.npz").exists()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_weak_scaling_shards_are_balanced(world):
    rng = np.random.default_rng(2)
    lengths = rng.integers(32, 513, size=32 * world)
    shards = shard_sequences(lengths, world, causal=True)
    assert all(abs(len(s) - 32) <= 8 for s in shards)
