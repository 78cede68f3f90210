"""Sequence sharding across the GPUs of one node.

Attention never mixes sequences (kernels.metal:86-91 indexes every load by its own
batch row), so a batch splits into independent shards with no collective on the data
path.  Sequences are assigned longest-processing-time first: sorted by attention cost
(n(n+1)/2 causal, n^2 bidirectional) and each placed on the least-loaded rank.
"""

from __future__ import annotations

import heapq

import numpy as np
from numpy.typing import NDArray


def sequence_cost(lengths: NDArray, causal: bool) -> NDArray[np.int64]:
    n = np.asarray(lengths, dtype=np.int64)
    return n * (n + 1) // 2 if causal else n * n


def shard_sequences(lengths: NDArray, world: int, causal: bool = True) -> list[NDArray[np.int64]]:
    """Returns, per rank, the (sorted) indices of the sequences it owns."""
    return shard_by_cost(sequence_cost(lengths, causal), world)


def shard_by_cost(cost: NDArray, world: int) -> list[NDArray[np.int64]]:
    """Longest-processing-time assignment of items with these costs to `world` ranks:
    per rank, the (sorted) indices of the items it owns."""
    if world < 1:
        raise ValueError("world must be positive")
    cost = np.asarray(cost, dtype=np.int64)
    order = np.argsort(-cost, kind="stable")
    heap = [(0, r) for r in range(world)]
    owned: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        owned[r].append(int(i))
        heapq.heappush(heap, (load + int(cost[i]), r))
    return [np.array(sorted(o), dtype=np.int64) for o in owned]


def shard_ranges(cost: NDArray, world: int) -> list[tuple[int, int]]:
    """Contiguous, cost-balanced split of items [0, n) into `world` ranges [a, b): cut
    where the running cost crosses each multiple of total / world.  The ranges of a
    packed or padded batch are contiguous in memory, so a shard needs no gather; the
    imbalance is at most about one item's cost."""
    if world < 1:
        raise ValueError("world must be positive")
    cost = np.asarray(cost, dtype=np.float64)
    prefix = np.concatenate([[0.0], np.cumsum(cost)])
    total = prefix[-1]
    cuts = [0]
    for r in range(1, world):
        target = total * r / world
        c = int(np.searchsorted(prefix, target))
        # The cut nearer to the target, kept monotone.
        if c > 0 and abs(prefix[c - 1] - target) <= abs(prefix[min(c, cost.size)] - target):
            c -= 1
        cuts.append(min(max(c, cuts[-1]), cost.size))
    cuts.append(cost.size)
    return [(cuts[r], cuts[r + 1]) for r in range(world)]


def pack(lengths: NDArray) -> NDArray[np.int32]:
    """cu_seqlens for sequences laid end to end."""
    n = np.asarray(lengths, dtype=np.int64)
    cu = np.zeros(n.size + 1, dtype=np.int64)
    cu[1:] = np.cumsum(n)
    if cu[-1] >= 2**31:
        raise ValueError("too many tokens for int32 offsets")
    return cu.astype(np.int32)


def gather_shard(tensor: NDArray, cu_seqlens: NDArray, owned: NDArray) -> tuple[NDArray,
                                                                                 NDArray]:
    """Rows of the owned sequences of a packed tensor, and their cu_seqlens."""
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    pieces = [tensor[cu[i]:cu[i + 1]] for i in owned]
    lengths = np.array([cu[i + 1] - cu[i] for i in owned], dtype=np.int64)
    rows = np.concatenate(pieces, axis=0) if pieces else tensor[:0]
    return rows, pack(lengths)
