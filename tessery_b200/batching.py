"""Varlen packing that replaces the reference's padded execution buckets.

The reference buckets inputs so that no row is padded to more than twice its length
and the bucket stays under a padded-token budget, then pads bucket widths to multiples
of 8 where that enables its tiled attention (batching.py:9-69, called from
api.py:225-242).  Packed (cu_seqlens) attention has no padded rows, so the only limits
left are the token budget and the sequence count per forward.
"""

from __future__ import annotations

from collections.abc import Iterator

import numpy as np
from numpy.typing import NDArray

from .partition import pack


def varlen_batches(
    lengths: NDArray, max_tokens: int, max_sequences: int | None = None
) -> Iterator[tuple[NDArray[np.intp], NDArray[np.int32]]]:
    """Yields (row indices, cu_seqlens) groups in input order.

    Each group holds whole sequences whose total length is at most `max_tokens` (a
    single longer sequence forms its own group) and at most `max_sequences` rows.
    """
    lengths = np.asarray(lengths, dtype=np.int64)
    if np.any(lengths <= 0):
        raise ValueError("lengths must be positive")
    start = 0
    while start < lengths.size:
        end, tokens = start, 0
        while end < lengths.size:
            nxt = tokens + int(lengths[end])
            if end > start and (nxt > max_tokens or (max_sequences and end - start >= max_sequences)):
                break
            tokens = nxt
            end += 1
        rows = np.arange(start, end, dtype=np.intp)
        yield rows, pack(lengths[start:end])
        start = end


def pack_rows(ids: NDArray, lengths: NDArray) -> tuple[NDArray, NDArray[np.int32]]:
    """Right-padded [B, W] rows -> packed [sum(lengths)] rows and cu_seqlens."""
    ids = np.asarray(ids)
    lengths = np.asarray(lengths, dtype=np.int64)
    if ids.ndim < 2 or lengths.shape != (ids.shape[0],) or np.any(lengths > ids.shape[1]):
        raise ValueError("bad padded batch")
    packed = np.concatenate([ids[b, : lengths[b]] for b in range(ids.shape[0])], axis=0)
    return packed, pack(lengths)


def unpack_rows(packed: NDArray, cu_seqlens: NDArray, width: int, fill=0) -> NDArray:
    """Packed rows -> right-padded [B, width, ...] rows (inverse of pack_rows)."""
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    batch = cu.size - 1
    out = np.full((batch, width) + packed.shape[1:], fill, dtype=packed.dtype)
    for b in range(batch):
        out[b, : cu[b + 1] - cu[b]] = packed[cu[b]:cu[b + 1]]
    return out
