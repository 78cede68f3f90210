"""Sequence shards across the GPUs of one node, driven from one host process.

The reference runs on one Apple GPU and has no multi-device code; what makes this
sharding exact is that its attention never mixes sequences (kernels.metal:86-91 indexes
every load by its own batch row) and its embedding forward is per text
(qwen3.py:112-296).  So a batch splits into independent shards, every device runs its
shard on its own context and stream, and no collective is needed on the data path.  The
attention splits a batch into contiguous ranges of sequences balanced by cost
(partition.shard_ranges): each device's inputs and outputs are then views of the
caller's arrays, moved without a host-side gather (at full link speed when the arrays
are page-locked).  The forward, whose inputs are token ids, assigns texts longest first
(partition.shard_by_cost) and copies back only the pooled embeddings.

One host thread per device issues that device's calls.  Every call into the native
library releases the interpreter lock for its whole duration (the host-buffer attention
call moves its inputs, runs the kernels and reads back before it returns; the forward is
one native call that queues all of its launches), so the devices work at the same time.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from concurrent.futures import ThreadPoolExecutor
from typing import Any

import numpy as np
from numpy.typing import NDArray

from . import native
from .attention import attention
from .errors import CudaUnavailableError, InvalidInputError
from .partition import sequence_cost, shard_by_cost, shard_ranges
from .runtime import CudaRuntime


def device_count() -> int:
    """CUDA devices visible to this process (0 when none)."""
    return int(native.load().tx_device_count())


class DeviceGroup:
    """One CudaRuntime (context + stream) per device and one worker thread per device."""

    def __init__(self, devices: Sequence[int] | None = None) -> None:
        if devices is None:
            count = device_count()
            if count < 1:
                raise CudaUnavailableError()
            devices = range(count)
        self.devices = [int(d) for d in devices]
        if not self.devices or len(set(self.devices)) != len(self.devices):
            raise InvalidInputError()
        self.runtimes: list[CudaRuntime] = []
        self._pool: ThreadPoolExecutor | None = None
        try:
            for d in self.devices:
                self.runtimes.append(CudaRuntime(d))
            self._pool = ThreadPoolExecutor(max_workers=len(self.devices),
                                            thread_name_prefix="tessery-device")
        except BaseException:
            self.close()
            raise

    def __len__(self) -> int:
        return len(self.devices)

    def run(self, fn: Callable[[CudaRuntime, Any], Any], work: Sequence[Any]) -> list[Any]:
        """fn(runtime, work[i]) for every device i at the same time; results in device
        order.  Work items that are None are skipped (their result is None).  Every
        device finishes before the first error, if any, is raised."""
        if self._pool is None:
            raise InvalidInputError()
        if len(work) != len(self.runtimes):
            raise InvalidInputError()
        futures = [None if item is None else self._pool.submit(fn, rt, item)
                   for rt, item in zip(self.runtimes, work, strict=True)]
        results: list[Any] = []
        error: BaseException | None = None
        for f in futures:
            if f is None:
                results.append(None)
                continue
            try:
                results.append(f.result())
            except BaseException as e:  # noqa: BLE001 - re-raised below, after the others
                results.append(None)
                error = error or e
        if error is not None:
            raise error
        return results

    def close(self) -> None:
        if self._pool is not None:
            self._pool.shutdown(wait=True)
            self._pool = None
        for rt in self.runtimes:
            rt.close()
        self.runtimes = []

    def __enter__(self) -> DeviceGroup:
        return self

    def __exit__(self, *_: object) -> None:
        self.close()


def attention_sharded(
    q: NDArray,
    k: NDArray,
    v: NDArray,
    *,
    group: DeviceGroup,
    lengths: NDArray | None = None,
    cu_seqlens: NDArray | None = None,
    causal: bool = True,
    scale: float | None = None,
    q_norm_weight: NDArray | None = None,
    k_norm_weight: NDArray | None = None,
    eps: float = 1e-6,
    theta: float = 1e6,
    out_dtype: str = "float32",
    out: NDArray | None = None,
) -> NDArray:
    """tessery_b200.attention with the sequences split across the group's devices.

    Same arguments, layouts and result as `attention` (padded q [B, L, H, d] with
    lengths [B], or packed q [T, H, d] with cu_seqlens [B+1]); the result is the same
    array the one-device call returns, bit for bit (each sequence goes through the same
    kernels with the same inputs).
    """
    if (lengths is None) == (cu_seqlens is None):
        raise InvalidInputError()
    out_np = {"float32": np.float32, "bf16": np.uint16}.get(out_dtype)
    if out_np is None:
        raise InvalidInputError()
    q, k, v = np.asarray(q), np.asarray(k), np.asarray(v)
    if out is None:
        out = np.empty(q.shape, dtype=out_np)
    elif out.shape != q.shape or out.dtype != out_np:
        raise InvalidInputError()
    common = dict(causal=causal, scale=scale, q_norm_weight=q_norm_weight,
                  k_norm_weight=k_norm_weight, eps=eps, theta=theta, out_dtype=out_dtype)
    if lengths is not None:
        lens = np.asarray(lengths)
        if lens.ndim != 1 or q.ndim != 4 or lens.size != q.shape[0]:
            raise InvalidInputError()
        ranges = shard_ranges(sequence_cost(lens, causal), len(group))

        def padded(rt: CudaRuntime, span: tuple[int, int]) -> None:
            a, b = span
            attention(q[a:b], k[a:b], v[a:b], lengths=lens[a:b], runtime=rt, out=out[a:b],
                      **common)

        group.run(padded, [r if r[1] > r[0] else None for r in ranges])
        return out
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    if cu.ndim != 1 or cu.size < 2 or q.ndim != 3 or int(cu[-1]) != q.shape[0]:
        raise InvalidInputError()
    lens = np.diff(cu)
    if np.any(lens <= 0):
        raise InvalidInputError()
    ranges = shard_ranges(sequence_cost(lens, causal), len(group))

    def packed(rt: CudaRuntime, span: tuple[int, int]) -> None:
        a, b = span
        r0, r1 = int(cu[a]), int(cu[b])
        attention(q[r0:r1], k[r0:r1], v[r0:r1], cu_seqlens=(cu[a:b + 1] - r0).astype(np.int32),
                  runtime=rt, out=out[r0:r1], **common)

    group.run(packed, [r if r[1] > r[0] else None for r in ranges])
    return out


class ShardedEncoder:
    """An embedding model with the texts of a batch split across devices: one encoder
    (its own copy of the weights, built by `factory(runtime)`) per device, texts assigned
    longest first by the encoder's forward cost, only the pooled rows copied back."""

    def __init__(self, factory: Callable[[CudaRuntime], Any], group: DeviceGroup) -> None:
        self.group = group
        loaded: list[Any] = [None] * len(group)

        def load(rt: CudaRuntime, i: int) -> None:
            loaded[i] = factory(rt)

        self.encoders = loaded
        try:
            group.run(load, list(range(len(group))))
        except BaseException:
            self.close()
            raise

    def _forward(self, ids: NDArray, lengths: NDArray, width: int, **kw: Any
                 ) -> NDArray[np.float32]:
        ids, lens = np.asarray(ids), np.asarray(lengths)
        if ids.ndim != 2 or lens.shape != (ids.shape[0],):
            raise InvalidInputError()
        costs = np.array([self.encoders[0].flops([n]) for n in lens], dtype=np.int64)
        owned = shard_by_cost(costs, len(self.group))
        result = np.empty((lens.size, width), dtype=np.float32)
        by_runtime = {id(e.rt): e for e in self.encoders}

        def run(rt: CudaRuntime, texts: NDArray[np.int64]) -> None:
            result[texts] = by_runtime[id(rt)].forward(ids[texts], lens[texts], **kw)

        self.group.run(run, [o if o.size else None for o in owned])
        return result

    def close(self) -> None:
        for e in self.encoders:
            if e is not None:
                e.close()
        self.encoders = []


class ShardedQwen3Encoder(ShardedEncoder):
    """Qwen3Encoder (qwen3.py:112-296) over every device of a group."""

    def __init__(self, weights: dict[str, NDArray], cfg: Any = None, *,
                 group: DeviceGroup, precise: bool = False) -> None:
        from .qwen3 import Qwen3Config, Qwen3Encoder

        self.cfg = cfg or Qwen3Config()
        super().__init__(lambda rt: Qwen3Encoder(weights, self.cfg, runtime=rt,
                                                 precise=precise), group)

    def forward(self, ids: NDArray, lengths: NDArray, *, dimensions: int | None = None
                ) -> NDArray[np.float32]:
        """Pooled, L2-normalised embeddings [batch, dimensions] of right-padded ids
        [batch, seq] with lengths [batch] (Qwen3Encoder.forward, sharded)."""
        dims = self.cfg.hidden if dimensions is None else int(dimensions)
        return self._forward(ids, lengths, dims, dimensions=dims)


class ShardedBertEncoder(ShardedEncoder):
    """BertEncoder (bert.py:104-235) over every device of a group."""

    def __init__(self, weights: dict[str, NDArray], cfg: Any = None, *,
                 group: DeviceGroup, precise: bool = True) -> None:
        from .bert import BertConfig, BertEncoder

        self.cfg = cfg or BertConfig()
        super().__init__(lambda rt: BertEncoder(weights, self.cfg, runtime=rt,
                                                precise=precise), group)

    def forward(self, ids: NDArray, lengths: NDArray) -> NDArray[np.float32]:
        """CLS embeddings [batch, hidden] of right-padded ids [batch, seq] (sharded)."""
        return self._forward(ids, lengths, self.cfg.hidden)
