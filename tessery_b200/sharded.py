"""Sequence shards across the GPUs of one node, driven from one host process.

The reference runs on one Apple GPU and has no multi-device code; what makes this
sharding exact is that its attention never mixes sequences (kernels.metal:86-91 indexes
every load by its own batch row) and its embedding forward is per text
(qwen3.py:112-296).  So a batch splits into independent shards: sequences are assigned
longest-processing-time first by their cost (partition.shard_by_cost), every device runs
its shard on its own context and stream, and no collective is needed on the data path.
Only results come back: the attention rows of each shard, or just the pooled embeddings
of the forward.

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
from .host import pinned_empty
from .partition import pack, sequence_cost, shard_by_cost
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
        self._staging: dict[tuple[int, str], NDArray] = {}
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

    def staging(self, index: int, name: str, shape: tuple[int, ...], dtype: Any) -> NDArray:
        """A page-locked host array of this shape for device `index`, reused across calls
        (grown when too small): the host side of that device's copies."""
        dtype = np.dtype(dtype)
        nbytes = int(np.prod(shape)) * dtype.itemsize
        key = (index, name)
        buf = self._staging.get(key)
        if buf is None or buf.nbytes < nbytes:
            buf = pinned_empty((max(nbytes, 1),), np.uint8)
            self._staging[key] = buf
        return buf[:nbytes].view(dtype).reshape(shape)

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
        self._staging.clear()

    def __enter__(self) -> DeviceGroup:
        return self

    def __exit__(self, *_: object) -> None:
        self.close()


def _gather(dst: NDArray, src: NDArray, starts: NDArray[np.int64], counts: NDArray[np.int64]
            ) -> None:
    """dst = the blocks src[starts[i] : starts[i] + counts[i]] laid end to end along axis
    0 (one contiguous copy per block: sequences are contiguous in both layouts)."""
    at = 0
    for a, n in zip(starts.tolist(), counts.tolist(), strict=True):
        dst[at:at + n] = src[a:a + n]
        at += n


def _scatter(dst: NDArray, src: NDArray, starts: NDArray[np.int64],
             counts: NDArray[np.int64]) -> None:
    """The inverse of _gather."""
    at = 0
    for a, n in zip(starts.tolist(), counts.tolist(), strict=True):
        dst[a:a + n] = src[at:at + n]
        at += n


def _stage(group: DeviceGroup, i: int, starts: NDArray[np.int64], counts: NDArray[np.int64],
           q: NDArray, k: NDArray, v: NDArray, out_dtype: Any
           ) -> tuple[NDArray, NDArray, NDArray, NDArray]:
    """Device i's blocks of q, k and v gathered into its page-locked staging arrays, and a
    staging array for its output rows."""
    rows = int(counts.sum())
    staged = []
    for name, a in (("q", q), ("k", k), ("v", v)):
        s = group.staging(i, name, (rows, *a.shape[1:]), a.dtype)
        _gather(s, a, starts, counts)
        staged.append(s)
    staged.append(group.staging(i, "out", (rows, *q.shape[1:]), out_dtype))
    return staged[0], staged[1], staged[2], staged[3]


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
        owned = shard_by_cost(sequence_cost(lens, causal), len(group))

        def padded(rt: CudaRuntime, job: tuple[int, NDArray[np.int64]]) -> None:
            i, seqs = job
            ones = np.ones_like(seqs)
            qs, ks, vs, os_ = _stage(group, i, seqs, ones, q, k, v, out_np)
            attention(qs, ks, vs, lengths=lens[seqs], runtime=rt, out=os_, **common)
            _scatter(out, os_, seqs, ones)

        group.run(padded, [(i, o) if o.size else None for i, o in enumerate(owned)])
        return out
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    if cu.ndim != 1 or cu.size < 2 or q.ndim != 3 or int(cu[-1]) != q.shape[0]:
        raise InvalidInputError()
    lens = np.diff(cu)
    if np.any(lens <= 0):
        raise InvalidInputError()
    owned = shard_by_cost(sequence_cost(lens, causal), len(group))

    def packed(rt: CudaRuntime, job: tuple[int, NDArray[np.int64]]) -> None:
        i, seqs = job
        qs, ks, vs, os_ = _stage(group, i, cu[seqs], lens[seqs], q, k, v, out_np)
        attention(qs, ks, vs, cu_seqlens=pack(lens[seqs]), runtime=rt, out=os_, **common)
        _scatter(out, os_, cu[seqs], lens[seqs])

    group.run(packed, [(i, o) if o.size else None for i, o in enumerate(owned)])
    return out


class ShardedQwen3Encoder:
    """The Qwen3 embedding forward with the texts of a batch split across devices: one
    Qwen3Encoder (its own copy of the weights) per device, texts assigned longest
    first by their forward cost, only the pooled rows copied back."""

    def __init__(self, weights: dict[str, NDArray], cfg: Any = None, *,
                 group: DeviceGroup, precise: bool = False) -> None:
        from .qwen3 import Qwen3Config, Qwen3Encoder

        self.cfg = cfg or Qwen3Config()
        self.group = group
        loaded: list[Any] = [None] * len(group)

        def load(rt: CudaRuntime, i: int) -> None:
            loaded[i] = Qwen3Encoder(weights, self.cfg, runtime=rt, precise=precise)

        self.encoders = loaded
        try:
            group.run(load, list(range(len(group))))
        except BaseException:
            self.close()
            raise

    def forward(self, ids: NDArray, lengths: NDArray, *, dimensions: int | None = None
                ) -> NDArray[np.float32]:
        """Pooled, L2-normalised embeddings [batch, dimensions] of right-padded ids
        [batch, seq] with lengths [batch] (Qwen3Encoder.forward, sharded)."""
        ids, lens = np.asarray(ids), np.asarray(lengths)
        if ids.ndim != 2 or lens.shape != (ids.shape[0],):
            raise InvalidInputError()
        dims = self.cfg.hidden if dimensions is None else int(dimensions)
        costs = np.array([self.encoders[0].flops([n]) for n in lens], dtype=np.int64)
        owned = shard_by_cost(costs, len(self.group))
        result = np.empty((lens.size, dims), dtype=np.float32)
        by_runtime = {id(e.rt): e for e in self.encoders}

        def run(rt: CudaRuntime, texts: NDArray[np.int64]) -> None:
            result[texts] = by_runtime[id(rt)].forward(ids[texts], lens[texts], dimensions=dims)

        self.group.run(run, [o if o.size else None for o in owned])
        return result

    def close(self) -> None:
        for e in self.encoders:
            if e is not None:
                e.close()
        self.encoders = []
