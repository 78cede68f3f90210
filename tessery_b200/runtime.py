"""CudaRuntime: the MetalRuntime-shaped host API over libtessattn.so.

It keeps the surface the reference's model adapters and kernel tests use on the
attention path (metal.py:94-119 Buffer, :169-414 runtime/command, :532-648
_attention/_dispatch, :650-662 read), so code written against MetalRuntime for these
operations runs unchanged; commands are CUDA stream-ordered instead of Metal command
buffers.  It adds typed entry points that take device pointers (bf16 inputs, varlen
packing, the fused q/k prologue).  NumPy in, NumPy out; no PyTorch dependency.
"""

from __future__ import annotations

import ctypes as ct
import struct
import threading
from collections import Counter
from collections.abc import Iterator, Sequence
from contextlib import contextmanager
from typing import Any
from weakref import WeakSet

import numpy as np
from numpy.typing import NDArray

from . import native
from .errors import (
    ClosedError,
    CudaUnavailableError,
    DeviceTimeoutError,
    InferenceError,
    InvalidInputError,
)

ATTENTION_KERNELS = (
    "attention",
    "attention_tiled",
    "attention_tail_32",
    "attention_tail_128",
    "attention_d32",
)


def _raise_for(rc: int) -> None:
    if rc == native.TX_OK:
        return
    if rc == native.TX_EINVAL:
        raise InvalidInputError()
    if rc == native.TX_ETIMEOUT:
        raise DeviceTimeoutError()
    raise InferenceError()


class Buffer:
    """Owned device buffer (counterpart of metal.py:94-119)."""

    def __init__(self, runtime: CudaRuntime, size: int, data: NDArray[Any] | None) -> None:
        self.runtime = runtime
        self.size = size
        self.pointer: int | None = runtime._lib.tx_buffer(
            runtime._pointer, None if data is None else data.ctypes.data, size
        )
        if not self.pointer:
            raise InferenceError()
        runtime.active_bytes += size
        runtime._allocations += 1
        runtime._allocated_bytes += size
        runtime.peak_bytes = max(runtime.peak_bytes, runtime.active_bytes)
        runtime._buffers.add(self)

    @property
    def device_ptr(self) -> int:
        if not self.pointer:
            raise ClosedError()
        return int(self.runtime._lib.tx_buffer_device_ptr(self.pointer))

    def write(self, data: NDArray[Any]) -> None:
        data = np.ascontiguousarray(data)
        if data.nbytes > self.size:
            raise InvalidInputError()
        _raise_for(self.runtime._lib.tx_write(self.pointer, data.ctypes.data, data.nbytes))

    def close(self) -> None:
        with self.runtime._lock:
            if getattr(self, "pointer", None):
                self.runtime._lib.tx_free(self.pointer)
                self.pointer = None
                self.runtime.active_bytes -= self.size

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


class CudaRuntime:
    """Stream-ordered command owner on one B200; commands are serialised per instance."""

    def __init__(self, device: int = 0) -> None:
        self._lib = native.load()
        self._pointer: int | None = self._lib.tx_create(device)
        if not self._pointer:
            raise CudaUnavailableError()
        self.device = device
        self._lock = threading.RLock()
        self._recording = False
        self._buffers: WeakSet[Buffer] = WeakSet()
        self._workspace: dict[str, Buffer] = {}
        self.active_bytes = 0
        self.peak_bytes = 0
        self._allocations = 0
        self._allocated_bytes = 0
        self._commands = 0
        self._gpu_samples = 0
        self._gpu_seconds = 0.0
        self._dispatches: Counter[str] = Counter()
        self._profile: list[dict[str, Any]] | None = None
        self._profile_command: list[dict[str, Any]] = []

    # ---- bookkeeping ------------------------------------------------------------------
    @property
    def sms(self) -> int:
        return int(self._lib.tx_device_sms(self._pointer))

    def last_kernel(self) -> str:
        """Route of the last attention call: "tc_bf16_d128", "simt" or "d32" (or "pool_project")."""
        raw = self._lib.tx_last_kernel(self._pointer)
        return raw.decode() if raw else ""

    def launch_count(self) -> int:
        """Kernels launched by this runtime's context so far."""
        return int(self._lib.tx_launch_count(self._pointer))

    def last_error(self) -> str:
        raw = self._lib.tx_last_error(self._pointer)
        return raw.decode() if raw else ""

    def diagnostics(self) -> dict[str, Any]:
        with self._lock:
            return {
                "native_library_sha256": self._lib._tessery_sha256,
                "native_library_path": self._lib._tessery_path,
                "allocations": self._allocations,
                "allocated_bytes": self._allocated_bytes,
                "completed_commands": self._commands,
                "gpu_timed_commands": self._gpu_samples,
                "gpu_seconds": self._gpu_seconds,
                "dispatches": dict(self._dispatches),
                "active_bytes": self.active_bytes,
                "peak_bytes": self.peak_bytes,
            }

    def _check_open(self) -> None:
        if not self._pointer:
            raise ClosedError()

    # ---- buffers (metal.py:354-373, 650-662) -------------------------------------------
    def buffer(self, size: int, data: NDArray[Any] | None = None) -> Buffer:
        with self._lock:
            self._check_open()
            if type(size) is not int or not 0 < size <= 2**40:
                raise InvalidInputError()
            if data is not None and (not data.flags.c_contiguous or data.nbytes != size):
                raise InvalidInputError()
            return Buffer(self, size, data)

    def read(self, buffer: Buffer, shape: tuple[int, ...], dtype=np.float32) -> NDArray[Any]:
        with self._lock:
            self._check_open()
            if self._recording or buffer.runtime is not self or not buffer.pointer:
                raise InferenceError()
            result = np.empty(shape, dtype=dtype)
            if result.nbytes != buffer.size:
                raise InferenceError()
            _raise_for(self._lib.tx_read(buffer.pointer, result.ctypes.data, result.nbytes))
            return result

    def workspace(self, name: str, size: int) -> Buffer:
        """Named, reusable device buffer of at least `size` bytes."""
        with self._lock:
            cached = self._workspace.get(name)
            if cached is not None and cached.pointer and cached.size >= size:
                return cached
            if cached is not None:
                cached.close()
            buffer = self.buffer(max(size, 256))
            self._workspace[name] = buffer
            return buffer

    # ---- commands (metal.py:375-414) --------------------------------------------------
    @contextmanager
    def command(self) -> Iterator[None]:
        with self._lock:
            self._check_open()
            if self._recording:
                raise InferenceError()
            if self._lib.tx_begin(self._pointer):
                self._lib.tx_abort(self._pointer)
                raise InferenceError()
            self._recording = True
            self._profile_command.clear()
            try:
                yield
                rc = self._lib.tx_finish(self._pointer)
                if rc:
                    _raise_for(rc)
                if self._profile is not None:
                    timings = (ct.c_double * len(self._profile_command))()
                    if self._lib.tx_profile_read(self._pointer, timings, len(timings)):
                        raise InferenceError()
                    self._profile.extend(
                        dict(record, gpu_seconds=float(seconds))
                        for record, seconds in zip(self._profile_command, timings, strict=True)
                    )
                self._commands += 1
                gpu_seconds = self._lib.tx_gpu_seconds(self._pointer)
                if gpu_seconds >= 0:
                    self._gpu_seconds += gpu_seconds
                    self._gpu_samples += 1
            finally:
                self._lib.tx_abort(self._pointer)
                self._recording = False
                self._profile_command.clear()

    @contextmanager
    def profile_kernels(self) -> Iterator[list[dict[str, Any]]]:
        """Per-dispatch device timings (CUDA events), counterpart of metal.py:236-258."""
        with self._lock:
            self._check_open()
            if self._recording or self._profile is not None:
                raise InferenceError()
            if self._lib.tx_profile_enable(self._pointer, 1):
                raise InferenceError()
            records: list[dict[str, Any]] = []
            self._profile = records
            try:
                yield records
            finally:
                self._lib.tx_profile_enable(self._pointer, 0)
                self._profile = None
                self._profile_command.clear()

    # ---- kernel routing (metal.py:532-648) ----------------------------------------------
    def _attention(
        self,
        buffers: Sequence[Buffer],
        *,
        tokens: int,
        seq: int,
        heads: int,
        kv_heads: int,
        dim: int,
        bidirectional: int = 0,
    ) -> None:
        """float32 attention over [q, k, v, lengths, out] in the padded layout.

        Same arguments and semantics as MetalRuntime._attention.  head_dim 32 goes to
        the bandwidth-oriented fp32 kernel; every other head_dim to the general kernel
        (kernels.metal:78-103 semantics).  bf16 tensor-core attention is reached through
        attention_padded_device / attention_varlen_device.
        """
        name = "attention_d32" if dim == 32 else "attention"
        self._dispatch(
            name,
            buffers,
            threads=tokens * heads * 32,
            group_size=32,
            seq=seq,
            heads=heads,
            kv_heads=kv_heads,
            dim=dim,
            scale=dim**-0.5,
            bidirectional=bidirectional,
        )

    def _dispatch(
        self,
        name: str,
        buffers: Sequence[Buffer],
        *,
        threads: int,
        group_size: int = 256,
        n: int = 0,
        rows: int = 0,
        cols: int = 0,
        k: int = 0,
        heads: int = 0,
        kv_heads: int = 0,
        seq: int = 0,
        batch: int = 0,
        dim: int = 0,
        group: int = 64,
        eps: float = 1e-6,
        theta: float = 1e6,
        scale: float = 1.0,
        bidirectional: int = 0,
        first_token: int = 0,
    ) -> None:
        if not self._recording or any(not b.pointer or b.runtime is not self for b in buffers):
            raise InferenceError()
        parameters = struct.pack(
            "<12I4f",
            n, rows, cols, k, heads, kv_heads, seq, batch, dim, group,
            int(bidirectional), int(first_token), eps, theta, scale, 0.0,
        )
        pointers = (ct.c_void_p * len(buffers))(*(b.pointer for b in buffers))
        rc = self._lib.tx_dispatch(
            self._pointer, name.encode("ascii"), pointers, len(buffers), parameters,
            len(parameters), threads, group_size,
        )
        if rc:
            _raise_for(rc)
        self._dispatches[name] += 1
        if self._profile is not None:
            self._profile_command.append(
                {"kernel": name, "rows": rows, "cols": cols, "seq": seq, "heads": heads,
                 "threads": threads}
            )

    # ---- typed entry points (host arrays) ------------------------------------------------
    def attention_host(
        self,
        q: NDArray[Any],
        k: NDArray[Any],
        v: NDArray[Any],
        out: NDArray[Any],
        *,
        lengths: NDArray[np.uint32] | None = None,
        cu_seqlens: NDArray[np.int32] | None = None,
        in_dtype: int,
        out_dtype: int,
        causal: bool = True,
        scale: float | None = None,
        q_norm_weight: NDArray[np.uint16] | None = None,
        k_norm_weight: NDArray[np.uint16] | None = None,
        eps: float = 1e-6,
        theta: float = 1e6,
    ) -> None:
        """Attention from host arrays into the host array `out` (tx_attention_*_host): the
        sequences go through in chunks whose copies in, kernels and copies out overlap.
        Arrays must be C-contiguous; padded q [B, L, H, d] with lengths [B] (uint32), or
        packed q [T, H, d] with cu_seqlens [nseq+1] (int32)."""
        self._check_open()
        arrays = [q, k, v, out] + [a for a in (lengths, cu_seqlens, q_norm_weight, k_norm_weight)
                                   if a is not None]
        if any(not a.flags.c_contiguous for a in arrays):
            raise InvalidInputError()
        qw = None if q_norm_weight is None else q_norm_weight.ctypes.data
        kw = None if k_norm_weight is None else k_norm_weight.ctypes.data
        dim = q.shape[-1]
        sc = dim**-0.5 if scale is None else scale
        if lengths is not None:
            batch, seq, heads = q.shape[:3]
            rc = self._lib.tx_attention_padded_host(
                self._pointer, q.ctypes.data, k.ctypes.data, v.ctypes.data, lengths.ctypes.data,
                out.ctypes.data, batch, seq, heads, k.shape[2], dim, in_dtype, out_dtype,
                int(bool(causal)), sc, qw, kw, eps, theta,
            )
        else:
            total, heads = q.shape[:2]
            rc = self._lib.tx_attention_varlen_host(
                self._pointer, q.ctypes.data, k.ctypes.data, v.ctypes.data, cu_seqlens.ctypes.data,
                cu_seqlens.size - 1, total, out.ctypes.data, heads, k.shape[1], dim, in_dtype,
                out_dtype, int(bool(causal)), sc, qw, kw, eps, theta,
            )
        _raise_for(rc)

    # ---- typed entry points (device pointers) -------------------------------------------
    def attention_padded_device(
        self,
        q: int,
        k: int,
        v: int,
        lengths: int,
        out: int,
        *,
        batch: int,
        seq: int,
        heads: int,
        kv_heads: int,
        dim: int,
        in_dtype: int = native.TX_BF16,
        out_dtype: int = native.TX_F32,
        causal: bool = True,
        scale: float | None = None,
        lengths_host: NDArray[np.uint32] | None = None,
        q_norm_weight: int | None = None,
        k_norm_weight: int | None = None,
        eps: float = 1e-6,
        theta: float = 1e6,
        stream: int | None = None,
    ) -> None:
        """Queues padded-layout attention on device pointers (tx_attention_padded)."""
        self._check_open()
        lh = None
        if lengths_host is not None:
            lh = np.ascontiguousarray(lengths_host, dtype=np.uint32)
            if lh.shape != (batch,):
                raise InvalidInputError()
        rc = self._lib.tx_attention_padded(
            self._pointer, q, k, v, lengths, None if lh is None else lh.ctypes.data, out,
            batch, seq, heads, kv_heads, dim, in_dtype, out_dtype, int(bool(causal)),
            dim**-0.5 if scale is None else scale, q_norm_weight, k_norm_weight, eps, theta,
            stream,
        )
        _raise_for(rc)

    def attention_varlen_device(
        self,
        q: int,
        k: int,
        v: int,
        cu_seqlens: int,
        out: int,
        *,
        nseq: int,
        total: int,
        max_len: int,
        heads: int,
        kv_heads: int,
        dim: int,
        in_dtype: int = native.TX_BF16,
        out_dtype: int = native.TX_F32,
        causal: bool = True,
        scale: float | None = None,
        cu_seqlens_host: NDArray[np.int32] | None = None,
        q_norm_weight: int | None = None,
        k_norm_weight: int | None = None,
        eps: float = 1e-6,
        theta: float = 1e6,
        stream: int | None = None,
    ) -> None:
        """Queues packed (cu_seqlens) attention on device pointers (tx_attention_varlen)."""
        self._check_open()
        ch = None
        if cu_seqlens_host is not None:
            ch = np.ascontiguousarray(cu_seqlens_host, dtype=np.int32)
            if ch.shape != (nseq + 1,):
                raise InvalidInputError()
        rc = self._lib.tx_attention_varlen(
            self._pointer, q, k, v, cu_seqlens, None if ch is None else ch.ctypes.data, nseq,
            total, max_len, out, heads, kv_heads, dim, in_dtype, out_dtype, int(bool(causal)),
            dim**-0.5 if scale is None else scale, q_norm_weight, k_norm_weight, eps, theta,
            stream,
        )
        _raise_for(rc)

    def qk_norm_rope_device(
        self,
        q: int | None,
        k: int | None,
        q_out: int | None,
        k_out: int | None,
        *,
        tokens: int,
        seq: int,
        heads: int,
        kv_heads: int,
        dim: int,
        q_norm_weight: int | None,
        k_norm_weight: int | None,
        cu_seqlens: int | None = None,
        nseq: int = 0,
        lengths: int | None = None,
        in_dtype: int = native.TX_BF16,
        out_dtype: int = native.TX_BF16,
        eps: float = 1e-6,
        theta: float = 1e6,
        stream: int | None = None,
    ) -> None:
        """Queues the fused q/k RMSNorm + RoPE prologue (tx_qk_norm_rope); q or k may be
        None.  `lengths` (padded layout) skips the rows past each sequence's length."""
        self._check_open()
        rc = self._lib.tx_qk_norm_rope(
            self._pointer, q, k, q_out, k_out, tokens, seq, cu_seqlens, nseq, lengths, heads,
            kv_heads, dim, in_dtype, out_dtype, q_norm_weight, k_norm_weight, eps, theta, stream,
        )
        _raise_for(rc)

    def pool_project_device(
        self,
        x: int,
        out: int,
        *,
        batch: int,
        cols: int,
        dim: int,
        seq: int = 0,
        lengths: int | None = None,
        cu_seqlens: int | None = None,
        first_token: bool = False,
        norm_weight: int | None = None,
        eps: float = 1e-6,
        in_dtype: int = native.TX_F32,
        stream: int | None = None,
    ) -> None:
        """Queues embedding pooling on device pointers (tx_pool_project): one row per
        sequence (last valid token, or the first with first_token), RMSNorm with
        norm_weight when given, L2 normalisation of the first `dim` columns into
        out [batch, dim] fp32."""
        self._check_open()
        rc = self._lib.tx_pool_project(
            self._pointer, x, in_dtype, lengths, cu_seqlens, out, batch, seq, cols, dim,
            int(bool(first_token)), norm_weight, eps, stream,
        )
        _raise_for(rc)

    def sync(self, stream: int | None = None) -> None:
        """Waits for queued work and reports kernel errors (tx_sync)."""
        self._check_open()
        _raise_for(self._lib.tx_sync(self._pointer, stream))

    # ---- lifecycle ----------------------------------------------------------------------
    def close(self) -> None:
        with self._lock:
            if self._recording or self._profile is not None:
                raise InferenceError()
            if self._pointer:
                for buffer in list(self._buffers):
                    buffer.close()
                self._workspace.clear()
                self._lib.tx_destroy(self._pointer)
                self._pointer = None

    def __enter__(self) -> CudaRuntime:
        return self

    def __exit__(self, *_: object) -> None:
        self.close()

    def __del__(self) -> None:
        if getattr(self, "_pointer", None) and hasattr(self, "_lock"):
            try:
                self.close()
            except Exception:
                pass

