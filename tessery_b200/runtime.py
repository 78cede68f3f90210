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
    """Handle of one device allocation made by the native context (the role of
    metal.py:94-119's Buffer).  The context owns the memory and its accounting
    (tx_memory_stats); this object only names the allocation for the Python side."""

    def __init__(self, runtime: CudaRuntime, handle: int, size: int) -> None:
        self.runtime = runtime
        self.pointer: int | None = handle
        self.size = size

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
        handle, self.pointer = self.pointer, None
        if handle:
            with self.runtime._lock:
                self.runtime._lib.tx_free(handle)

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


class _Params(ct.Structure):
    """The 64-byte kernel parameter block of kernels.metal:5-8 (twelve uint32, four
    float), laid out field by field as the library's Params64 reads it."""

    _fields_ = [(name, ct.c_uint32) for name in (
        "n", "rows", "cols", "k", "heads", "kv_heads", "seq", "batch", "dim", "group",
        "bidirectional", "first_token")] + [
        (name, ct.c_float) for name in ("eps", "theta", "scale", "reserved")]


class _Command:
    """One open command: what was dispatched into it, for the profile and the counters.
    Closing it either commits (tx_finish) or discards (tx_abort) the queued work."""

    def __init__(self, runtime: CudaRuntime) -> None:
        self.runtime = runtime
        self.log: list[dict[str, Any]] = []

    def commit(self) -> None:
        rt = self.runtime
        _raise_for(rt._lib.tx_finish(rt._pointer))
        if rt._profile is not None:
            seconds = (ct.c_double * len(self.log))()
            if rt._lib.tx_profile_read(rt._pointer, seconds, len(self.log)) != native.TX_OK:
                raise InferenceError()
            for entry, t in zip(self.log, seconds, strict=True):
                rt._profile.append({**entry, "gpu_seconds": float(t)})
        rt._commands += 1
        t = rt._lib.tx_gpu_seconds(rt._pointer)
        if t >= 0:
            rt._gpu_seconds += t
            rt._gpu_samples += 1

    def discard(self) -> None:
        self.runtime._lib.tx_abort(self.runtime._pointer)


class CudaRuntime:
    """Stream-ordered command owner on one B200; commands are serialised per instance."""

    def __init__(self, device: int = 0) -> None:
        self._lib = native.load()
        self._pointer: int | None = self._lib.tx_create(device)
        if not self._pointer:
            raise CudaUnavailableError()
        self.device = device
        self._lock = threading.RLock()
        self._open: _Command | None = None
        self._buffers: WeakSet[Buffer] = WeakSet()
        self._workspace: dict[str, Buffer] = {}
        self._commands = 0
        self._gpu_samples = 0
        self._gpu_seconds = 0.0
        self._dispatches: Counter[str] = Counter()
        self._profile: list[dict[str, Any]] | None = None

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

    def kernel_timing(self, enabled: bool) -> None:
        """While enabled, each kernel launch of the typed attention calls is bracketed by
        a CUDA event pair (tx_kernel_timing); kernel_times() reads the last call's."""
        self._check_open()
        _raise_for(self._lib.tx_kernel_timing(self._pointer, int(bool(enabled))))

    def kernel_times(self) -> list[float]:
        """Device seconds of each kernel of the last typed attention call, in launch
        order (the q/k prologue when it ran, then the attention kernel); waits for them."""
        self._check_open()
        seconds = (ct.c_double * 8)()
        count = ct.c_uint32(0)
        _raise_for(self._lib.tx_kernel_times(self._pointer, seconds, 8, ct.byref(count)))
        return [float(seconds[i]) for i in range(count.value)]

    def host_copy_bytes(self) -> tuple[int, int]:
        """(host-to-device, device-to-host) bytes the last host-buffer attention call
        copied (tx_host_copy_bytes)."""
        self._check_open()
        out = (ct.c_uint64 * 2)()
        _raise_for(self._lib.tx_host_copy_bytes(self._pointer, out))
        return int(out[0]), int(out[1])

    def set_wait_limit(self, cycles: int) -> None:
        """Limit, in SM clock cycles, of each bounded wait of the tensor-core kernel
        (0 restores the default, about a second).  A wait that runs out is reported as
        DeviceTimeoutError by the next sync; the runtime stays usable."""
        self._check_open()
        _raise_for(self._lib.tx_set_wait_limit(self._pointer, int(cycles)))

    def last_error(self) -> str:
        raw = self._lib.tx_last_error(self._pointer)
        return raw.decode() if raw else ""

    def _memory(self) -> tuple[int, int, int, int]:
        """(live bytes, peak live bytes, allocations, allocated bytes) of the context."""
        stats = (ct.c_uint64 * 4)()
        if not self._pointer or self._lib.tx_memory_stats(self._pointer, stats) != native.TX_OK:
            return (0, 0, 0, 0)
        return tuple(int(x) for x in stats)  # type: ignore[return-value]

    @property
    def active_bytes(self) -> int:
        return self._memory()[0]

    @property
    def peak_bytes(self) -> int:
        return self._memory()[1]

    def diagnostics(self) -> dict[str, Any]:
        """Counters under the key names of MetalRuntime.diagnostics (metal.py:208-234)."""
        with self._lock:
            live, peak, count, total = self._memory()
            return {
                "native_library_sha256": self._lib._tessery_sha256,
                "native_library_path": self._lib._tessery_path,
                "allocations": count,
                "allocated_bytes": total,
                "completed_commands": self._commands,
                "gpu_timed_commands": self._gpu_samples,
                "gpu_seconds": self._gpu_seconds,
                "dispatches": dict(self._dispatches),
                "active_bytes": live,
                "peak_bytes": peak,
            }

    def _check_open(self) -> None:
        if not self._pointer:
            raise ClosedError()

    # ---- buffers (metal.py:354-373, 650-662) -------------------------------------------
    def buffer(self, size: int, data: NDArray[Any] | None = None) -> Buffer:
        """A device buffer of `size` bytes, filled from `data` (C-contiguous, exactly
        `size` bytes) or with zeros."""
        size_ok = type(size) is int and 0 < size <= 2**40
        data_ok = data is None or (data.flags.c_contiguous and data.nbytes == size)
        if not (size_ok and data_ok):
            raise InvalidInputError()
        with self._lock:
            self._check_open()
            source = None if data is None else data.ctypes.data
            handle = self._lib.tx_buffer(self._pointer, source, size)
            if not handle:
                raise InferenceError()
            made = Buffer(self, handle, size)
            self._buffers.add(made)
            return made

    def read(self, buffer: Buffer, shape: tuple[int, ...], dtype=np.float32) -> NDArray[Any]:
        with self._lock:
            self._check_open()
            if self._open is not None or buffer.runtime is not self or not buffer.pointer:
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
        """Brackets dispatches into one stream-ordered command.  A clean exit waits for
        the command and raises its error, if any; an exception discards it."""
        with self._lock:
            self._check_open()
            if self._open is not None:
                raise InferenceError()
            if self._lib.tx_begin(self._pointer) != native.TX_OK:
                raise InferenceError()
            current = self._open = _Command(self)
            try:
                yield
            except BaseException:
                current.discard()
                raise
            else:
                try:
                    current.commit()
                except BaseException:
                    current.discard()
                    raise
            finally:
                self._open = None

    @contextmanager
    def profile_kernels(self) -> Iterator[list[dict[str, Any]]]:
        """Per-dispatch device timings (CUDA events), counterpart of metal.py:236-258:
        one record per dispatch of the commands run inside the block."""
        with self._lock:
            self._check_open()
            if self._open is not None or self._profile is not None:
                raise InferenceError()
            if self._lib.tx_profile_enable(self._pointer, 1) != native.TX_OK:
                raise InferenceError()
            self._profile = records = []
            try:
                yield records
            finally:
                self._profile = None
                self._lib.tx_profile_enable(self._pointer, 0)

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
        current = self._open
        if current is None:
            raise InferenceError()
        handles = []
        for b in buffers:
            if b.runtime is not self or not b.pointer:
                raise InferenceError()
            handles.append(b.pointer)
        block = _Params(n=n, rows=rows, cols=cols, k=k, heads=heads, kv_heads=kv_heads, seq=seq,
                        batch=batch, dim=dim, group=group, bidirectional=int(bidirectional),
                        first_token=int(first_token), eps=eps, theta=theta, scale=scale)
        slots = (ct.c_void_p * max(len(handles), 1))(*handles)
        _raise_for(self._lib.tx_dispatch(self._pointer, name.encode("ascii"), slots, len(handles),
                                         ct.addressof(block), ct.sizeof(block), threads,
                                         group_size))
        self._dispatches[name] += 1
        current.log.append({"kernel": name, "rows": rows, "cols": cols, "seq": seq,
                            "heads": heads, "threads": threads})

    def _matmul_f32(self, buffers: Sequence[Buffer], *, rows: int, cols: int, k: int) -> None:
        """out [rows, cols] = a [rows, k] . bt [cols, k]^T over [a, bt, out]: the call shape of
        MetalRuntime._matmul_f32 (metal.py:664-700), one fp32 dispatch covering every row."""
        self._dispatch("matmul_f32", buffers, threads=((rows + 3) // 4) * cols * 32,
                       group_size=32, rows=rows, cols=cols, k=k)

    def _matmul_bias_f32(self, buffers: Sequence[Buffer], *, rows: int, cols: int,
                         k: int) -> None:
        """The affine projection over [a, bt, out, bias] (metal.py:702-731)."""
        self._dispatch("matmul_bias_f32", buffers, threads=((rows + 3) // 4) * cols * 32,
                       group_size=32, rows=rows, cols=cols, k=k)

    def add(self, a: NDArray[np.float32], b: NDArray[np.float32]) -> NDArray[np.float32]:
        """Elementwise a + b on the device (MetalRuntime.add, metal.py:733-748)."""
        if a.shape != b.shape or a.dtype != np.float32 or b.dtype != np.float32 or not a.size:
            raise InferenceError()
        with self._lock:
            bufs = [self.buffer(x.nbytes, np.ascontiguousarray(x)) for x in (a, b)]
            bufs.append(self.buffer(a.nbytes))
            try:
                with self.command():
                    self._dispatch("add", bufs, threads=a.size, n=a.size)
                return self.read(bufs[-1], a.shape)
            finally:
                for x in bufs:
                    x.close()

    def matmul(self, a: NDArray[np.float32], b: NDArray[np.float32]) -> NDArray[np.float32]:
        """General float32 [M, K] @ [K, N] on the device (MetalRuntime.matmul,
        metal.py:750-780)."""
        if (a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0] or a.dtype != np.float32
                or b.dtype != np.float32 or not a.size or not b.size):
            raise InferenceError()
        m, k = a.shape
        n = b.shape[1]
        with self._lock:
            bufs = [self.buffer(x.nbytes, np.ascontiguousarray(x)) for x in (a, b.T)]
            bufs.append(self.buffer(m * n * 4))
            try:
                with self.command():
                    self._matmul_f32(bufs, rows=m, cols=n, k=k)
                return self.read(bufs[-1], (m, n))
            finally:
                for x in bufs:
                    x.close()

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

    # ---- the Qwen3 forward around the attention (device pointers) -----------------------
    def dequant4_device(self, packed: int, scales: int, biases: int, out: int, *, rows: int,
                        cols: int, out_lo: int | None = None, stream: int | None = None) -> None:
        """uint4 weights (weight4, kernels.metal:11-19) into bf16 [rows, cols], and their
        rounding residues into out_lo when given (tx_dequant4)."""
        self._check_open()
        _raise_for(self._lib.tx_dequant4(self._pointer, packed, scales, biases, out, out_lo, rows,
                                         cols, stream))

    def split_bf16_device(self, x: int, out: int, *, n: int, stream: int | None = None) -> None:
        """fp32 x [n] as a bf16 pair: out [n] = bf16(x), out + n: the residue (tx_split_bf16)."""
        self._check_open()
        _raise_for(self._lib.tx_split_bf16(self._pointer, x, out, n, stream))

    def embedding4_device(self, ids: int, out: int, *, tokens: int, packed: int, scales: int,
                          biases: int, cols: int, vocab: int, stream: int | None = None) -> None:
        """Token rows of a uint4 embedding table as fp32 (embedding4, kernels.metal:21-28)."""
        self._check_open()
        _raise_for(self._lib.tx_embedding4(self._pointer, ids, tokens, packed, scales, biases,
                                           out, cols, vocab, stream))

    def rms_norm_rows_device(self, x: int, weight: int, out: int, *, rows: int, cols: int,
                             eps: float = 1e-6, out_dtype: int = native.TX_BF16,
                             stream: int | None = None) -> None:
        """Row RMSNorm of fp32 x with a bf16 weight (kernels.metal:53-63) (tx_rms_norm_rows)."""
        self._check_open()
        _raise_for(self._lib.tx_rms_norm_rows(self._pointer, x, weight, out, out_dtype, rows,
                                              cols, eps, stream))

    def linear_device(self, x: int, w: int, out: int, *, m: int, n: int, k: int, mode: int,
                      x_lo: int | None = None, w_lo: int | None = None,
                      bias: int | None = None, fmt: int = native.TX_BF16,
                      part: int | None = None, stream: int | None = None) -> None:
        """Tensor-core x [m, k] . w [n, k]^T (+ bias) with a TX_LINEAR_* epilogue; fmt
        TX_BF16 or TX_F32 (TF32 operands); with the lo parts of split operands (x_lo and
        w_lo), the three-product form; part: output column-block width (tx_linear)."""
        self._check_open()
        _raise_for(self._lib.tx_linear(self._pointer, x, x_lo, w, w_lo, bias, out, m, n, k, mode,
                                       fmt, n if part is None else part, stream))

    def qwen3_forward_device(self, model: Any, ids: int, cu_seqlens: int,
                             cu_host: NDArray[np.int32], pooled: int, dimensions: int,
                             workspace: int, workspace_bytes: int,
                             stream: int | None = None) -> None:
        """Queues the whole Qwen3 embedding forward (tx_qwen3_forward): `model` is a
        reference to a native.TxQwen3Model, `cu_host` the host copy of the packed
        sequences' cu_seqlens."""
        self._check_open()
        cu_host = np.ascontiguousarray(cu_host, dtype=np.int32)
        _raise_for(self._lib.tx_qwen3_forward(
            self._pointer, model, ids, cu_seqlens, cu_host.ctypes.data, cu_host.size - 1,
            pooled, dimensions, workspace, workspace_bytes, stream))

    # ---- the BERT fp32 forward around the attention (device pointers) -------------------
    def split_tf32_device(self, x: int, out: int, *, n: int, stream: int | None = None) -> None:
        """fp32 x [n] as a TF32 operand pair out [2][n] (tx_split_tf32)."""
        self._check_open()
        _raise_for(self._lib.tx_split_tf32(self._pointer, x, out, n, stream))

    def layer_norm_rows_device(self, x: int, weight: int, bias: int, out: int, *, rows: int,
                               cols: int, eps: float, pair: int | None = None,
                               split: int = native.TX_F32, stream: int | None = None) -> None:
        """Row LayerNorm (kernels.metal:362-373), optionally writing the next GEMM's split
        operand `pair` (tx_layer_norm_rows)."""
        self._check_open()
        _raise_for(self._lib.tx_layer_norm_rows(self._pointer, x, weight, bias, out, pair, split,
                                                rows, cols, eps, stream))

    def bert_embed_device(self, ids: int, out: int, *, tokens: int, cols: int, words: int,
                          positions: int, types: int, vocab: int, max_pos: int, ln_w: int,
                          ln_b: int, eps: float, cu_seqlens: int | None = None, nseq: int = 0,
                          seq: int = 0, pair: int | None = None, split: int = native.TX_F32,
                          stream: int | None = None) -> None:
        """Word + type + position embeddings, LayerNorm'd (tx_bert_embed)."""
        self._check_open()
        _raise_for(self._lib.tx_bert_embed(self._pointer, ids, cu_seqlens, nseq, seq, tokens,
                                           words, positions, types, vocab, max_pos, ln_w, ln_b,
                                           eps, out, pair, split, cols, stream))

    def bert_forward_device(self, model: Any, ids: int, cu_seqlens: int,
                            cu_host: NDArray[np.int32], pooled: int, workspace: int,
                            workspace_bytes: int, stream: int | None = None) -> None:
        """Queues the whole BERT forward (tx_bert_forward); `model` is a reference to a
        native.TxBertModel."""
        self._check_open()
        cu_host = np.ascontiguousarray(cu_host, dtype=np.int32)
        _raise_for(self._lib.tx_bert_forward(self._pointer, model, ids, cu_seqlens,
                                             cu_host.ctypes.data, cu_host.size - 1, pooled,
                                             workspace, workspace_bytes, stream))

    def sync(self, stream: int | None = None) -> None:
        """Waits for queued work and reports kernel errors (tx_sync)."""
        self._check_open()
        _raise_for(self._lib.tx_sync(self._pointer, stream))

    # ---- lifecycle ----------------------------------------------------------------------
    def close(self) -> None:
        with self._lock:
            if self._open is not None or self._profile is not None:
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

