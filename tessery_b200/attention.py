"""NumPy-in / NumPy-out attention on a B200 (the operator behind
MetalRuntime._attention, metal.py:532-569, with the Qwen3 q/k prologue of
qwen3.py:216-237 optionally fused in front).

Inputs are float32 arrays, or uint16 arrays holding bf16 bit patterns (the convention
the reference uses for bf16 data, kernels.metal:10).  Device memory is reused across
calls (the runtime's named workspace buffers, and for attention the context's own copy
buffers); results are copied back to host.
"""

from __future__ import annotations

import threading

import numpy as np
from numpy.typing import NDArray

from . import native
from .errors import InvalidInputError
from .host import result_empty
from .runtime import CudaRuntime, _raise_for

_default: CudaRuntime | None = None
_default_lock = threading.Lock()


def default_runtime(device: int = 0) -> CudaRuntime:
    """Process-wide runtime on `device`, created on first use."""
    global _default
    with _default_lock:
        if _default is None or not _default._pointer or _default.device != device:
            _default = CudaRuntime(device)
        return _default


def _dtype_code(a: NDArray) -> int:
    if a.dtype == np.float32:
        return native.TX_F32
    if a.dtype == np.uint16:
        return native.TX_BF16
    raise InvalidInputError()


def _upload(rt: CudaRuntime, name: str, a: NDArray) -> int:
    a = np.ascontiguousarray(a)
    buffer = rt.workspace(name, a.nbytes)
    buffer.write(a)
    return buffer.device_ptr


def attention(
    q: NDArray,
    k: NDArray,
    v: NDArray,
    *,
    lengths: NDArray | None = None,
    cu_seqlens: NDArray | None = None,
    causal: bool = True,
    scale: float | None = None,
    q_norm_weight: NDArray | None = None,
    k_norm_weight: NDArray | None = None,
    eps: float = 1e-6,
    theta: float = 1e6,
    out_dtype: str = "float32",
    runtime: CudaRuntime | None = None,
    out: NDArray | None = None,
) -> NDArray:
    """Attention with per-sequence lengths (padded) or cu_seqlens (packed).

    Padded: q [B, L, H, d], k/v [B, L, Hkv, d], lengths [B].
    Packed: q [T, H, d], k/v [T, Hkv, d], cu_seqlens [nseq+1] (int32, cu[0] = 0).
    q_norm_weight/k_norm_weight: uint16 bf16 bits [d]; when given, that input is
    RMSNorm'd and rotated (RoPE, positions = padded index or index within the sequence)
    first.
    Returns float32 (or uint16 bf16 bits when out_dtype == "bf16") in q's layout,
    written into `out` when given (e.g. a page-locked array from host.pinned_empty), else
    into a new array (page-locked memory recycled from dropped results, host.result_empty).
    Pageable inputs are copied through the library's page-locked staging.
    """
    rt = runtime or default_runtime()
    q, k, v = (np.ascontiguousarray(a) for a in (q, k, v))
    code = _dtype_code(q)
    if _dtype_code(k) != code or _dtype_code(v) != code:
        raise InvalidInputError()
    out_code = {"float32": native.TX_F32, "bf16": native.TX_BF16}.get(out_dtype)
    if out_code is None:
        raise InvalidInputError()
    qw = kw = None
    if q_norm_weight is not None:
        qw = np.ascontiguousarray(q_norm_weight, dtype=np.uint16)
        if qw.shape != (q.shape[-1],):
            raise InvalidInputError()
    if k_norm_weight is not None:
        kw = np.ascontiguousarray(k_norm_weight, dtype=np.uint16)
        if kw.shape != (q.shape[-1],):
            raise InvalidInputError()
    out_np_dtype = np.float32 if out_code == native.TX_F32 else np.uint16
    if (lengths is None) == (cu_seqlens is None):
        raise InvalidInputError()
    sel: dict = {}
    if lengths is not None:
        if q.ndim != 4 or k.ndim != 4 or k.shape != v.shape:
            raise InvalidInputError()
        batch, seq, heads, dim = q.shape
        if k.shape[:2] != (batch, seq) or k.shape[3] != dim:
            raise InvalidInputError()
        sel["lengths"] = np.ascontiguousarray(lengths, dtype=np.uint32)
        if sel["lengths"].shape != (batch,):
            raise InvalidInputError()
    else:
        if q.ndim != 3 or k.ndim != 3 or k.shape != v.shape:
            raise InvalidInputError()
        total, heads, dim = q.shape
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        if cu.ndim != 1 or cu.size < 2 or k.shape[0] != total or k.shape[2] != dim:
            raise InvalidInputError()
        if int(np.max(np.diff(cu))) <= 0:
            raise InvalidInputError()
        sel["cu_seqlens"] = cu
    if out is None:
        out = result_empty(q.shape, out_np_dtype)
    elif out.shape != q.shape or out.dtype != out_np_dtype or not out.flags.c_contiguous:
        raise InvalidInputError()
    # Host arrays straight into the host-buffer entry point: the library moves the
    # sequences through in chunks whose copies in, kernels and copies out overlap
    # (pageable arrays through its page-locked staging).
    rt.attention_host(q, k, v, out, in_dtype=code, out_dtype=out_code, causal=causal,
                      scale=scale, q_norm_weight=qw, k_norm_weight=kw, eps=eps, theta=theta,
                      **sel)
    return out


def qk_norm_rope(
    q: NDArray,
    k: NDArray,
    q_norm_weight: NDArray,
    k_norm_weight: NDArray,
    *,
    seq: int | None = None,
    cu_seqlens: NDArray | None = None,
    eps: float = 1e-6,
    theta: float = 1e6,
    out_dtype: str | None = None,
    runtime: CudaRuntime | None = None,
) -> tuple[NDArray, NDArray]:
    """Fused q/k RMSNorm + RoPE.  q [tokens, H, d], k [tokens, Hkv, d] (padded batches
    flattened, positions = token % seq) or packed with cu_seqlens."""
    rt = runtime or default_runtime()
    q, k = np.ascontiguousarray(q), np.ascontiguousarray(k)
    if q.ndim != 3 or k.ndim != 3 or q.shape[0] != k.shape[0] or q.shape[2] != k.shape[2]:
        raise InvalidInputError()
    code = _dtype_code(q)
    if _dtype_code(k) != code:
        raise InvalidInputError()
    out_code = code if out_dtype is None else {"float32": native.TX_F32, "bf16": native.TX_BF16}[
        out_dtype]
    tokens, heads, dim = q.shape
    qw = _upload(rt, "q_norm_weight", np.asarray(q_norm_weight, dtype=np.uint16))
    kw = _upload(rt, "k_norm_weight", np.asarray(k_norm_weight, dtype=np.uint16))
    qp, kp = _upload(rt, "q", q), _upload(rt, "k", k)
    esz = 4 if out_code == native.TX_F32 else 2
    qo = rt.workspace("q_out", q.size * esz)
    ko = rt.workspace("k_out", k.size * esz)
    cu_ptr, nseq = None, 0
    if cu_seqlens is not None:
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        cu_ptr, nseq = _upload(rt, "cu", cu), cu.size - 1
        seq = seq or int(np.max(np.diff(cu)))
    if not seq:
        raise InvalidInputError()
    rt.qk_norm_rope_device(
        qp, kp, qo.device_ptr, ko.device_ptr, tokens=tokens, seq=seq, heads=heads,
        kv_heads=k.shape[1], dim=dim, q_norm_weight=qw, k_norm_weight=kw, cu_seqlens=cu_ptr,
        nseq=nseq, in_dtype=code, out_dtype=out_code, eps=eps, theta=theta,
    )
    rt.sync()
    np_dtype = np.float32 if out_code == native.TX_F32 else np.uint16
    qr = np.empty(q.shape, dtype=np_dtype)
    kr = np.empty(k.shape, dtype=np_dtype)
    rt._lib.tx_read(qo.pointer, qr.ctypes.data, qr.nbytes)
    rt._lib.tx_read(ko.pointer, kr.ctypes.data, kr.nbytes)
    return qr, kr


def pool_project(
    x: NDArray,
    *,
    dim: int | None = None,
    lengths: NDArray | None = None,
    cu_seqlens: NDArray | None = None,
    first_token: bool = False,
    norm_weight: NDArray | None = None,
    eps: float = 1e-6,
    runtime: CudaRuntime | None = None,
    out: NDArray | None = None,
) -> NDArray:
    """Embeddings from final hidden states (kernels.metal:339-349, with the final
    rms_norm of qwen3.py:281-290 fused when norm_weight is given).

    x: float32 or bf16 bits, padded [B, seq, cols] with lengths [B], or packed
    [total, cols] with cu_seqlens [B+1].  Row per sequence: the last valid token, or the
    first when first_token (BERT CLS).  norm_weight: bf16 bits [cols].  Returns
    float32 [B, dim] (dim defaults to cols), each row of unit L2 norm.
    """
    rt = runtime or default_runtime()
    x = np.ascontiguousarray(x)
    code = _dtype_code(x)
    if (lengths is None) == (cu_seqlens is None):
        raise InvalidInputError()
    if lengths is not None:
        if x.ndim != 3:
            raise InvalidInputError()
        batch, seq, cols = x.shape
        sel = np.ascontiguousarray(lengths, dtype=np.uint32)
        if sel.shape != (batch,):
            raise InvalidInputError()
    else:
        if x.ndim != 2:
            raise InvalidInputError()
        seq, cols = 0, x.shape[1]
        sel = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        if sel.ndim != 1 or sel.size < 2 or int(sel[0]) != 0 or int(sel[-1]) > x.shape[0] \
                or np.any(np.diff(sel) < 0):
            raise InvalidInputError()
        batch = sel.size - 1
    dim = cols if dim is None else int(dim)
    if not 0 < dim <= cols:
        raise InvalidInputError()
    xp = _upload(rt, "pool_x", x)
    sp = _upload(rt, "pool_sel", sel)
    wp = None
    if norm_weight is not None:
        w = np.ascontiguousarray(norm_weight, dtype=np.uint16)
        if w.shape != (cols,):
            raise InvalidInputError()
        wp = _upload(rt, "pool_norm_weight", w)
    dev_out = rt.workspace("pool_out", batch * dim * 4)
    rt.pool_project_device(
        xp, dev_out.device_ptr, batch=batch, cols=cols, dim=dim, seq=seq,
        lengths=sp if lengths is not None else None,
        cu_seqlens=sp if cu_seqlens is not None else None, first_token=first_token,
        norm_weight=wp, eps=eps, in_dtype=code,
    )
    rt.sync()
    if out is None:
        out = np.empty((batch, dim), dtype=np.float32)
    elif out.shape != (batch, dim) or out.dtype != np.float32 or not out.flags.c_contiguous:
        raise InvalidInputError()
    _raise_for(rt._lib.tx_read(dev_out.pointer, out.ctypes.data, out.nbytes))
    return out
