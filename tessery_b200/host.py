"""Page-locked host arrays for fast, asynchronous host<->device copies."""

from __future__ import annotations

import ctypes as ct
import threading
import weakref

import numpy as np

from . import native
from .errors import InferenceError


def pinned_empty(shape, dtype) -> np.ndarray:
    """Uninitialised NumPy array in page-locked memory (cudaHostAlloc); freed when the
    array is garbage-collected."""
    lib = native.load()
    dtype = np.dtype(dtype)
    nbytes = int(np.prod(shape)) * dtype.itemsize
    ptr = lib.tx_host_alloc(max(nbytes, 1))
    if not ptr:
        raise InferenceError()
    raw = (ct.c_uint8 * max(nbytes, 1)).from_address(ptr)
    array = np.frombuffer(raw, dtype=np.uint8, count=nbytes).view(dtype).reshape(shape)
    weakref.finalize(raw, lib.tx_host_free, ptr)
    return array


def pinned_copy(a: np.ndarray) -> np.ndarray:
    out = pinned_empty(a.shape, a.dtype)
    out[...] = a
    return out


# Result arrays of the NumPy entry points: page-locked, so that the device writes them
# with a plain DMA (no staging copy, no first-touch page faults of a fresh array), and
# recycled: the memory of a result the caller has dropped is kept, by exact size, for
# the next result of that size.  Both the bytes of live results and the bytes kept are
# bounded; past the live bound a result is an ordinary (pageable) NumPy array.
_RESULT_LIVE_LIMIT = 1 << 30
_RESULT_KEEP_LIMIT = 1 << 30
_result_lock = threading.Lock()
_result_free: dict[int, list[int]] = {}
_result_state = {"live": 0, "kept": 0}


def _result_release(ptr: int, nbytes: int) -> None:
    lib = native.load()
    with _result_lock:
        _result_state["live"] -= nbytes
        if _result_state["kept"] + nbytes <= _RESULT_KEEP_LIMIT:
            _result_free.setdefault(nbytes, []).append(ptr)
            _result_state["kept"] += nbytes
            return
    lib.tx_host_free(ptr)


def result_empty(shape, dtype) -> np.ndarray:
    """Uninitialised array for a result: page-locked recycled memory while the live
    results stay under 1 GiB, else np.empty."""
    dtype = np.dtype(dtype)
    nbytes = max(int(np.prod(shape)) * dtype.itemsize, 1)
    ptr = 0
    with _result_lock:
        if _result_state["live"] + nbytes > _RESULT_LIVE_LIMIT:
            return np.empty(shape, dtype)
        free = _result_free.get(nbytes)
        if free:
            ptr = free.pop()
            _result_state["kept"] -= nbytes
        _result_state["live"] += nbytes
    if not ptr:
        ptr = native.load().tx_host_alloc(nbytes)
        if not ptr:
            with _result_lock:
                _result_state["live"] -= nbytes
            return np.empty(shape, dtype)
    raw = (ct.c_uint8 * nbytes).from_address(ptr)
    array = np.frombuffer(raw, dtype=np.uint8, count=int(np.prod(shape)) * dtype.itemsize)
    weakref.finalize(raw, _result_release, ptr, nbytes)
    return array.view(dtype).reshape(shape)
