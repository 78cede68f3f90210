"""Page-locked host arrays for fast, asynchronous host<->device copies."""

from __future__ import annotations

import ctypes as ct
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
