"""Result arrays of the NumPy API (tessery_b200.host.result_empty): page-locked memory
recycled by exact size once a result is dropped, bounded live and kept bytes, and a
plain NumPy array past the bounds or when page-locked memory is unavailable.  A fake
allocator stands in for tx_host_alloc / tx_host_free, so this runs without a GPU."""

from __future__ import annotations

import ctypes as ct
import gc

import numpy as np
import pytest

from tessery_b200 import host


class FakeLib:
    def __init__(self):
        self.blocks: dict[int, ct.Array] = {}
        self.allocs = 0
        self.frees = 0

    def tx_host_alloc(self, size):
        buf = (ct.c_uint8 * int(size))()
        self.blocks[ct.addressof(buf)] = buf
        self.allocs += 1
        return ct.addressof(buf)

    def tx_host_free(self, ptr):
        self.frees += 1
        del self.blocks[ptr]


@pytest.fixture
def fake(monkeypatch):
    lib = FakeLib()
    monkeypatch.setattr(host.native, "load", lambda: lib)
    monkeypatch.setattr(host, "_result_free", {})
    monkeypatch.setattr(host, "_result_state", {"live": 0, "kept": 0})
    return lib


def test_dropped_result_memory_is_reused(fake):
    a = host.result_empty((4, 8), np.float32)
    a[...] = 1.0
    first = a.ctypes.data
    assert fake.allocs == 1 and host._result_state["live"] == 128
    del a
    gc.collect()
    assert host._result_state == {"live": 0, "kept": 128}
    b = host.result_empty((8, 4), np.float32)  # same size, other shape
    assert b.ctypes.data == first and fake.allocs == 1
    assert b.shape == (8, 4) and b.dtype == np.float32 and b.flags.c_contiguous
    c = host.result_empty((3,), np.float32)  # other size: a new block
    assert c.ctypes.data != first and fake.allocs == 2


def test_live_bound_falls_back_to_numpy(fake, monkeypatch):
    monkeypatch.setattr(host, "_RESULT_LIVE_LIMIT", 256)
    a = host.result_empty((64,), np.float32)  # 256 bytes: at the bound
    b = host.result_empty((1,), np.float32)  # past it: ordinary array
    assert fake.allocs == 1
    assert b.base is None or not isinstance(b.base, ct.Array)
    del a, b


def test_kept_bound_frees_the_rest(fake, monkeypatch):
    monkeypatch.setattr(host, "_RESULT_KEEP_LIMIT", 100)
    a = host.result_empty((16,), np.float32)  # 64 bytes
    b = host.result_empty((16,), np.float32)
    del a, b
    gc.collect()
    assert host._result_state["kept"] == 64 and fake.frees == 1


def test_failed_allocation_gives_a_numpy_array(monkeypatch):
    class NoMemory(FakeLib):
        def tx_host_alloc(self, size):
            return 0

    monkeypatch.setattr(host.native, "load", lambda: NoMemory())
    monkeypatch.setattr(host, "_result_state", {"live": 0, "kept": 0})
    a = host.result_empty((2, 2), np.float32)
    assert a.shape == (2, 2) and host._result_state["live"] == 0
