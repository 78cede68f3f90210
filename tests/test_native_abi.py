"""The C-ABI library loads on a machine without a GPU and exports every declared entry
point; the loader refuses stale or incomplete builds (as metal.py:27-91 does)."""

import ctypes as ct
import re
from pathlib import Path
from types import SimpleNamespace

import pytest

from tessery_b200 import native
from tessery_b200.errors import CudaUnavailableError, NativeBuildError

HEADER = Path(__file__).resolve().parents[1] / "include" / "tessattn.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(tx_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("tx_create", "tx_buffer", "tx_read", "tx_begin", "tx_dispatch", "tx_finish",
                     "tx_abort", "tx_attention_padded", "tx_attention_varlen", "tx_qk_norm_rope"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ct.CDLL(str(native.library_path()))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(native.SIGNATURES) == set(declared_functions())


def test_loader_binds_and_checks_version():
    lib = native.load()
    assert lib.tx_abi_version() == native.ABI_VERSION
    assert len(lib._tessery_sha256) == 64


def test_no_device_is_a_stable_error():
    lib = native.load()
    count = ct.c_int(0)
    try:
        cudart_has_gpu = ct.CDLL("libcuda.so.1") is not None
    except OSError:
        cudart_has_gpu = False
    if cudart_has_gpu:
        pytest.skip("a CUDA driver is present")
    from tessery_b200 import CudaRuntime

    with pytest.raises(CudaUnavailableError):
        CudaRuntime(0)
    assert lib.tx_last_error(None)
    del count


def test_null_handles_are_rejected_without_a_device():
    lib = native.load()
    assert lib.tx_begin(None) == native.TX_EINVAL
    assert lib.tx_finish(None) == native.TX_EINVAL
    assert lib.tx_read(None, None, 0) == native.TX_EINVAL
    assert lib.tx_sync(None, None) == native.TX_EINVAL
    assert lib.tx_buffer(None, None, 16) is None
    assert lib.tx_gpu_seconds(None) == -1.0
    assert lib.tx_launch_count(None) == 0
    # The host-buffer attention entry points refuse a missing context before touching
    # any pointer.
    assert lib.tx_attention_padded_host(None, None, None, None, None, None, 1, 1, 1, 1, 128, 1,
                                        0, 1, 0.1, None, None, 1e-6, 1e6) == native.TX_EINVAL
    assert lib.tx_attention_varlen_host(None, None, None, None, None, 1, 1, None, 1, 1, 128, 1,
                                        0, 1, 0.1, None, None, 1e-6, 1e6) == native.TX_EINVAL


@pytest.mark.parametrize("changed_during_load", [False, True])
def test_missing_symbols_or_changing_library_raise(tmp_path, monkeypatch, changed_during_load):
    library = tmp_path / native.LIBRARY_NAME
    library.write_bytes(b"placeholder")
    monkeypatch.setattr(native, "library_path", lambda: library)
    monkeypatch.setattr(native, "_lib", None)

    def fake_load(path):
        if changed_during_load:
            library.write_bytes(b"changed")
        return SimpleNamespace()  # no symbols

    monkeypatch.setattr(native.ct, "CDLL", fake_load)
    with pytest.raises(NativeBuildError):
        native.load()


def test_missing_library_raises(tmp_path, monkeypatch):
    monkeypatch.setattr(native, "library_path", lambda: tmp_path / "absent.so")
    monkeypatch.setattr(native, "_lib", None)
    with pytest.raises(NativeBuildError):
        native.load()
