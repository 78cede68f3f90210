"""ctypes binding of libtessattn.so (counterpart of metal.py:27-91).

Loads exactly one in-tree library, checks that its bytes do not change while it is
being loaded, binds every entry point declared in include/tessattn.h and checks the ABI
version.  A missing library, symbol or version mismatch raises NativeBuildError; there
is no fallback implementation.
"""

from __future__ import annotations

import ctypes as ct
import hashlib
import threading
from pathlib import Path
from typing import Any

from .errors import NativeBuildError

ABI_VERSION = 10
LIBRARY_NAME = "libtessattn.so"

TX_OK, TX_EINVAL, TX_ECUDA, TX_ETIMEOUT = 0, 1, 2, 3
TX_F32, TX_BF16, TX_BF16X2 = 0, 1, 2
TX_LINEAR_STORE_F32, TX_LINEAR_STORE_BF16, TX_LINEAR_ADD_F32, TX_LINEAR_GATED_BF16 = 0, 1, 2, 3
TX_LINEAR_GELU_SPLIT = 4

_vp, _u32, _u64, _i32, _f32 = ct.c_void_p, ct.c_uint32, ct.c_uint64, ct.c_int, ct.c_float


class TxQwen3Layer(ct.Structure):
    """Device pointers of one layer's weights (TxQwen3Layer in tessattn.h)."""

    _fields_ = [(name, _vp) for name in (
        "input_norm", "post_norm", "q_norm", "k_norm", "q_proj", "k_proj", "v_proj", "o_proj",
        "gate_up", "down")]


class TxQwen3Model(ct.Structure):
    """Shape and weights of a Qwen3 embedding model (TxQwen3Model in tessattn.h)."""

    _fields_ = [
        *[(name, _u32) for name in ("hidden", "intermediate", "layers", "heads", "kv_heads",
                                    "head_dim", "vocab")],
        ("eps", _f32), ("theta", _f32), ("precise", _i32),
        ("embed_packed", _vp), ("embed_scales", _vp), ("embed_biases", _vp),
        ("final_norm", _vp), ("layer", ct.POINTER(TxQwen3Layer)),
    ]


class TxBertLayer(ct.Structure):
    """Device pointers of one BERT layer's weights (TxBertLayer in tessattn.h)."""

    _fields_ = [(name, _vp) for name in (
        "qkv_w", "qkv_b", "o_w", "o_b", "ln1_w", "ln1_b", "i_w", "i_b", "out_w", "out_b",
        "ln2_w", "ln2_b")]


class TxBertModel(ct.Structure):
    """Shape and weights of a BERT encoder (TxBertModel in tessattn.h)."""

    _fields_ = [
        *[(name, _u32) for name in ("hidden", "intermediate", "layers", "heads", "vocab",
                                    "max_pos")],
        ("eps", _f32), ("precise", _i32),
        ("words", _vp), ("positions", _vp), ("types", _vp), ("ln_w", _vp), ("ln_b", _vp),
        ("layer", ct.POINTER(TxBertLayer)),
    ]


SIGNATURES: dict[str, tuple[list[Any], Any]] = {
    "tx_abi_version": ([], _u32),
    "tx_create": ([_i32], _vp),
    "tx_destroy": ([_vp], None),
    "tx_last_error": ([_vp], ct.c_char_p),
    "tx_device_sms": ([_vp], _i32),
    "tx_set_wait_limit": ([_vp, ct.c_int64], _i32),
    "tx_last_kernel": ([_vp], ct.c_char_p),
    "tx_launch_count": ([_vp], _u64),
    "tx_buffer": ([_vp, _vp, _u64], _vp),
    "tx_free": ([_vp], None),
    "tx_memory_stats": ([_vp, ct.POINTER(_u64)], _i32),
    "tx_host_copy_bytes": ([_vp, ct.POINTER(_u64)], _i32),
    "tx_read": ([_vp, _vp, _u64], _i32),
    "tx_write": ([_vp, _vp, _u64], _i32),
    "tx_buffer_device_ptr": ([_vp], _vp),
    "tx_buffer_size": ([_vp], _u64),
    "tx_host_alloc": ([_u64], _vp),
    "tx_host_free": ([_vp], None),
    "tx_begin": ([_vp], _i32),
    "tx_dispatch": ([_vp, ct.c_char_p, ct.POINTER(_vp), _u32, _vp, _u32, _u64, _u32], _i32),
    "tx_finish": ([_vp], _i32),
    "tx_abort": ([_vp], None),
    "tx_gpu_seconds": ([_vp], ct.c_double),
    "tx_profile_enable": ([_vp, _i32], _i32),
    "tx_profile_read": ([_vp, ct.POINTER(ct.c_double), _u32], _i32),
    "tx_kernel_timing": ([_vp, _i32], _i32),
    "tx_kernel_times": ([_vp, ct.POINTER(ct.c_double), _u32, ct.POINTER(_u32)], _i32),
    "tx_attention_padded": (
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _i32, _i32, _i32,
         _f32, _vp, _vp, _f32, _f32, _vp],
        _i32,
    ),
    "tx_attention_varlen": (
        [_vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp, _u32, _u32, _u32, _i32, _i32,
         _i32, _f32, _vp, _vp, _f32, _f32, _vp],
        _i32,
    ),
    "tx_attention_padded_host": (
        [_vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _i32, _i32, _i32, _f32,
         _vp, _vp, _f32, _f32],
        _i32,
    ),
    "tx_attention_varlen_host": (
        [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _vp, _u32, _u32, _u32, _i32, _i32, _i32, _f32,
         _vp, _vp, _f32, _f32],
        _i32,
    ),
    "tx_qk_norm_rope": (
        [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _vp, _u32, _vp, _u32, _u32, _u32, _i32, _i32, _vp,
         _vp, _f32, _f32, _vp],
        _i32,
    ),
    "tx_pool_project": (
        [_vp, _vp, _i32, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _i32, _vp, _f32, _vp],
        _i32,
    ),
    "tx_sync": ([_vp, _vp], _i32),
    "tx_device_count": ([], _i32),
    "tx_split_tf32": ([_vp, _vp, _vp, _u64, _vp], _i32),
    "tx_layer_norm_rows": ([_vp, _vp, _vp, _vp, _vp, _vp, _i32, _u32, _u32, _f32, _vp], _i32),
    "tx_bert_embed": (
        [_vp, _vp, _vp, _u32, _u32, _u32, _vp, _vp, _vp, _u32, _u32, _vp, _vp, _f32, _vp, _vp,
         _i32, _u32, _vp], _i32),
    "tx_bert_workspace_bytes": ([ct.POINTER(TxBertModel), _u32], _u64),
    "tx_bert_forward": (
        [_vp, ct.POINTER(TxBertModel), _vp, _vp, _vp, _u32, _vp, _vp, _u64, _vp], _i32),
    "tx_qwen3_workspace_bytes": ([ct.POINTER(TxQwen3Model), _u32], _u64),
    "tx_qwen3_forward": (
        [_vp, ct.POINTER(TxQwen3Model), _vp, _vp, _vp, _u32, _vp, _u32, _vp, _u64, _vp], _i32),
    "tx_dequant4": ([_vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _vp], _i32),
    "tx_split_bf16": ([_vp, _vp, _vp, _u64, _vp], _i32),
    "tx_embedding4": ([_vp, _vp, _u32, _vp, _vp, _vp, _vp, _u32, _u32, _vp], _i32),
    "tx_rms_norm_rows": ([_vp, _vp, _vp, _vp, _i32, _u32, _u32, _f32, _vp], _i32),
    "tx_linear": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _i32, _i32, _u32, _vp],
                  _i32),
    "tx_attention_padded_noalloc": (
        [_vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _i32, _i32, _f32, _vp, _f32,
         _f32, _vp, _vp],
        _i32,
    ),
}

_lock = threading.Lock()
_lib: Any = None


def library_path() -> Path:
    return Path(__file__).resolve().parent / LIBRARY_NAME


def load() -> Any:
    """Returns the bound library, loading it once per process."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise NativeBuildError()
        try:
            before = path.read_bytes()
            lib: Any = ct.CDLL(str(path))
            if path.read_bytes() != before:
                raise NativeBuildError()
        except OSError:
            raise NativeBuildError() from None
        try:
            for name, (args, result) in SIGNATURES.items():
                function = getattr(lib, name)
                function.argtypes, function.restype = args, result
        except AttributeError:
            raise NativeBuildError() from None
        if lib.tx_abi_version() != ABI_VERSION:
            raise NativeBuildError()
        lib._tessery_sha256 = hashlib.sha256(before).hexdigest()
        lib._tessery_path = str(path)
        _lib = lib
        return lib
