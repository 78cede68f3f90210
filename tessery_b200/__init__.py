"""tessery_b200: B200-native encoder attention with Tessery's operator contract.

Host side: NumPy in, NumPy out, no PyTorch dependency, a thin ctypes binding of
libtessattn.so (hand-written CUDA for sm_100a).  See include/tessattn.h for the C ABI.
"""

from .attention import attention, default_runtime, pool_project, qk_norm_rope
from .batching import pack_rows, unpack_rows, varlen_batches
from .errors import (
    ClosedError,
    CudaUnavailableError,
    DeviceTimeoutError,
    EmbeddingError,
    InferenceError,
    InvalidInputError,
    NativeBuildError,
)
from .native import TX_BF16, TX_F32
from .partition import gather_shard, pack, shard_sequences
from .runtime import Buffer, CudaRuntime

__all__ = [
    "Buffer",
    "ClosedError",
    "CudaRuntime",
    "CudaUnavailableError",
    "DeviceTimeoutError",
    "EmbeddingError",
    "InferenceError",
    "InvalidInputError",
    "NativeBuildError",
    "TX_BF16",
    "TX_F32",
    "attention",
    "default_runtime",
    "gather_shard",
    "pack",
    "pack_rows",
    "pool_project",
    "qk_norm_rope",
    "shard_sequences",
    "unpack_rows",
    "varlen_batches",
]
