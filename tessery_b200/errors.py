"""Stable, payload-free errors (same codes as the reference's errors.py:4-59).

The native library's one-line reason for the last failure is available from
``CudaRuntime.last_error()``; it is never attached to the exception, as the reference
keeps payloads out of its errors.
"""


class EmbeddingError(Exception):
    code = "embedding_error"
    http_status = 500

    def __init__(self) -> None:
        super().__init__(self.code)


class InvalidInputError(EmbeddingError):
    code = "invalid_input"
    http_status = 400


class InferenceError(EmbeddingError):
    code = "inference_failed"


class DeviceTimeoutError(InferenceError):
    """A bounded device-side wait gave up; the context stays usable."""

    code = "device_timeout"


class ClosedError(EmbeddingError):
    code = "closed"


class CudaUnavailableError(EmbeddingError):
    """No usable sm_100 device (counterpart of MetalUnavailableError)."""

    code = "cuda_unavailable"


class NativeBuildError(EmbeddingError):
    code = "native_engine_not_built"
