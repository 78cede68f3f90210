"""CPU oracle for the encoder-attention hot path (test infrastructure only).

This package restates, in NumPy, the semantics of the reference's Metal kernels on the
attention path.  It is the checker for the CUDA library and the CPU baseline of the
benchmark: only the test suite, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg may import it.  The product (``tessery_b200``) never calls it and has no
CPU fallback.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own kernel tests
(tests/real_metal/test_kernels.py in the reference) against a fake runtime backed by
this oracle, records the reference's expected values and the verdicts, and commits
them as fixtures under ``tests/golden/``.
"""

from .attention import (  # noqa: F401
    attention_padded,
    attention_reference_loop,
    attention_varlen,
    bf16_bits,
    bf16_bits_to_f32,
    bf16_round,
    pool_project,
    pool_project_packed,
    qk_norm_rope,
    rms_norm,
    rope,
    rope_inv_freq,
)
