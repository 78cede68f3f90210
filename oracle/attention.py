"""NumPy restatement of the reference's attention-path kernels (test infrastructure).

Each function names the reference source it follows (paths inside the reference
project).  Arithmetic is float64 by default ("exact" oracle, as the reference's own
f64 tests use) or float32 when ``dtype=np.float32`` (the reference's float32 NumPy
formula, used as the CPU baseline).
"""

from __future__ import annotations

import numpy as np
from numpy.typing import NDArray


# ---- bf16 helpers ----------------------------------------------------------------------
def bf16_bits(x: NDArray) -> NDArray[np.uint16]:
    """float32 -> bf16 bit patterns, round to nearest even (as cvt.rn.bf16 does)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(bits: NDArray) -> NDArray[np.float32]:
    """bf16 bit patterns -> float32 (kernels.metal:10, `bf16()`)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: NDArray) -> NDArray[np.float32]:
    """Rounds float32 values to the nearest bf16 value, returned as float32."""
    return bf16_bits_to_f32(bf16_bits(x))


# ---- prologue -------------------------------------------------------------------------
def rms_norm(x: NDArray, w_bits: NDArray, eps: float, dtype=np.float64) -> NDArray:
    """Row RMSNorm with a bf16 weight: x * rsqrt(mean(x^2) + eps) * w.

    Follows kernels.metal:53-63 (`rms_norm`), applied per (token, head) row as
    qwen3.py:216-226 calls it for q and k.
    """
    x = np.asarray(x, dtype=dtype)
    w = bf16_bits_to_f32(w_bits).astype(dtype)
    inv = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + dtype(eps))
    return x * inv * w


def rope_inv_freq(theta: float, dim: int) -> NDArray[np.float32]:
    """Per-column inverse frequency theta^(-2c/dim), rounded once to float32.

    kernels.metal:70 evaluates ``pow(theta, -2c/dim)`` in float; the CUDA kernels and
    this oracle both use the float nearest to the exact value.
    """
    c = np.arange(dim // 2, dtype=np.float64)
    return (float(theta) ** (-2.0 * c / dim)).astype(np.float32)


def rope_angles(positions: NDArray, theta: float, dim: int) -> NDArray[np.float32]:
    """float32 angle = float(position) * inv_freq[c] (kernels.metal:70)."""
    pos = np.asarray(positions, dtype=np.float32)
    return (pos[..., None] * rope_inv_freq(theta, dim)).astype(np.float32)


def rope(x: NDArray, positions: NDArray, theta: float, dtype=np.float64) -> NDArray:
    """Split-half rotation (kernels.metal:65-74).

    x: [..., tokens, heads, dim]; positions: [..., tokens] (the padded index for the
    padded layout, kernels.metal:68; the index within the sequence for varlen).
    """
    x = np.asarray(x, dtype=dtype)
    dim = x.shape[-1]
    half = dim // 2
    ang = rope_angles(positions, theta, dim).astype(np.float64)[..., None, :]
    cos, sin = np.cos(ang).astype(dtype), np.sin(ang).astype(dtype)
    a, b = x[..., :half], x[..., half:]
    return np.concatenate((a * cos - b * sin, a * sin + b * cos), axis=-1)


def qk_norm_rope(q, k, q_w_bits, k_w_bits, eps, theta, positions, dtype=np.float64):
    """q/k RMSNorm followed by RoPE, in the order of qwen3.py:216-237."""
    qn = rope(rms_norm(q, q_w_bits, eps, dtype), positions, theta, dtype)
    kn = rope(rms_norm(k, k_w_bits, eps, dtype), positions, theta, dtype)
    return qn, kn


# ---- attention ------------------------------------------------------------------------
def _softmax_rows(scores: NDArray) -> NDArray:
    probs = np.exp(scores - scores.max(axis=-1, keepdims=True))
    probs /= probs.sum(axis=-1, keepdims=True)
    return probs


def _attend(q_rows, k_rows, v_rows, positions, n, causal, scale, dtype):
    """q_rows [r, d] at `positions`; keys/values [n, d]; returns [r, d]."""
    if n == 0:
        return np.full(q_rows.shape, np.nan, dtype=dtype)
    scores = (q_rows.astype(dtype) @ k_rows.astype(dtype).T) * dtype(scale)
    if causal:
        keys = np.arange(n)
        scores = np.where(keys[None, :] > np.asarray(positions)[:, None], -np.inf, scores)
    return _softmax_rows(scores) @ v_rows.astype(dtype)


def attention_padded(q, k, v, lengths, causal: bool, scale: float, dtype=np.float64):
    """Padded-layout attention, kernels.metal:78-103 (and :108-298, same semantics).

    q/out [B, L, H, d]; k/v [B, L, Hkv, d]; lengths [B].  A query at position p of a
    sequence of length n attends to keys [0, causal ? min(p+1, n) : n); padded query
    rows (p >= n) attend to [0, n) (tests/real_metal/test_kernels.py:196-209);
    kv head = h // (H // Hkv) (kernels.metal:87).  Length 0 gives NaN rows (0/0).
    """
    q, k, v = np.asarray(q), np.asarray(k), np.asarray(v)
    b_, l_, h_, d_ = q.shape
    hkv = k.shape[2]
    group = h_ // hkv
    out = np.empty((b_, l_, h_, d_), dtype=dtype)
    pos = np.arange(l_)
    for b in range(b_):
        n = min(int(lengths[b]), l_)
        for g in range(hkv):
            kk, vv = k[b, :n, g], v[b, :n, g]
            for h in range(g * group, (g + 1) * group):
                out[b, :, h] = _attend(q[b, :, h], kk, vv, pos, n, causal, scale, dtype)
    return out


def attention_varlen(q, k, v, cu_seqlens, causal: bool, scale: float, dtype=np.float64):
    """Packed (cu_seqlens) attention with the same semantics; positions are the index
    within each sequence, and there are no padded rows."""
    q, k, v = np.asarray(q), np.asarray(k), np.asarray(v)
    total, h_, d_ = q.shape
    hkv = k.shape[1]
    group = h_ // hkv
    out = np.empty((total, h_, d_), dtype=dtype)
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    for s in range(len(cu) - 1):
        a, b = int(cu[s]), int(cu[s + 1])
        n = b - a
        if n == 0:
            continue
        pos = np.arange(n)
        for g in range(hkv):
            kk, vv = k[a:b, g], v[a:b, g]
            for h in range(g * group, (g + 1) * group):
                out[a:b, h] = _attend(q[a:b, h], kk, vv, pos, n, causal, scale, dtype)
    return out


def attention_reference_loop(q, k, v, lengths, causal: bool, scale: float):
    """Per-key float32 online softmax, operation for operation as kernels.metal:78-103
    (scalar `attention`).  Pure-Python loops: small cases only."""
    q, k, v = (np.asarray(a, dtype=np.float32) for a in (q, k, v))
    b_, l_, h_, d_ = q.shape
    group = h_ // k.shape[2]
    out = np.empty_like(q)
    f = np.float32
    for b in range(b_):
        n = min(int(lengths[b]), l_)
        for p in range(l_):
            end = min(p + 1, n) if causal else n
            for h in range(h_):
                g = h // group
                acc = np.zeros(d_, np.float32)
                maximum, denom = f(-np.inf), f(0.0)
                for key in range(end):
                    score = f(np.dot(q[b, p, h], k[b, key, g])) * f(scale)
                    nxt = max(maximum, score)
                    corr, prob = f(np.exp(maximum - nxt)), f(np.exp(score - nxt))
                    denom = denom * corr + prob
                    acc = acc * corr + prob * v[b, key, g]
                    maximum = nxt
                with np.errstate(invalid="ignore", divide="ignore"):
                    out[b, p, h] = acc / denom
    return out


def pool_project(x, lengths, dim: int, first_token: bool, dtype=np.float64):
    """Last-token (or first-token) pooling and L2 normalisation of the first `dim`
    columns, kernels.metal:339-349 (`pool_project`).  x: [B, seq, cols]."""
    x = np.asarray(x, dtype=dtype)
    b_ = x.shape[0]
    rows = np.zeros(b_, dtype=np.int64) if first_token else np.asarray(lengths, np.int64) - 1
    picked = x[np.arange(b_), rows, :dim]
    return picked / np.sqrt(np.sum(picked * picked, axis=-1, keepdims=True))


def pool_project_packed(x, cu_seqlens, dim: int, first_token: bool, dtype=np.float64):
    """pool_project (kernels.metal:339-349) on packed rows: sequence b spans rows
    cu[b]..cu[b+1]-1 of x [total, cols]; its last row (or first, first_token) is picked
    and its first `dim` columns L2-normalised."""
    x = np.asarray(x, dtype=dtype)
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    rows = cu[:-1] if first_token else cu[1:] - 1
    picked = x[rows, :dim]
    return picked / np.sqrt(np.sum(picked * picked, axis=-1, keepdims=True))
