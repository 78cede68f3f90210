"""NumPy restatement of the reference's Qwen3 embedding forward (test infrastructure).

Follows Qwen3Backend.forward (qwen3.py:112-296) kernel call by kernel call, in the padded
layout the reference uses, with the arithmetic of each kernel:

- weight4 / embedding4 (kernels.metal:11-28): element (r, c) = code * scale + bias, with
  code i of a packed word in bits 4i..4i+3 and one bf16 scale/bias per 64 columns;
- linear4 (kernels.metal:32-51): x . W^T;
- rms_norm (kernels.metal:53-63), rope (:65-74), attention (:78-103), add (:300-304);
- gated4 + silu_gate (kernels.metal:333-337): silu(x . Wg^T) * (x . Wu^T);
- the final rms_norm and pool_project (qwen3.py:281-290, kernels.metal:339-349).

float64 by default; float32 gives the reference's own number format (used as the CPU
baseline).  Weights are dequantised one matrix at a time.
"""

from __future__ import annotations

import numpy as np
from numpy.typing import NDArray

from .attention import attention_padded, bf16_bits_to_f32, pool_project, rms_norm, rope


def dequant4(packed: NDArray, scales: NDArray, biases: NDArray, dtype=np.float64) -> NDArray:
    """[rows, cols] weights of a uint4 matrix (weight4, kernels.metal:11-19)."""
    packed = np.asarray(packed, dtype=np.uint32)
    rows, words = packed.shape
    shifts = np.arange(8, dtype=np.uint32) * np.uint32(4)
    codes = ((packed[:, :, None] >> shifts) & np.uint32(15)).reshape(rows, words * 8)
    s = np.repeat(bf16_bits_to_f32(scales).astype(dtype), 64, axis=1)
    b = np.repeat(bf16_bits_to_f32(biases).astype(dtype), 64, axis=1)
    return codes.astype(dtype) * s + b


def _matrix(weights, name, dtype):
    return dequant4(weights[name + ".weight"], weights[name + ".scales"],
                    weights[name + ".biases"], dtype)


def silu_gate(gate: NDArray, up: NDArray) -> NDArray:
    """silu_gate (kernels.metal:333-337): gate / (1 + exp(-gate)) * up."""
    return gate / (1.0 + np.exp(-gate)) * up


def qwen3_forward(weights: dict, cfg, ids: NDArray, lengths: NDArray, dimensions: int,
                  dtype=np.float64) -> NDArray:
    """Pooled, L2-normalised embeddings [batch, dimensions] of right-padded ids [batch, seq]
    (qwen3.py:112-296).  `cfg` carries hidden, intermediate, layers, heads, kv_heads,
    head_dim, eps and theta."""
    ids = np.asarray(ids, dtype=np.int64)
    lengths = np.asarray(lengths)
    batch, seq = ids.shape
    tokens = batch * seq
    H, KV, D = cfg.heads, cfg.kv_heads, cfg.head_dim
    # embedding4 (qwen3.py:166-173): only the rows the ids select are dequantised.
    flat = ids.reshape(-1)
    x = dequant4(weights["model.embed_tokens.weight"][flat],
                 weights["model.embed_tokens.scales"][flat],
                 weights["model.embed_tokens.biases"][flat], dtype)
    positions = np.broadcast_to(np.arange(seq), (batch, seq))
    for layer in range(cfg.layers):
        p = f"model.layers.{layer}"
        a = p + ".self_attn"
        normalized = rms_norm(x, weights[p + ".input_layernorm.weight"], cfg.eps, dtype)
        q = normalized @ _matrix(weights, a + ".q_proj", dtype).T
        k = normalized @ _matrix(weights, a + ".k_proj", dtype).T
        v = normalized @ _matrix(weights, a + ".v_proj", dtype).T
        q = q.reshape(batch, seq, H, D)
        k = k.reshape(batch, seq, KV, D)
        v = v.reshape(batch, seq, KV, D)
        q = rope(rms_norm(q, weights[a + ".q_norm.weight"], cfg.eps, dtype), positions,
                 cfg.theta, dtype)
        k = rope(rms_norm(k, weights[a + ".k_norm.weight"], cfg.eps, dtype), positions,
                 cfg.theta, dtype)
        attended = attention_padded(q, k, v, lengths, True, D**-0.5, dtype)
        x = x + attended.reshape(tokens, H * D) @ _matrix(weights, a + ".o_proj", dtype).T
        normalized = rms_norm(x, weights[p + ".post_attention_layernorm.weight"], cfg.eps,
                              dtype)
        gated = silu_gate(normalized @ _matrix(weights, p + ".mlp.gate_proj", dtype).T,
                          normalized @ _matrix(weights, p + ".mlp.up_proj", dtype).T)
        x = x + gated @ _matrix(weights, p + ".mlp.down_proj", dtype).T
    normalized = rms_norm(x, weights["model.norm.weight"], cfg.eps, dtype)
    return pool_project(normalized.reshape(batch, seq, cfg.hidden), lengths, dimensions, False,
                        dtype)
