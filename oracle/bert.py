"""NumPy restatement of the reference's BERT fp32 embedding forward (test infrastructure).

Follows BertBackend.forward (bert.py:104-235) dispatch by dispatch, in the padded layout
the reference uses, with the arithmetic of each kernel:

- embedding_position (kernels.metal:353-361): (word + token type 0) + position, the
  position of a token being its padded index;
- layer_norm (kernels.metal:362-373): (x - mean) / sqrt(mean((x - mean)^2) + eps) * w + b;
- matmul_bias_f32 (kernels.metal:438-487): x . W^T + bias;
- attention (kernels.metal:78-103), bidirectional over each sequence's valid keys;
- add (:300-304), gelu_f32 (:381-391: the erf form, evaluated here with math.erf, which
  the reference's Abramowitz-Stegun 7.1.26 approximates to 1.5e-7);
- pool_project with first_token (:339-349): the CLS row, L2-normalised.

float64 by default; float32 gives the reference's own number format (the CPU baseline).
"""

from __future__ import annotations

import math

import numpy as np
from numpy.typing import NDArray

from .attention import attention_padded, pool_project

_erf = np.vectorize(math.erf, otypes=[np.float64])


def layer_norm(x: NDArray, w: NDArray, b: NDArray, eps: float, dtype=np.float64) -> NDArray:
    """layer_norm (kernels.metal:362-373) over the last axis."""
    x = np.asarray(x, dtype=dtype)
    mean = x.mean(axis=-1, keepdims=True)
    d = x - mean
    inv = 1.0 / np.sqrt((d * d).mean(axis=-1, keepdims=True) + dtype(eps))
    return d * inv * np.asarray(w, dtype) + np.asarray(b, dtype)


def gelu(x: NDArray, dtype=np.float64) -> NDArray:
    """The erf form of gelu_f32 (kernels.metal:381-391): 0.5 x (1 + erf(x / sqrt 2))."""
    x = np.asarray(x, dtype=dtype)
    return (0.5 * x * (1.0 + _erf(x.astype(np.float64) / math.sqrt(2.0)))).astype(dtype)


def gelu_as(x: NDArray) -> NDArray[np.float32]:
    """gelu_f32 evaluated as the reference evaluates it, in float32: erf from the rational
    approximation 7.1.26 of Abramowitz and Stegun (kernels.metal:384-390)."""
    x = np.asarray(x, dtype=np.float32)
    z = np.abs(x) * np.float32(math.sqrt(0.5))
    t = np.float32(1) / (np.float32(1) + np.float32(0.3275911) * z)
    poly = ((((np.float32(1.061405429) * t - np.float32(1.453152027)) * t
              + np.float32(1.421413741)) * t - np.float32(0.284496736)) * t
            + np.float32(0.254829592)) * t
    tail = poly * np.exp(-z * z)
    return np.float32(0.5) * x * np.where(x < 0, tail, np.float32(2) - tail)


def embedding_position(ids: NDArray, words: NDArray, positions: NDArray, types: NDArray,
                       dtype=np.float64) -> NDArray:
    """embedding_position (kernels.metal:353-361) of padded ids [batch, seq]."""
    ids = np.asarray(ids, dtype=np.int64)
    seq = ids.shape[1]
    w = np.asarray(words, dtype)[ids]
    return (w + np.asarray(types, dtype)[0]) + np.asarray(positions, dtype)[:seq]


def linear(x: NDArray, weights: dict, name: str, dtype) -> NDArray:
    """matmul_bias_f32 (kernels.metal:438-487): x . W^T + bias."""
    return x @ np.asarray(weights[name + ".weight"], dtype).T + np.asarray(
        weights[name + ".bias"], dtype)


def bert_forward(weights: dict, cfg, ids: NDArray, lengths: NDArray, dtype=np.float64
                 ) -> NDArray:
    """CLS embeddings [batch, hidden], L2-normalised, of right-padded ids [batch, seq]
    (bert.py:104-235).  `cfg` carries hidden, heads, layers, eps."""
    ids = np.asarray(ids, dtype=np.int64)
    lengths = np.asarray(lengths)
    batch, seq = ids.shape
    H, D = cfg.heads, cfg.hidden // cfg.heads
    x = embedding_position(ids, weights["embeddings.word_embeddings.weight"],
                           weights["embeddings.position_embeddings.weight"],
                           weights["embeddings.token_type_embeddings.weight"], dtype)
    x = layer_norm(x, weights["embeddings.LayerNorm.weight"],
                   weights["embeddings.LayerNorm.bias"], cfg.eps, dtype)
    for layer in range(cfg.layers):
        p = f"encoder.layer.{layer}"
        q = linear(x, weights, p + ".attention.self.query", dtype).reshape(batch, seq, H, D)
        k = linear(x, weights, p + ".attention.self.key", dtype).reshape(batch, seq, H, D)
        v = linear(x, weights, p + ".attention.self.value", dtype).reshape(batch, seq, H, D)
        attended = attention_padded(q, k, v, lengths, False, D**-0.5, dtype)
        x = x + linear(attended.reshape(batch, seq, H * D), weights,
                       p + ".attention.output.dense", dtype)
        x = layer_norm(x, weights[p + ".attention.output.LayerNorm.weight"],
                       weights[p + ".attention.output.LayerNorm.bias"], cfg.eps, dtype)
        act = gelu(linear(x, weights, p + ".intermediate.dense", dtype), dtype)
        x = x + linear(act, weights, p + ".output.dense", dtype)
        x = layer_norm(x, weights[p + ".output.LayerNorm.weight"],
                       weights[p + ".output.LayerNorm.bias"], cfg.eps, dtype)
    return pool_project(x, lengths, cfg.hidden, True, dtype)
