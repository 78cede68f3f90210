"""Seeded synthetic workloads with the shapes and value distributions of the benchmark
configurations (Qwen3-Embedding-0.6B and BGE-small attention layers).  No datasets or
weights are involved: every tensor is drawn from numpy.random.default_rng(seed).

bf16 tensors are carried as uint16 bit patterns (round to nearest even), the same
convention the reference uses for its bf16 weights (kernels.metal:10).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
from numpy.typing import NDArray


def to_bf16_bits(x: NDArray) -> NDArray[np.uint16]:
    """float32 -> bf16 bit patterns, round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16)


def from_bf16_bits(bits: NDArray) -> NDArray[np.float32]:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclass
class Workload:
    """One attention problem: inputs plus the description needed to run and score it."""

    name: str
    layout: str  # "padded" or "varlen"
    q: NDArray
    k: NDArray
    v: NDArray
    heads: int
    kv_heads: int
    dim: int
    causal: bool
    scale: float
    in_dtype: str  # "f32" or "bf16" (uint16 bit patterns)
    seq: int  # padded L, or max_len for varlen
    lengths: NDArray[np.uint32] | None = None
    cu_seqlens: NDArray[np.int32] | None = None
    q_norm_weight: NDArray[np.uint16] | None = None
    k_norm_weight: NDArray[np.uint16] | None = None
    eps: float = 1e-6
    theta: float = 1e6
    seed: int = 0
    notes: dict = field(default_factory=dict)

    @property
    def seq_lengths(self) -> NDArray[np.int64]:
        if self.layout == "padded":
            return np.minimum(self.lengths.astype(np.int64), self.seq)
        return np.diff(self.cu_seqlens.astype(np.int64))

    @property
    def batch(self) -> int:
        return int(self.seq_lengths.size)

    @property
    def rows(self) -> int:
        """Query rows present in the layout (padded rows included)."""
        return int(self.q.shape[0] * self.q.shape[1]) if self.layout == "padded" else int(
            self.q.shape[0])

    def valid_tokens(self) -> int:
        return int(self.seq_lengths.sum())

    def useful_pairs(self) -> int:
        """(query, key) pairs of valid query rows: n(n+1)/2 causal, n^2 bidirectional."""
        n = self.seq_lengths
        return int((n * (n + 1) // 2).sum() if self.causal else (n * n).sum())

    def useful_flops(self) -> int:
        """4 * d * heads per useful pair (QK^T and PV, 2 flops per multiply-add)."""
        return 4 * self.dim * self.heads * self.useful_pairs()

    def io_bytes(self, out_bytes_per_elem: int = 4) -> int:
        """Contract I/O: read q, k, v (and the prologue weights), write the output."""
        b = self.q.nbytes + self.k.nbytes + self.v.nbytes
        if self.q_norm_weight is not None:
            b += self.q_norm_weight.nbytes + self.k_norm_weight.nbytes
        out_elems = self.q.size
        return int(b + out_elems * out_bytes_per_elem)


def _normal(rng, shape, scale=1.0) -> NDArray[np.float32]:
    x = rng.standard_normal(size=shape, dtype=np.float32)
    if scale != 1.0:
        x *= np.float32(scale)
    return x


def _qwen_weights(rng, dim):
    q_w = to_bf16_bits(1.0 + 0.02 * rng.standard_normal(dim).astype(np.float32))
    k_w = to_bf16_bits(1.0 + 0.02 * rng.standard_normal(dim).astype(np.float32))
    return q_w, k_w


def bge(batch: int = 4, seq: int = 128, seed: int = 1, min_len: int = 16) -> Workload:
    """BGE-small attention block: 12 heads x 32, bidirectional, fp32, key-padding mask
    by length ~ U[min_len, seq], Q/K/V ~ N(0,1)/sqrt(32), scale 1/sqrt(32)."""
    rng = np.random.default_rng(seed)
    heads, dim = 12, 32
    lengths = rng.integers(min_len, seq + 1, size=batch).astype(np.uint32)
    s = 1.0 / np.sqrt(dim)
    q = _normal(rng, (batch, seq, heads, dim), s)
    k = _normal(rng, (batch, seq, heads, dim), s)
    v = _normal(rng, (batch, seq, heads, dim), s)
    return Workload("bge_d32_padded", "padded", q, k, v, heads, heads, dim, False, dim**-0.5,
                    "f32", seq, lengths=lengths, seed=seed)


def qwen_padded(batch: int = 32, seq: int = 512, seed: int = 2, min_len: int = 32,
                lengths: NDArray | None = None, dtype: str = "bf16") -> Workload:
    """Qwen3-0.6B attention layer: 16q/8kv heads x 128, causal, right-padded lengths
    ~ U[min_len, seq], Q/K/V ~ N(0,1) in bf16 (dtype "f32": the same draws kept in
    float32, the reference adapter's float buffers), q/k RMSNorm weights 1+N(0,0.02)
    (bf16), eps 1e-6, RoPE theta 1e6."""
    rng = np.random.default_rng(seed)
    heads, kv, dim = 16, 8, 128
    if lengths is None:
        lengths = rng.integers(min_len, seq + 1, size=batch)
    lengths = np.asarray(lengths, dtype=np.uint32)
    cast = to_bf16_bits if dtype == "bf16" else (lambda a: a)
    q = cast(_normal(rng, (batch, seq, heads, dim)))
    k = cast(_normal(rng, (batch, seq, kv, dim)))
    v = cast(_normal(rng, (batch, seq, kv, dim)))
    q_w, k_w = _qwen_weights(rng, dim)
    name = "qwen_d128_padded" if dtype == "bf16" else "qwen_d128_padded_f32"
    return Workload(name, "padded", q, k, v, heads, kv, dim, True, dim**-0.5, dtype, seq,
                    lengths=lengths, q_norm_weight=q_w, k_norm_weight=k_w, seed=seed)


def varlen_lengths(nseq: int, seed: int, median: float = 96.0, sigma: float = 0.8,
                   lo: int = 2, hi: int = 512) -> NDArray[np.int64]:
    rng = np.random.default_rng(seed)
    raw = rng.lognormal(np.log(median), sigma, size=nseq)
    return np.clip(np.round(raw), lo, hi).astype(np.int64)


def qwen_varlen(nseq: int = 256, seed: int = 3, lengths: NDArray | None = None) -> Workload:
    """Ragged Qwen3-shape attention: sequences packed by cu_seqlens (no padding),
    lengths log-normal (median 96, sigma 0.8) clipped to [2, 512]."""
    if lengths is None:
        lengths = varlen_lengths(nseq, seed)
    lengths = np.asarray(lengths, dtype=np.int64)
    rng = np.random.default_rng(seed + 1000)
    heads, kv, dim = 16, 8, 128
    cu = np.zeros(lengths.size + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lengths)
    total = int(cu[-1])
    q = to_bf16_bits(_normal(rng, (total, heads, dim)))
    k = to_bf16_bits(_normal(rng, (total, kv, dim)))
    v = to_bf16_bits(_normal(rng, (total, kv, dim)))
    q_w, k_w = _qwen_weights(rng, dim)
    return Workload("qwen_d128_varlen", "varlen", q, k, v, heads, kv, dim, True, dim**-0.5,
                    "bf16", int(lengths.max()), cu_seqlens=cu, q_norm_weight=q_w,
                    k_norm_weight=k_w, seed=seed)


def short_tails(kind: str = "qwen", batch: int = 32, seed: int = 4, lo: int = 2,
                hi: int = 32) -> Workload:
    """Short-sequence tails: lengths ~ U[2, 32], bf16 N(0,1) inputs, packed varlen.
    kind "qwen": 16q/8kv x 128 causal with the q/k prologue; "bge": 12 x 32
    bidirectional."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(lo, hi + 1, size=batch).astype(np.int64)
    cu = np.zeros(batch + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lengths)
    total = int(cu[-1])
    if kind == "qwen":
        heads, kv, dim, causal = 16, 8, 128, True
    else:
        heads, kv, dim, causal = 12, 12, 32, False
    q = to_bf16_bits(_normal(rng, (total, heads, dim)))
    k = to_bf16_bits(_normal(rng, (total, kv, dim)))
    v = to_bf16_bits(_normal(rng, (total, kv, dim)))
    q_w = k_w = None
    if kind == "qwen":
        q_w, k_w = _qwen_weights(rng, dim)
    return Workload(f"{kind}_short_tails", "varlen", q, k, v, heads, kv, dim, causal,
                    dim**-0.5, "bf16", int(lengths.max()), cu_seqlens=cu, q_norm_weight=q_w,
                    k_norm_weight=k_w, seed=seed)


def benchmark_workload(name: str, rank: int = 0, world: int = 1,
                       scaled_batch: int = 4096) -> Workload:
    """The seeded input of one benchmark workload as rank `rank` of `world` sees it.

    qwen_padded: 32 sequences per rank, lengths ~ U[32, 512] from seed 2 over all ranks,
    assigned longest first; qwen_f32: the same batch with float32 inputs; qwen_varlen:
    the 256 log-normal sequences of seed 3, split across the ranks; bge / bge_scaled: batch 4 / `scaled_batch`, seed 1; tails_qwen /
    tails_bge: 32 sequences of U[2, 32], seed 4.  Ranks other than 0 draw their tensors
    from seed + 1000 * rank.
    """
    from .partition import shard_sequences

    if name == "qwen_padded":
        lengths = np.random.default_rng(2).integers(32, 513, size=32 * world)
        owned = shard_sequences(lengths, world, causal=True)[rank]
        return qwen_padded(batch=len(owned), seq=512, seed=2 + 1000 * rank,
                           lengths=lengths[owned])
    if name == "qwen_f32":
        lengths = np.random.default_rng(2).integers(32, 513, size=32 * world)
        owned = shard_sequences(lengths, world, causal=True)[rank]
        return qwen_padded(batch=len(owned), seq=512, seed=2 + 1000 * rank,
                           lengths=lengths[owned], dtype="f32")
    if name == "qwen_varlen":
        lengths = varlen_lengths(256, 3)
        owned = shard_sequences(lengths, world, causal=True)[rank]
        return qwen_varlen(seed=3 + 1000 * rank, lengths=lengths[owned])
    if name == "bge":
        return bge(batch=4, seq=128, seed=1 + 1000 * rank)
    if name == "bge_scaled":
        return bge(batch=scaled_batch, seq=128, seed=1 + 1000 * rank)
    if name == "tails_qwen":
        return short_tails("qwen", batch=32, seed=4 + 1000 * rank)
    if name == "tails_bge":
        return short_tails("bge", batch=32, seed=4 + 1000 * rank)
    raise ValueError(name)
