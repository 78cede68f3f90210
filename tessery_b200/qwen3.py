"""Qwen3 embedding forward on one B200: the layer loop of Qwen3Backend.forward
(qwen3.py:112-296 in the reference) around this library's attention.

Per layer, as the reference (qwen3.py:191-280): RMSNorm of the hidden rows, q/k/v
projections, q/k RMSNorm + RoPE and causal GQA attention, o projection added to the
residual, RMSNorm, SiLU-gated MLP, down projection added to the residual; then the final
RMSNorm of each sequence's last token, its first `dimensions` columns L2-normalised
(qwen3.py:281-290).  Differences, all of layout or number format:

- sequences are packed by cu_seqlens (no padded rows; the reference pads to the longest
  sequence, and padded rows never reach a valid token's output in a causal model);
- uint4 weights (qwen3.py:70-73) are dequantised once at load to bf16, the tensor-core
  operand format; activations entering a projection are bf16, accumulation and the
  residual stream are fp32 (the reference is fp32 throughout);
- only the pooled rows leave the GPU.

NumPy in, NumPy out; device work through the C ABI of libtessattn.so.
"""

from __future__ import annotations

import ctypes as ct
from dataclasses import dataclass

import numpy as np
from numpy.typing import NDArray

from . import native
from .errors import InvalidInputError
from .runtime import Buffer, CudaRuntime
from .workloads import to_bf16_bits


@dataclass(frozen=True)
class Qwen3Config:
    """Shape of a Qwen3 embedding model (Qwen3-Embedding-0.6B by default)."""

    hidden: int = 1024
    intermediate: int = 3072
    layers: int = 28
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    vocab: int = 151669
    eps: float = 1e-6
    theta: float = 1e6

    def check(self) -> None:
        """The shapes the kernels take (the reference's own checks are qwen3.py:36-44)."""
        if (self.head_dim != 128 or self.heads % self.kv_heads or self.hidden % 256
                or self.intermediate % 128 or (self.heads * self.head_dim) % 256
                or (self.kv_heads * self.head_dim) % 256 or self.hidden % 64):
            raise InvalidInputError()


def quantised_names(cfg: Qwen3Config) -> dict[str, tuple[int, int]]:
    """(outputs, inputs) of every uint4 matrix, under the reference's tensor names
    (qwen3.py:68-89)."""
    names = {"model.embed_tokens": (cfg.vocab, cfg.hidden)}
    for layer in range(cfg.layers):
        prefix = f"model.layers.{layer}"
        names[prefix + ".self_attn.q_proj"] = (cfg.heads * cfg.head_dim, cfg.hidden)
        names[prefix + ".self_attn.k_proj"] = (cfg.kv_heads * cfg.head_dim, cfg.hidden)
        names[prefix + ".self_attn.v_proj"] = (cfg.kv_heads * cfg.head_dim, cfg.hidden)
        names[prefix + ".self_attn.o_proj"] = (cfg.hidden, cfg.heads * cfg.head_dim)
        names[prefix + ".mlp.gate_proj"] = (cfg.intermediate, cfg.hidden)
        names[prefix + ".mlp.up_proj"] = (cfg.intermediate, cfg.hidden)
        names[prefix + ".mlp.down_proj"] = (cfg.hidden, cfg.intermediate)
    return names


def norm_names(cfg: Qwen3Config) -> dict[str, int]:
    names = {"model.norm": cfg.hidden}
    for layer in range(cfg.layers):
        prefix = f"model.layers.{layer}"
        names[prefix + ".input_layernorm"] = cfg.hidden
        names[prefix + ".post_attention_layernorm"] = cfg.hidden
        names[prefix + ".self_attn.q_norm"] = cfg.head_dim
        names[prefix + ".self_attn.k_norm"] = cfg.head_dim
    return names


def random_weights(cfg: Qwen3Config, seed: int) -> dict[str, NDArray]:
    """Seeded random weights in the reference's storage format: per uint4 matrix
    `.weight` uint32 [out, in/8] (random 4-bit codes), `.scales` bf16 N(0, 0.02) and
    `.biases` bf16 N(0, 0.01) [out, in/64]; per norm `.weight` bf16 1 + N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    weights: dict[str, NDArray] = {}
    for name, (out, inp) in quantised_names(cfg).items():
        weights[name + ".weight"] = rng.integers(0, 2**32, size=(out, inp // 8), dtype=np.uint32)
        weights[name + ".scales"] = to_bf16_bits(
            0.02 * rng.standard_normal((out, inp // 64), dtype=np.float32))
        weights[name + ".biases"] = to_bf16_bits(
            0.01 * rng.standard_normal((out, inp // 64), dtype=np.float32))
    for name, dims in norm_names(cfg).items():
        weights[name + ".weight"] = to_bf16_bits(
            1.0 + 0.02 * rng.standard_normal(dims, dtype=np.float32))
    return weights


def interleave_gate_up(gate: NDArray, up: NDArray, block: int = 128) -> NDArray:
    """Rows of two [out, ...] arrays in blocks of `block`: gate block 0, up block 0, gate
    block 1, ... -- the row order of the fused gated projection (TX_LINEAR_GATED_BF16)."""
    out = gate.shape[0]
    g = gate.reshape(out // block, block, *gate.shape[1:])
    u = up.reshape(out // block, block, *up.shape[1:])
    return np.ascontiguousarray(np.stack([g, u], axis=1).reshape(2 * out, *gate.shape[1:]))


class Qwen3Encoder:
    """The Qwen3 embedding forward on one device (counterpart of Qwen3Backend,
    qwen3.py:15-304, and of its Backend protocol, backend.py:23-32).

    `weights` maps the reference's tensor names to arrays in its storage format (see
    random_weights).  Loading uploads every tensor, dequantises the projection matrices
    to bf16 on the device (the gate and up projections interleaved into one fused
    matrix) and keeps the embedding table in uint4.
    """

    def __init__(self, weights: dict[str, NDArray], cfg: Qwen3Config = Qwen3Config(),
                 runtime: CudaRuntime | None = None, precise: bool = False) -> None:
        cfg.check()
        self.cfg = cfg
        # precise: every projection operand as a bf16 pair (hi + lo, about 16 significant
        # bits, three tensor-core products) and the attention in fp32 (the general
        # kernel), for results within the reference's fp32 tolerance; else bf16 operands
        # and the tensor-core attention.
        self.precise = precise
        self.rt = runtime or CudaRuntime(0)
        self._owns_runtime = runtime is None
        self._dev: dict[str, Buffer] = {}
        rt = self.rt

        def upload(a: NDArray) -> Buffer:
            a = np.ascontiguousarray(a)
            return rt.buffer(a.nbytes, a)

        try:
            for suffix in ("weight", "scales", "biases"):
                self._dev["embed." + suffix] = upload(weights[f"model.embed_tokens.{suffix}"])
            for name, dims in norm_names(cfg).items():
                self._dev[name] = upload(weights[name + ".weight"])
            for layer in range(cfg.layers):
                prefix = f"model.layers.{layer}"
                for proj in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                             "self_attn.o_proj", "mlp.down_proj"):
                    self._dev[f"{prefix}.{proj}"] = self._dequantised(
                        *(weights[f"{prefix}.{proj}.{s}"] for s in ("weight", "scales", "biases")))
                fused = [interleave_gate_up(weights[f"{prefix}.mlp.gate_proj.{s}"],
                                            weights[f"{prefix}.mlp.up_proj.{s}"])
                         for s in ("weight", "scales", "biases")]
                self._dev[f"{prefix}.mlp.gate_up"] = self._dequantised(*fused)
            rt.sync()
            self._model = self._describe()
        except BaseException:
            self.close()
            raise

    def _dequantised(self, packed: NDArray, scales: NDArray, biases: NDArray) -> Buffer:
        """bf16 [rows, cols] weights on the device (followed by their rounding residues,
        another [rows, cols], in precise mode)."""
        rows, cols = packed.shape[0], packed.shape[1] * 8
        rt = self.rt
        parts = [rt.buffer(a.nbytes, np.ascontiguousarray(a)) for a in (packed, scales, biases)]
        out = rt.buffer(rows * cols * 2 * (2 if self.precise else 1))
        try:
            rt.dequant4_device(*(b.device_ptr for b in parts), out.device_ptr, rows=rows, cols=cols,
                               out_lo=out.device_ptr + rows * cols * 2 if self.precise else None)
            rt.sync()
        finally:
            for b in parts:
                b.close()
        return out

    # ---- forward ---------------------------------------------------------------------------
    def forward(self, ids: NDArray, lengths: NDArray, *, dimensions: int | None = None
                ) -> NDArray[np.float32]:
        """Pooled, L2-normalised embeddings [batch, dimensions] of right-padded token ids
        [batch, seq] with valid lengths [batch] (qwen3.py:112-296)."""
        cfg = self.cfg
        dims = cfg.hidden if dimensions is None else dimensions
        ids = np.asarray(ids)
        lengths = np.asarray(lengths)
        if (ids.ndim != 2 or lengths.shape != (ids.shape[0],) or not 1 <= dims <= cfg.hidden
                or ids.shape[0] < 1 or np.any(lengths < 1) or np.any(lengths > ids.shape[1])
                or np.any(ids < 0)):
            raise InvalidInputError()
        lens = lengths.astype(np.int64)
        cu = np.zeros(lens.size + 1, dtype=np.int32)
        cu[1:] = np.cumsum(lens)
        tokens = np.concatenate([ids[b, :lens[b]] for b in range(lens.size)]).astype(np.uint32)
        return self.forward_packed(tokens, cu, dimensions=dims)

    def forward_packed(self, tokens: NDArray[np.uint32], cu_seqlens: NDArray[np.int32], *,
                       dimensions: int) -> NDArray[np.float32]:
        """The same forward on sequences packed end to end (cu_seqlens [batch + 1])."""
        cfg, rt = self.cfg, self.rt
        T, B = int(tokens.size), int(cu_seqlens.size - 1)
        if B < 1 or int(cu_seqlens[-1]) != T or not 1 <= dimensions <= cfg.hidden:
            raise InvalidInputError()
        ids_b = rt.workspace("qwen.ids", T * 4)
        cu_b = rt.workspace("qwen.cu", (B + 1) * 4)
        ids_b.write(np.ascontiguousarray(tokens, dtype=np.uint32))
        cu_b.write(np.ascontiguousarray(cu_seqlens, dtype=np.int32))
        pooled = rt.buffer(B * dimensions * 4)
        try:
            self.enqueue(ids_b.device_ptr, cu_b.device_ptr, cu_seqlens, pooled.device_ptr,
                         dimensions)
            rt.sync()
            result = rt.read(pooled, (B, dimensions))
        finally:
            pooled.close()
        # The reference's output check (qwen3.py:292-295).
        if not np.isfinite(result).all() or not np.allclose(
                np.linalg.norm(result, axis=1), 1.0, atol=1e-4, rtol=0.0):
            raise InvalidInputError()
        return result

    def enqueue(self, ids: int, cu: int, cu_seqlens: NDArray[np.int32], pooled: int,
                dimensions: int, stream: int | None = None) -> None:
        """Queues the whole forward on `stream` (None: the context's stream) without
        waiting: token ids `ids` (device uint32 [T]) packed by `cu` (device int32
        [batch + 1], host copy `cu_seqlens`) to pooled embeddings `pooled` (device fp32
        [batch, dimensions]).  One native call (tx_qwen3_forward) queues every launch;
        the activations live in the runtime's workspace "qwen.forward"."""
        rt = self.rt
        cu_host = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        need = int(rt._lib.tx_qwen3_workspace_bytes(ct.byref(self._model), int(cu_host[-1])))
        if not need:
            raise InvalidInputError()
        ws = rt.workspace("qwen.forward", need)
        rt.qwen3_forward_device(ct.byref(self._model), ids, cu, cu_host, pooled, dimensions,
                                ws.device_ptr, ws.size, stream=stream)

    def _describe(self) -> native.TxQwen3Model:
        """The native model description: shapes and the device pointers of every weight."""
        cfg, d = self.cfg, self._dev
        layers = (native.TxQwen3Layer * cfg.layers)()
        for layer in range(cfg.layers):
            p = f"model.layers.{layer}"
            ptr = {key: d[name].device_ptr for key, name in (
                ("input_norm", p + ".input_layernorm"),
                ("post_norm", p + ".post_attention_layernorm"),
                ("q_norm", p + ".self_attn.q_norm"), ("k_norm", p + ".self_attn.k_norm"),
                ("q_proj", p + ".self_attn.q_proj"), ("k_proj", p + ".self_attn.k_proj"),
                ("v_proj", p + ".self_attn.v_proj"), ("o_proj", p + ".self_attn.o_proj"),
                ("gate_up", p + ".mlp.gate_up"), ("down", p + ".mlp.down_proj"))}
            layers[layer] = native.TxQwen3Layer(**ptr)
        self._layers = layers  # the description points into this array
        return native.TxQwen3Model(
            hidden=cfg.hidden, intermediate=cfg.intermediate, layers=cfg.layers,
            heads=cfg.heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim, vocab=cfg.vocab,
            eps=cfg.eps, theta=cfg.theta, precise=int(self.precise),
            embed_packed=d["embed.weight"].device_ptr, embed_scales=d["embed.scales"].device_ptr,
            embed_biases=d["embed.biases"].device_ptr, final_norm=d["model.norm"].device_ptr,
            layer=ct.cast(layers, ct.POINTER(native.TxQwen3Layer)))

    def flops(self, lengths: NDArray) -> int:
        """Multiply-add work of one forward over sequences of these lengths, counted as 2
        flops each: the projections over every token plus the causal attention pairs."""
        cfg = self.cfg
        n = np.asarray(lengths, dtype=np.int64)
        qd, kd = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
        per_token = cfg.hidden * (qd + 2 * kd) + qd * cfg.hidden + 3 * cfg.hidden * cfg.intermediate
        pairs = int((n * (n + 1) // 2).sum())
        return cfg.layers * (2 * per_token * int(n.sum()) + 4 * cfg.head_dim * cfg.heads * pairs)

    def close(self) -> None:
        for b in self._dev.values():
            b.close()
        self._dev.clear()
        if self._owns_runtime:
            self.rt.close()
