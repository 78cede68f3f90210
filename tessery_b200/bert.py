"""BERT (BGE-small) fp32 embedding forward on one B200: the layer loop of
BertBackend.forward (bert.py:104-235 in the reference) around this library's head_dim-32
attention.

Per layer, as the reference (bert.py:191-231): q, k and v projections (+ bias),
bidirectional attention over each sequence's valid tokens, output projection added to
the residual stream and LayerNorm, intermediate projection with GELU, output projection
added and LayerNorm; then the CLS row of each sequence, L2-normalised (bert.py:232-241).
Differences, all of layout or number format:

- sequences are packed by cu_seqlens (no padded rows: with the key-padding mask a padded
  row never reaches a valid row's output);
- the projections run on tensor cores with TF32 split operands (three products: about 22
  significant bits per operand, fp32-level results); `precise=False` uses one TF32
  product per projection;
- the three q/k/v projections are one GEMM over their stacked weights;
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


@dataclass(frozen=True)
class BertConfig:
    """Shape of a BERT encoder (BGE-small-en-v1.5 by default)."""

    hidden: int = 384
    intermediate: int = 1536
    layers: int = 12
    heads: int = 12
    vocab: int = 30522
    max_pos: int = 512
    types: int = 2
    eps: float = 1e-12

    def check(self) -> None:
        """The shapes the kernels take (the reference's own checks are bert.py:23-47)."""
        if (self.hidden % 128 or self.hidden > 1024 or self.hidden % self.heads
                or self.intermediate % 128 or not self.layers or self.vocab < 1
                or self.max_pos < 1 or self.types < 1):
            raise InvalidInputError()

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


def weight_shapes(cfg: BertConfig) -> dict[str, tuple[int, ...]]:
    """Every fp32 tensor of the model under the reference's names (bert.py:49-75)."""
    shapes: dict[str, tuple[int, ...]] = {
        "embeddings.word_embeddings.weight": (cfg.vocab, cfg.hidden),
        "embeddings.position_embeddings.weight": (cfg.max_pos, cfg.hidden),
        "embeddings.token_type_embeddings.weight": (cfg.types, cfg.hidden),
        "embeddings.LayerNorm.weight": (cfg.hidden,),
        "embeddings.LayerNorm.bias": (cfg.hidden,),
    }
    for layer in range(cfg.layers):
        p = f"encoder.layer.{layer}"
        for name, out, inp in (("attention.self.query", cfg.hidden, cfg.hidden),
                               ("attention.self.key", cfg.hidden, cfg.hidden),
                               ("attention.self.value", cfg.hidden, cfg.hidden),
                               ("attention.output.dense", cfg.hidden, cfg.hidden),
                               ("intermediate.dense", cfg.intermediate, cfg.hidden),
                               ("output.dense", cfg.hidden, cfg.intermediate)):
            shapes[f"{p}.{name}.weight"] = (out, inp)
            shapes[f"{p}.{name}.bias"] = (out,)
        for name in ("attention.output.LayerNorm", "output.LayerNorm"):
            shapes[f"{p}.{name}.weight"] = (cfg.hidden,)
            shapes[f"{p}.{name}.bias"] = (cfg.hidden,)
    return shapes


def random_weights(cfg: BertConfig, seed: int) -> dict[str, NDArray[np.float32]]:
    """Seeded random fp32 weights in the reference's layout: matrices and embeddings
    N(0, 0.02^2), biases N(0, 0.02^2), LayerNorm weights 1 + N(0, 0.02^2) and biases
    N(0, 0.02^2)."""
    rng = np.random.default_rng(seed)
    weights: dict[str, NDArray[np.float32]] = {}
    for name, shape in weight_shapes(cfg).items():
        w = 0.02 * rng.standard_normal(shape, dtype=np.float32)
        if name.endswith("LayerNorm.weight"):
            w += np.float32(1.0)
        weights[name] = w.astype(np.float32)
    return weights


class BertEncoder:
    """The BERT embedding forward on one device (counterpart of BertBackend,
    bert.py:13-248).  `weights` maps the reference's tensor names to fp32 arrays."""

    def __init__(self, weights: dict[str, NDArray], cfg: BertConfig = BertConfig(),
                 runtime: CudaRuntime | None = None, precise: bool = True) -> None:
        cfg.check()
        self.cfg = cfg
        self.precise = precise
        self.rt = runtime or CudaRuntime(0)
        self._owns_runtime = runtime is None
        self._dev: dict[str, Buffer] = {}
        shapes = weight_shapes(cfg)
        for name, shape in shapes.items():
            if np.asarray(weights[name]).shape != shape:
                raise InvalidInputError()
        try:
            for name in shapes:  # tables, LayerNorms and the dense biases as they are
                if "attention.self." not in name and not self._is_projection(name):
                    self._dev[name] = self._upload(weights[name])
            for layer in range(cfg.layers):
                p = f"encoder.layer.{layer}"
                a = p + ".attention.self."
                stacked = np.concatenate([weights[a + s + ".weight"] for s in
                                          ("query", "key", "value")])
                self._dev[p + ".qkv.weight"] = self._split(stacked)
                self._dev[p + ".qkv.bias"] = self._upload(np.concatenate(
                    [weights[a + s + ".bias"] for s in ("query", "key", "value")]))
                for name in ("attention.output.dense", "intermediate.dense", "output.dense"):
                    self._dev[f"{p}.{name}.weight"] = self._split(weights[f"{p}.{name}.weight"])
            self.rt.sync()
            self._model = self._describe()
        except BaseException:
            self.close()
            raise

    @staticmethod
    def _is_projection(name: str) -> bool:
        """A projection matrix (uploaded as a TF32 operand pair)."""
        return name.endswith(".weight") and ("attention.self." in name or ".dense." in name)

    def _upload(self, a: NDArray) -> Buffer:
        a = np.ascontiguousarray(a, dtype=np.float32)
        return self.rt.buffer(a.nbytes, a)

    def _split(self, w: NDArray) -> Buffer:
        """fp32 [n, k] weights as a TF32 operand pair on the device: hi then lo."""
        w = np.ascontiguousarray(w, dtype=np.float32)
        raw = self._upload(w)
        try:
            pair = self.rt.buffer(2 * w.nbytes)
            self.rt.split_tf32_device(raw.device_ptr, pair.device_ptr, n=w.size)
            self.rt.sync()
        finally:
            raw.close()
        return pair

    def _describe(self) -> native.TxBertModel:
        cfg, d = self.cfg, self._dev
        layers = (native.TxBertLayer * cfg.layers)()
        for layer in range(cfg.layers):
            p = f"encoder.layer.{layer}"
            ln1, ln2 = p + ".attention.output.LayerNorm", p + ".output.LayerNorm"
            layers[layer] = native.TxBertLayer(
                qkv_w=d[p + ".qkv.weight"].device_ptr, qkv_b=d[p + ".qkv.bias"].device_ptr,
                o_w=d[p + ".attention.output.dense.weight"].device_ptr,
                o_b=d[p + ".attention.output.dense.bias"].device_ptr,
                ln1_w=d[ln1 + ".weight"].device_ptr, ln1_b=d[ln1 + ".bias"].device_ptr,
                i_w=d[p + ".intermediate.dense.weight"].device_ptr,
                i_b=d[p + ".intermediate.dense.bias"].device_ptr,
                out_w=d[p + ".output.dense.weight"].device_ptr,
                out_b=d[p + ".output.dense.bias"].device_ptr,
                ln2_w=d[ln2 + ".weight"].device_ptr, ln2_b=d[ln2 + ".bias"].device_ptr)
        self._layers = layers  # the description points into this array
        e = "embeddings."
        return native.TxBertModel(
            hidden=cfg.hidden, intermediate=cfg.intermediate, layers=cfg.layers, heads=cfg.heads,
            vocab=cfg.vocab, max_pos=cfg.max_pos, eps=cfg.eps, precise=int(self.precise),
            words=d[e + "word_embeddings.weight"].device_ptr,
            positions=d[e + "position_embeddings.weight"].device_ptr,
            types=d[e + "token_type_embeddings.weight"].device_ptr,
            ln_w=d[e + "LayerNorm.weight"].device_ptr, ln_b=d[e + "LayerNorm.bias"].device_ptr,
            layer=ct.cast(layers, ct.POINTER(native.TxBertLayer)))

    # ---- forward ---------------------------------------------------------------------------
    def forward(self, ids: NDArray, lengths: NDArray) -> NDArray[np.float32]:
        """CLS embeddings [batch, hidden], L2-normalised, of right-padded token ids
        [batch, seq] with valid lengths [batch] (bert.py:104-248)."""
        ids, lengths = np.asarray(ids), np.asarray(lengths)
        if (ids.ndim != 2 or lengths.shape != (ids.shape[0],) or ids.shape[0] < 1
                or np.any(lengths < 1) or np.any(lengths > ids.shape[1])
                or np.any(lengths > self.cfg.max_pos) or np.any(ids < 0)):
            raise InvalidInputError()
        lens = lengths.astype(np.int64)
        cu = np.zeros(lens.size + 1, dtype=np.int32)
        cu[1:] = np.cumsum(lens)
        tokens = np.concatenate([ids[b, :lens[b]] for b in range(lens.size)]).astype(np.uint32)
        return self.forward_packed(tokens, cu)

    def forward_packed(self, tokens: NDArray[np.uint32], cu_seqlens: NDArray[np.int32]
                       ) -> NDArray[np.float32]:
        """The same forward on sequences packed end to end (cu_seqlens [batch + 1])."""
        rt = self.rt
        T, B = int(tokens.size), int(cu_seqlens.size - 1)
        if B < 1 or int(cu_seqlens[-1]) != T:
            raise InvalidInputError()
        ids_b = rt.workspace("bert.ids", T * 4)
        cu_b = rt.workspace("bert.cu", (B + 1) * 4)
        ids_b.write(np.ascontiguousarray(tokens, dtype=np.uint32))
        cu_b.write(np.ascontiguousarray(cu_seqlens, dtype=np.int32))
        pooled = rt.buffer(B * self.cfg.hidden * 4)
        try:
            self.enqueue(ids_b.device_ptr, cu_b.device_ptr, cu_seqlens, pooled.device_ptr)
            rt.sync()
            result = rt.read(pooled, (B, self.cfg.hidden))
        finally:
            pooled.close()
        # The reference's output check (bert.py:242-246).
        if not np.isfinite(result).all() or not np.allclose(
                np.linalg.norm(result, axis=1), 1.0, atol=1e-4, rtol=0.0):
            raise InvalidInputError()
        return result

    def enqueue(self, ids: int, cu: int, cu_seqlens: NDArray[np.int32], pooled: int,
                stream: int | None = None) -> None:
        """Queues the whole forward on `stream` (None: the context's stream) without
        waiting: token ids `ids` (device uint32 [T]) packed by `cu` (device int32
        [batch + 1], host copy `cu_seqlens`) to CLS embeddings `pooled` (device fp32
        [batch, hidden]).  One native call (tx_bert_forward)."""
        rt = self.rt
        cu_host = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        need = int(rt._lib.tx_bert_workspace_bytes(ct.byref(self._model), int(cu_host[-1])))
        if not need:
            raise InvalidInputError()
        ws = rt.workspace("bert.forward", need)
        rt.bert_forward_device(ct.byref(self._model), ids, cu, cu_host, pooled, ws.device_ptr,
                               ws.size, stream=stream)

    def flops(self, lengths: NDArray) -> int:
        """Multiply-add work of one forward, 2 flops each: the projections over every
        valid token plus the bidirectional attention pairs."""
        cfg = self.cfg
        n = np.asarray(lengths, dtype=np.int64)
        per_token = 4 * cfg.hidden * cfg.hidden + 2 * cfg.hidden * cfg.intermediate
        pairs = int((n * n).sum())
        return cfg.layers * (2 * per_token * int(n.sum()) + 4 * cfg.hidden * pairs)

    def close(self) -> None:
        for b in self._dev.values():
            b.close()
        self._dev.clear()
        if self._owns_runtime:
            self.rt.close()
