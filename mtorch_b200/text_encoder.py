"""CLIP text encoder (SD-1.5's ViT-L/14 text tower shape) on the device path.

The reference has no text-encoder model; its Stable-Diffusion workload composes one from public ops
(tests/compat/benchmarking.py:5194-5244: token + position embedding, LayerNorm, causal multi-head
attention, output projection; 7690-7715: the pre-LN layer with the quick-GELU MLP).  This module
composes the same ops at SD-1.5's text-encoder shape: vocabulary 49408, 77 positions, width 768,
12 layers of 12 heads (head dim 64), MLP 3072, final LayerNorm.

Kernels per layer: LayerNorm; one QKV GEMM (bias in the epilogue) whose output the attention kernel
reads as strided head views; causal flash attention writing heads-merged rows; the output projection
with the residual add in its epilogue; LayerNorm; the MLP-in GEMM with quick-GELU in its epilogue;
the MLP-out GEMM with the residual add in its epilogue.  The token and position embeddings are
gathered and summed by one kernel.
"""
from __future__ import annotations

import numpy as np

from . import _lib as L
from . import ops
from .nn import LayerNorm, Linear, Module, ModuleList, init
from .tensor import Tensor, _new, empty, tensor


class CLIPEncoderLayer(Module):
    def __init__(self, width=768, heads=12, mlp=3072, device=None, dtype=None):
        super().__init__()
        kw = dict(device=device, dtype=dtype)
        self.width, self.heads = width, heads
        self.norm1 = LayerNorm(width, **kw)
        self.qkv = Linear(width, 3 * width, **kw)
        self.out = Linear(width, width, **kw)
        self.norm2 = LayerNorm(width, **kw)
        self.fc1 = Linear(width, mlp, **kw)
        self.fc2 = Linear(mlp, width, **kw)

    def forward(self, h: Tensor, n: int, s: int) -> Tensor:
        """h: [n*s, width] token rows -> [n*s, width]."""
        c, H = self.width, self.heads
        D = c // H
        y = self.norm1(h)
        qkv = ops.linear(y, self.qkv.weight, self.qkv.bias)
        p = qkv.stride(0)

        def heads(t):
            return t._view((n, H, s, D), (s * p, D, p, 1))

        a = _new((n * s, c), h.dtype, h.device)
        av = a._view((n, H, s, D), (s * c, D, c, 1))
        ops.scaled_dot_product_attention(heads(qkv[:, 0:c]), heads(qkv[:, c:2 * c]), heads(qkv[:, 2 * c:3 * c]),
                                         is_causal=True, out=av)
        h = ops.linear(a, self.out.weight, self.out.bias, residual=h)
        y = self.norm2(h)
        y = ops.linear(y, self.fc1.weight, self.fc1.bias, epilogue=L.EPI_QUICK_GELU)
        return ops.linear(y, self.fc2.weight, self.fc2.bias, residual=h)


class CLIPTextEncoder(Module):
    """input_ids [n, s] (host or device int64) -> last hidden state [n, s, width] after the final
    LayerNorm (what the UNet's cross-attention consumes).  Weights are random-init: embeddings
    N(0, 0.02), linear layers with the module default."""

    def __init__(self, vocab=49408, positions=77, width=768, layers=12, heads=12, mlp=3072, device=None,
                 dtype=None):
        super().__init__()
        kw = dict(device=device, dtype=dtype)
        self.width, self.positions = width, positions
        self.register_parameter("token_embedding", empty(vocab, width, **kw))
        self.register_parameter("position_embedding", empty(positions, width, **kw))
        init.normal_(self.token_embedding, 0.0, 0.02)
        init.normal_(self.position_embedding, 0.0, 0.02)
        self.layers = ModuleList([CLIPEncoderLayer(width, heads, mlp, **kw) for _ in range(layers)])
        self.final_norm = LayerNorm(width, **kw)
        self._pos_ids = {}

    def _positions(self, n, s, dev):
        key = (n, s, str(dev))
        if key not in self._pos_ids:
            self._pos_ids[key] = tensor(np.broadcast_to(np.arange(s, dtype=np.int64), (n, s)).copy()).to(dev)
        return self._pos_ids[key]

    def forward(self, input_ids: Tensor) -> Tensor:
        n, s = input_ids.shape
        if s > self.positions:
            raise ValueError(f"CLIPTextEncoder: sequence of {s} tokens exceeds {self.positions} positions")
        dev = self.token_embedding.device
        h = ops.embedding(input_ids, self.token_embedding, add_weight=self.position_embedding,
                          add_input=self._positions(n, s, dev))
        h = h.reshape(n * s, self.width)
        for layer in self.layers:
            h = layer(h, n, s)
        return self.final_norm(h).reshape(n, s, self.width)


def clip_text_flops(seq=77, width=768, layers=12, mlp=3072) -> float:
    """FLOPs (2 per MAC) of one sequence: the four projections per layer and the attention
    products counted over the full S x S (the causal half is still computed)."""
    per_layer = 2.0 * seq * width * (3 * width + width + 2 * mlp) + 4.0 * seq * seq * width
    return layers * per_layer
