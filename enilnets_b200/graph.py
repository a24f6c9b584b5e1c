"""Padding-mask-aware multi-head self-attention with the reference graph
layer's interface (graph/sequence.py:23-29, :90-183), on the B200 kernels.

Inference only: forward returns the output without building an autograd
graph. The masking rule is the graph layer's additive -1e9 per violated term
(padding, and causal/window), which the kernel applies exactly even for rows
whose every key is masked.
"""
from __future__ import annotations

from typing import Any, Optional

import numpy as np

from . import attention
from .backend import to_device, to_numpy
from .layers import _validate_num_kv_heads, init_weights


def lengths_to_mask(lengths: Any, max_len: Optional[int] = None) -> np.ndarray:
    """Per-example lengths -> boolean padding mask (batch, max_len), True
    where a token is real (graph/sequence.py:23-29)."""
    lengths = np.asarray(lengths).astype(np.int64)
    if max_len is None:
        max_len = int(lengths.max())
    return np.arange(max_len)[None, :] < lengths[:, None]


class Parameter:
    """Holds a weight array as `.data`, like the reference's graph Parameter."""

    def __init__(self, data: np.ndarray, name: str = "") -> None:
        self.data = data
        self.name = name


class Output:
    """Forward result: `.data` is the (batch, seq, embed_dim) NumPy array."""

    def __init__(self, data: np.ndarray) -> None:
        self.data = data

    @property
    def shape(self):
        return self.data.shape


class MultiHeadAttention:
    """graph.MultiHeadAttention(embed_dim, num_heads=4, causal=False,
    init_method="xavier_uniform", num_kv_heads=None, window_size=None);
    weights Wq/bq..Wo/bo drawn in the reference order and shareable with an
    nn/ layer dict."""

    def __init__(self, embed_dim: int, num_heads: int = 4, causal: bool = False,
                 init_method: str = "xavier_uniform", num_kv_heads: Optional[int] = None,
                 window_size: Optional[int] = None) -> None:
        if embed_dim % num_heads != 0:
            raise ValueError(
                f"embed_dim ({embed_dim}) must be divisible by num_heads ({num_heads})")
        self.embed_dim = embed_dim
        self.num_heads = num_heads
        self.num_kv_heads = _validate_num_kv_heads(num_heads, num_kv_heads, "MultiHeadAttention")
        self.head_dim = embed_dim // num_heads
        self.causal = causal
        if window_size is not None and window_size < 0:
            raise ValueError(f"window_size must be >= 0 or None, got {window_size}")
        self.window_size = window_size
        kv_dim = self.num_kv_heads * self.head_dim
        for name, out_dim in (("Wq", embed_dim), ("Wk", kv_dim), ("Wv", kv_dim),
                              ("Wo", embed_dim)):
            w, b = init_weights(embed_dim, out_dim, method=init_method)
            setattr(self, name, Parameter(w, name=name))
            bname = "b" + name[1:].lower()
            setattr(self, bname, Parameter(b, name=bname))

    def _layer(self) -> dict:
        return {"type": "multihead_attention", "embed_dim": self.embed_dim,
                "num_heads": self.num_heads, "num_kv_heads": self.num_kv_heads,
                "head_dim": self.head_dim, "causal": self.causal,
                "window_size": self.window_size, "positional_scheme": "absolute",
                "Wq": self.Wq.data, "bq": self.bq.data, "Wk": self.Wk.data, "bk": self.bk.data,
                "Wv": self.Wv.data, "bv": self.bv.data, "Wo": self.Wo.data, "bo": self.bo.data}

    def forward_device(self, x, key_padding_mask=None):
        import torch
        xd = x if hasattr(x, "is_cuda") else to_device(getattr(x, "data", x), torch.float32)
        return attention.self_attention(self._layer(), xd, key_padding_mask=key_padding_mask,
                                        mask_mode="additive")

    def forward(self, x, key_padding_mask=None) -> Output:
        """x (batch, seq, embed_dim); key_padding_mask (batch, seq) bool, True =
        real token (graph/sequence.py:144-183)."""
        return Output(to_numpy(self.forward_device(x, key_padding_mask)))

    __call__ = forward
