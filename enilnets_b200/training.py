"""Training path of the attention layer on the B200 kernels.

The reference trains a multihead_attention layer with Forward(training=True),
which caches (Q, K, V, Qh, Kh, Vh, attn, context, x_in), and
nn/backward.py:241-327 (multihead_attention_backward), which forms the
projection gradients around the attention core's dQh, dKh, dVh and returns dx.
Here the forward keeps what the backward kernels need (the bf16 Q, K, V the
attention core read, its output and LSE) and the backward runs K5
(enl_attn_backward) for the core:

  d_Wo = dout^T context, d_bo = sum dout, dcontext = dout Wo
  dQh, dKh, dVh = K5(Q, K, V, O, LSE, dcontext)     (GQA already summed)
  RoPE layers: dQh, dKh rotated back by -angle     (nn/backward.py:300-308)
  d_Wq = dQ^T x_in, d_bq = sum dQ, ... ; dx = dQ Wq + dK Wk + dV Wv.

The projections run in fp32 GEMMs. The attention core follows set_precision
in both directions: under "fp32" (the reference's float32 models) Q, K, V,
the output and dO stay fp32 and K1 / K5 split them into bf16 hi/lo planes
(three MMAs per product), for head dims up to 64, where the split backward
fits in shared memory; wider heads, and the "bf16" precision, run the core
on bf16 operands with fp32 accumulation. Softmax layers only (plain and tiled_block_size, which compute the same function);
linearized kernels, sparse patterns and attention dropout raise ValueError.
"""
from __future__ import annotations

from typing import Any, Dict, Tuple

import numpy as np

from . import attention, backend, kernels
from .backend import to_device, to_numpy

_NEG_SIN: dict = {}


def _check_trainable(layer: Dict[str, Any]) -> None:
    if layer.get("type", "multihead_attention") != "multihead_attention":
        raise ValueError(f"training covers multihead_attention layers, not {layer.get('type')!r}")
    if layer.get("attention_kernel", "softmax") != "softmax":
        raise ValueError("the attention backward covers attention_kernel='softmax' layers "
                         f"(got {layer.get('attention_kernel')!r})")
    if layer.get("sparse_pattern") is not None:
        raise ValueError("the attention backward does not cover sparse_pattern layers")
    if layer.get("dropout", 0.0) > 0:
        raise ValueError("attention dropout at training=True is not supported by the B200 "
                         "attention path")


def _unrotate(t, pos0: int = 0):
    """Rotate (B, S, H, D) fp32 in place by the negated RoPE angles: the
    transpose of the forward rotation (nn/backward.py:300-308)."""
    import torch
    cos, sin = attention.rope_tables(pos0 + t.shape[1], t.shape[-1])
    key = (sin.data_ptr(), sin.shape[0])
    neg = _NEG_SIN.get(key)
    if neg is None:
        _NEG_SIN.clear()
        neg = _NEG_SIN[key] = torch.neg(sin)
    kernels.rope_(t, cos, neg, pos0)
    return t


def _core_dtype(head_dim: int):
    """Operand dtype of the attention core for this precision and head dim."""
    import torch
    if backend.compute_dtype() == torch.float32 and head_dim <= 64:
        return torch.float32
    return torch.bfloat16


def _weights_f32(layer, names):
    import torch
    return attention._WEIGHTS.get(layer, names, "w", torch.float32)


def self_attention_forward_train(layer: Dict[str, Any], x) -> Tuple[Any, Dict[str, Any]]:
    """Forward of one multihead_attention layer on a (B, S, E) device tensor,
    returning the fp32 output and the cache the backward needs."""
    import torch
    import torch.nn.functional as F
    _check_trainable(layer)
    B, S, E = x.shape
    H, D = layer["num_heads"], layer["head_dim"]
    Hkv = layer.get("num_kv_heads") or H
    x = x.float()
    w = _weights_f32(layer, ("Wq", "Wk", "Wv"))
    b = attention._WEIGHTS.get(layer, ("bq", "bk", "bv"), "b", torch.float32)
    core = _core_dtype(D)
    qkv = F.linear(x, w, b).to(core)
    q = attention.split_heads(qkv, H, D, 0)
    k = attention.split_heads(qkv, Hkv, D, H * D)
    v = attention.split_heads(qkv, Hkv, D, H * D + Hkv * D)
    scheme = layer.get("positional_scheme", "absolute")
    if scheme == "rope":
        attention.apply_rope(q, 0)
        attention.apply_rope(k, 0)
    causal = bool(layer.get("causal", False))
    window = layer.get("window_size")
    slopes = attention.alibi_tensor(H) if scheme == "alibi" else None
    o, lse = kernels.attention_prefill(q, k, v, causal=causal, window=window,
                                       alibi_slopes=slopes, out_dtype=core,
                                       return_lse=True)
    ctx = o.flatten(-2).float()
    wo = _weights_f32(layer, ("Wo",))
    bo = attention._WEIGHTS.get(layer, ("bo",), "b", torch.float32)
    y = F.linear(ctx, wo, bo)
    cache = {"x": x, "q": q, "k": k, "v": v, "o": o, "lse": lse, "ctx": ctx,
             "causal": causal, "window": window, "slopes": slopes, "rope": scheme == "rope"}
    return y, cache


def self_attention_backward(layer: Dict[str, Any], cache: Dict[str, Any],
                            dout) -> Tuple[Any, Dict[str, Any]]:
    """(dx, grads) of the layer for dout (B, S, E) on the device: grads holds
    d_Wq, d_bq, d_Wk, d_bk, d_Wv, d_bv, d_Wo, d_bo as fp32 device tensors."""
    import torch
    B, S, E = dout.shape
    H, D = layer["num_heads"], layer["head_dim"]
    Hkv = layer.get("num_kv_heads") or H
    kv_dim = Hkv * D
    dout = dout.float()
    d2 = dout.reshape(-1, E)
    grads = {"d_Wo": d2.T @ cache["ctx"].reshape(-1, E), "d_bo": d2.sum(0)}
    dctx = (dout @ _weights_f32(layer, ("Wo",))).unflatten(-1, (H, D)).to(cache["q"].dtype)
    dq, dk, dv = kernels.attention_backward(cache["q"], cache["k"], cache["v"], cache["o"],
                                            cache["lse"], dctx, causal=cache["causal"],
                                            window=cache["window"],
                                            alibi_slopes=cache["slopes"])
    if cache["rope"]:
        _unrotate(dq)
        _unrotate(dk)
    x2 = cache["x"].reshape(-1, E)
    dQ, dK, dV = dq.reshape(-1, E), dk.reshape(-1, kv_dim), dv.reshape(-1, kv_dim)
    for name, g in (("q", dQ), ("k", dK), ("v", dV)):
        grads[f"d_W{name}"] = g.T @ x2
        grads[f"d_b{name}"] = g.sum(0)
    dx = dQ @ _weights_f32(layer, ("Wq",)) + dK @ _weights_f32(layer, ("Wk",)) + \
        dV @ _weights_f32(layer, ("Wv",))
    return dx.reshape(B, S, E), grads


def multihead_attention_forward_train(layer: Dict[str, Any], x) -> Tuple[np.ndarray, Dict]:
    """NumPy in, NumPy out: the layer's training forward and its cache."""
    import torch
    _check_trainable(layer)  # before any device work
    y, cache = self_attention_forward_train(layer, to_device(np.asarray(x), torch.float32))
    return to_numpy(y), cache


def multihead_attention_backward(dout, layer: Dict[str, Any], cache: Dict[str, Any]) -> np.ndarray:
    """nn/backward.py:241-327 for a softmax layer: stores d_Wq, d_bq, d_Wk,
    d_bk, d_Wv, d_bv, d_Wo, d_bo on `layer` (NumPy, the weights' dtype) and
    returns dx, the gradient of the layer's input."""
    import torch
    dx, grads = self_attention_backward(layer, cache,
                                        to_device(np.asarray(dout), torch.float32))
    for name, g in grads.items():
        ref = layer[name.replace("d_", "", 1)]
        layer[name] = to_numpy(g).astype(np.asarray(ref).dtype, copy=False)
    return to_numpy(dx)
