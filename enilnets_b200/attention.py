"""Layer-level attention on the B200 kernels.

Mirrors the reference's attention branches layer by layer:
  * self-attention           nn/forward.py:423-556 (projections, RoPE/ALiBi,
                             GQA, causal/window masks, softmax, Wo)
  * cross-attention          nn/forward.py:557-591
  * key-padding (graph MHA)  graph/sequence.py:144-183 (additive -1e9 rule)
  * linearized kernels       nn/forward.py:456-480
  * block-sparse patterns    nn/forward.py:482-502
The projections run on the K6 tcgen05 GEMM (kernels.project) in the
precision that backend.set_precision selects: bf16 operands, or fp32 through
split-bf16 planes (hi*hi + hi*lo + lo*hi). The bias and, for RoPE layers, the
rotation of Q and K are fused into its epilogue. Q/K/V are never copied or
expanded: the prefill kernel (K1) reads them as strided head views of the
fused QKV projection output and indexes K/V heads group-major
(nn/forward.py:165-171) instead of repeating them.
"""
from __future__ import annotations

import math
from typing import Optional

import numpy as np

from . import kernels, sparse
from .backend import compute_dtype, device, to_device

SINUSOIDAL_BASE = 10000.0  # core/constants.py:70


LINEAR_KERNELS = ("linear", "performer")


def check_supported(layer: dict, training: bool = False) -> None:
    """Raise ValueError for options the B200 kernels do not implement, naming
    the option, instead of falling back to another backend."""
    kernel = layer.get("attention_kernel", "softmax")
    if kernel != "softmax" and kernel not in LINEAR_KERNELS:
        raise ValueError(f"attention_kernel={kernel!r} is not supported by the B200 attention "
                         "path (softmax, linear and performer only).")
    if training and layer.get("dropout", 0.0) > 0:
        raise ValueError("attention dropout at training=True is not supported by the B200 "
                         "attention path (inference only).")


# --------------------------------------------------------------- caches
class _LayerWeights:
    """Device copies (in the compute dtype) of one layer's concatenated
    projections, rebuilt whenever an array in the layer dict is replaced."""

    def __init__(self):
        self._store = {}

    def get(self, layer: dict, names, kind, dtype):
        """kind "w": the weights stacked on their output axis, in dtype; "b":
        the biases concatenated; "split": (hi, lo) bf16 planes of the fp32
        weights, the operand of the split-bf16 projection."""
        arrays = tuple(layer[n] for n in names)
        key = (kind, dtype, device().index) + tuple(id(a) for a in arrays)
        hit = self._store.get(key)
        if hit is not None and all(x is y for x, y in zip(hit[0], arrays)):
            return hit[1]
        import torch
        if kind in ("w", "split"):
            host = np.concatenate([np.asarray(a, np.float32) for a in arrays], axis=0)
        else:
            host = np.concatenate([np.asarray(a, np.float32).reshape(-1) for a in arrays])
        if kind == "split":
            t = kernels.split_bf16(to_device(host, torch.float32))
        else:
            t = to_device(host, dtype)
        self._store[key] = (arrays, t)
        return t


_WEIGHTS = _LayerWeights()
_ALIBI: dict = {}
_ROPE: dict = {}


def alibi_slopes(num_heads: int) -> np.ndarray:
    """Geometric ALiBi slopes, nn/forward.py:90-100."""
    def pow2(n):
        start = 2.0 ** (-8.0 / n)
        return [start ** (i + 1) for i in range(n)]
    if num_heads & (num_heads - 1) == 0:
        return np.array(pow2(num_heads))
    closest = 2 ** int(np.floor(np.log2(num_heads)))
    return np.array(pow2(closest) + pow2(2 * closest)[0::2][: num_heads - closest])


def alibi_tensor(num_heads: int):
    import torch
    key = (num_heads, device().index)
    if key not in _ALIBI:
        _ALIBI[key] = to_device(alibi_slopes(num_heads).astype(np.float32), torch.float32)
    return _ALIBI[key]


def rope_tables(n_rows: int, head_dim: int):
    """(cos, sin) device tables of at least n_rows rows, computed in float64
    exactly as nn/forward.py:46-55 computes the angles."""
    import torch
    key = (head_dim, device().index)
    have = _ROPE.get(key)
    if have is None or have[0].shape[0] < n_rows:
        rows = max(n_rows, 2 * (have[0].shape[0] if have is not None else 0), 256)
        half = head_dim // 2
        theta = SINUSOIDAL_BASE ** (-2.0 * np.arange(half) / head_dim)
        angles = np.arange(rows, dtype=np.float64)[:, None] * theta[None, :]
        have = (to_device(np.cos(angles).astype(np.float32), torch.float32),
                to_device(np.sin(angles).astype(np.float32), torch.float32))
        _ROPE[key] = have
    return have


def apply_rope(t, pos0: int):
    """Rotate (B, S, H, D) in place at absolute positions pos0.. (nn/forward.py:80-88)."""
    cos, sin = rope_tables(pos0 + t.shape[1], t.shape[-1])
    kernels.rope_(t, cos, sin, pos0)
    return t


# ---------------------------------------------------------- projections
FUSED_ROPE_HEAD_DIMS = (8, 16, 32, 64, 128)


def project(x, layer: dict, which: str, rope_pos0: Optional[int] = None, out_dtype=None):
    """x @ W.T + b for W in {"q", "kv", "qkv", "o"} as one K6 GEMM in the
    compute dtype (nn/forward.py:428-430, :551); fp32 runs the split-bf16
    path. With rope_pos0 (a "qkv" projection of a RoPE layer) the Q and K
    columns come out rotated at positions rope_pos0 + s (nn/forward.py:80-88),
    fused into the GEMM's epilogue; returns (y, rotated) so that head dims the
    epilogue does not cover fall back to apply_rope. out_dtype defaults to the
    compute dtype; the layers' output projections ask for fp32, which the
    epilogue writes directly (no bf16 rounding, no separate cast)."""
    import torch
    names = {"q": (("Wq",), ("bq",)), "kv": (("Wk", "Wv"), ("bk", "bv")),
             "qkv": (("Wq", "Wk", "Wv"), ("bq", "bk", "bv")), "o": (("Wo",), ("bo",))}[which]
    dt = compute_dtype()
    b = _WEIGHTS.get(layer, names[1], "b", torch.float32)
    rope = None
    if rope_pos0 is not None:
        H, D = layer["num_heads"], layer["head_dim"]
        Hkv = layer.get("num_kv_heads") or H
        if D in FUSED_ROPE_HEAD_DIMS:
            S = x.shape[-2]
            cos, sin = rope_tables(rope_pos0 + S, D)
            rope = (cos, sin, (H + Hkv) * D, D, S, rope_pos0)
    out_dtype = out_dtype or dt
    if dt == torch.float32:
        hi, lo = _WEIGHTS.get(layer, names[0], "split", dt)
        y = kernels.project(x.float(), hi, b, w_lo=lo, out_dtype=out_dtype, rope=rope)
    else:
        w = _WEIGHTS.get(layer, names[0], "w", dt)
        y = kernels.project(x.to(dt), w, b, out_dtype=out_dtype, rope=rope)
    return (y, rope is not None) if rope_pos0 is not None else y


def split_heads(t, heads: int, head_dim: int, offset: int = 0):
    """(B, S, *) -> strided (B, S, heads, head_dim) view at column offset."""
    return t[..., offset:offset + heads * head_dim].unflatten(-1, (heads, head_dim))


def classify_key_mask(mask, B: int, S: int):
    """A boolean key-padding mask (True = real token) as the kernel takes it.

    graph/sequence.py:162-168 adds -1e9 for any (batch, seq) mask. A mask
    whose real tokens form a prefix in every row (what lengths_to_mask,
    graph/sequence.py:23-29, builds) becomes ("lengths", int32 (B,)); any
    other mask (left padding, holes) ("words", int64 (B, ceil(S/64)) packed
    bits). Host arrays; raises ValueError for a wrong shape, as the
    reference does."""
    m = np.asarray(mask if not hasattr(mask, "detach") else mask.detach().cpu().numpy())
    if m.shape != (B, S):
        raise ValueError(f"key_padding_mask shape {m.shape} must be (batch, seq) = {(B, S)}")
    m = m.astype(bool)
    lengths = m.sum(axis=1)
    if np.array_equal(m, np.arange(S)[None, :] < lengths[:, None]):
        return "lengths", lengths.astype(np.int32)
    return "words", kernels.key_mask_words(m)


def key_mask_args(mask, B: int, S: int) -> dict:
    """classify_key_mask as attention_prefill keyword arguments on the device."""
    import torch
    kind, arr = classify_key_mask(mask, B, S)
    if kind == "lengths":
        return {"kv_valid_len": to_device(arr, torch.int32)}
    return {"kv_mask": torch.from_numpy(arr).to(device())}


def omega_tensor(layer: dict):
    """The Performer projection of a layer as a device fp32 tensor."""
    import torch
    return _WEIGHTS.get(layer, ("omega",), "w", torch.float32)


def linearized(layer: dict, q, k, v, causal: bool):
    """phi(Q) (phi(K)^T V) / (phi(Q) . sum phi(K)) for a linear or performer
    layer (nn/forward.py:456-478): queries take the row stabilizer, keys one
    global stabilizer per (batch, kv head), the same as the reference's per
    expanded head since a group's heads are copies."""
    kernel = layer["attention_kernel"]
    omega = omega_tensor(layer) if kernel == "performer" else None
    Df = omega.shape[0] if omega is not None else q.shape[3]
    # On the tensor-core path the maps write phi as the bf16 planes the
    # attention reads (no fp32 phi round trip).
    planes = kernels.linear_planes_ok(v.shape[3], Df)
    qp, _ = kernels.linear_feature_map(q, kernel, omega, planes=planes)
    kp, _ = kernels.linear_feature_map(k, kernel, omega, global_stab=True, planes=planes)
    return kernels.linear_attention(qp, kp, v, causal=causal, out_dtype=compute_dtype(),
                                    num_features=Df)


# ------------------------------------------------------------- forward
def self_attention(layer: dict, x, key_padding_mask=None, mask_mode: Optional[str] = None):
    """One multihead_attention layer on a (B, S, E) device tensor; returns
    the (B, S, E) fp32 output. With key_padding_mask, masking follows the
    graph layer's additive -1e9 rule (graph/sequence.py:162-176); without it,
    the nn/ layer's -inf masks (nn/forward.py:539-543)."""
    import torch
    check_supported(layer)
    B, S, E = x.shape
    H, D = layer["num_heads"], layer["head_dim"]
    Hkv = layer.get("num_kv_heads") or H
    scheme = layer.get("positional_scheme", "absolute")
    if scheme == "rope":
        qkv, rotated = project(x, layer, "qkv", rope_pos0=0)
    else:
        qkv, rotated = project(x, layer, "qkv"), True
    q = split_heads(qkv, H, D, 0)
    k = split_heads(qkv, Hkv, D, H * D)
    v = split_heads(qkv, Hkv, D, H * D + Hkv * D)
    if not rotated:
        apply_rope(q, 0)
        apply_rope(k, 0)
    if layer.get("attention_kernel", "softmax") in LINEAR_KERNELS:
        if key_padding_mask is not None:
            raise ValueError("key_padding_mask is not supported with a linearized "
                             "attention_kernel (it builds no score matrix to mask)")
        ctx = linearized(layer, q, k, v, bool(layer.get("causal", False)))
        return project(ctx.flatten(-2), layer, "o", out_dtype=torch.float32)
    if layer.get("sparse_pattern") is not None:
        if key_padding_mask is not None:
            raise ValueError("key_padding_mask is not supported with sparse_pattern (the "
                             "pattern is the whole mask)")
        ctx = sparse.attention(q, k, v, sparse.normalize_pattern(layer["sparse_pattern"]),
                               causal=bool(layer.get("causal", False)),
                               alibi_slopes=alibi_tensor(H) if scheme == "alibi" else None,
                               out_dtype=compute_dtype())
        return project(ctx.flatten(-2), layer, "o", out_dtype=torch.float32)
    masks = {}
    mode = mask_mode or "exclude"
    if key_padding_mask is not None:
        masks = key_mask_args(key_padding_mask, B, S)
        mode = mask_mode or "additive"
    ctx = kernels.attention_prefill(
        q, k, v, causal=bool(layer.get("causal", False)), window=layer.get("window_size"),
        alibi_slopes=alibi_tensor(H) if scheme == "alibi" else None,
        mask_mode=mode, out_dtype=compute_dtype(), **masks)
    return project(ctx.flatten(-2), layer, "o", out_dtype=torch.float32)


def cross_attention(layer: dict, x, memory, memory_key_padding_mask=None):
    """One cross_attention layer (nn/forward.py:557-591): Q from x (B, Sq, E),
    K/V from memory (B, Skv, E), non-causal. memory_key_padding_mask (True =
    real) applies the graph layer's -1e9 key-padding rule to the memory keys."""
    import torch
    check_supported(layer)
    B, Sq, E = x.shape
    Skv = memory.shape[1]
    H, D = layer["num_heads"], layer["head_dim"]
    Hkv = layer.get("num_kv_heads") or H
    q = split_heads(project(x, layer, "q"), H, D)
    kv = project(memory, layer, "kv")
    k = split_heads(kv, Hkv, D, 0)
    v = split_heads(kv, Hkv, D, Hkv * D)
    masks = {}
    mode = "exclude"
    if memory_key_padding_mask is not None:
        masks = key_mask_args(memory_key_padding_mask, B, Skv)
        mode = "additive"
    ctx = kernels.attention_prefill(q, k, v, causal=False, mask_mode=mode,
                                    out_dtype=compute_dtype(), **masks)
    return project(ctx.flatten(-2), layer, "o", out_dtype=torch.float32)
