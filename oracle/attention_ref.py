"""CPU float64 oracle for the Enilnets attention inference path.

TEST INFRASTRUCTURE ONLY. Nothing in the product (enilnets_b200/) imports or
calls this module; only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline use it, and only as the checker or the timed CPU baseline.

It restates, in NumPy float64, the reference's algorithms (Enilnets v4.11.0;
paths relative to the reference package):

* plain softmax attention          nn/forward.py:525-551
* streaming ("flash") softmax      nn/flash_attention.py:42-80
* causal / window masks            nn/forward.py:102-117, flash_attention.py:24-39
* ALiBi slopes and bias            nn/forward.py:90-100, :526-535
* RoPE angles and rotation         nn/forward.py:46-55, :80-88
* GQA head mapping                 nn/forward.py:165-171
* additive -1e9 key-padding rule   graph/sequence.py:159-183
* cross attention                  nn/forward.py:557-591
* one-token cached step            nn/kvcache.py:156-213
* KVCache reorder                  nn/kvcache.py:42-66
* attention backward (dQ, dK, dV)  nn/flash_attention.py:83-114

Parity is pinned: tests/test_oracle_golden.py checks every function here
against golden vectors produced by running the reference itself
(tests/golden/make_golden.py).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np

MASK_VALUE = -1e9  # graph/sequence.py:107, nn/flash_attention.py:21
SINUSOIDAL_BASE = 10000.0  # core/constants.py:70


# --------------------------------------------------------------------- bf16
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round to the nearest bfloat16 (ties to even); returns float32 values
    that are exactly representable in bf16. NaN stays NaN."""
    f = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = rounded.view(np.float32).copy()
    out[np.isnan(f)] = np.nan
    return out


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """uint16 bit patterns of bf16_round(x) (the storage NumPy lacks)."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def seeded_normal(seed: int, shape, bf16: bool = True) -> np.ndarray:
    """Seeded N(0,1) activations, bf16-rounded when the path computes in bf16,
    returned as float64 so the oracle measures kernel error only."""
    x = np.random.RandomState(seed).standard_normal(shape).astype(np.float32)
    return (bf16_round(x) if bf16 else x).astype(np.float64)


# ------------------------------------------------------ positional helpers
def alibi_slopes(num_heads: int) -> np.ndarray:
    """Geometric ALiBi slopes, nn/forward.py:90-100."""
    def pow2(n):
        start = 2.0 ** (-8.0 / n)
        return [start ** (i + 1) for i in range(n)]
    if num_heads & (num_heads - 1) == 0:
        return np.array(pow2(num_heads))
    closest = 2 ** int(np.floor(np.log2(num_heads)))
    return np.array(pow2(closest) + pow2(2 * closest)[0::2][: num_heads - closest])


def rope_tables(n_pos: int, head_dim: int, base: float = SINUSOIDAL_BASE):
    """(cos, sin), each (n_pos, head_dim/2), nn/forward.py:46-55."""
    half = head_dim // 2
    theta = base ** (-2.0 * np.arange(half) / head_dim)
    angles = np.arange(n_pos, dtype=np.float64)[:, None] * theta[None, :]
    return np.cos(angles), np.sin(angles)


def rope_rotate(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """rotate_half on the last axis, nn/forward.py:80-88. x (..., S, D) with
    cos/sin (S, D/2)."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], axis=-1)


# ------------------------------------------------------------- attention
def _blocked(q_pos, k_pos, causal, window):
    """Causal/window rule of nn/forward.py:102-117 (True = masked)."""
    diff = q_pos[:, None] - k_pos[None, :]
    blocked = diff < 0 if causal else np.zeros(diff.shape, dtype=bool)
    if window is not None and window >= 0:
        blocked = blocked | (np.abs(diff) > window)
    return blocked


def attention_ref(q, k, v, *, causal=False, window=None, kv_valid_len=None,
                  alibi=None, q_pos0=0, k_pos0=0, mask_mode="exclude",
                  scale=None, key_mask=None) -> Tuple[np.ndarray, np.ndarray]:
    """Softmax attention in float64.

    q (B, Sq, H, D), k/v (B, Skv, Hkv, D); query head h reads kv head
    h // (H // Hkv). Query row i sits at q_pos0 + i, key j at k_pos0 + j.
    mask_mode "exclude": masked scores are -inf (nn/forward.py:539-543).
    mask_mode "additive": padded keys add -1e9, and causal/window violations
    add another -1e9 (graph/sequence.py:162-176).
    key_mask: (B, Skv) bool, True = real key; any pattern (left padding,
    holes), the key_padding_mask of graph/sequence.py:162-168. A key is
    padding when it is masked here or at/after kv_valid_len.
    alibi: (H,) slopes; bias -slope * (i - j) if causal else -slope * |i - j|
    (nn/forward.py:526-535, nn/kvcache.py:199-203).
    Returns (o (B, Sq, H, D), lse (B, H, Sq)).
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    B, Sq, H, D = q.shape
    Skv, Hkv = k.shape[1], k.shape[2]
    rep = H // Hkv
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    q_pos = q_pos0 + np.arange(Sq)
    k_pos = k_pos0 + np.arange(Skv)
    blocked = _blocked(q_pos, k_pos, causal, window)
    dist = q_pos[:, None] - k_pos[None, :]
    dist = dist if causal else np.abs(dist)
    o = np.empty((B, Sq, H, D))
    lse = np.empty((B, H, Sq))
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        for b in range(B):
            L = Skv if kv_valid_len is None else int(np.clip(kv_valid_len[b], 0, Skv))
            pad = np.arange(Skv) >= L
            if key_mask is not None:
                pad = pad | ~np.asarray(key_mask[b], dtype=bool)
            for h in range(H):
                s = (q[b, :, h] @ k[b, :, h // rep].T) * scale
                if alibi is not None:
                    s = s - alibi[h] * dist
                if mask_mode == "additive":
                    s = s + np.where(pad, MASK_VALUE, 0.0)[None, :] + \
                        np.where(blocked, MASK_VALUE, 0.0)
                else:
                    s = np.where(blocked | pad[None, :], -np.inf, s)
                m = np.max(s, axis=-1, keepdims=True)
                e = np.exp(s - m)
                den = np.sum(e, axis=-1, keepdims=True)
                o[b, :, h] = (e @ v[b, :, h // rep]) / den
                lse[b, h] = (m + np.log(den))[:, 0]
    return o, lse


def flash_attention_ref(Qh, Kh, Vh, block_size, causal=False, window=None, slopes=None):
    """Streaming softmax over (B, H, S, D), nn/flash_attention.py:42-80, with
    the -1e9 block bias of nn/flash_attention.py:24-39. Returns (out,
    row_max, row_sum)."""
    B, H, S, Dh = Qh.shape
    scale = 1.0 / np.sqrt(Dh)
    out = np.zeros((B, H, S, Dh))
    row_max = np.full((B, H, S, 1), -np.inf)
    row_sum = np.zeros((B, H, S, 1))
    q_pos = np.arange(S)
    for start in range(0, S, block_size):
        stop = min(start + block_size, S)
        k_pos = np.arange(start, stop)
        scores = np.matmul(Qh, Kh[:, :, start:stop].transpose(0, 1, 3, 2)) * scale
        if causal or window is not None:
            scores = scores + np.where(_blocked(q_pos, k_pos, causal, window),
                                       MASK_VALUE, 0.0)[None, None]
        if slopes is not None:
            diff = q_pos[:, None] - k_pos[None, :]
            scores = scores - slopes[None, :, None, None] * \
                (diff if causal else np.abs(diff))[None, None]
        block_max = np.max(scores, axis=-1, keepdims=True)
        new_max = np.maximum(row_max, block_max)
        rescale = np.exp(row_max - new_max)
        p = np.exp(scores - new_max)
        row_sum = row_sum * rescale + np.sum(p, axis=-1, keepdims=True)
        out = out * rescale + np.matmul(p, Vh[:, :, start:stop])
        row_max = new_max
    return out / row_sum, row_max, row_sum


def attention_backward_ref(q, k, v, dout, *, causal=False, window=None, alibi=None,
                           scale=None):
    """Gradients of attention_ref's output in float64, as
    nn/flash_attention.py:83-114 forms them: P from the -1e9-masked scores,
    dV = P^T dO, dP = dO V^T, dS = P (dP - rowsum(dO * O)) scale,
    dQ = dS K, dK = dS^T Q. q/dout (B, Sq, H, D), k/v (B, Skv, Hkv, D); dK and
    dV of a kv head sum its query heads (the adjoint of the repeat,
    nn/forward.py:165-171). Returns (dq, dk, dv) in the inputs' layouts."""
    q, k, v, dout = (np.asarray(t, np.float64) for t in (q, k, v, dout))
    B, Sq, H, D = q.shape
    Skv, Hkv = k.shape[1], k.shape[2]
    rep = H // Hkv
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    q_pos, k_pos = np.arange(Sq), np.arange(Skv)
    bias = np.where(_blocked(q_pos, k_pos, causal, window), MASK_VALUE, 0.0)
    dist = q_pos[:, None] - k_pos[None, :]
    dist = dist if causal else np.abs(dist)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    for b in range(B):
        for h in range(H):
            kh, vh = k[b, :, h // rep], v[b, :, h // rep]
            s = (q[b, :, h] @ kh.T) * scale + bias
            if alibi is not None:
                s = s - alibi[h] * dist
            e = np.exp(s - s.max(axis=-1, keepdims=True))
            pr = e / e.sum(axis=-1, keepdims=True)
            o = pr @ vh
            g = dout[b, :, h]
            dv[b, :, h // rep] += pr.T @ g
            dp = g @ vh.T
            ds = pr * (dp - np.sum(g * o, axis=-1, keepdims=True)) * scale
            dq[b, :, h] = ds @ kh
            dk[b, :, h // rep] += ds.T @ q[b, :, h]
    return dq, dk, dv


def decode_ref(q, k_cache, v_cache, *, slot_begin, slot_end, pos_slot0, q_pos,
               window=None, alibi=None, scale=None):
    """One query token per (b, h) against cache slots [slot_begin, slot_end),
    nn/kvcache.py:198-213 (causal: keys after q_pos are masked; window:
    |q_pos - k_pos| > window masked). q (B, H, D), caches (B, Hkv, cap, D).
    Returns (o (B, H, D), lse (B, H))."""
    q = np.asarray(q, np.float64)
    B, H, D = q.shape
    Hkv = k_cache.shape[1]
    rep = H // Hkv
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    if slot_end <= slot_begin:  # no key at all: 0/0 output, zero-weight partial
        return np.full((B, H, D), np.nan), np.full((B, H), -np.inf)
    K = np.asarray(k_cache[:, :, slot_begin:slot_end], np.float64)
    V = np.asarray(v_cache[:, :, slot_begin:slot_end], np.float64)
    k_pos = pos_slot0 + np.arange(slot_begin, slot_end)
    blocked = _blocked(np.array([q_pos]), k_pos, True, window)[0]
    o = np.empty((B, H, D))
    lse = np.empty((B, H))
    with np.errstate(invalid="ignore", divide="ignore"):
        for h in range(H):
            s = np.einsum("bd,bsd->bs", q[:, h], K[:, h // rep]) * scale
            if alibi is not None:
                s = s - alibi[h] * (q_pos - k_pos)[None, :]
            s = np.where(blocked[None, :], -np.inf, s)
            m = np.max(s, axis=-1, keepdims=True)
            e = np.exp(s - m)
            den = np.sum(e, axis=-1, keepdims=True)
            o[:, h] = np.einsum("bs,bsd->bd", e, V[:, h // rep]) / den
            # No visible key: lse = -inf (the partial carries no weight in a
            # merge), the output stays NaN like the reference's 0/0.
            lse[:, h] = np.where(np.isneginf(m), -np.inf, m + np.log(den))[:, 0]
    return o, lse


def lse_merge_ref(part_o, part_lse):
    """Merge normalised partials: sum_i w_i o_i / sum_i w_i, w_i = e^{lse_i - max}.
    part_o (P, B, H, D), part_lse (P, B, H). No reference counterpart (the
    reference never splits the key sequence); this is the standard identity."""
    m = np.max(part_lse, axis=0)
    w = np.exp(part_lse - m[None])
    w = np.where(np.isfinite(part_lse), w, 0.0)
    den = np.sum(w, axis=0)
    o = np.einsum("pbh,pbhd->bhd", w, np.where(np.isfinite(part_o), part_o, 0.0)) / den[..., None]
    return o, m + np.log(den)


def kv_append_ref(cache, src, slot0):
    """cache[b, h, slot0 + t] = src[b, t, h]: the effect of the reference's
    concatenate-append (nn/kvcache.py:156-162) on a preallocated buffer."""
    out = np.array(cache, copy=True)
    n = src.shape[1]
    out[:, :, slot0:slot0 + n] = np.transpose(src, (0, 2, 1, 3))
    return out


def kv_gather_ref(src, index):
    """KVCache.reorder's batch-axis gather, nn/kvcache.py:42-61."""
    return np.asarray(src)[np.asarray(index)]


# ----------------------------------------------------------- layer level
def project(x, W, b):
    """x @ W.T + b (nn/forward.py:428-430)."""
    return np.asarray(x, np.float64) @ np.asarray(W, np.float64).T + np.asarray(b, np.float64)


def mha_layer_ref(layer: dict, x: np.ndarray, key_padding_mask: Optional[np.ndarray] = None,
                  mask_mode: Optional[str] = None) -> np.ndarray:
    """Full multi-head self-attention layer in float64: projections, optional
    RoPE/ALiBi, GQA, masks, softmax, context, Wo (nn/forward.py:423-556). With
    key_padding_mask (True = real) the graph path's additive rule applies
    (graph/sequence.py:144-183)."""
    x = np.asarray(x, np.float64)
    B, S, E = x.shape
    H, Dh = layer["num_heads"], layer["head_dim"]
    Hkv = layer.get("num_kv_heads") or H
    Q = project(x, layer["Wq"], layer["bq"]).reshape(B, S, H, Dh)
    K = project(x, layer["Wk"], layer["bk"]).reshape(B, S, Hkv, Dh)
    V = project(x, layer["Wv"], layer["bv"]).reshape(B, S, Hkv, Dh)
    scheme = layer.get("positional_scheme", "absolute")
    if scheme == "rope":
        cos, sin = rope_tables(S, Dh)
        Q = rope_rotate(Q.transpose(0, 2, 1, 3), cos, sin).transpose(0, 2, 1, 3)
        K = rope_rotate(K.transpose(0, 2, 1, 3), cos, sin).transpose(0, 2, 1, 3)
    slopes = alibi_slopes(H) if scheme == "alibi" else None
    mask = None if key_padding_mask is None else np.asarray(key_padding_mask, bool)
    mode = mask_mode or ("additive" if key_padding_mask is not None else "exclude")
    o, _ = attention_ref(Q, K, V, causal=layer.get("causal", False),
                         window=layer.get("window_size"), key_mask=mask, alibi=slopes,
                         mask_mode=mode)
    return project(o.reshape(B, S, H * Dh), layer["Wo"], layer["bo"])


def cross_layer_ref(layer: dict, x: np.ndarray, memory: np.ndarray,
                    memory_valid_len: Optional[np.ndarray] = None,
                    memory_key_mask: Optional[np.ndarray] = None) -> np.ndarray:
    """Cross attention (nn/forward.py:557-591): Q from x, K/V from memory,
    non-causal; memory_valid_len (prefix lengths) or memory_key_mask (any
    boolean (B, Skv) mask, True = real) applies the graph path's -1e9
    key-padding rule (graph/sequence.py:162-168) to the memory keys."""
    x = np.asarray(x, np.float64)
    mem = np.asarray(memory, np.float64)
    B, Sq, E = x.shape
    Skv = mem.shape[1]
    H, Dh = layer["num_heads"], layer["head_dim"]
    Hkv = layer.get("num_kv_heads") or H
    Q = project(x, layer["Wq"], layer["bq"]).reshape(B, Sq, H, Dh)
    K = project(mem, layer["Wk"], layer["bk"]).reshape(B, Skv, Hkv, Dh)
    V = project(mem, layer["Wv"], layer["bv"]).reshape(B, Skv, Hkv, Dh)
    masked = memory_valid_len is not None or memory_key_mask is not None
    o, _ = attention_ref(Q, K, V, kv_valid_len=memory_valid_len, key_mask=memory_key_mask,
                         mask_mode="additive" if masked else "exclude")
    return project(o.reshape(B, Sq, H * Dh), layer["Wo"], layer["bo"])
