"""KV-cache incremental decoding on the B200 kernels.

Same interface as the reference's nn/kvcache.py: `KVCache` (kv / linear /
residual / position, reorder, expand; nn/kvcache.py:23-66) and
`cached_forward_step(model, token_ids, cache, advance_position=True)`
(nn/kvcache.py:69-120), over the same layer dicts.

What changes is where the cache lives and how it grows. The reference keeps
host arrays and re-concatenates the whole cache every step
(nn/kvcache.py:156-162). Here each attention layer owns a preallocated device
buffer pair (B, Hkv, capacity, D) in bf16; a step appends only its new rows
(K3, enl_kv_append) and attends with the split-KV decode kernel (K2) for one
new token or the prefill kernel (K1, causal with position offsets) for a
multi-token step. Sliding-window eviction (nn/kvcache.py:169-180) advances
the start of the live slot range without moving data; the buffer is
compacted or doubled only when it fills.
"""
from __future__ import annotations

from typing import Any, Dict

import numpy as np

from . import attention, kernels, sparse
from .backend import device, to_device, to_numpy
from .network import dense, embed, layernorm, positional_table


class _LayerKV:
    """Device K/V of one attention layer: live slots [begin, end), slot s at
    absolute position base + s."""

    def __init__(self, B: int, Hkv: int, D: int, base: int, need: int, dtype):
        import torch
        cap = max(64, 1 << (max(need, 1) - 1).bit_length())
        self.k = torch.zeros((B, Hkv, cap, D), dtype=dtype, device=device())
        self.v = torch.zeros_like(self.k)
        self.begin = 0
        self.end = 0
        self.base = base

    @property
    def capacity(self) -> int:
        return self.k.shape[2]

    def reserve(self, n_new: int) -> None:
        """Make room for n_new more slots: compact evicted slots away, or
        double the buffer."""
        import torch
        if self.end + n_new <= self.capacity:
            return
        live = self.end - self.begin
        if live + n_new <= self.capacity and self.begin > 0:
            k = self.k[:, :, self.begin:self.end].clone()
            v = self.v[:, :, self.begin:self.end].clone()
            self.k[:, :, :live] = k
            self.v[:, :, :live] = v
        else:
            cap = 1 << (live + n_new - 1).bit_length()
            k = torch.zeros((self.k.shape[0], self.k.shape[1], cap, self.k.shape[3]),
                            dtype=self.k.dtype, device=self.k.device)
            v = torch.zeros_like(k)
            k[:, :, :live] = self.k[:, :, self.begin:self.end]
            v[:, :, :live] = self.v[:, :, self.begin:self.end]
            self.k, self.v = k, v
        self.base += self.begin
        self.end = live
        self.begin = 0

    def view(self):
        """(K, V, start) as the reference stores them: (B, Hkv, S_cached, D)
        views of the live slots and the absolute position of column 0."""
        return (self.k[:, :, self.begin:self.end], self.v[:, :, self.begin:self.end],
                self.base + self.begin)

    def gather(self, index) -> "_LayerKV":
        import torch
        out = _LayerKV.__new__(_LayerKV)
        B_out = index.shape[0]
        out.k = torch.zeros((B_out,) + tuple(self.k.shape[1:]), dtype=self.k.dtype,
                            device=self.k.device)
        out.v = torch.zeros_like(out.k)
        kernels.kv_gather(out.k, self.k, index, self.begin, self.end)
        kernels.kv_gather(out.v, self.v, index, self.begin, self.end)
        out.begin, out.end, out.base = self.begin, self.end, self.base
        return out


class _KVMapping:
    """Read-only mapping layer index -> (K, V, start), like the reference's
    `KVCache.kv` dict."""

    def __init__(self, store: Dict[int, _LayerKV]):
        self._store = store

    def __getitem__(self, idx):
        return self._store[idx].view()

    def __contains__(self, idx):
        return idx in self._store

    def __iter__(self):
        return iter(self._store)

    def __len__(self):
        return len(self._store)

    def keys(self):
        return self._store.keys()

    def items(self):
        return [(k, v.view()) for k, v in self._store.items()]

    def get(self, idx, default=None):
        return self._store[idx].view() if idx in self._store else default


class KVCache:
    """Per-stream decoding state (nn/kvcache.py:23-66): cached K/V per
    attention layer (device-resident), cached residual-save activations, and
    the absolute position of the next token."""

    def __init__(self) -> None:
        self._kv: Dict[int, _LayerKV] = {}
        self.linear: Dict[int, Any] = {}
        self.residual: Dict[int, Any] = {}
        self.position: int = 0

    @property
    def kv(self) -> _KVMapping:
        return _KVMapping(self._kv)

    def __repr__(self) -> str:
        return f"KVCache(position={self.position}, attention_layers={sorted(self._kv)})"

    def reorder(self, index) -> None:
        """Gather every cached tensor along the batch axis by `index`
        (beam search after pruning; nn/kvcache.py:42-61), on the device."""
        import torch
        idx = to_device(np.asarray(index, dtype=np.int64).reshape(-1), torch.int64)
        for key in list(self._kv):
            self._kv[key] = self._kv[key].gather(idx)
        for key in list(self.residual):
            self.residual[key] = self.residual[key].index_select(0, idx)
        for key in list(self.linear):
            self.linear[key] = tuple(None if t is None else t.index_select(0, idx)
                                     for t in self.linear[key])

    def expand(self, size: int) -> None:
        """Replicate a batch-1 cache to `size` rows (nn/kvcache.py:63-66)."""
        self.reorder([0] * int(size))


def attention_step(layer: Dict[str, Any], x, idx: int, cache: KVCache, B: int, S_new: int,
                   pos: int):
    """One attention layer's cached step (nn/kvcache.py:123-214): project the
    new tokens, append their K/V, attend over cached + new. Raises if the
    layer is non-causal, as the reference does."""
    import torch
    if not layer.get("causal", False):
        raise ValueError(
            f"KV-cache stepping requires causal attention; layer {idx} is non-causal (its full "
            "output at earlier positions would change when later tokens arrive, which a cache "
            "cannot represent).")
    attention.check_supported(layer)
    H, D = layer["num_heads"], layer["head_dim"]
    Hkv = layer.get("num_kv_heads") or H
    scheme = layer.get("positional_scheme", "absolute")
    window = layer.get("window_size")
    if scheme == "rope":
        # Rotated at absolute positions in the projection's epilogue; the
        # cache stores rotated K.
        qkv, rotated = attention.project(x, layer, "qkv", rope_pos0=pos)
    else:
        qkv, rotated = attention.project(x, layer, "qkv"), True
    q = attention.split_heads(qkv, H, D, 0)
    k_new = attention.split_heads(qkv, Hkv, D, H * D)
    v_new = attention.split_heads(qkv, Hkv, D, H * D + Hkv * D)
    if not rotated:
        attention.apply_rope(q, pos)
        attention.apply_rope(k_new, pos)
    if layer.get("attention_kernel", "softmax") in attention.LINEAR_KERNELS:
        return _linear_step(layer, q, k_new, v_new, idx, cache)
    lc = cache._kv.get(idx)
    if lc is None:
        lc = _LayerKV(B, Hkv, D, base=pos, need=S_new, dtype=qkv.dtype)
        cache._kv[idx] = lc
    elif lc.k.dtype != qkv.dtype:
        raise ValueError(f"the cache of layer {idx} holds {lc.k.dtype} K/V but the precision is "
                         f"now {qkv.dtype}; start a new KVCache after set_precision")
    lc.reserve(S_new)
    kernels.kv_append(lc.k, k_new, lc.end)
    kernels.kv_append(lc.v, v_new, lc.end)
    lc.end += S_new
    if window is not None:
        # Keep what the OLDEST query of this step still needs (nn/kvcache.py:171-180).
        drop = max(0, (pos - window) - (lc.base + lc.begin))
        lc.begin = min(lc.begin + drop, lc.end)
    slopes = attention.alibi_tensor(H) if scheme == "alibi" else None
    spec = layer.get("sparse_pattern")
    if spec is not None:
        # Block-sparse step (nn/kvcache.py:263-306): K1's sparse mode at the
        # step's absolute positions, for one new token or several; the cache
        # keeps every key since any earlier block may be selected.
        kv_k = lc.k[:, :, lc.begin:lc.end].permute(0, 2, 1, 3)
        kv_v = lc.v[:, :, lc.begin:lc.end].permute(0, 2, 1, 3)
        ctx = sparse.attention(q, kv_k, kv_v, sparse.normalize_pattern(spec), causal=True,
                               alibi_slopes=slopes, q_pos0=pos, k_pos0=lc.base + lc.begin,
                               out_dtype=qkv.dtype)
    elif S_new == 1:
        ctx = kernels.attention_decode(q[:, 0], lc.k, lc.v, slot_begin=lc.begin,
                                       slot_end=lc.end, pos_slot0=lc.base, q_pos=pos,
                                       window=window, alibi_slopes=slopes,
                                       out_dtype=qkv.dtype).unsqueeze(1)
    else:
        kv_k = lc.k[:, :, lc.begin:lc.end].permute(0, 2, 1, 3)
        kv_v = lc.v[:, :, lc.begin:lc.end].permute(0, 2, 1, 3)
        ctx = kernels.attention_prefill(q, kv_k, kv_v, causal=True, window=window,
                                        alibi_slopes=slopes, q_pos0=pos,
                                        k_pos0=lc.base + lc.begin, out_dtype=qkv.dtype)
    return attention.project(ctx.flatten(-2), layer, "o", out_dtype=torch.float32)


def _linear_step(layer: Dict[str, Any], q, k_new, v_new, idx: int, cache: KVCache):
    """Cached step of a linearized layer (nn/kvcache.py:217-260): causal
    linear attention is a linear RNN, so the whole history is the running
    sums sum phi(k) v^T and sum phi(k), kept on the device in cache.linear[idx]
    as (kv (B, Hkv, Df, D), ksum (B, Hkv, Df), stabilizer (B, Hkv) or None).
    Performer keys share one stabilizer across steps: the larger of the
    carried one and this step's, with the carried sums scaled down by
    exp(old - new) (the ratio is scale-invariant)."""
    import torch
    kernel = layer["attention_kernel"]
    prev = cache.linear.get(idx)
    omega = attention.omega_tensor(layer) if kernel == "performer" else None
    scale = None
    stab = None
    if kernel == "performer":
        floor = prev[2] if prev is not None else None
        kp, stab = kernels.linear_feature_map(k_new, kernel, omega, global_stab=True,
                                              stab_floor=floor)
        if prev is not None:
            scale = torch.exp(prev[2] - stab)
    else:
        kp, _ = kernels.linear_feature_map(k_new, kernel)
    qp, _ = kernels.linear_feature_map(q, kernel, omega)
    ctx, (kv, ksum) = kernels.linear_attention(
        qp, kp, v_new, causal=True, state=None if prev is None else (prev[0], prev[1]),
        state_scale=scale, return_state=True, out_dtype=q.dtype)
    cache.linear[idx] = (kv, ksum, stab)
    return attention.project(ctx.flatten(-2), layer, "o", out_dtype=torch.float32)


def cached_forward_step_device(model: Any, token_ids, cache: KVCache,
                               advance_position: bool = True):
    """cached_forward_step without the final device->host copy."""
    x = np.asarray(token_ids)
    if x.ndim == 1:
        x = x[None, :]
    B, S_new = int(x.shape[0]), int(x.shape[1])
    pos = cache.position
    for idx, layer in enumerate(model.layers):
        t = layer["type"]
        if t == "embedding":
            x = embed(x, layer)
        elif t == "positional_encoding":
            table = positional_table(layer)
            if pos + S_new > table.shape[0]:
                raise ValueError(f"positions {pos}..{pos + S_new - 1} exceed the positional "
                                 f"table ({table.shape[0]} rows) of layer {idx}")
            x = x + table[pos:pos + S_new][None]
        elif t == "layernorm":
            x = layernorm(x, layer)
        elif t in ("dense", "sparse"):
            x = dense(x, layer)
        elif t == "dropout":
            pass                                        # inference no-op
        elif t == "residual_save":
            cache.residual[idx] = x
        elif t == "residual_add":
            x = x + cache.residual[layer["save_index"]]
        elif t == "multihead_attention":
            x = attention_step(layer, x, idx, cache, B, S_new, pos)
        else:
            raise ValueError(
                f"KV-cache stepping doesn't support layer type '{t}' (layer {idx}); use a full "
                "Forward() for this architecture.")
    if advance_position:
        cache.position += S_new
    return x


def cached_forward_step(model: Any, token_ids, cache: KVCache,
                        advance_position: bool = True) -> np.ndarray:
    """Step `token_ids` ((batch, n_new) ints, or (n_new,) as batch 1) through
    `model`'s layers, reading and updating `cache`; returns the new positions'
    outputs (batch, n_new, out_dim) as a NumPy array (nn/kvcache.py:69-120)."""
    return to_numpy(cached_forward_step_device(model, token_ids, cache, advance_position))
