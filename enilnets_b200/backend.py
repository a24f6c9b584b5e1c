"""Process-global switches and host<->device plumbing, mirroring the
reference's core/backend.py (use_float64 / default_dtype, core/backend.py:126-141)
and core/utils.py:11 (set_seed).

Weights stay NumPy arrays in the layer dicts, exactly as the reference builds
and saves them (nn/io.py:9-19); this module stages them to the device once
and caches the device copy per array.
"""
from __future__ import annotations

import numpy as np

_STATE = {"float64": False, "precision": "fp32"}
_PRECISIONS = ("fp32", "bf16")


def use_float64(enabled: bool = True) -> None:
    """Default working precision of the NumPy side (weights built, arrays
    returned): float64 when enabled, else float32 (core/backend.py:126-130).
    The device arithmetic is chosen by set_precision."""
    _STATE["float64"] = bool(enabled)


def set_precision(mode: str) -> None:
    """Device arithmetic of the attention layers.

    "fp32" (default, the reference's float32 models): fp32 projection GEMMs,
    attention on the split-bf16 tensor-core path (hi*hi + hi*lo + lo*hi per
    product, about 2^-16 relative error), fp32 KV cache.
    "bf16": bf16 projections, bf16 attention inputs with fp32 accumulation,
    bf16 KV cache: the fast path, max abs error ~1e-2 per attention layer on
    unit-variance activations.
    """
    if mode not in _PRECISIONS:
        raise ValueError(f"precision must be one of {_PRECISIONS}, got {mode!r}")
    _STATE["precision"] = mode


def precision() -> str:
    return _STATE["precision"]


def compute_dtype():
    """torch dtype of projections, attention inputs and the KV cache."""
    import torch
    return torch.float32 if _STATE["precision"] == "fp32" else torch.bfloat16


def is_float64_enabled() -> bool:
    return _STATE["float64"]


def default_dtype():
    return np.float64 if _STATE["float64"] else np.float32


def set_seed(seed: int) -> None:
    """Seed NumPy's legacy global RNG, which the builders draw from in the
    same order as the reference, so the same seed gives the same weights."""
    np.random.seed(seed)


def device():
    """The current CUDA device; raises RuntimeError without one, like the
    reference's use_gpu(True) (core/backend.py:106-113). There is no CPU
    fallback for the attention path."""
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError(
            "No CUDA device is visible: the enilnets_b200 attention path runs only on a "
            "B200 (sm_100a) GPU and has no CPU fallback.")
    return torch.device("cuda", torch.cuda.current_device())


def to_device(x, dtype=None):
    """A CUDA tensor for `x`: NumPy arrays are copied through pinned memory,
    CUDA tensors and __cuda_array_interface__ objects (CuPy) are used in place
    (converted only if `dtype` differs)."""
    import torch
    dev = device()
    if isinstance(x, torch.Tensor):
        t = x if x.is_cuda else x.to(dev, non_blocking=True)
    elif hasattr(x, "__cuda_array_interface__"):
        t = torch.as_tensor(x, device=dev)
    else:
        arr = np.ascontiguousarray(np.asarray(x))
        if arr.dtype == np.float64:
            arr = arr.astype(np.float32)
        t = torch.from_numpy(arr)
        if t.numel() > (1 << 16):
            t = t.pin_memory()
        t = t.to(dev, non_blocking=True)
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t


def to_numpy(t) -> np.ndarray:
    """Host NumPy copy in the default working dtype (core/backend.py:152-157)."""
    return t.detach().float().cpu().numpy().astype(default_dtype(), copy=False)


class WeightCache:
    """Device copies of layer-dict arrays, keyed by the array object: a new
    array assigned into a layer dict is uploaded again; in-place edits of an
    array already uploaded are not seen (call clear() after such edits)."""

    def __init__(self):
        self._store = {}

    def get(self, arr: np.ndarray, dtype, make=None):
        key = (id(arr), dtype, make)
        hit = self._store.get(key)
        if hit is not None and hit[0] is arr:
            return hit[1]
        t = to_device(arr if make is None else make(arr), dtype)
        self._store[key] = (arr, t)
        return t

    def clear(self):
        self._store.clear()


WEIGHTS = WeightCache()
