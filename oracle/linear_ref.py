"""CPU oracle for the linearized attention kernels (test infrastructure only).

A float64 NumPy restatement of the reference's linear ("elu+1") and
Performer/FAVOR+ attention, used by tests/ to check the CUDA kernels
(enilnets_b200/csrc/enl_linear.cu). Parity is pinned by
tests/golden/linear_layers.npz, which the reference itself produced
(tests/golden/make_golden.py, case `linear`).

Reference lines restated:
  make_projection          nn/attention_kernels.py:23-35
  performer stabilizer     nn/attention_kernels.py:38-55
  feature_map              nn/attention_kernels.py:58-74
  linear_attention_forward nn/attention_kernels.py:119-143
  cached linear step       nn/kvcache.py:217-260
"""
from __future__ import annotations

import numpy as np


def make_projection(num_features: int, head_dim: int, rng=np.random) -> np.ndarray:
    """Orthogonal random features in blocks of head_dim, rescaled to the norms
    of i.i.d. Gaussian rows. The draws (one randn(head_dim, head_dim) per
    block, then one randn(num_features, head_dim)) come in the reference's
    order, so the same seed gives the same matrix."""
    blocks = []
    for _ in range((num_features + head_dim - 1) // head_dim):
        q, _ = np.linalg.qr(rng.randn(head_dim, head_dim))
        blocks.append(q.T)
    omega = np.concatenate(blocks, axis=0)[:num_features]
    norms = np.linalg.norm(rng.randn(num_features, head_dim), axis=1)
    return omega * norms[:, None]


def performer_proj(x: np.ndarray, omega: np.ndarray) -> np.ndarray:
    """w_f . x' with x' = x / head_dim^(1/4); x (..., S, Dh) -> (..., S, Df)."""
    xs = np.asarray(x, np.float64) / x.shape[-1] ** 0.25
    return xs @ np.asarray(omega, np.float64).T


def performer_stab(x: np.ndarray, omega: np.ndarray, stabilize: str) -> np.ndarray:
    """Row stabilizer (max over features) or global one (max over rows and
    features of each (batch, head)); keepdims like the reference."""
    proj = performer_proj(x, omega)
    axes = -1 if stabilize == "row" else (-2, -1)
    return np.max(proj, axis=axes, keepdims=True)


def feature_map(x: np.ndarray, kernel: str, omega=None, stabilize: str = "row",
                stab=None) -> np.ndarray:
    """phi(x) for x (B, H, S, Dh)."""
    x = np.asarray(x, np.float64)
    if kernel == "linear":
        return np.where(x > 0, x + 1.0, np.exp(np.minimum(x, 0.0)))
    if kernel == "performer":
        xs = x / x.shape[-1] ** 0.25
        proj = xs @ np.asarray(omega, np.float64).T
        sq = np.sum(xs * xs, axis=-1, keepdims=True) / 2.0
        if stab is None:
            axes = -1 if stabilize == "row" else (-2, -1)
            stab = np.max(proj, axis=axes, keepdims=True)
        return np.exp(proj - sq - stab) / np.sqrt(omega.shape[0])
    raise ValueError(f"Unknown attention feature map: {kernel!r}")


def linear_attention(qp: np.ndarray, kp: np.ndarray, v: np.ndarray, causal: bool,
                     kv0=None, ksum0=None, eps: float = 1e-20):
    """out = phi(Q) S_kv / (phi(Q) . s_k + eps) with S_kv = sum phi(k) v^T and
    s_k = sum phi(k), over keys s <= t when causal (prefix sums) or over all
    keys otherwise. qp, kp (B, H, S, Df), v (B, H, S, D). kv0 (B, H, Df, D) /
    ksum0 (B, H, Df) add a carried state to every prefix (causal only).
    Returns (out, kv_end, ksum_end)."""
    qp, kp, v = (np.asarray(a, np.float64) for a in (qp, kp, v))
    if causal:
        kv = np.cumsum(kp[..., :, None] * v[..., None, :], axis=2)
        ks = np.cumsum(kp, axis=2)
        if kv0 is not None:
            kv = kv + np.asarray(kv0, np.float64)[:, :, None]
            ks = ks + np.asarray(ksum0, np.float64)[:, :, None]
        num = np.einsum("bhsf,bhsfd->bhsd", qp, kv)
        den = np.sum(qp * ks, axis=-1, keepdims=True) + eps
        return num / den, kv[:, :, -1], ks[:, :, -1]
    kv = np.swapaxes(kp, -1, -2) @ v
    ks = np.sum(kp, axis=2)
    num = qp @ kv
    den = np.sum(qp * ks[:, :, None, :], axis=-1, keepdims=True) + eps
    return num / den, kv, ks


def linear_step(qh, kh, vh, kernel: str, omega, state=None):
    """One cached step (nn/kvcache.py:217-260) on (B, H, S_new, Dh) arrays whose
    K/V heads are already expanded to H. state = (kv, ksum, stab) or None.
    Returns (context (B, H, S_new, Dh), new_state)."""
    stab = None
    scale = None
    if kernel == "performer":
        stab_new = performer_stab(kh, omega, "global")
        if state is None:
            stab = stab_new
        else:
            stab = np.maximum(state[2], stab_new)
            scale = np.exp(state[2] - stab)[..., 0]         # (B, H, 1)
    qp = feature_map(qh, kernel, omega, "row")
    kp = feature_map(kh, kernel, omega, "global", stab=stab)
    kv0 = ksum0 = None
    if state is not None:
        kv0, ksum0 = state[0], state[1]
        if scale is not None:
            kv0 = kv0 * scale[..., None]
            ksum0 = ksum0 * scale
    out, kv, ks = linear_attention(qp, kp, vh, True, kv0, ksum0)
    return out, (kv, ks, stab)
