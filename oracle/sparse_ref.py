"""CPU oracle for block-sparse attention (test infrastructure only).

A float64 NumPy restatement of the reference's block-sparse attention, used
by tests/ to check K1's sparse mode (enilnets_b200/csrc/enl_prefill.cu with
the layouts of enl_sparse.cu). Instead of gathering key blocks it builds the
dense (queries x keys) visibility the pattern implies and runs a masked
softmax over all keys, the equivalence the reference's own test relies on
(test_enilnets.py:8096-8134). Parity is pinned by tests/golden/sparse.npz,
which the reference itself produced (tests/golden/make_golden.py, case
`sparse_cases`).

Reference lines restated:
  block_selection          nn/sparse_attention.py:48-84
  sparse_attention_forward nn/sparse_attention.py:96-142
  cached sparse step       nn/kvcache.py:263-306
"""
from __future__ import annotations

from typing import Dict, List, Optional

import numpy as np


def selection(spec: Dict[str, int], n_blocks: int, causal: bool) -> List[List[int]]:
    """Key blocks of every query block, ascending. One RandomState(seed) draws
    the random extras block after block, from the not yet chosen candidates
    in ascending order (blocks <= i when causal)."""
    rng = np.random.RandomState(spec["seed"])
    out = []
    for i in range(n_blocks):
        near = [i - d for d in range(1, spec["local"] + 1) if i - d >= 0]
        if not causal:
            near += [i + d for d in range(1, spec["local"] + 1) if i + d < n_blocks]
        cand = set([i] + near + list(range(min(spec["global"], n_blocks))))
        if causal:
            cand = {b for b in cand if b <= i}
        if spec["random"] > 0:
            rest = [b for b in range(i + 1 if causal else n_blocks) if b not in cand]
            if rest:
                take = rng.choice(len(rest), size=min(spec["random"], len(rest)), replace=False)
                cand |= {rest[int(t)] for t in np.ravel(take)}
        out.append(sorted(cand))
    return out


def visibility(spec: Dict[str, int], q_pos: np.ndarray, k_pos: np.ndarray, causal: bool,
               n_blocks: int) -> np.ndarray:
    """(len(q_pos), len(k_pos)) bool: key visible to query."""
    bs = spec["block_size"]
    sel = selection(spec, n_blocks, causal)
    allow = np.zeros((len(q_pos), len(k_pos)), dtype=bool)
    kb = np.asarray(k_pos) // bs
    for r, qp in enumerate(q_pos):
        allow[r] = np.isin(kb, sel[int(qp) // bs])
        if causal:
            allow[r] &= np.asarray(k_pos) <= qp
    return allow


def _masked_softmax_av(q, k, v, allow, bias):
    """softmax(q k^T / sqrt(D) + bias, -inf off `allow`) v over (..., S, D)."""
    s = np.einsum("...qd,...kd->...qk", q, k) / np.sqrt(q.shape[-1])
    if bias is not None:
        s = s + bias
    s = np.where(allow, s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    e = np.exp(s)
    return np.einsum("...qk,...kd->...qd", e / e.sum(axis=-1, keepdims=True), v)


def sparse_attention(Qh, Kh, Vh, spec: Dict[str, int], causal: bool,
                     alibi_slopes: Optional[np.ndarray] = None) -> np.ndarray:
    """(B, H, S, D) float64 context of a forward pass: block count
    ceil(S / bs), ALiBi -slope * distance (absolute distance when not
    causal), K/V heads already expanded to H."""
    S = Qh.shape[2]
    bs = spec["block_size"]
    pos = np.arange(S)
    allow = visibility(spec, pos, pos, causal, (S + bs - 1) // bs)
    bias = None
    if alibi_slopes is not None:
        dist = (pos[:, None] - pos[None, :]).astype(np.float64)
        if not causal:
            dist = np.abs(dist)
        bias = -np.asarray(alibi_slopes, np.float64)[:, None, None] * dist[None]
    return _masked_softmax_av(Qh, Kh, Vh, allow, bias)


def sparse_step(Qh, Kh_all, Vh_all, spec: Dict[str, int], q_pos: np.ndarray,
                k_pos: np.ndarray, alibi_slopes: Optional[np.ndarray] = None) -> np.ndarray:
    """(B, H, S_new, D) context of a cached step: causal, block count from the
    last key position, ALiBi by signed distance."""
    bs = spec["block_size"]
    allow = visibility(spec, q_pos, k_pos, True, int(k_pos[-1]) // bs + 1)
    bias = None
    if alibi_slopes is not None:
        dist = (np.asarray(q_pos)[:, None] - np.asarray(k_pos)[None, :]).astype(np.float64)
        bias = -np.asarray(alibi_slopes, np.float64)[:, None, None] * dist[None]
    return _masked_softmax_av(Qh, Kh_all, Vh_all, allow, bias)
