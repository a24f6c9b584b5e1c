"""Block-sparse attention patterns (nn/sparse_attention.py) on the K1 kernel.

The reference gathers, per query block, the key blocks its pattern selects
(local neighbours, leading global blocks, seeded random extras) and runs a
dense softmax over the gather (nn/sparse_attention.py:96-142). Here the
selection stays the reference's (same pattern contract, same seeded draws,
so layers built and saved by the reference attend to the same keys), and the
gather becomes a layout K1 walks directly:

- per 128-row query tile, the sorted 128-key tiles any of its rows needs
  (built here on the host, a few integers per tile);
- per (entry, tile half, row), a 64-bit mask of the keys that row may see
  (filled on the device by ``enl_sparse_build_masks``), which also carries
  the causal rule and the sequence end (:130-134).

Layouts depend only on the pattern, the lengths and the positions, so they
are cached and reused across layers, heads and calls.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Any, Dict, List, NamedTuple, Optional, Tuple

import numpy as np
import torch

from . import _native as nat

_KEYS = ("block_size", "local", "global", "random", "seed")


def normalize_pattern(pattern: Any) -> Dict[str, int]:
    """The reference's pattern contract (nn/sparse_attention.py:23-45): a dict
    with a required ``block_size`` >= 1 and optional ``local`` (1), ``global``
    (0), ``random`` (0), ``seed`` (0); ValueError otherwise, with its messages."""
    if not isinstance(pattern, dict):
        raise ValueError("sparse_pattern must be a dict, e.g. "
                         "{'block_size': 16, 'local': 1, 'global': 1, 'random': 2}")
    extra = sorted(set(pattern) - set(_KEYS))
    if extra:
        raise ValueError(f"Unknown sparse_pattern keys: {extra}")
    spec = {"local": 1, "global": 0, "random": 0, "seed": 0}
    spec.update(pattern)
    if "block_size" not in pattern or int(spec["block_size"]) < 1:
        raise ValueError("sparse_pattern needs a block_size >= 1")
    for key in ("local", "global", "random"):
        if int(spec[key]) < 0:
            raise ValueError(f"sparse_pattern['{key}'] must be >= 0")
    if not (spec["local"] or spec["global"] or spec["random"]):
        raise ValueError(
            "sparse_pattern selects no blocks at all (local/global/random are all 0), which "
            "would leave every query with nothing to attend to.")
    return {k: int(spec[k]) for k in spec}


def _spec_key(spec: Dict[str, int]) -> Tuple[int, ...]:
    return tuple(int(spec[k]) for k in _KEYS)


class _Selector:
    """Per-block key-block sets of one pattern, in the reference's draw order
    (nn/sparse_attention.py:57-75): block i takes itself, its `local`
    neighbours (both sides unless causal), the first `global` blocks, drops
    later blocks when causal, then `random` distinct extras drawn from the
    remaining candidates in ascending order with one RandomState(seed) shared
    by all blocks in turn. Under a causal mask block i's set does not depend
    on how many blocks follow, so the causal selector keeps its generator and
    extends the table as sequences grow."""

    def __init__(self, spec: Dict[str, int], n_blocks: int, causal: bool):
        self.spec, self.causal, self.n_blocks = spec, causal, n_blocks
        self.rng = np.random.RandomState(spec["seed"])
        self.rows: List[List[int]] = []

    def extend(self, n: int) -> None:
        sp, causal = self.spec, self.causal
        while len(self.rows) < n:
            i = len(self.rows)
            picked = {i}
            for d in range(1, sp["local"] + 1):
                if i - d >= 0:
                    picked.add(i - d)
                if not causal and i + d < self.n_blocks:
                    picked.add(i + d)
            picked.update(range(min(sp["global"], self.n_blocks)))
            if causal:
                picked = {b for b in picked if b <= i}
            if sp["random"]:
                limit = i + 1 if causal else self.n_blocks
                free = [b for b in range(limit) if b not in picked]
                if free:
                    draw = self.rng.choice(len(free), size=min(sp["random"], len(free)),
                                           replace=False)
                    picked.update(free[int(x)] for x in np.asarray(draw).reshape(-1))
            self.rows.append(sorted(picked))


_selectors: "OrderedDict[tuple, _Selector]" = OrderedDict()


def _selection_rows(spec: Dict[str, int], n_blocks: int, causal: bool) -> List[List[int]]:
    """Rows 0..n_blocks-1 of the selection (cached per pattern)."""
    # Causal rows never look past their own block (the clip of the global
    # range to n_blocks, :66, removes only blocks > i), so one selector serves
    # every length; non-causal tables depend on n_blocks through the right
    # neighbours and the random pool.
    key = (_spec_key(spec), causal, -1 if causal else n_blocks)
    sel = _selectors.get(key)
    if sel is None:
        sel = _Selector(spec, (1 << 62) if causal else n_blocks, causal)
        _selectors[key] = sel
        while len(_selectors) > 64:
            _selectors.popitem(last=False)
    else:
        _selectors.move_to_end(key)
    sel.extend(n_blocks)
    return sel.rows[:n_blocks]


def block_selection(spec: Dict[str, int], n_blocks: int, causal: bool) -> Tuple[Any, Any]:
    """(index, valid), both (n_blocks, width), as nn/sparse_attention.py:48-84
    returns them: row i lists block i's key blocks in ascending order, padded
    with i where `valid` is False."""
    rows = _selection_rows(spec, n_blocks, causal)
    width = max(len(r) for r in rows)
    index = np.repeat(np.arange(n_blocks, dtype=np.int64)[:, None], width, axis=1)
    valid = np.zeros((n_blocks, width), dtype=bool)
    for i, r in enumerate(rows):
        index[i, :len(r)] = r
        valid[i, :len(r)] = True
    return index, valid


class SparseLayout:
    """K1's view of a pattern for one (seq_q, seq_kv, q_pos0, k_pos0): device
    int32 tile_ptr (n_qtiles + 1), int32 tile_kt (n_entries), int64 masks
    (n_entries, 2, 128); `pairs` is the number of (query, key) pairs the
    pattern allows (the attention's useful work)."""

    def __init__(self, tile_ptr, tile_kt, masks, *, n_entries: int, seq_q: int, seq_kv: int,
                 q_pos0: int, k_pos0: int, pairs: int):
        self.tile_ptr, self.tile_kt, self.masks = tile_ptr, tile_kt, masks
        self.n_entries = n_entries
        self.seq_q, self.seq_kv, self.q_pos0, self.k_pos0 = seq_q, seq_kv, q_pos0, k_pos0
        self.pairs = pairs

    def native(self) -> nat.SparseLayout:
        lay = nat.SparseLayout()
        lay.tile_ptr, lay.tile_kt = self.tile_ptr.data_ptr(), self.tile_kt.data_ptr()
        lay.masks, lay.n_entries = self.masks.data_ptr(), self.n_entries
        return lay


def _pairs(qlo: int, qhi: int, klo: int, khi: int, causal: bool) -> int:
    """Allowed (q, k) pairs for query positions [qlo, qhi] and key positions
    [klo, khi] (empty ranges give 0)."""
    if qhi < qlo or khi < klo:
        return 0
    width = khi - klo + 1
    if not causal:
        return (qhi - qlo + 1) * width
    # row q sees keys [klo, min(khi, q)]
    a, b = max(qlo, klo), min(qhi, khi)
    ramp = (b - a + 1) * (a - klo + 1 + b - klo + 1) // 2 if b >= a else 0
    flat = max(0, qhi - max(qlo, khi + 1) + 1) * width
    return ramp + flat


class TilePlan(NamedTuple):
    """Host half of a layout: the selection of the query blocks in range as a
    CSR (sel_ptr, sel_kb over blocks qb0 ..), the key tiles of every query
    tile (tile_ptr, tile_kt) and the number of allowed (query, key) pairs."""
    qb0: int
    sel_ptr: np.ndarray
    sel_kb: np.ndarray
    tile_ptr: np.ndarray
    tile_kt: np.ndarray
    pairs: int


def plan_tiles(spec: Dict[str, int], seq_q: int, seq_kv: int, *, causal: bool,
               q_pos0: int = 0, k_pos0: int = 0) -> TilePlan:
    """Key tiles for query positions [q_pos0, q_pos0 + seq_q) against keys at
    [k_pos0, k_pos0 + seq_kv). The block count is the one the reference
    derives: ceil(S / bs) for a forward pass (nn/sparse_attention.py:104) and
    last key position // bs + 1 for a cached step (nn/kvcache.py:275), which
    are the same number. A tile is listed when at least one of the query
    tile's rows may see one of its keys."""
    bs = spec["block_size"]
    n_blocks = (k_pos0 + seq_kv - 1) // bs + 1
    qb0 = q_pos0 // bs
    qb1 = (q_pos0 + seq_q - 1) // bs
    if not causal and qb1 >= n_blocks:
        raise ValueError(f"non-causal sparse attention needs the queries inside the keys' "
                         f"{n_blocks} blocks (query block {qb1})")
    sel = _selection_rows(spec, max(n_blocks, qb1 + 1), causal)[qb0:qb1 + 1]
    sel_ptr = np.zeros(len(sel) + 1, dtype=np.int32)
    sel_ptr[1:] = np.cumsum([len(r) for r in sel])
    sel_kb = np.asarray([kb for r in sel for kb in r], dtype=np.int32)

    n_qt = (seq_q + 127) // 128
    tile_ptr = np.zeros(n_qt + 1, dtype=np.int32)
    tiles: List[int] = []
    pairs = 0
    for t in range(n_qt):
        p_lo = q_pos0 + t * 128
        p_hi = q_pos0 + min(seq_q, t * 128 + 128) - 1
        need = set()
        for qb in range(p_lo // bs, p_hi // bs + 1):
            rq_lo, rq_hi = max(qb * bs, p_lo), min(qb * bs + bs - 1, p_hi)
            for kb in sel[qb - qb0]:
                j_lo = max(kb * bs - k_pos0, 0)
                j_hi = min(kb * bs + bs - 1 - k_pos0, seq_kv - 1)
                if causal:
                    j_hi = min(j_hi, rq_hi - k_pos0)
                if j_hi < j_lo:
                    continue
                need.update(range(j_lo // 128, j_hi // 128 + 1))
                pairs += _pairs(rq_lo, rq_hi, j_lo + k_pos0, j_hi + k_pos0, causal)
        tiles.extend(sorted(need))
        tile_ptr[t + 1] = len(tiles)
    return TilePlan(qb0, sel_ptr, sel_kb, tile_ptr, np.asarray(tiles, dtype=np.int32), pairs)


_layouts: "OrderedDict[tuple, SparseLayout]" = OrderedDict()


def build_layout(spec: Dict[str, int], seq_q: int, seq_kv: int, *, causal: bool,
                 device: torch.device, q_pos0: int = 0, k_pos0: int = 0) -> SparseLayout:
    """plan_tiles on the host, then the column masks on the device
    (enl_sparse_build_masks). Cached per (pattern, lengths, positions,
    causal, device)."""
    from . import kernels
    device = torch.device(device)
    key = (_spec_key(spec), seq_q, seq_kv, q_pos0, k_pos0, bool(causal), str(device))
    lay = _layouts.get(key)
    if lay is not None:
        _layouts.move_to_end(key)
        return lay
    plan = plan_tiles(spec, seq_q, seq_kv, causal=causal, q_pos0=q_pos0, k_pos0=k_pos0)
    # At least one (unused) element keeps every device pointer non-null.
    n_entries, n_sel = plan.tile_kt.size, plan.sel_kb.size
    dev_i32 = dict(dtype=torch.int32, device=device)
    t_ptr = torch.as_tensor(plan.tile_ptr, **dev_i32)
    t_kt = torch.as_tensor(plan.tile_kt if n_entries else np.zeros(1, np.int32), **dev_i32)
    masks = torch.zeros((max(n_entries, 1), 2, 128), dtype=torch.int64, device=device)
    s_ptr = torch.as_tensor(plan.sel_ptr, **dev_i32)
    s_kb = torch.as_tensor(plan.sel_kb if n_sel else np.zeros(1, np.int32), **dev_i32)
    if n_entries:
        kernels.sparse_build_masks(t_ptr, t_kt[:n_entries], masks[:n_entries], s_ptr,
                                   s_kb[:n_sel], qb0=plan.qb0, block_size=spec["block_size"],
                                   seq_q=seq_q, seq_kv=seq_kv, q_pos0=q_pos0, k_pos0=k_pos0,
                                   causal=causal)
    lay = SparseLayout(t_ptr, t_kt, masks, n_entries=n_entries, seq_q=seq_q, seq_kv=seq_kv,
                       q_pos0=q_pos0, k_pos0=k_pos0, pairs=plan.pairs)
    _layouts[key] = lay
    while len(_layouts) > 32:
        _layouts.popitem(last=False)
    return lay


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, spec: Dict[str, int], *,
              causal: bool, alibi_slopes: Optional[torch.Tensor] = None, q_pos0: int = 0,
              k_pos0: int = 0, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Block-sparse attention on (B, S, H, D) device views through K1
    (nn/sparse_attention.py:96-142; with positions, the scores of
    nn/kvcache.py:263-306). Scale 1/sqrt(D), ALiBi signed when causal and
    absolute otherwise."""
    from . import kernels
    lay = build_layout(spec, q.shape[1], k.shape[1], causal=causal, device=q.device,
                       q_pos0=q_pos0, k_pos0=k_pos0)
    return kernels.attention_prefill(q, k, v, causal=causal, alibi_slopes=alibi_slopes,
                                     q_pos0=q_pos0, k_pos0=k_pos0, out_dtype=out_dtype,
                                     sparse=lay)
