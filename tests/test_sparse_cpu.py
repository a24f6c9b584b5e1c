"""Block-sparse attention host logic and oracle, on the CPU.

- The oracle (oracle/sparse_ref.py) and the product's pattern code
  (enilnets_b200/sparse.py) reproduce the reference's block_selection tables
  and forward outputs (tests/golden/sparse.npz, made by the reference).
- The tile plan lists every (query, key) pair the pattern allows, and its
  pair count is the oracle's.
- Pattern validation raises the reference's errors (test_enilnets.py:8207-8226).
"""
import json

import numpy as np
import pytest

from enilnets_b200 import sparse as sp
from oracle import sparse_ref as sr


@pytest.fixture(scope="module")
def golden(golden_dir):
    data = np.load(golden_dir / "sparse.npz")
    return data, json.loads(str(data["meta"]))


def test_selection_tables_match_reference(golden):
    data, meta = golden
    for i, (pat, nb, causal) in enumerate(meta["sel"]):
        spec = sp.normalize_pattern(pat)
        index, valid = sp.block_selection(spec, nb, causal)
        assert np.array_equal(index, data[f"sel{i}_index"]), (pat, nb, causal)
        assert np.array_equal(valid, data[f"sel{i}_valid"]), (pat, nb, causal)
        rows = sr.selection(spec, nb, causal)
        ref_rows = [sorted(int(x) for x, v in zip(ix, vl) if v)
                    for ix, vl in zip(data[f"sel{i}_index"], data[f"sel{i}_valid"])]
        assert rows == ref_rows


def test_causal_selection_is_prefix_stable():
    """A causal block's selection does not depend on how many blocks follow
    (test_enilnets.py:8239-8250); the cached selector extends in place."""
    spec = sp.normalize_pattern({"block_size": 2, "local": 1, "global": 1, "random": 1})
    small = sp.block_selection(spec, 4, True)
    large = sp.block_selection(spec, 9, True)
    again = sp.block_selection(spec, 4, True)
    for i in range(4):
        a = sorted(int(x) for x, v in zip(small[0][i], small[1][i]) if v)
        b = sorted(int(x) for x, v in zip(large[0][i], large[1][i]) if v)
        assert a == b
    assert np.array_equal(small[0], again[0])
    assert sr.selection(spec, 9, True)[:4] == sr.selection(spec, 4, True)


def test_oracle_matches_reference_forward(golden):
    data, meta = golden
    for i, c in enumerate(meta["core"]):
        rs = np.random.RandomState(3100 + i)
        shape = (c["B"], c["H"], c["S"], c["Dh"])
        q, k, v = (rs.standard_normal(shape) for _ in range(3))
        from oracle.attention_ref import alibi_slopes
        slopes = alibi_slopes(c["H"]) if c["alibi"] else None
        out = sr.sparse_attention(q, k, v, sp.normalize_pattern(c["pattern"]), c["causal"],
                                  slopes)
        assert np.max(np.abs(out - data[f"core{i}_y"])) < 1e-6, c


def test_oracle_step_equals_forward_rows():
    """A cached step at positions [p, p + n) over keys [0, p + n) gives the
    forward pass's rows p .. p + n - 1 (causal)."""
    rs = np.random.RandomState(5)
    spec = sp.normalize_pattern({"block_size": 3, "local": 1, "global": 1, "random": 1})
    q, k, v = (rs.standard_normal((1, 2, 14, 8)) for _ in range(3))
    full = sr.sparse_attention(q, k, v, spec, True)
    for p, n in ((0, 1), (5, 1), (9, 5), (13, 1)):
        step = sr.sparse_step(q[:, :, p:p + n], k[:, :, :p + n], v[:, :, :p + n], spec,
                              np.arange(p, p + n), np.arange(p + n))
        assert np.allclose(step, full[:, :, p:p + n], atol=1e-12)


CASES = [
    ({"block_size": 3, "local": 1, "global": 1, "random": 1}, 10, 10, 0, 0, False),
    ({"block_size": 16, "local": 2, "global": 1, "random": 2, "seed": 4}, 300, 300, 0, 0, False),
    ({"block_size": 64, "local": 1, "global": 1}, 700, 700, 0, 0, True),
    ({"block_size": 100, "local": 1, "random": 1}, 333, 333, 0, 0, True),
    ({"block_size": 1, "local": 5, "global": 2}, 200, 200, 0, 0, True),
    ({"block_size": 256, "local": 1}, 600, 600, 0, 0, True),
    ({"block_size": 3, "local": 1, "global": 1, "random": 1}, 1, 9, 8, 0, True),   # one-token step
    ({"block_size": 4, "local": 1, "random": 2, "seed": 9}, 4, 9, 5, 0, True),      # multi-token
    ({"block_size": 8, "local": 1, "global": 1}, 3, 40, 200, 163, True),            # cache from 163
]


@pytest.mark.parametrize("pat,Sq,Skv,q0,k0,causal", CASES)
def test_tile_plan_covers_exactly_the_allowed_pairs(pat, Sq, Skv, q0, k0, causal):
    spec = sp.normalize_pattern(pat)
    plan = sp.plan_tiles(spec, Sq, Skv, causal=causal, q_pos0=q0, k_pos0=k0)
    q_pos, k_pos = np.arange(q0, q0 + Sq), np.arange(k0, k0 + Skv)
    n_blocks = (k0 + Skv - 1) // spec["block_size"] + 1
    allow = sr.visibility(spec, q_pos, k_pos, causal, n_blocks)
    assert plan.pairs == int(allow.sum())
    assert plan.tile_ptr[0] == 0 and plan.tile_ptr[-1] == plan.tile_kt.size
    assert plan.tile_ptr.size == (Sq + 127) // 128 + 1
    for t in range(plan.tile_ptr.size - 1):
        kts = plan.tile_kt[plan.tile_ptr[t]:plan.tile_ptr[t + 1]]
        assert list(kts) == sorted(set(kts.tolist()))
        rows = allow[t * 128:(t + 1) * 128]
        needed = sorted(set((np.nonzero(rows.any(axis=0))[0] // 128).tolist()))
        assert list(kts) == needed  # every listed tile is used, every used tile listed


def test_every_query_sees_its_own_key():
    spec = sp.normalize_pattern({"block_size": 4, "local": 1, "global": 1})
    allow = sr.visibility(spec, np.arange(40), np.arange(40), True, 10)
    assert allow.diagonal().all() and allow.mean() < 0.35
    assert allow[4:, :4].all()


@pytest.mark.parametrize("bad", [{}, {"block_size": 0}, {"block_size": 4, "local": -1},
                                 {"block_size": 4, "local": 0, "global": 0, "random": 0},
                                 {"block_size": 4, "bogus": 1}, "not-a-dict"])
def test_invalid_patterns_rejected(bad):
    with pytest.raises(ValueError):
        sp.normalize_pattern(bad)


def test_normalized_pattern_defaults():
    assert sp.normalize_pattern({"block_size": 16}) == {
        "local": 1, "global": 0, "random": 0, "seed": 0, "block_size": 16}
