"""The attention-backward oracle against the reference's own
flash_attention_backward outputs (tests/golden/flash_backward.npz, made by
the reference, nn/flash_attention.py:83-114), plus a GQA property: with the
kv heads repeated, the summed group gradients equal the per-head ones."""
import json

import numpy as np

from oracle import attention_ref as ar


def _inputs(i, c):
    rs = np.random.RandomState(4000 + i)
    shape = (c["B"], c["H"], c["S"], c["Dh"])
    return [rs.standard_normal(shape).transpose(0, 2, 1, 3) for _ in range(4)]


def test_backward_oracle_matches_reference(golden_dir):
    data = np.load(golden_dir / "flash_backward.npz")
    meta = json.loads(str(data["meta"]))
    for i, c in enumerate(meta):
        q, k, v, do = _inputs(i, c)
        slopes = ar.alibi_slopes(c["H"]) if c["alibi"] else None
        dq, dk, dv = ar.attention_backward_ref(q, k, v, do, causal=c["causal"],
                                               window=c["window"], alibi=slopes)
        for name, got in (("dq", dq), ("dk", dk), ("dv", dv)):
            ref = data[f"{name}{i}"].transpose(0, 2, 1, 3)
            assert np.max(np.abs(got - ref)) <= 1e-5 * max(1.0, np.abs(ref).max()), (c, name)


def test_backward_oracle_gqa_sums_the_group():
    rs = np.random.RandomState(3)
    B, S, H, Hkv, D = 1, 20, 4, 2, 8
    q = rs.standard_normal((B, S, H, D))
    k = rs.standard_normal((B, S, Hkv, D))
    v = rs.standard_normal((B, S, Hkv, D))
    do = rs.standard_normal((B, S, H, D))
    dq, dk, dv = ar.attention_backward_ref(q, k, v, do, causal=True)
    kr, vr = np.repeat(k, 2, axis=2), np.repeat(v, 2, axis=2)
    dq2, dk2, dv2 = ar.attention_backward_ref(q, kr, vr, do, causal=True)
    assert np.allclose(dq, dq2)
    assert np.allclose(dk, dk2.reshape(B, S, Hkv, 2, D).sum(axis=3))
    assert np.allclose(dv, dv2.reshape(B, S, Hkv, 2, D).sum(axis=3))
