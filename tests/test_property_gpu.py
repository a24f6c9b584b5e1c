"""Randomised parity: hypothesis draws shapes and masking options, and K1/K2
must match the float64 oracle on each draw. The search is derandomised (a
fixed example sequence) so that the suite is reproducible.

Drawn for the prefill:
- B, H (with Hkv dividing H), Sq, Skv, head dims 8-128;
- causal, window, per-batch valid lengths and either mask rule;
- ALiBi, position offsets, bf16 or fp32 inputs.

Drawn for the decode: the same head options with the slot range and split
count.

Tolerance: 2e-2 for bf16 inputs, 1e-3 for fp32."""
import numpy as np
import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import HealthCheck, given, settings, strategies as st  # noqa: E402

from oracle import attention_ref as ref  # noqa: E402

pytestmark = pytest.mark.gpu
SETTINGS = settings(max_examples=60, deadline=None, derandomize=True,
                    suppress_health_check=list(HealthCheck))


@st.composite
def prefill_case(draw):
    G = draw(st.sampled_from([1, 2, 4]))
    Hkv = draw(st.integers(1, 3))
    B = draw(st.integers(1, 3))
    D = 8 * draw(st.integers(1, 16))
    causal = draw(st.booleans())
    Sq = draw(st.integers(1, 300))
    Skv = Sq if (causal and draw(st.booleans())) else draw(st.integers(1, 300))
    window = draw(st.one_of(st.none(), st.integers(0, 200)))
    lens = draw(st.one_of(st.none(), st.lists(st.integers(0, Skv), min_size=B, max_size=B)))
    mode = draw(st.sampled_from(["exclude", "additive"]))
    alibi = draw(st.booleans())
    q_pos0 = draw(st.integers(0, 64))
    k_pos0 = draw(st.integers(0, 64)) if draw(st.booleans()) else q_pos0
    fp32 = draw(st.booleans())
    seed = draw(st.integers(0, 10 ** 6))
    return dict(B=B, H=G * Hkv, Hkv=Hkv, D=D, Sq=Sq, Skv=Skv, causal=causal, window=window,
                lens=lens, mode=mode, alibi=alibi, q_pos0=q_pos0, k_pos0=k_pos0, fp32=fp32,
                seed=seed)


@given(case=prefill_case())
@SETTINGS
def test_prefill_matches_oracle(cuda, case):
    import torch
    from enilnets_b200 import _native, kernels
    c = case
    bf16 = not c["fp32"]
    q = ref.seeded_normal(c["seed"], (c["B"], c["Sq"], c["H"], c["D"]), bf16=bf16)
    k = ref.seeded_normal(c["seed"] + 1, (c["B"], c["Skv"], c["Hkv"], c["D"]), bf16=bf16)
    v = ref.seeded_normal(c["seed"] + 2, (c["B"], c["Skv"], c["Hkv"], c["D"]), bf16=bf16)
    dt = torch.float32 if c["fp32"] else torch.bfloat16
    t = lambda a: torch.from_numpy(a.astype(np.float32)).cuda().to(dt)
    slopes = ref.alibi_slopes(c["H"]) if c["alibi"] else None
    out = kernels.attention_prefill(
        t(q), t(k), t(v), causal=c["causal"], window=c["window"],
        kv_valid_len=None if c["lens"] is None else torch.tensor(c["lens"], dtype=torch.int32).cuda(),
        alibi_slopes=None if slopes is None else torch.tensor(slopes, dtype=torch.float32).cuda(),
        q_pos0=c["q_pos0"], k_pos0=c["k_pos0"], mask_mode=c["mode"], out_dtype=torch.float32)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    oref, _ = ref.attention_ref(q, k, v, causal=c["causal"], window=c["window"],
                                kv_valid_len=c["lens"], alibi=slopes, q_pos0=c["q_pos0"],
                                k_pos0=c["k_pos0"], mask_mode=c["mode"])
    o = out.cpu().numpy().astype(np.float64)
    finite = np.isfinite(oref)
    assert np.array_equal(finite, np.isfinite(o)), "NaN pattern differs"
    tol = 1e-3 if c["fp32"] else 2e-2
    if finite.any():
        assert np.max(np.abs(o[finite] - oref[finite])) <= tol


@st.composite
def decode_case(draw):
    G = draw(st.sampled_from([1, 2, 4, 8]))
    Hkv = draw(st.integers(1, 3))
    B = draw(st.integers(1, 4))
    D = 8 * draw(st.integers(1, 16))
    cap = draw(st.integers(1, 2000))
    begin = draw(st.integers(0, cap))
    end = draw(st.integers(begin, cap))
    pos_slot0 = draw(st.integers(0, 100))
    q_pos = draw(st.integers(0, pos_slot0 + cap + 10))
    window = draw(st.one_of(st.none(), st.integers(0, 500)))
    splits = draw(st.sampled_from([0, 1, 3, 7]))
    alibi = draw(st.booleans())
    fp32 = draw(st.booleans())
    seed = draw(st.integers(0, 10 ** 6))
    return dict(B=B, H=G * Hkv, Hkv=Hkv, D=D, cap=cap, begin=begin, end=end,
                pos_slot0=pos_slot0, q_pos=q_pos, window=window, splits=splits, alibi=alibi,
                fp32=fp32, seed=seed)


@given(case=decode_case())
@SETTINGS
def test_decode_matches_oracle(cuda, case):
    import torch
    from enilnets_b200 import _native, kernels
    c = case
    bf16 = not c["fp32"]
    q = ref.seeded_normal(c["seed"], (c["B"], c["H"], c["D"]), bf16=bf16)
    K = ref.seeded_normal(c["seed"] + 1, (c["B"], c["Hkv"], c["cap"], c["D"]), bf16=bf16)
    V = ref.seeded_normal(c["seed"] + 2, (c["B"], c["Hkv"], c["cap"], c["D"]), bf16=bf16)
    dt = torch.float32 if c["fp32"] else torch.bfloat16
    t = lambda a: torch.from_numpy(a.astype(np.float32)).cuda().to(dt)
    slopes = ref.alibi_slopes(c["H"]) if c["alibi"] else None
    o = kernels.attention_decode(
        t(q), t(K), t(V), slot_begin=c["begin"], slot_end=c["end"], pos_slot0=c["pos_slot0"],
        q_pos=c["q_pos"], window=c["window"], n_splits=c["splits"],
        alibi_slopes=None if slopes is None else torch.tensor(slopes, dtype=torch.float32).cuda(),
        out_dtype=torch.float32)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    oref, _ = ref.decode_ref(q, K, V, slot_begin=c["begin"], slot_end=c["end"],
                             pos_slot0=c["pos_slot0"], q_pos=c["q_pos"], window=c["window"],
                             alibi=slopes)
    on = o.cpu().numpy().astype(np.float64)
    finite = np.isfinite(oref)
    assert np.array_equal(finite, np.isfinite(on)), "NaN pattern differs"
    tol = 1e-3 if c["fp32"] else 2e-2
    if finite.any():
        assert np.max(np.abs(on[finite] - oref[finite])) <= tol
