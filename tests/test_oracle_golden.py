"""Pin the CPU oracle to the reference: every oracle function must reproduce
the golden vectors that tests/golden/make_golden.py produced by running the
reference itself (float64). CPU only."""
import json

import numpy as np
import pytest

from oracle import attention_ref as ref


def _load(golden_dir, name):
    data = np.load(golden_dir / name)
    return data, json.loads(str(data["meta"]))


def _layer(data, i, **cfg):
    layer = {k: data[f"{k}{i}"] for k in ("Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo")}
    H = cfg["num_heads"]
    E = cfg["embed_dim"]
    layer.update(num_heads=H, head_dim=E // H, embed_dim=E,
                 num_kv_heads=cfg.get("num_kv_heads") or H,
                 causal=cfg.get("causal", False), window_size=cfg.get("window_size"),
                 positional_scheme=cfg.get("positional_scheme", "absolute"))
    return layer


def test_bf16_round_is_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.005859375, 1.0078125, -2.5, 3.0e38, np.inf, 0.0],
                 np.float32)
    r = ref.bf16_round(x)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7 -> even (1.0); 1 + 1.5*2^-8 rounds up.
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == np.float32(1.0078125)
    assert r[3] == np.float32(1.0078125) and r[4] == -2.5 and r[6] == np.inf
    assert np.all((r.view(np.uint32) & 0xFFFF) == 0)
    assert np.isnan(ref.bf16_round(np.array([np.nan], np.float32)))[0]


def test_alibi_slopes_match_published_geometric_sequence():
    assert np.allclose(ref.alibi_slopes(8), [2.0 ** (-(i + 1)) for i in range(8)])
    s6 = ref.alibi_slopes(6)
    assert s6.shape == (6,) and np.all(np.diff(s6[:4]) < 0)


def test_flash_attention_oracle_matches_reference(golden_dir):
    data, meta = _load(golden_dir, "flash_attention.npz")
    for i, m in enumerate(meta):
        Q, K, V = data[f"q{i}"], data[f"k{i}"], data[f"v{i}"]
        slopes = ref.alibi_slopes(Q.shape[1]) if m["alibi"] else None
        o, rmax, rsum = ref.flash_attention_ref(Q, K, V, m["block"], m["causal"], m["window"],
                                                slopes)
        np.testing.assert_allclose(o, data[f"o{i}"], atol=1e-12)
        np.testing.assert_allclose(rmax, data[f"rowmax{i}"], atol=1e-12)
        np.testing.assert_allclose(rsum, data[f"rowsum{i}"], rtol=1e-12)
        # The kernel-facing oracle (-inf exclusion, (B, S, H, D) layout) agrees
        # with the reference's streaming path wherever a row has a visible key.
        t = lambda a: a.transpose(0, 2, 1, 3)  # noqa: E731
        o2, lse = ref.attention_ref(t(Q), t(K), t(V), causal=m["causal"], window=m["window"],
                                    alibi=slopes)
        np.testing.assert_allclose(t(o2), data[f"o{i}"], atol=1e-10)
        np.testing.assert_allclose(lse, (rmax + np.log(rsum))[..., 0], atol=1e-10)


def test_mha_layer_oracle_matches_reference(golden_dir):
    data, meta = _load(golden_dir, "mha_layer.npz")
    for i, cfg in enumerate(meta):
        layer = _layer(data, i, **cfg)
        y = ref.mha_layer_ref(layer, data[f"x{i}"])
        np.testing.assert_allclose(y, data[f"y{i}"], atol=1e-10, err_msg=str(cfg))


def test_graph_padding_oracle_matches_reference(golden_dir):
    data, meta = _load(golden_dir, "graph_padding.npz")
    for i, cfg in enumerate(meta):
        layer = _layer(data, i, **cfg)
        S = data[f"x{i}"].shape[1]
        mask = np.arange(S)[None, :] < data[f"len{i}"][:, None]
        y = ref.mha_layer_ref(layer, data[f"x{i}"], key_padding_mask=mask)
        # The reference adds -1e9 in float64, which keeps scores to ~1e-7.
        np.testing.assert_allclose(y, data[f"y{i}"], atol=1e-6, err_msg=str(cfg))


def graph_mask_layer(i, cfg):
    """Weights of graph_mask.npz layer case i, drawn in the reference's order
    from its seed by enilnets_b200's graph builder (host-side NumPy)."""
    import enilnets_b200 as enl
    from enilnets_b200.graph import MultiHeadAttention
    enl.set_seed(3600 + i)
    g = MultiHeadAttention(cfg["embed_dim"], cfg["num_heads"], causal=cfg["causal"],
                           window_size=cfg["window_size"])
    layer = g._layer()
    layer["window_size"] = cfg["window_size"]
    return layer


def test_graph_arbitrary_mask_oracle_matches_reference(golden_dir):
    """Left padding, holes and fully masked rows (graph/sequence.py:162-168
    accepts any boolean key_padding_mask), with and without causal/window."""
    data, meta = _load(golden_dir, "graph_mask.npz")
    for i, cfg in enumerate(meta["layer"]):
        layer = graph_mask_layer(i, cfg)
        mask = data[f"layer_mask{i}"]
        assert not np.array_equal(mask, np.arange(mask.shape[1])[None, :] <
                                  mask.sum(axis=1)[:, None]), "golden masks are not prefixes"
        x = np.random.RandomState(3700 + i).standard_normal((3, 33, 64))
        y = ref.mha_layer_ref(layer, x, key_padding_mask=mask)
        np.testing.assert_allclose(y, data[f"layer_y{i}"], atol=1e-6, err_msg=str(cfg))
    for j, c in enumerate(meta["kernel"]):
        y = graph_mask_kernel_oracle(c, data[f"kernel_mask{j}"])
        # stored as float16 (about 5e-4 relative)
        np.testing.assert_allclose(y, data[f"kernel_y{j}"].astype(np.float64), atol=2e-3,
                                   rtol=2e-3, err_msg=str(c))


def graph_mask_kernel_oracle(c, mask):
    """Oracle output of a graph_mask.npz kernel case (identity projections:
    q = k = v = x split into heads)."""
    E = c["H"] * c["D"]
    x = ref.seeded_normal(c["seed"], (c["B"], c["S"], E))
    qkv = x.reshape(c["B"], c["S"], c["H"], c["D"])
    o, _ = ref.attention_ref(qkv, qkv, qkv, causal=c["causal"], window=c["window"],
                             key_mask=mask, mask_mode="additive")
    return o.reshape(c["B"], c["S"], E)


def test_cross_attention_oracle_matches_reference(golden_dir):
    data, meta = _load(golden_dir, "cross_layer.npz")
    for i, cfg in enumerate(meta):
        layer = _layer(data, i, **cfg)
        y = ref.cross_layer_ref(layer, data[f"qin{i}"], data[f"x{i}"])
        np.testing.assert_allclose(y, data[f"y{i}"], atol=1e-10, err_msg=str(cfg))


def prefill_case_inputs(c):
    """Inputs of a kernel_prefill.npz case: identity projections make
    q = k = v = x split into heads."""
    E = c["H"] * c["D"]
    x = ref.seeded_normal(c["seed"], (c["B"], c["S"], E))
    qkv = x.reshape(c["B"], c["S"], c["H"], c["D"])
    return x, qkv


def prefill_case_oracle(c):
    _, qkv = prefill_case_inputs(c)
    if c["kind"] == "nn":
        slopes = ref.alibi_slopes(c["H"]) if c["scheme"] == "alibi" else None
        o, _ = ref.attention_ref(qkv, qkv, qkv, causal=c["causal"], window=c["window"],
                                 alibi=slopes, mask_mode="exclude")
    else:
        o, _ = ref.attention_ref(qkv, qkv, qkv, causal=c["causal"], window=c["window"],
                                 kv_valid_len=np.array(c["lengths"]), mask_mode="additive")
    return o.reshape(c["B"], c["S"], c["H"] * c["D"])


def test_kernel_shaped_prefill_oracle_matches_reference(golden_dir):
    data, meta = _load(golden_dir, "kernel_prefill.npz")
    for i, c in enumerate(meta):
        y = prefill_case_oracle(c)
        np.testing.assert_allclose(y, data[f"y{i}"], atol=2e-6, err_msg=str(c))


def decode_case_inputs(c):
    B, H, Hkv, D, ctx = c["B"], c["H"], c["Hkv"], c["D"], c["ctx"]
    Kc = ref.seeded_normal(c["seed"], (B, Hkv, ctx, D))
    Vc = ref.seeded_normal(c["seed"] + 1000, (B, Hkv, ctx, D))
    x = ref.seeded_normal(c["seed"] + 2000, (B, 1, H * D))
    q = x.reshape(B, H, D)
    new = x[:, :, :Hkv * D].reshape(B, 1, Hkv, D)
    return Kc, Vc, q, new


def decode_case_oracle(c):
    Kc, Vc, q, new = decode_case_inputs(c)
    ctx = c["ctx"]
    K = ref.kv_append_ref(np.concatenate([Kc, np.zeros_like(Kc[:, :, :1])], axis=2), new, ctx)
    V = ref.kv_append_ref(np.concatenate([Vc, np.zeros_like(Vc[:, :, :1])], axis=2), new, ctx)
    slopes = ref.alibi_slopes(c["H"]) if c["scheme"] == "alibi" else None
    o, _ = ref.decode_ref(q, K, V, slot_begin=0, slot_end=ctx + 1, pos_slot0=0, q_pos=ctx,
                          window=c["window"], alibi=slopes)
    return o.reshape(c["B"], 1, c["H"] * c["D"])


def test_kernel_shaped_decode_oracle_matches_reference(golden_dir):
    data, meta = _load(golden_dir, "kernel_decode.npz")
    for i, c in enumerate(meta):
        y = decode_case_oracle(c)
        np.testing.assert_allclose(y, data[f"y{i}"], atol=2e-6, err_msg=str(c))
        # Window eviction keeps exactly the slots the mask would allow.
        if c["window"] is not None:
            assert int(data[f"start{i}"]) == c["ctx"] - c["window"]


def test_lse_merge_identity_recovers_unsplit_attention():
    rng = np.random.RandomState(0)
    q = rng.standard_normal((2, 3, 16))
    K = rng.standard_normal((2, 3, 50, 16))
    V = rng.standard_normal((2, 3, 50, 16))
    full, lse = ref.decode_ref(q, K, V, slot_begin=0, slot_end=50, pos_slot0=0, q_pos=49)
    parts = [ref.decode_ref(q, K, V, slot_begin=a, slot_end=b, pos_slot0=0, q_pos=49)
             for a, b in ((0, 7), (7, 30), (30, 50))]
    o, l2 = ref.lse_merge_ref(np.stack([p[0] for p in parts]), np.stack([p[1] for p in parts]))
    np.testing.assert_allclose(o, full, atol=1e-12)
    np.testing.assert_allclose(l2, lse, atol=1e-12)


def test_query_zero_of_a_causal_stream_is_v0():
    # Known answer from the reference's own tests: causal query 0 sees only key 0.
    rng = np.random.RandomState(2)
    q, k, v = (rng.standard_normal((1, 6, 1, 4)) for _ in range(3))
    o, _ = ref.attention_ref(q, k, v, causal=True)
    np.testing.assert_allclose(o[0, 0, 0], v[0, 0, 0], atol=1e-12)
