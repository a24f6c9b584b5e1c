"""Host-side layer API checks (no GPU): the builders draw exactly the
reference's weights, validate like the reference, and the layer-level oracle
reproduces the reference's outputs on models rebuilt by our builders."""
import hashlib
import json

import numpy as np
import pytest

import enilnets_b200 as enl
from enilnets_b200 import attention, layers
from enilnets_b200.graph import MultiHeadAttention, lengths_to_mask
from oracle import attention_ref as ref


@pytest.fixture
def float64():
    enl.use_float64(True)
    yield
    enl.use_float64(False)


def test_config1_weights_are_bit_identical_to_the_reference(golden_dir):
    """set_seed(0) + add_multihead_attention(256, 8, causal=True) at the
    reference's default float32 gives the reference's exact weights."""
    data = np.load(golden_dir / "config1.npz")
    digests = json.loads(str(data["digests"]))
    enl.use_float64(False)
    enl.set_seed(0)
    m = enl.AttentionNet()
    m.add_multihead_attention(embed_dim=256, num_heads=8, causal=True)
    for k, d in digests.items():
        got = hashlib.sha256(np.ascontiguousarray(m.layers[0][k]).tobytes()).hexdigest()
        assert got == d, k


def test_layer_dict_contract():
    m = enl.AttentionNet()
    m.add_multihead_attention(embed_dim=64, num_heads=4, num_kv_heads=2, causal=True,
                              window_size=3, positional_scheme="rope")
    layer = m.layers[0]
    for key in ("type", "embed_dim", "num_heads", "num_kv_heads", "head_dim", "dropout",
                "causal", "window_size", "attention_kernel", "sparse_pattern",
                "tiled_block_size", "positional_scheme", "Wq", "bq", "Wk", "bk", "Wv", "bv",
                "Wo", "bo"):
        assert key in layer
    assert layer["Wk"].shape == (2 * 16, 64) and layer["Wq"].shape == (64, 64)
    m.add_cross_attention(kv_source_index=-1, num_heads=4)
    assert m.layers[1]["type"] == "cross_attention" and m.layers[1]["embed_dim"] == 64


@pytest.mark.parametrize("kwargs,match", [
    (dict(embed_dim=8, num_heads=4, num_kv_heads=3), "num_kv_heads=3"),
    (dict(embed_dim=8, num_heads=2, window_size=-1), "window_size"),
    (dict(embed_dim=6, num_heads=2, positional_scheme="rope"), "even head_dim"),
    (dict(embed_dim=8, num_heads=2, positional_scheme="sinusoid"), "positional_scheme"),
    (dict(embed_dim=8, num_heads=2, tiled_block_size=0), "tiled_block_size"),
    (dict(embed_dim=8, num_heads=2, tiled_block_size=4, dropout=0.1), "dropout"),
    (dict(embed_dim=8, num_heads=2, attention_kernel="cosine"), "Unknown attention_kernel"),
    (dict(embed_dim=8, num_heads=2, attention_kernel="linear", positional_scheme="alibi"),
     "incompatible with positional_scheme='alibi'"),
    (dict(embed_dim=8, num_heads=2, attention_kernel="performer", window_size=2),
     "incompatible with window_size"),
    (dict(embed_dim=8, num_heads=2, attention_kernel="linear", dropout=0.1),
     "incompatible with dropout"),
    (dict(embed_dim=8, num_heads=2, attention_kernel="linear", sparse_pattern={"block_size": 2}),
     "nothing to sparsify"),
    (dict(embed_dim=8, num_heads=2, attention_kernel="linear", tiled_block_size=4),
     "nothing to tile"),
    (dict(embed_dim=8, num_heads=2, sparse_pattern={"block_size": 2}, window_size=3),
     "window_size"),
    (dict(embed_dim=8, num_heads=2, sparse_pattern={"block_size": 2}, tiled_block_size=2),
     "nothing to tile"),
    (dict(embed_dim=8, num_heads=2, sparse_pattern={"block_size": 0}), "block_size >= 1"),
    (dict(embed_dim=8, num_heads=2, sparse_pattern="local"), "must be a dict"),
])
def test_builder_validation_matches_reference_errors(kwargs, match):
    with pytest.raises(ValueError, match=match):
        enl.AttentionNet().add_multihead_attention(**kwargs)


def test_cross_attention_source_index_is_validated():
    m = enl.AttentionNet()
    m.add_dense(8, 8, activation="linear")
    with pytest.raises(ValueError, match="out of range"):
        m.add_cross_attention(kv_source_index=1, embed_dim=8, num_heads=2)


def test_lengths_to_mask_and_prefix_lengths():
    mask = lengths_to_mask([3, 1, 0], 4)
    assert mask.tolist() == [[True, True, True, False], [True, False, False, False],
                             [False] * 4]
    kind, lens = attention.classify_key_mask(mask, 3, 4)
    assert kind == "lengths" and lens.tolist() == [3, 1, 0]
    with pytest.raises(ValueError, match="shape"):
        attention.classify_key_mask(mask, 3, 5)


def test_non_prefix_masks_become_packed_key_words():
    """Left padding and holes (any boolean mask, graph/sequence.py:162-168)
    go to the kernel as bits: bit c of word w = key 64 w + c."""
    rng = np.random.RandomState(0)
    for S in (3, 64, 65, 200):
        m = rng.rand(3, S) < 0.6
        m[0, : S // 2] = False  # left padding
        m[0, S // 2:] = True
        kind, words = attention.classify_key_mask(m, 3, S)
        assert kind == "words" and words.dtype == np.int64
        assert words.shape == (3, (S + 63) // 64)
        u = words.view(np.uint64)
        bits = np.array([[(int(u[b, j // 64]) >> (j % 64)) & 1 for j in range(S)]
                         for b in range(3)], dtype=bool)
        np.testing.assert_array_equal(bits, m)
        pad = [(int(u[b, -1]) >> c) & 1 for b in range(3) for c in range(S % 64 or 64, 64)]
        assert not any(pad), "bits past the sequence end must be clear"


def _rebuild_mha(i, cfg):
    enl.set_seed(1100 + i)
    m = enl.AttentionNet()
    m.add_multihead_attention(**cfg)
    x = np.random.RandomState(1200 + i).standard_normal((2, 40, cfg["embed_dim"]))
    return m, x


def test_layer_oracle_on_rebuilt_models_matches_reference(golden_dir, float64):
    """Our float64 builders + the oracle reproduce the reference's layer
    outputs: pins the builders' RNG order and the oracle together."""
    data = np.load(golden_dir / "layer_b200.npz")
    meta = json.loads(str(data["meta"]))
    for i, cfg in enumerate(meta["mha"]):
        m, x = _rebuild_mha(i, cfg)
        y = ref.mha_layer_ref(m.layers[0], x)
        np.testing.assert_allclose(y, data[f"mha{i}_y"], atol=1e-5, err_msg=str(cfg))
    for i, cfg in enumerate(meta["graph"]):
        enl.set_seed(1300 + i)
        g = MultiHeadAttention(64, 4, causal=cfg["causal"], window_size=cfg["window_size"])
        x = np.random.RandomState(1400 + i).standard_normal((3, 33, 64))
        y = ref.mha_layer_ref(g._layer(), x, key_padding_mask=lengths_to_mask(cfg["lengths"], 33))
        np.testing.assert_allclose(y, data[f"graph{i}_y"], atol=1e-5, err_msg=str(cfg))


def test_transformer_block_layer_sequence():
    m = enl.AttentionNet()
    m.add_embedding(vocab_size=11, embed_dim=16)
    m.add_transformer_block(16, num_heads=2, causal=True)
    types = [l["type"] for l in m.layers]
    assert types == ["embedding", "residual_save", "layernorm", "multihead_attention",
                     "residual_add", "residual_save", "layernorm", "dense", "dense",
                     "residual_add"]
    assert m.layers[4]["save_index"] == 1 and m.layers[9]["save_index"] == 5


def test_linearized_layers_draw_the_projection_before_the_weights():
    """nn/layers.py:294: every linearized kernel draws its random-feature
    matrix (head_dim * 4 rows unless num_features) before Wq..Wo, so the same
    seed gives the reference's weights; only the Performer uses it."""
    from oracle import linear_ref
    for kernel, nf in (("linear", None), ("performer", 24)):
        enl.set_seed(5)
        m = enl.AttentionNet()
        m.add_multihead_attention(embed_dim=32, num_heads=2, attention_kernel=kernel,
                                  num_features=nf)
        np.random.seed(5)
        omega = linear_ref.make_projection(nf or 16 * 4, 16)
        assert np.allclose(m.layers[0]["omega"], omega, atol=1e-6)
        enl.set_seed(5)
        ref = enl.AttentionNet()
        ref.add_multihead_attention(embed_dim=32, num_heads=2)
        # the softmax layer's Wq comes first in the stream, the linearized one after omega
        assert not np.array_equal(m.layers[0]["Wq"], ref.layers[0]["Wq"])
