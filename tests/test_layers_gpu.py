"""Layer-level parity on the GPU: models built by enilnets_b200's builders
from the reference's seeds run through AttentionNet.Forward,
graph.MultiHeadAttention and cached_forward_step, against outputs the
reference itself produced (tests/golden/layer_b200.npz, config1.npz).

Both device precisions run (enilnets_b200.set_precision):
  fp32 (default): max abs error <= 1e-3, the north-star bar for fp32 inputs;
  bf16:           max abs error <= 2e-2 per attention layer. Through a whole
                  transformer block, layernorm and the logits projection the
                  bf16 roundings compound, so those model-level outputs are
                  held to 5e-2 in bf16 (and to 1e-3 in fp32)."""
import json

import numpy as np
import pytest

import enilnets_b200 as enl
from enilnets_b200.graph import MultiHeadAttention, lengths_to_mask

pytestmark = pytest.mark.gpu
TOL = {"fp32": 1e-3, "bf16": 2e-2}
TOL_MODEL = {"fp32": 1e-3, "bf16": 5e-2}


@pytest.fixture
def float64():
    enl.use_float64(True)
    yield
    enl.use_float64(False)


@pytest.fixture(params=["fp32", "bf16"])
def precision(request):
    enl.set_precision(request.param)
    yield request.param
    enl.set_precision("fp32")


def _golden(golden_dir):
    data = np.load(golden_dir / "layer_b200.npz")
    return data, json.loads(str(data["meta"]))


def _err(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def test_mha_layers_forward(cuda, golden_dir, float64, precision):
    """fp32: against the reference's own outputs at 1e-3. bf16: against the
    float64 oracle (pinned to the reference, test_oracle_golden.py) run on the
    bf16-rounded input and weights, so that 2e-2 measures the device path
    rather than the quantisation of its inputs, and against the reference's
    outputs at the model-level 5e-2."""
    from oracle import attention_ref as ref
    data, meta = _golden(golden_dir)
    for i, cfg in enumerate(meta["mha"]):
        enl.set_seed(1100 + i)
        m = enl.AttentionNet()
        m.add_multihead_attention(**cfg)
        x = np.random.RandomState(1200 + i).standard_normal((2, 40, cfg["embed_dim"]))
        y = m.Forward(x, training=False)
        err = _err(y, data[f"mha{i}_y"])
        if precision == "fp32":
            assert err <= TOL["fp32"], f"{cfg}: {err:.3e}"
            continue
        assert err <= TOL_MODEL["bf16"], f"{cfg}: {err:.3e} against the reference"
        layer = dict(m.layers[0])
        for k in ("Wq", "Wk", "Wv", "Wo"):
            layer[k] = ref.bf16_round(layer[k]).astype(np.float64)
        y_ref = ref.mha_layer_ref(layer, ref.bf16_round(x).astype(np.float64))
        err_q = _err(y, y_ref)
        assert err_q <= TOL["bf16"], f"{cfg}: {err_q:.3e} against bf16-rounded inputs"


def test_graph_padding_layers(cuda, golden_dir, float64, precision):
    data, meta = _golden(golden_dir)
    for i, cfg in enumerate(meta["graph"]):
        enl.set_seed(1300 + i)
        g = MultiHeadAttention(64, 4, causal=cfg["causal"], window_size=cfg["window_size"])
        x = np.random.RandomState(1400 + i).standard_normal((3, 33, 64))
        y = g(x, key_padding_mask=lengths_to_mask(cfg["lengths"], 33)).data
        err = _err(y, data[f"graph{i}_y"])
        assert err <= TOL[precision], f"{cfg}: {err:.3e}"


def test_graph_padding_garbage_invariance(cuda, precision):
    """graph/sequence.py contract (reference test_enilnets.py:6791-6801):
    garbage in padded slots does not change real-token outputs."""
    enl.set_seed(0)
    g = MultiHeadAttention(64, 4, causal=True)
    x = np.random.RandomState(0).standard_normal((3, 20, 64))
    mask = lengths_to_mask([20, 13, 5], 20)
    clean = g(x, key_padding_mask=mask).data
    bad = x.copy()
    bad[~mask] = 999.0
    dirty = g(bad, key_padding_mask=mask).data
    assert np.allclose(clean[mask], dirty[mask], atol=1e-6)


def test_cross_attention_layers(cuda, golden_dir, float64, precision):
    data, meta = _golden(golden_dir)
    for i, cfg in enumerate(meta["cross"]):
        enl.set_seed(1500 + i)
        m = enl.AttentionNet()
        m.add_dense(64, 64, activation="linear")
        m.add_cross_attention(kv_source_index=-1, embed_dim=64, num_heads=4,
                              num_kv_heads=cfg["num_kv_heads"])
        x = np.random.RandomState(1600 + i).standard_normal((2, 24, 64))
        err = _err(m.Forward(x, training=False), data[f"cross{i}_y"])
        assert err <= TOL[precision], f"{cfg}: {err:.3e}"


def _kv_model(i, cfg):
    enl.set_seed(1700 + i)
    m = enl.AttentionNet()
    m.add_embedding(vocab_size=17, embed_dim=64)
    if cfg["scheme"] == "absolute":
        m.add_positional_encoding(max_seq_len=32, learnable=False)
    m.add_transformer_block(64, num_heads=4, causal=True, positional_scheme=cfg["scheme"],
                            num_kv_heads=cfg["num_kv_heads"], window_size=cfg["window_size"])
    m.add_layernorm()
    m.add_dense(n_out=17, activation="linear")
    toks = np.random.RandomState(1800 + i).randint(0, 17, size=(3, 9))
    return m, toks


def test_kv_cache_stepping_matches_reference(cuda, golden_dir, float64, precision):
    """Primed 4-token step then 5 single-token steps (nn/kvcache.py:69-214)
    equal both the reference's stepped outputs and its full Forward; the
    cache stores the unexpanded Hkv heads and evicts outside the window."""
    data, meta = _golden(golden_dir)
    for i, cfg in enumerate(meta["kv"]):
        m, toks = _kv_model(i, cfg)
        full = m.Forward(toks, training=False)
        assert _err(full, data[f"kv{i}_full"]) <= TOL_MODEL[precision], cfg
        cache = enl.KVCache()
        pieces = [enl.cached_forward_step(m, toks[:, :4], cache)]
        pieces += [enl.cached_forward_step(m, toks[:, j:j + 1], cache) for j in range(4, 9)]
        stepped = np.concatenate(pieces, axis=1)
        assert _err(stepped, data[f"kv{i}_stepped"]) <= TOL_MODEL[precision], cfg
        assert _err(stepped, full) <= TOL_MODEL[precision], cfg
        attn_idx = [j for j, l in enumerate(m.layers) if l["type"] == "multihead_attention"][0]
        k, v, start = cache.kv[attn_idx]
        assert tuple(k.shape) == tuple(data[f"kv{i}_kshape"]), cfg
        assert start == int(data[f"kv{i}_start"]), cfg
        assert cache.position == 9


def test_kv_cache_reorder_and_expand(cuda, golden_dir, float64, precision):
    """KVCache.expand/reorder gather by parent on the device
    (nn/kvcache.py:42-66; reference test_enilnets.py:10539-10556)."""
    data, meta = _golden(golden_dir)
    for i, cfg in enumerate(meta["kv"]):
        m, toks = _kv_model(i, cfg)
        cache = enl.KVCache()
        enl.cached_forward_step(m, toks[:1, :4], cache)
        cache.expand(3)
        attn_idx = [j for j, l in enumerate(m.layers) if l["type"] == "multihead_attention"][0]
        assert cache.kv[attn_idx][0].shape[0] == 3
        enl.cached_forward_step(m, np.array([[5], [6], [7]]), cache)
        cache.reorder([2, 2, 0])
        out = enl.cached_forward_step(m, np.array([[9], [9], [9]]), cache)
        assert _err(out, data[f"kv{i}_reordered"]) <= TOL_MODEL[precision], cfg
        assert np.allclose(out[0], out[1], atol=1e-6)


def test_non_causal_layer_cannot_be_stepped(cuda):
    m = enl.AttentionNet()
    m.add_embedding(vocab_size=5, embed_dim=16)
    m.add_multihead_attention(embed_dim=16, num_heads=2, causal=False)
    with pytest.raises(ValueError, match="requires causal attention"):
        enl.cached_forward_step(m, np.array([[1, 2]]), enl.KVCache())


def test_config1_layer_output(cuda, golden_dir, precision):
    """set_seed(0), add_multihead_attention(256, 8,
    causal=True), x ~ RandomState(1) (4, 256, 256), default float32; <= 1e-3
    on the fp32 path (the default), <= 2e-2 on the bf16 path."""
    data = np.load(golden_dir / "config1.npz")
    enl.use_float64(False)
    enl.set_seed(0)
    m = enl.AttentionNet()
    m.add_multihead_attention(embed_dim=256, num_heads=8, causal=True)
    x = np.random.RandomState(1).standard_normal((4, 256, 256))
    y = m.Forward(x, training=False)
    assert y.dtype == np.float32 and y.shape == (4, 256, 256)
    err = _err(y[0], data["y0"])
    assert err <= TOL[precision], err
