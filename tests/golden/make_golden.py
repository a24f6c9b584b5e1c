"""Generate the golden vectors that pin the oracle (and the kernels) to the
reference, by running the reference itself.

Run in a container that has the reference checked out, naming its source
tree (the directory that holds the Enilnets package):

    ENILNETS_REFERENCE=/path/to/reference python tests/golden/make_golden.py [case ...]

Writes tests/golden/*.npz. The reference must never be imported at test time; the
committed .npz files are all the tests use.

Every case runs the reference in float64 (``use_float64(True)``). To expose
the attention core through the reference's own layer code, the projection
weights are set to identity and the biases to zero, so a layer's output is
exactly the concatenated per-head context (nn/forward.py:428-551,
graph/sequence.py:144-183, nn/kvcache.py:123-214). Inputs of the larger,
kernel-shaped cases are regenerated from their seeds by
``oracle.attention_ref.seeded_normal`` and are therefore not stored.
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
REF = os.environ.get("ENILNETS_REFERENCE")
if not REF:
    raise SystemExit("set ENILNETS_REFERENCE to the reference source tree (the directory that "
                     "holds the Enilnets package)")
sys.path.insert(0, REF)

from oracle.attention_ref import seeded_normal  # noqa: E402

import Enilnets  # noqa: E402
from Enilnets import NeuralNet  # noqa: E402
from Enilnets.core import backend  # noqa: E402
from Enilnets.nn import flash_attention as fa  # noqa: E402
from Enilnets.nn import kvcache as kvc  # noqa: E402
from Enilnets.graph import MultiHeadAttention, Tensor, lengths_to_mask  # noqa: E402

backend.use_float64(True)


def identity_layer(layer: dict) -> None:
    E = layer["embed_dim"]
    kv = layer["num_kv_heads"] * layer["head_dim"]
    layer["Wq"] = np.eye(E)
    layer["Wo"] = np.eye(E)
    layer["Wk"] = np.eye(kv, E)
    layer["Wv"] = np.eye(kv, E)
    for b, n in (("bq", E), ("bk", kv), ("bv", kv), ("bo", E)):
        layer[b] = np.zeros(n)


def flash_cases():
    """nn/flash_attention.py:42-80 on random (B, H, S, D) inputs."""
    out = {}
    meta = []
    rng = np.random.RandomState(1234)
    i = 0
    for causal in (False, True):
        for window in (None, 3):
            for alibi in (False, True):
                Q, K, V = (rng.standard_normal((2, 4, 11, 8)) for _ in range(3))
                slopes = Enilnets.nn.forward._alibi_slopes(4) if alibi else None
                o, cache = fa.flash_attention_forward(Q, K, V, 4, causal, window, slopes)
                out[f"q{i}"], out[f"k{i}"], out[f"v{i}"], out[f"o{i}"] = Q, K, V, o
                out[f"rowmax{i}"], out[f"rowsum{i}"] = cache[4], cache[5]
                meta.append({"causal": causal, "window": window, "alibi": alibi, "block": 4})
                i += 1
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "flash_attention.npz", **out)


def mha_layer_cases():
    """Full MHA layers (nn/forward.py:423-556) with random weights, float64."""
    out = {}
    meta = []
    i = 0
    configs = [
        dict(embed_dim=16, num_heads=4, causal=True),
        dict(embed_dim=16, num_heads=4, causal=False),
        dict(embed_dim=16, num_heads=4, causal=True, window_size=2),
        dict(embed_dim=16, num_heads=4, causal=True, positional_scheme="rope"),
        dict(embed_dim=16, num_heads=4, causal=False, positional_scheme="alibi"),
        dict(embed_dim=16, num_heads=4, causal=True, positional_scheme="alibi"),
        dict(embed_dim=16, num_heads=4, causal=True, num_kv_heads=2),
        dict(embed_dim=16, num_heads=4, causal=True, num_kv_heads=1, window_size=3,
             positional_scheme="rope"),
    ]
    for cfg in configs:
        Enilnets.core.utils.set_seed(100 + i)
        m = NeuralNet()
        m.add_multihead_attention(**cfg)
        x = np.random.RandomState(200 + i).standard_normal((2, 9, 16))
        y = m.Forward(x, training=False)
        layer = m.layers[0]
        for key in ("Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo"):
            out[f"{key}{i}"] = layer[key]
        out[f"x{i}"], out[f"y{i}"] = x, y
        meta.append(cfg)
        i += 1
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "mha_layer.npz", **out)


def graph_padding_cases():
    """graph.MultiHeadAttention with key_padding_mask (graph/sequence.py:144-183)."""
    out = {}
    meta = []
    i = 0
    for causal in (False, True):
        for window in (None, 2):
            for lengths in ([9, 5, 1], [9, 4, 0]):
                Enilnets.core.utils.set_seed(300 + i)
                g = MultiHeadAttention(16, 4, causal=causal, window_size=window)
                x = np.random.RandomState(400 + i).standard_normal((3, 9, 16))
                mask = np.asarray(lengths_to_mask(lengths, 9))
                y = g(Tensor(x), key_padding_mask=mask).data
                for key in ("Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo"):
                    out[f"{key}{i}"] = getattr(g, key).data
                out[f"x{i}"], out[f"y{i}"], out[f"len{i}"] = x, y, np.array(lengths)
                meta.append({"causal": causal, "window_size": window, "embed_dim": 16,
                             "num_heads": 4, "lengths": lengths})
                i += 1
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "graph_padding.npz", **out)


def _mask_patterns(B, S, rng):
    """Key-padding masks that are not prefixes: left padding, random holes,
    a fully masked row, and a row whose only real keys sit at the end."""
    pats = []
    left = np.ones((B, S), dtype=bool)
    for b in range(B):
        left[b, : (b * S) // (2 * B) + b] = False  # left padding of growing width
    pats.append(("left", left))
    holes = rng.rand(B, S) < 0.7
    holes[:, 0] = rng.rand(B) < 0.5
    pats.append(("holes", holes))
    mixed = rng.rand(B, S) < 0.5
    mixed[0] = False                      # every key of row 0 is padding
    mixed[-1] = False
    mixed[-1, S - max(1, S // 10):] = True  # row B-1: only its last keys are real
    pats.append(("mixed", mixed))
    return pats


def graph_mask_cases():
    """graph.MultiHeadAttention with key_padding_mask patterns that are not
    prefixes (graph/sequence.py:162-168 adds -1e9 for any boolean mask).

    layer{i}: MultiHeadAttention(64, 4) layers with the reference's own
    seeded weights (set_seed 3600 + i; any builder that draws in the
    reference's order rebuilds them), x = RandomState(3700 + i) (3, 33, 64);
    mask and output (float32) stored. kernel{i}: identity projections at
    kernel head dims, x = seeded_normal(seed, (B, S, E)) (not stored), mask
    and output (float16) stored."""
    out = {}
    meta = {"layer": [], "kernel": []}
    rng = np.random.RandomState(3500)
    i = 0
    for causal, window in ((False, None), (True, None), (True, 3), (False, 2)):
        for name, mask in _mask_patterns(3, 33, rng):
            Enilnets.core.utils.set_seed(3600 + i)
            g = MultiHeadAttention(64, 4, causal=causal, window_size=window)
            x = np.random.RandomState(3700 + i).standard_normal((3, 33, 64))
            y = g(Tensor(x), key_padding_mask=mask).data
            out[f"layer_y{i}"] = y.astype(np.float32)
            out[f"layer_mask{i}"] = mask
            meta["layer"].append({"causal": causal, "window_size": window, "embed_dim": 64,
                                  "num_heads": 4, "pattern": name})
            i += 1
    cases = [dict(B=2, S=160, H=1, D=64, causal=True, window=None),
             dict(B=2, S=160, H=1, D=64, causal=False, window=None),
             dict(B=2, S=130, H=1, D=128, causal=True, window=None),
             dict(B=2, S=160, H=1, D=64, causal=True, window=40),
             dict(B=2, S=130, H=1, D=128, causal=False, window=25)]
    j = 0
    for c in cases:
        for name, mask in _mask_patterns(c["B"], c["S"], rng):
            seed = 3800 + j
            E = c["H"] * c["D"]
            x = seeded_normal(seed, (c["B"], c["S"], E))
            g = MultiHeadAttention(E, c["H"], causal=c["causal"], window_size=c["window"])
            for wname in ("Wq", "Wk", "Wv", "Wo"):
                getattr(g, wname).data = np.eye(E)
                getattr(g, "b" + wname[1:].lower()).data = np.zeros(E)
            y = g(Tensor(x), key_padding_mask=mask).data
            out[f"kernel_y{j}"] = y.astype(np.float16)  # kernel bar 2e-2; keeps the file small
            out[f"kernel_mask{j}"] = mask
            meta["kernel"].append(dict(c, seed=seed, pattern=name))
            j += 1
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "graph_mask.npz", **out)


def cross_cases():
    """cross_attention layers (nn/forward.py:557-591): Q from a dense layer's
    output, K/V from the raw network input."""
    out = {}
    meta = []
    for i, hkv in enumerate((None, 2)):
        Enilnets.core.utils.set_seed(500 + i)
        m = NeuralNet()
        m.add_dense(16, 16, activation="linear")
        m.add_cross_attention(kv_source_index=-1, embed_dim=16, num_heads=4, num_kv_heads=hkv)
        x = np.random.RandomState(600 + i).standard_normal((2, 7, 16))
        y = m.Forward(x, training=False)
        q_in = m.outputs[1]
        layer = m.layers[1]
        for key in ("Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo"):
            out[f"{key}{i}"] = layer[key]
        out[f"x{i}"], out[f"qin{i}"], out[f"y{i}"] = x, q_in, y
        meta.append({"num_kv_heads": hkv, "embed_dim": 16, "num_heads": 4})
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "cross_layer.npz", **out)


def kernel_prefill_cases():
    """Attention core at kernel shapes (head_dim 64/128), produced by the
    reference's own layers with identity projections. Inputs come from
    seeded_normal(seed, (B, S, E)) and are not stored."""
    out = {}
    meta = []
    cases = [
        dict(kind="nn", B=1, S=160, H=2, D=64, causal=True, window=None, scheme="absolute"),
        dict(kind="nn", B=1, S=160, H=2, D=64, causal=False, window=None, scheme="absolute"),
        dict(kind="nn", B=1, S=200, H=1, D=128, causal=True, window=None, scheme="absolute"),
        dict(kind="nn", B=1, S=160, H=2, D=64, causal=True, window=40, scheme="alibi"),
        dict(kind="nn", B=1, S=130, H=2, D=64, causal=False, window=None, scheme="alibi"),
        dict(kind="graph", B=2, S=150, H=2, D=64, causal=True, window=None,
             lengths=[150, 70]),
        dict(kind="graph", B=2, S=150, H=2, D=64, causal=False, window=None,
             lengths=[131, 0]),
        dict(kind="graph", B=2, S=150, H=2, D=64, causal=True, window=20,
             lengths=[150, 90]),
    ]
    for i, c in enumerate(cases):
        seed = 700 + i
        E = c["H"] * c["D"]
        x = seeded_normal(seed, (c["B"], c["S"], E))
        if c["kind"] == "nn":
            m = NeuralNet()
            m.add_multihead_attention(embed_dim=E, num_heads=c["H"], causal=c["causal"],
                                      window_size=c["window"], positional_scheme=c["scheme"])
            identity_layer(m.layers[0])
            y = m.Forward(x, training=False)
        else:
            g = MultiHeadAttention(E, c["H"], causal=c["causal"], window_size=c["window"])
            for name, n_out in (("Wq", E), ("Wk", E), ("Wv", E), ("Wo", E)):
                getattr(g, name).data = np.eye(n_out, E)
                getattr(g, "b" + name[1:].lower()).data = np.zeros(n_out)
            mask = np.asarray(lengths_to_mask(c["lengths"], c["S"]))
            y = g(Tensor(x), key_padding_mask=mask).data
        out[f"y{i}"] = y.astype(np.float32)
        meta.append(dict(c, seed=seed))
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "kernel_prefill.npz", **out)


def kernel_decode_cases():
    """One-token cached steps through nn/kvcache.py:_attention_step at kernel
    shapes, identity projections: the new token's q = k = v = x, the cache is
    seeded N(0,1) (bf16-rounded) K/V."""
    out = {}
    meta = []
    cases = [
        dict(B=2, H=2, Hkv=2, D=64, ctx=300, scheme="absolute", window=None),
        dict(B=2, H=4, Hkv=2, D=64, ctx=257, scheme="alibi", window=None),
        dict(B=1, H=2, Hkv=2, D=128, ctx=200, scheme="absolute", window=64),
        dict(B=2, H=4, Hkv=1, D=64, ctx=129, scheme="absolute", window=None),
    ]
    for i, c in enumerate(cases):
        seed = 800 + i
        B, H, Hkv, D, ctx = c["B"], c["H"], c["Hkv"], c["D"], c["ctx"]
        E = H * D
        m = NeuralNet()
        m.add_multihead_attention(embed_dim=E, num_heads=H, causal=True, num_kv_heads=Hkv,
                                  window_size=c["window"], positional_scheme=c["scheme"])
        layer = m.layers[0]
        identity_layer(layer)
        Kc = seeded_normal(seed, (B, Hkv, ctx, D))
        Vc = seeded_normal(seed + 1000, (B, Hkv, ctx, D))
        x = seeded_normal(seed + 2000, (B, 1, E))
        cache = kvc.KVCache()
        cache.kv[0] = (Kc, Vc, 0)
        y = kvc._attention_step(layer, x, 0, cache, B, 1, ctx)
        out[f"y{i}"] = y.astype(np.float32)
        out[f"start{i}"] = np.array(cache.kv[0][2])
        out[f"len{i}"] = np.array(cache.kv[0][0].shape[2])
        meta.append(dict(c, seed=seed))
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "kernel_decode.npz", **out)


def kvcache_cases():
    """Token-by-token and primed stepping through cached_forward_step of a
    small causal stack (nn/kvcache.py:69-120) against its full Forward."""
    out = {}
    meta = []
    i = 0
    for scheme in ("absolute", "rope", "alibi"):
        for hkv, window in ((None, None), (1, 2)):
            Enilnets.core.utils.set_seed(900 + i)
            m = NeuralNet()
            m.add_embedding(vocab_size=17, embed_dim=8)
            if scheme == "absolute":
                m.add_positional_encoding(max_seq_len=32, learnable=False)
            m.add_transformer_block(8, num_heads=2, causal=True, positional_scheme=scheme,
                                    num_kv_heads=hkv, window_size=window)
            m.add_layernorm()
            m.add_dense(n_out=17, activation="linear")
            toks = np.random.RandomState(950 + i).randint(0, 17, size=(3, 6))
            full = m.Forward(toks, training=False)
            cache = kvc.KVCache()
            pieces = [kvc.cached_forward_step(m, toks[:, :4], cache)]
            pieces += [kvc.cached_forward_step(m, toks[:, j:j + 1], cache) for j in (4, 5)]
            stepped = np.concatenate(pieces, axis=1)
            out[f"toks{i}"], out[f"full{i}"], out[f"stepped{i}"] = toks, full, stepped
            attn_idx = [j for j, l in enumerate(m.layers) if l["type"] == "multihead_attention"][0]
            out[f"kshape{i}"] = np.array(cache.kv[attn_idx][0].shape)
            out[f"start{i}"] = np.array(cache.kv[attn_idx][2])
            layers = []
            for j, l in enumerate(m.layers):
                rec = {k: v for k, v in l.items() if not isinstance(v, np.ndarray)
                       and k not in ("sparse_pattern",) and not k.startswith("_")
                       and isinstance(v, (int, float, str, bool, type(None), tuple, list))}
                rec["_pos_type"] = l.get("_pos_type")
                layers.append(rec)
                for k, v in l.items():
                    if isinstance(v, np.ndarray):
                        out[f"L{i}_{j}_{k}"] = v
            meta.append({"scheme": scheme, "num_kv_heads": hkv, "window_size": window,
                         "layers": layers})
            i += 1
    out["meta"] = np.array(json.dumps(meta, default=str))
    np.savez_compressed(HERE / "kvcache_stepping.npz", **out)


def layer_b200_cases():
    """Layer-level cases at head dims the kernels take (multiples of 8): full
    MHA layers, graph padding, cross attention and KV-cache stepping, run by
    the reference in float64 with its own seeded weights. Only outputs are
    stored: the tests rebuild each model from the same seed with the
    reference-order builders of enilnets_b200.layers (seeds: 1100+i for MHA
    weights, 1200+i for its input; 1300+i / 1400+i graph; 1500+i / 1600+i
    cross; 1700+i / 1800+i KV stepping)."""
    out = {}
    meta = {"mha": [], "graph": [], "cross": [], "kv": []}
    configs = [
        dict(embed_dim=64, num_heads=4, causal=True),
        dict(embed_dim=64, num_heads=4, causal=False),
        dict(embed_dim=64, num_heads=4, causal=True, window_size=5),
        dict(embed_dim=64, num_heads=4, causal=True, positional_scheme="rope"),
        dict(embed_dim=64, num_heads=4, causal=False, positional_scheme="alibi"),
        dict(embed_dim=64, num_heads=4, causal=True, positional_scheme="alibi", window_size=9),
        dict(embed_dim=64, num_heads=4, causal=True, num_kv_heads=2),
        dict(embed_dim=64, num_heads=4, causal=True, num_kv_heads=1, positional_scheme="rope"),
        dict(embed_dim=128, num_heads=2, causal=True),
    ]
    for i, cfg in enumerate(configs):
        Enilnets.core.utils.set_seed(1100 + i)
        m = NeuralNet()
        m.add_multihead_attention(**cfg)
        x = np.random.RandomState(1200 + i).standard_normal((2, 40, cfg["embed_dim"]))
        y = m.Forward(x, training=False)
        out[f"mha{i}_y"] = y.astype(np.float32)
        meta["mha"].append(cfg)
    i = 0
    for causal in (False, True):
        for window in (None, 3):
            for lengths in ([33, 17, 1], [33, 20, 0]):
                Enilnets.core.utils.set_seed(1300 + i)
                g = MultiHeadAttention(64, 4, causal=causal, window_size=window)
                x = np.random.RandomState(1400 + i).standard_normal((3, 33, 64))
                mask = np.asarray(lengths_to_mask(lengths, 33))
                y = g(Tensor(x), key_padding_mask=mask).data
                out[f"graph{i}_y"] = y.astype(np.float32)
                meta["graph"].append({"causal": causal, "window_size": window,
                                      "embed_dim": 64, "num_heads": 4, "lengths": lengths})
                i += 1
    for i, hkv in enumerate((None, 2)):
        Enilnets.core.utils.set_seed(1500 + i)
        m = NeuralNet()
        m.add_dense(64, 64, activation="linear")
        m.add_cross_attention(kv_source_index=-1, embed_dim=64, num_heads=4, num_kv_heads=hkv)
        x = np.random.RandomState(1600 + i).standard_normal((2, 24, 64))
        y = m.Forward(x, training=False)
        out[f"cross{i}_y"] = y.astype(np.float32)
        meta["cross"].append({"num_kv_heads": hkv})
    i = 0
    for scheme in ("absolute", "rope", "alibi"):
        for hkv, window in ((None, None), (2, 3)):
            Enilnets.core.utils.set_seed(1700 + i)
            m = NeuralNet()
            m.add_embedding(vocab_size=17, embed_dim=64)
            if scheme == "absolute":
                m.add_positional_encoding(max_seq_len=32, learnable=False)
            m.add_transformer_block(64, num_heads=4, causal=True, positional_scheme=scheme,
                                    num_kv_heads=hkv, window_size=window)
            m.add_layernorm()
            m.add_dense(n_out=17, activation="linear")
            toks = np.random.RandomState(1800 + i).randint(0, 17, size=(3, 9))
            full = m.Forward(toks, training=False)
            cache = kvc.KVCache()
            pieces = [kvc.cached_forward_step(m, toks[:, :4], cache)]
            pieces += [kvc.cached_forward_step(m, toks[:, j:j + 1], cache) for j in range(4, 9)]
            out[f"kv{i}_full"] = full.astype(np.float32)
            out[f"kv{i}_stepped"] = np.concatenate(pieces, axis=1).astype(np.float32)
            attn_idx = [j for j, l in enumerate(m.layers) if l["type"] == "multihead_attention"][0]
            out[f"kv{i}_kshape"] = np.array(cache.kv[attn_idx][0].shape)
            out[f"kv{i}_start"] = np.array(cache.kv[attn_idx][2])
            # reorder: expand row 0 to 3 beams, one step, gather by parents, one step
            cache2 = kvc.KVCache()
            kvc.cached_forward_step(m, toks[:1, :4], cache2)
            cache2.expand(3)
            kvc.cached_forward_step(m, np.array([[5], [6], [7]]), cache2)
            cache2.reorder([2, 2, 0])
            out[f"kv{i}_reordered"] = kvc.cached_forward_step(
                m, np.array([[9], [9], [9]]), cache2).astype(np.float32)
            meta["kv"].append({"scheme": scheme, "num_kv_heads": hkv, "window_size": window})
            i += 1
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "layer_b200.npz", **out)


def config1_case():
    """BASELINE config 1 exactly: set_seed(0), add_multihead_attention(256, 8,
    causal=True) at the reference's default float32, x ~ RandomState(1);
    the output of batch row 0 from the float64 path, plus SHA-256 digests of
    the seeded float32 weights (to pin the builders' RNG order)."""
    import hashlib
    backend.use_float64(False)
    Enilnets.core.utils.set_seed(0)
    m = NeuralNet()
    m.add_multihead_attention(embed_dim=256, num_heads=8, causal=True)
    digests = {k: hashlib.sha256(np.ascontiguousarray(m.layers[0][k]).tobytes()).hexdigest()
               for k in ("Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo")}
    layer = {k: np.asarray(v, np.float64) if isinstance(v, np.ndarray) else v
             for k, v in m.layers[0].items()}
    backend.use_float64(True)
    m64 = NeuralNet()
    m64.layers = [layer]
    x = np.random.RandomState(1).standard_normal((4, 256, 256))
    y = m64.Forward(x, training=False)
    np.savez_compressed(HERE / "config1.npz", y0=y[0].astype(np.float32),
                        digests=np.array(json.dumps(digests)))


TEXTGEN_CORPUS = [
    "attention reads keys and values; the cache keeps them close.",
    "a small model writes one letter at a time, then looks back.",
    "keys fade, values stay, and the window slides along.",
]
TEXTGEN_PROMPTS = ["the cache", "a small", "keys and", "values"]


def textgen_case():
    """The reference's TextGenerator (generative/text_generation.py) on a
    char-level tokenizer, float64, seed 42: greedy ids with and without the
    KV cache, beam-search ids, batched greedy ids, perplexity, and each
    greedy step's top-1 / top-2 probability margin (for tie-aware
    comparison). Also SHA-256 digests of every weight array, to pin the
    builders' RNG order for the whole stack."""
    import hashlib
    from Enilnets.generative.text_generation import TextGenerator
    from Enilnets.text.text_utils import Tokenizer
    backend.use_float64(True)
    tok = Tokenizer(level="char").fit(TEXTGEN_CORPUS)
    Enilnets.core.utils.set_seed(42)
    gen = TextGenerator(tok, embed_dim=32, num_heads=4, num_layers=2, max_seq_len=48)
    digests = []
    for layer in gen.network.layers:
        for k in sorted(layer):
            v = layer[k]
            if isinstance(v, np.ndarray):
                digests.append(hashlib.sha256(np.ascontiguousarray(v).tobytes()).hexdigest())
    out = {"vocab": np.array(json.dumps(tok.word_to_idx)),
           "digests": np.array(json.dumps(digests))}
    start = tok.word_to_idx[tok.start_token]
    for i, prompt in enumerate(TEXTGEN_PROMPTS[:2]):
        ids = [start] + tok.encode(prompt, add_special_tokens=False).tolist()
        # greedy path with margins, via the reference's own uncached loop
        margins = []
        cur = list(ids)
        for _ in range(12):
            probs = gen.network.Forward(np.array([cur[-48:]]), training=False)[0, -1]
            top = np.sort(probs)[::-1]
            margins.append(float(top[0] - top[1]))
            nxt = int(np.argmax(probs))
            if nxt == tok.word_to_idx[tok.end_token]:
                break
            cur.append(nxt)
        out[f"greedy{i}_text"] = np.array(gen.generate(prompt, max_new_tokens=12, greedy=True))
        out[f"greedy{i}_text_nocache"] = np.array(
            gen.generate(prompt, max_new_tokens=12, greedy=True, use_cache=False))
        out[f"greedy{i}_ids"] = np.array(cur)
        out[f"greedy{i}_margins"] = np.array(margins)
        out[f"beam{i}_text"] = np.array(
            gen.generate_beam(prompt, beam_width=3, max_new_tokens=8))
    out["batch_texts"] = np.array(json.dumps(
        gen.generate_batch(TEXTGEN_PROMPTS, max_new_tokens=6, greedy=True)))
    out["perplexity"] = np.array(gen.perplexity(TEXTGEN_CORPUS[0]))
    np.savez_compressed(HERE / "textgen.npz", **out)


def linear_cases():
    """Linearized attention kernels ("linear" elu+1 and "performer" FAVOR+),
    run by the reference in float64 (nn/attention_kernels.py, nn/forward.py:
    456-478, nn/kvcache.py:217-260).

    core{i}: identity-weight layers, so the output is the attention context of
        x itself; the Performer's projection matrix is stored as core{i}_omega
        and the input regenerates from RandomState(2100 + i).
    mha{i}: full layers with the reference's own seeded weights (set_seed
        2200 + i, input RandomState(2300 + i)); the tests rebuild them with
        enilnets_b200.layers, which draws the projection before the weights as
        the reference does.
    kv{i}: a transformer block with a linearized kernel stepped through the
        cache (prime 4 tokens, then 5 single steps) against its full Forward,
        and the step after expanding to 3 beams and reordering
        (set_seed 2400 + i, tokens RandomState(2500 + i))."""
    out = {}
    meta = {"core": [], "mha": [], "kv": []}
    core = [
        dict(embed_dim=32, num_heads=2, causal=False, attention_kernel="linear"),
        dict(embed_dim=32, num_heads=2, causal=True, attention_kernel="linear"),
        dict(embed_dim=32, num_heads=2, causal=False, attention_kernel="performer"),
        dict(embed_dim=32, num_heads=2, causal=True, attention_kernel="performer",
             num_features=24),
    ]
    for i, cfg in enumerate(core):
        Enilnets.core.utils.set_seed(2000 + i)
        m = NeuralNet()
        m.add_multihead_attention(**cfg)
        identity_layer(m.layers[0])
        x = np.random.RandomState(2100 + i).standard_normal((2, 21, cfg["embed_dim"]))
        out[f"core{i}_y"] = m.Forward(x, training=False)
        if "omega" in m.layers[0]:
            out[f"core{i}_omega"] = np.asarray(m.layers[0]["omega"])
        meta["core"].append(cfg)
    mha = [
        dict(embed_dim=64, num_heads=4, causal=True, attention_kernel="linear"),
        dict(embed_dim=64, num_heads=4, causal=False, attention_kernel="linear", num_kv_heads=2),
        dict(embed_dim=64, num_heads=4, causal=True, attention_kernel="performer"),
        dict(embed_dim=64, num_heads=4, causal=False, attention_kernel="performer",
             num_kv_heads=1, num_features=40),
        dict(embed_dim=64, num_heads=4, causal=True, attention_kernel="linear",
             positional_scheme="rope"),
    ]
    for i, cfg in enumerate(mha):
        Enilnets.core.utils.set_seed(2200 + i)
        m = NeuralNet()
        m.add_multihead_attention(**cfg)
        x = np.random.RandomState(2300 + i).standard_normal((2, 40, cfg["embed_dim"]))
        out[f"mha{i}_y"] = m.Forward(x, training=False).astype(np.float32)
        meta["mha"].append(cfg)
    kv = [
        dict(attention_kernel="linear", num_kv_heads=None, positional_scheme="absolute"),
        dict(attention_kernel="performer", num_kv_heads=None, positional_scheme="absolute"),
        dict(attention_kernel="performer", num_kv_heads=2, positional_scheme="rope"),
        dict(attention_kernel="linear", num_kv_heads=2, positional_scheme="rope"),
    ]
    for i, cfg in enumerate(kv):
        Enilnets.core.utils.set_seed(2400 + i)
        m = NeuralNet()
        m.add_embedding(vocab_size=17, embed_dim=64)
        if cfg["positional_scheme"] == "absolute":
            m.add_positional_encoding(max_seq_len=32, learnable=False)
        m.add_transformer_block(64, num_heads=4, causal=True, **cfg)
        m.add_layernorm()
        m.add_dense(n_out=17, activation="linear")
        toks = np.random.RandomState(2500 + i).randint(0, 17, size=(3, 9))
        full = m.Forward(toks, training=False)
        cache = kvc.KVCache()
        pieces = [kvc.cached_forward_step(m, toks[:, :4], cache)]
        pieces += [kvc.cached_forward_step(m, toks[:, j:j + 1], cache) for j in range(4, 9)]
        out[f"kv{i}_full"] = full.astype(np.float32)
        out[f"kv{i}_stepped"] = np.concatenate(pieces, axis=1).astype(np.float32)
        cache2 = kvc.KVCache()
        kvc.cached_forward_step(m, toks[:1, :4], cache2)
        cache2.expand(3)
        kvc.cached_forward_step(m, np.array([[5], [6], [7]]), cache2)
        cache2.reorder([2, 2, 0])
        out[f"kv{i}_reordered"] = kvc.cached_forward_step(
            m, np.array([[9], [9], [9]]), cache2).astype(np.float32)
        meta["kv"].append(cfg)
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "linear_layers.npz", **out)


def sparse_cases():
    """Block-sparse attention (sparse_pattern), run by the reference in float64
    (nn/sparse_attention.py:48-142, nn/forward.py:482-502,
    nn/kvcache.py:263-306).

    sel{i}: block_selection(index, valid) tables, random draws included.
    core{i}: sparse_attention_forward on (B, H, S, Dh) inputs regenerated from
        RandomState(3100 + i) (q, k, v drawn in that order), ALiBi slopes of
        the reference's _alibi_slopes(H) when the case asks for them.
    mha{i}: full layers with the reference's seeded weights (set_seed 3200 + i,
        input RandomState(3300 + i)).
    kv{i}: the reference test's stepping model (set_seed 3400 + i, tokens
        RandomState(3500 + i)): full Forward, one-token steps, and a 5 + 4
        split."""
    from Enilnets.nn import sparse_attention as sa
    from Enilnets.nn.forward import _alibi_slopes
    out = {}
    meta = {"sel": [], "core": [], "mha": [], "kv": []}
    sel = [
        ({"block_size": 3, "local": 1, "global": 1, "random": 1}, 12, True),
        ({"block_size": 3, "local": 1, "global": 1, "random": 1}, 12, False),
        ({"block_size": 2, "local": 1, "random": 2, "seed": 7}, 8, True),
        ({"block_size": 16, "local": 2, "global": 2, "random": 3, "seed": 5}, 40, True),
        ({"block_size": 16, "local": 2, "global": 2, "random": 3, "seed": 5}, 40, False),
        ({"block_size": 4, "local": 0, "global": 0, "random": 2, "seed": 11}, 25, False),
    ]
    for i, (pat, nb, causal) in enumerate(sel):
        index, valid = sa.block_selection(sa.normalize_pattern(pat), nb, causal)
        out[f"sel{i}_index"], out[f"sel{i}_valid"] = index, valid
        meta["sel"].append([pat, nb, causal])
    core = [
        dict(B=2, H=2, S=10, Dh=4, pattern={"block_size": 3, "local": 1, "global": 1,
                                            "random": 1}, causal=False, alibi=False),
        dict(B=2, H=2, S=10, Dh=4, pattern={"block_size": 4, "local": 1}, causal=True,
             alibi=False),
        dict(B=2, H=2, S=77, Dh=32, pattern={"block_size": 8, "local": 1, "global": 1,
                                             "random": 2}, causal=True, alibi=False),
        dict(B=1, H=3, S=300, Dh=64, pattern={"block_size": 16, "local": 2, "global": 1,
                                              "random": 2, "seed": 4}, causal=False,
             alibi=False),
        dict(B=1, H=2, S=260, Dh=128, pattern={"block_size": 64, "local": 1, "global": 1},
             causal=True, alibi=True),
        dict(B=1, H=2, S=333, Dh=64, pattern={"block_size": 100, "local": 1, "random": 1},
             causal=False, alibi=True),
        dict(B=1, H=2, S=200, Dh=16, pattern={"block_size": 1, "local": 5, "global": 2},
             causal=True, alibi=False),
        dict(B=1, H=1, S=600, Dh=64, pattern={"block_size": 256, "local": 1}, causal=True,
             alibi=False),
    ]
    for i, c in enumerate(core):
        rs = np.random.RandomState(3100 + i)
        shape = (c["B"], c["H"], c["S"], c["Dh"])
        q, k, v = (rs.standard_normal(shape) for _ in range(3))
        slopes = _alibi_slopes(c["H"]) if c["alibi"] else None
        ctx, _ = sa.sparse_attention_forward(q, k, v, sa.normalize_pattern(c["pattern"]),
                                             c["causal"], slopes)
        out[f"core{i}_y"] = ctx.astype(np.float32)
        meta["core"].append(c)
    mha = [
        dict(causal=True, positional_scheme="absolute", num_kv_heads=None,
             sparse_pattern={"block_size": 8, "local": 1, "global": 1, "random": 1}),
        dict(causal=False, positional_scheme="rope", num_kv_heads=2,
             sparse_pattern={"block_size": 16, "local": 1, "random": 2, "seed": 3}),
        dict(causal=True, positional_scheme="alibi", num_kv_heads=1,
             sparse_pattern={"block_size": 5, "local": 2, "global": 1}),
        dict(causal=False, positional_scheme="alibi", num_kv_heads=None,
             sparse_pattern={"block_size": 12, "local": 1, "global": 2}),
        dict(causal=True, positional_scheme="absolute", num_kv_heads=None,
             sparse_pattern={"block_size": 40}),
    ]
    for i, cfg in enumerate(mha):
        Enilnets.core.utils.set_seed(3200 + i)
        m = NeuralNet()
        m.add_multihead_attention(embed_dim=64, num_heads=4, **cfg)
        x = np.random.RandomState(3300 + i).standard_normal((2, 40, 64))
        out[f"mha{i}_y"] = m.Forward(x, training=False).astype(np.float32)
        meta["mha"].append(cfg)
    kv = [
        dict(pattern={"block_size": 2, "local": 1}, scheme="absolute"),
        dict(pattern={"block_size": 3, "local": 1, "global": 1, "random": 1}, scheme="rope"),
        dict(pattern={"block_size": 3, "local": 1, "global": 1, "random": 1}, scheme="alibi"),
        dict(pattern={"block_size": 4, "local": 1, "random": 2, "seed": 9}, scheme="absolute"),
    ]
    for i, cfg in enumerate(kv):
        Enilnets.core.utils.set_seed(3400 + i)
        m = NeuralNet()
        m.add_embedding(vocab_size=13, embed_dim=32)
        if cfg["scheme"] == "absolute":
            m.add_positional_encoding(max_seq_len=16, learnable=False)
        m.add_multihead_attention(embed_dim=32, num_heads=4, causal=True,
                                  positional_scheme=cfg["scheme"],
                                  sparse_pattern=cfg["pattern"])
        m.add_dense(n_out=13, activation="linear")
        toks = np.random.RandomState(3500 + i).randint(0, 13, size=(2, 9))
        out[f"kv{i}_full"] = m.Forward(toks, training=False).astype(np.float32)
        c1 = kvc.KVCache()
        out[f"kv{i}_one"] = np.concatenate(
            [kvc.cached_forward_step(m, toks[:, j:j + 1], c1) for j in range(9)],
            axis=1).astype(np.float32)
        c2 = kvc.KVCache()
        out[f"kv{i}_multi"] = np.concatenate(
            [kvc.cached_forward_step(m, toks[:, :5], c2),
             kvc.cached_forward_step(m, toks[:, 5:], c2)], axis=1).astype(np.float32)
        meta["kv"].append(cfg)
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "sparse.npz", **out)


def flash_backward_cases():
    """nn/flash_attention.py:83-114 (flash_attention_backward) after its
    forward, on (B, H, S, Dh) inputs regenerated from RandomState(4000 + i)
    (q, k, v, dout drawn in that order); dQ, dK, dV stored as float32."""
    out = {}
    meta = []
    cases = []
    for causal in (False, True):
        for window in (None, 3):
            for alibi in (False, True):
                cases.append(dict(B=2, H=2, S=11, Dh=8, causal=causal, window=window,
                                  alibi=alibi, block=4))
    cases.append(dict(B=1, H=2, S=150, Dh=64, causal=True, window=None, alibi=True, block=32))
    cases.append(dict(B=1, H=1, S=140, Dh=128, causal=False, window=40, alibi=False, block=64))
    for i, c in enumerate(cases):
        rs = np.random.RandomState(4000 + i)
        shape = (c["B"], c["H"], c["S"], c["Dh"])
        Q, K, V, dO = (rs.standard_normal(shape) for _ in range(4))
        slopes = Enilnets.nn.forward._alibi_slopes(c["H"]) if c["alibi"] else None
        _, cache = fa.flash_attention_forward(Q, K, V, c["block"], c["causal"], c["window"],
                                              slopes)
        dq, dk, dv = fa.flash_attention_backward(dO, cache)
        out[f"dq{i}"], out[f"dk{i}"], out[f"dv{i}"] = (t.astype(np.float32)
                                                       for t in (dq, dk, dv))
        meta.append(c)
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "flash_backward.npz", **out)


def mha_backward_cases():
    """nn/backward.py:241-327 (multihead_attention_backward) after
    Forward(training=True) on one-layer models (set_seed 4500 + i, input and
    dout from RandomState(4600 + i), x first): dx and the eight parameter
    gradients, float32."""
    from Enilnets.nn import backward as bw
    out = {}
    meta = []
    cfgs = [
        dict(embed_dim=64, num_heads=4, causal=True),
        dict(embed_dim=64, num_heads=4, causal=True, positional_scheme="rope", num_kv_heads=2),
        dict(embed_dim=64, num_heads=4, causal=False, positional_scheme="alibi"),
        dict(embed_dim=64, num_heads=2, causal=True, window_size=7, num_kv_heads=1),
        dict(embed_dim=128, num_heads=2, causal=True, tiled_block_size=16,
             positional_scheme="rope"),
    ]
    for i, cfg in enumerate(cfgs):
        Enilnets.core.utils.set_seed(4500 + i)
        m = NeuralNet()
        m.add_multihead_attention(**cfg)
        rs = np.random.RandomState(4600 + i)
        x = rs.standard_normal((2, 37, cfg["embed_dim"]))
        dout = rs.standard_normal((2, 37, cfg["embed_dim"]))
        m.Forward(x, training=True)
        layer = m.layers[0]
        dx = bw.multihead_attention_backward(dout, layer, m.attention_cache[0])
        out[f"dx{i}"] = dx.astype(np.float32)
        for name in ("d_Wq", "d_bq", "d_Wk", "d_bk", "d_Wv", "d_bv", "d_Wo", "d_bo"):
            out[f"{name}{i}"] = np.asarray(layer[name]).astype(np.float32)
        meta.append(cfg)
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / "mha_backward.npz", **out)


def main():
    if len(sys.argv) > 1:
        for name in sys.argv[1:]:
            globals()[name]()
        return
    flash_cases()
    mha_layer_cases()
    graph_padding_cases()
    graph_mask_cases()
    cross_cases()
    kernel_prefill_cases()
    kernel_decode_cases()
    kvcache_cases()
    layer_b200_cases()
    config1_case()
    textgen_case()
    linear_cases()
    sparse_cases()
    flash_backward_cases()
    mha_backward_cases()
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
