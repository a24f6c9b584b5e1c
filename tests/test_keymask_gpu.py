"""Arbitrary key-padding masks on the GPU.

graph/sequence.py:162-168 adds -1e9 for every key a boolean (batch, seq)
key_padding_mask marks as padding, whatever the pattern: left padding, holes,
fully masked rows. Masks whose real tokens are not a prefix reach K1 as
packed bits (kv_mask); these tests hold that path to the reference's own
outputs (tests/golden/graph_mask.npz) and to the float64 oracle, at the
bf16 bar (2e-2) and the fp32 bar (1e-3), including the rows whose every key
is masked, where only the keys with the fewest -1e9 terms survive."""
import json

import numpy as np
import pytest

from oracle import attention_ref as ref

pytestmark = pytest.mark.gpu
TOL = {"bf16": 2e-2, "fp32": 1e-3}


def _dev(x, dtype):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    return t.to(torch.bfloat16) if dtype == "bf16" else t


def _run(q, k, v, mask, dtype="bf16", lens=None, **kw):
    import torch
    from enilnets_b200 import kernels, _native
    out, lse = kernels.attention_prefill(
        _dev(q, dtype), _dev(k, dtype), _dev(v, dtype),
        kv_mask=None if mask is None else kernels.pack_key_mask(mask, "cuda"),
        kv_valid_len=None if lens is None else torch.tensor(lens, dtype=torch.int32).cuda(),
        out_dtype=torch.float32, return_lse=True, **kw)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    return out.cpu().numpy().astype(np.float64), lse.cpu().numpy().astype(np.float64)


def _check(q, k, v, mask, dtype="bf16", lens=None, **kw):
    o, lse = _run(q, k, v, mask, dtype, lens, **kw)
    oref, lref = ref.attention_ref(q, k, v, key_mask=mask, kv_valid_len=lens, **kw)
    finite = np.isfinite(oref)
    assert np.array_equal(finite, np.isfinite(o)), f"NaN pattern differs for {kw}"
    err = np.max(np.abs(o[finite] - oref[finite])) if finite.any() else 0.0
    assert err <= TOL[dtype], f"max abs err {err:.3e} > {TOL[dtype]} for {dtype} {kw}"
    if kw.get("mask_mode") == "exclude":
        lf = np.isfinite(lref)
        assert np.max(np.abs(lse[lf] - lref[lf]), initial=0.0) <= 2e-2
    return err


def _patterns(B, S, seed):
    rng = np.random.RandomState(seed)
    left = np.ones((B, S), dtype=bool)
    for b in range(B):
        left[b, : (b * S) // (2 * B) + 3 * b] = False
    holes = rng.rand(B, S) < 0.6
    mixed = rng.rand(B, S) < 0.3
    mixed[0] = False
    mixed[-1] = False
    mixed[-1, -5:] = True
    sparse_runs = np.zeros((B, S), dtype=bool)
    for b in range(B):  # a few runs of real keys separated by whole padded tiles
        for start in rng.randint(0, S, size=3):
            sparse_runs[b, start:start + 20] = True
    return {"left": left, "holes": holes, "mixed": mixed, "runs": sparse_runs}


def test_golden_graph_mask_kernel_cases(cuda, golden_dir):
    """The reference's own graph MHA outputs (identity projections) for left
    padding, holes and fully masked rows, causal/window included."""
    data = np.load(golden_dir / "graph_mask.npz")
    meta = json.loads(str(data["meta"]))
    for j, c in enumerate(meta["kernel"]):
        E = c["H"] * c["D"]
        x = ref.seeded_normal(c["seed"], (c["B"], c["S"], E))
        qkv = x.reshape(c["B"], c["S"], c["H"], c["D"])
        o, _ = _run(qkv, qkv, qkv, data[f"kernel_mask{j}"], causal=c["causal"],
                    window=c["window"], mask_mode="additive")
        y = o.reshape(c["B"], c["S"], E)
        err = np.max(np.abs(y - data[f"kernel_y{j}"].astype(np.float64)))
        assert err <= TOL["bf16"], f"{c}: {err:.3e}"


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("mode", ["additive", "exclude"])
def test_random_masks_against_oracle(cuda, D, mode):
    B, S, H, Hkv = 3, 300, 4, 2
    q = ref.seeded_normal(21, (B, S, H, D))
    k = ref.seeded_normal(22, (B, S, Hkv, D))
    v = ref.seeded_normal(23, (B, S, Hkv, D))
    for name, mask in _patterns(B, S, 24).items():
        for causal, window in ((False, None), (True, None), (True, 30), (False, 50)):
            _check(q, k, v, mask, causal=causal, window=window, mask_mode=mode)


def test_masks_with_fp32_inputs(cuda):
    """The fp32 (split-bf16) path, the reference's default float32 models."""
    B, S, H, D = 2, 200, 2, 64
    q = ref.seeded_normal(31, (B, S, H, D), bf16=False)
    k = ref.seeded_normal(32, (B, S, H, D), bf16=False)
    v = ref.seeded_normal(33, (B, S, H, D), bf16=False)
    for name, mask in _patterns(B, S, 34).items():
        for causal, window in ((False, None), (True, None), (True, 25)):
            _check(q, k, v, mask, dtype="fp32", causal=causal, window=window,
                   mask_mode="additive")


def test_mask_combined_with_valid_lengths_and_offsets(cuda):
    """A key must pass both kv_mask and kv_valid_len; query/key position
    offsets shift the causal diagonal (the cached multi-token step)."""
    B, S, Sq, H, D = 2, 260, 130, 2, 128
    q = ref.seeded_normal(41, (B, Sq, H, D))
    k = ref.seeded_normal(42, (B, S, H, D))
    v = ref.seeded_normal(43, (B, S, H, D))
    mask = _patterns(B, S, 44)["holes"]
    for mode in ("additive", "exclude"):
        _check(q, k, v, mask, lens=[200, 77], causal=True, q_pos0=130, mask_mode=mode)
        _check(q, k, v, mask, lens=[260, 5], causal=False, window=40, q_pos0=60,
               mask_mode=mode)


def test_prefix_mask_as_bits_equals_length_path(cuda):
    """A prefix mask given as bits selects exactly the keys the length path
    selects."""
    B, S, H, D = 3, 333, 2, 128
    q = ref.seeded_normal(51, (B, S, H, D))
    k = ref.seeded_normal(52, (B, S, H, D))
    v = ref.seeded_normal(53, (B, S, H, D))
    lens = np.array([333, 140, 0])
    mask = np.arange(S)[None, :] < lens[:, None]
    for causal, window in ((True, None), (False, None), (True, 20)):
        a, _ = _run(q, k, v, mask, causal=causal, window=window, mask_mode="additive")
        b, _ = _run(q, k, v, None, lens=list(lens), causal=causal, window=window,
                    mask_mode="additive")
        fin = np.isfinite(b)
        assert np.array_equal(np.isfinite(a), fin)
        assert np.max(np.abs(a[fin] - b[fin])) <= 1e-6


def test_garbage_in_masked_keys_does_not_change_the_output(cuda):
    """graph/sequence.py padding contract (reference test_enilnets.py:
    6791-6801), for holes: values under masked keys never reach the output
    of rows that have an unmasked key."""
    B, S, H, D = 2, 190, 2, 64
    q = ref.seeded_normal(61, (B, S, H, D))
    k = ref.seeded_normal(62, (B, S, H, D))
    v = ref.seeded_normal(63, (B, S, H, D))
    mask = _patterns(B, S, 64)["holes"]
    o1, _ = _run(q, k, v, mask, causal=True, mask_mode="additive")
    k2, v2 = k.copy(), v.copy()
    k2[~mask] = 999.0
    v2[~mask] = -999.0
    o2, _ = _run(q, k2, v2, mask, causal=True, mask_mode="additive")
    pos = np.arange(S)
    has_key = np.array([[mask[b, : i + 1].any() for i in pos] for b in range(B)])
    assert np.array_equal(o1[has_key], o2[has_key])


@pytest.fixture(params=["fp32", "bf16"])
def precision(request):
    import enilnets_b200 as enl
    enl.set_precision(request.param)
    yield request.param
    enl.set_precision("fp32")


def test_graph_layer_with_non_prefix_masks(cuda, golden_dir, precision):
    """graph.MultiHeadAttention(64, 4) with the reference's seeded weights
    and left-padded, holed and fully masked rows, against the reference's
    own outputs."""
    import enilnets_b200 as enl
    from enilnets_b200.graph import MultiHeadAttention
    data = np.load(golden_dir / "graph_mask.npz")
    meta = json.loads(str(data["meta"]))
    enl.use_float64(True)
    try:
        for i, cfg in enumerate(meta["layer"]):
            enl.set_seed(3600 + i)
            g = MultiHeadAttention(64, 4, causal=cfg["causal"], window_size=cfg["window_size"])
            x = np.random.RandomState(3700 + i).standard_normal((3, 33, 64))
            y = g(x, key_padding_mask=data[f"layer_mask{i}"]).data
            err = float(np.max(np.abs(np.asarray(y, np.float64) - data[f"layer_y{i}"])))
            assert err <= TOL[precision], f"{cfg}: {err:.3e}"
    finally:
        enl.use_float64(False)


def test_cross_attention_memory_mask_with_holes(cuda):
    """The cross-attention layer applies the same -1e9 rule to a memory mask
    with holes and left padding (the oracle's cross_layer_ref)."""
    import enilnets_b200 as enl
    from enilnets_b200 import attention
    from enilnets_b200.backend import to_device
    import torch
    enl.set_seed(77)
    m = enl.AttentionNet()
    m.add_dense(64, 64, activation="linear")
    m.add_cross_attention(kv_source_index=-1, embed_dim=64, num_heads=4)
    layer = m.layers[1]
    rng = np.random.RandomState(78)
    x = rng.standard_normal((2, 24, 64))
    mem = rng.standard_normal((2, 150, 64))
    mask = _patterns(2, 150, 79)["mixed"]
    y = attention.cross_attention(layer, to_device(x, torch.float32),
                                  to_device(mem, torch.float32),
                                  memory_key_padding_mask=mask).cpu().numpy()
    yref = ref.cross_layer_ref(layer, x, mem, memory_key_mask=mask)
    assert np.max(np.abs(y - yref)) <= TOL["fp32"]
