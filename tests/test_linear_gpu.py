"""Linearized attention kernels (K4, enl_linear.cu) on the GPU.

Kernel level: the feature map and the linear-attention kernel against the
float64 oracle (oracle/linear_ref.py) on the same inputs, including ragged
chunk and column counts, GQA and a carried decode state. Layer level: models
rebuilt from the reference's seeds against the reference's own outputs
(tests/golden/linear_layers.npz), full forward and cached stepping.

Arithmetic is fp32: max abs error <= 1e-3 (the north-star bar for fp32
inputs); the kernel-level cases on fp32 inputs hold to 1e-4."""
import json

import numpy as np
import pytest

import enilnets_b200 as enl
from oracle import linear_ref as lr

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _t(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()
    return t if dtype is None else t.to(dtype)


def _np(t):
    return t.float().cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("kernel", ["linear", "performer"])
@pytest.mark.parametrize("Dh,Df", [(8, 24), (32, 128), (64, 256), (128, 256), (192, 256),
                                   (128, 512)])
def test_feature_map_matches_oracle(cuda, kernel, Dh, Df):
    from enilnets_b200 import _native, kernels
    rng = np.random.RandomState(Dh + Df)
    B, S, H = 2, 37, 3
    x = rng.standard_normal((B, S, H, Dh))
    omega = lr.make_projection(Df, Dh, np.random.RandomState(Dh))
    xt = _t(x)
    om = _t(omega) if kernel == "performer" else None
    phi, _ = kernels.linear_feature_map(xt, kernel, om)
    ref = lr.feature_map(x.transpose(0, 2, 1, 3), kernel, omega, "row")
    assert np.max(np.abs(_np(phi) - ref)) <= 1e-4 * max(1.0, np.abs(ref).max())
    if kernel == "performer":
        phk, stab = kernels.linear_feature_map(xt, kernel, om, global_stab=True)
        st = lr.performer_stab(x.transpose(0, 2, 1, 3), omega, "global")
        assert np.max(np.abs(_np(stab) - st[..., 0, 0])) <= 1e-4 * max(1.0, np.abs(st).max())
        refk = lr.feature_map(x.transpose(0, 2, 1, 3), kernel, omega, "global")
        assert np.max(np.abs(_np(phk) - refk)) <= 1e-4 * max(1.0, np.abs(refk).max())
        # a floor above the data's own maximum wins
        floor = st[..., 0, 0] + 3.0
        _, stab2 = kernels.linear_feature_map(xt, kernel, om, global_stab=True,
                                              stab_floor=_t(floor))
        assert np.allclose(_np(stab2), floor, atol=1e-5)
    torch_sync()
    _native.raise_on_device_error()


def torch_sync():
    import torch
    torch.cuda.synchronize()


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("S,D,Df,H,Hkv", [
    (1, 8, 8, 2, 2), (5, 40, 40, 4, 2), (16, 32, 32, 2, 1), (37, 64, 256, 4, 4),
    (300, 128, 128, 2, 2), (129, 72, 512, 4, 1),
    # odd head dim (scalar V loads) and odd feature count (last feature pair half used)
    (45, 37, 33, 2, 1),
    # long enough for the causal pass to run in parallel sequence segments
    (1500, 64, 96, 4, 2), (2048, 32, 32, 1, 1)])
def test_linear_attention_matches_oracle(cuda, causal, S, D, Df, H, Hkv):
    from enilnets_b200 import _native, kernels
    rng = np.random.RandomState(S + D + Df)
    B = 2
    qp = np.exp(rng.standard_normal((B, H, S, Df)) * 0.5)   # positive features
    kp = np.exp(rng.standard_normal((B, Hkv, S, Df)) * 0.5)
    v = rng.standard_normal((B, S, Hkv, D))
    out = kernels.linear_attention(_t(qp), _t(kp), _t(v), causal=causal)
    G = H // Hkv
    kph = np.repeat(kp, G, axis=1)
    vh = np.repeat(v.transpose(0, 2, 1, 3), G, axis=1)
    ref, _, _ = lr.linear_attention(qp, kph, vh, causal)
    torch_sync()
    _native.raise_on_device_error()
    assert np.max(np.abs(_np(out).transpose(0, 2, 1, 3) - ref)) <= 1e-4


def test_linear_attention_bf16_values_and_output(cuda):
    import torch
    from enilnets_b200 import kernels
    rng = np.random.RandomState(9)
    B, S, H, D, Df = 2, 50, 2, 64, 64
    qp = np.exp(rng.standard_normal((B, H, S, Df)) * 0.5)
    kp = np.exp(rng.standard_normal((B, H, S, Df)) * 0.5)
    v = rng.standard_normal((B, S, H, D))
    vb = _t(v, torch.bfloat16)
    out = kernels.linear_attention(_t(qp), _t(kp), vb, causal=True, out_dtype=torch.bfloat16)
    ref, _, _ = lr.linear_attention(qp, kp, _np(vb).transpose(0, 2, 1, 3), True)
    assert np.max(np.abs(_np(out).transpose(0, 2, 1, 3) - ref)) <= 2e-2


def test_carried_state_equals_one_pass(cuda):
    """Prefix sums split across calls (state out -> scaled state in) equal one
    causal pass: the decode step's state algebra."""
    from enilnets_b200 import kernels
    rng = np.random.RandomState(4)
    B, H, Hkv, S, D, Df = 2, 4, 2, 23, 48, 96
    qp = np.exp(rng.standard_normal((B, H, S, Df)) * 0.5)
    kp = np.exp(rng.standard_normal((B, Hkv, S, Df)) * 0.5)
    v = rng.standard_normal((B, S, Hkv, D))
    full = _np(kernels.linear_attention(_t(qp), _t(kp), _t(v), causal=True))
    cut = 9
    o1, st = kernels.linear_attention(_t(qp[:, :, :cut]), _t(kp[:, :, :cut]), _t(v[:, :cut]),
                                      causal=True, return_state=True)
    # a common scale on the carried sums and the new keys cancels in the ratio
    scale = np.full((B, Hkv), 0.25)
    o2, _ = kernels.linear_attention(_t(qp[:, :, cut:]), _t(kp[:, :, cut:] * 0.25),
                                     _t(v[:, cut:]), causal=True, state=st,
                                     state_scale=_t(scale), return_state=True)
    stepped = np.concatenate([_np(o1), _np(o2)], axis=1)
    assert np.max(np.abs(stepped - full)) <= 1e-4
    kv_ref = np.einsum("bhsf,bshd->bhfd", kp, v)
    assert np.max(np.abs(_np(st[0]) - np.einsum("bhsf,bshd->bhfd", kp[:, :, :cut],
                                                 v[:, :cut]))) <= 1e-3
    assert kv_ref.shape == tuple(st[0].shape)


@pytest.fixture
def float64():
    enl.use_float64(True)
    yield
    enl.use_float64(False)


def _golden(golden_dir):
    data = np.load(golden_dir / "linear_layers.npz")
    return data, json.loads(str(data["meta"]))


def test_linear_layers_match_reference(cuda, golden_dir, float64):
    data, meta = _golden(golden_dir)
    for i, cfg in enumerate(meta["mha"]):
        enl.set_seed(2200 + i)
        m = enl.AttentionNet()
        m.add_multihead_attention(**cfg)
        x = np.random.RandomState(2300 + i).standard_normal((2, 40, cfg["embed_dim"]))
        err = float(np.max(np.abs(m.Forward(x, training=False) - data[f"mha{i}_y"])))
        assert err <= TOL, (cfg, err)


def _kv_model(i, cfg):
    enl.set_seed(2400 + i)
    m = enl.AttentionNet()
    m.add_embedding(vocab_size=17, embed_dim=64)
    if cfg["positional_scheme"] == "absolute":
        m.add_positional_encoding(max_seq_len=32, learnable=False)
    m.add_transformer_block(64, num_heads=4, causal=True, **cfg)
    m.add_layernorm()
    m.add_dense(n_out=17, activation="linear")
    return m, np.random.RandomState(2500 + i).randint(0, 17, size=(3, 9))


def test_linear_kv_stepping_matches_reference(cuda, golden_dir, float64):
    """Prime 4 tokens, then 5 single steps (nn/kvcache.py:217-260): equal to the
    reference's stepped outputs and its full Forward; the state lives in
    cache.linear, no K/V cache grows."""
    data, meta = _golden(golden_dir)
    for i, cfg in enumerate(meta["kv"]):
        m, toks = _kv_model(i, cfg)
        full = m.Forward(toks, training=False)
        assert np.max(np.abs(full - data[f"kv{i}_full"])) <= TOL, cfg
        cache = enl.KVCache()
        pieces = [enl.cached_forward_step(m, toks[:, :4], cache)]
        pieces += [enl.cached_forward_step(m, toks[:, j:j + 1], cache) for j in range(4, 9)]
        stepped = np.concatenate(pieces, axis=1)
        assert np.max(np.abs(stepped - data[f"kv{i}_stepped"])) <= TOL, cfg
        assert len(cache.kv) == 0 and len(cache.linear) == 1


def test_linear_kv_reorder_matches_reference(cuda, golden_dir, float64):
    data, meta = _golden(golden_dir)
    for i, cfg in enumerate(meta["kv"]):
        m, toks = _kv_model(i, cfg)
        cache = enl.KVCache()
        enl.cached_forward_step(m, toks[:1, :4], cache)
        cache.expand(3)
        enl.cached_forward_step(m, np.array([[5], [6], [7]]), cache)
        cache.reorder([2, 2, 0])
        out = enl.cached_forward_step(m, np.array([[9], [9], [9]]), cache)
        assert np.max(np.abs(out - data[f"kv{i}_reordered"])) <= TOL, cfg
        assert np.allclose(out[0], out[1], atol=1e-6)


@pytest.mark.parametrize("S,cut", [(1500, 700), (2100, 1030)])
def test_segmented_carried_state_equals_one_pass(cuda, S, cut):
    """Long calls run in sequence segments (per-segment sums, a scan that
    starts from the carried, scaled state, then the outputs): split at `cut`
    with the state handed over, they equal one pass, and the returned state
    is the total."""
    from enilnets_b200 import _native, kernels
    rng = np.random.RandomState(S)
    B, H, Hkv, D, Df = 2, 4, 2, 64, 48
    qp = np.exp(rng.standard_normal((B, H, S, Df)) * 0.5)
    kp = np.exp(rng.standard_normal((B, Hkv, S, Df)) * 0.5)
    v = rng.standard_normal((B, S, Hkv, D))
    full, st_full = kernels.linear_attention(_t(qp), _t(kp), _t(v), causal=True,
                                             return_state=True)
    o1, st = kernels.linear_attention(_t(qp[:, :, :cut]), _t(kp[:, :, :cut]), _t(v[:, :cut]),
                                      causal=True, return_state=True)
    scale = np.full((B, Hkv), 0.5)
    o2, st2 = kernels.linear_attention(_t(qp[:, :, cut:]), _t(kp[:, :, cut:] * 0.5),
                                       _t(v[:, cut:]), causal=True, state=st,
                                       state_scale=_t(scale), return_state=True)
    torch_sync()
    _native.raise_on_device_error()
    stepped = np.concatenate([_np(o1), _np(o2)], axis=1)
    assert np.max(np.abs(stepped - _np(full))) <= 1e-4
    kv_ref = np.einsum("bhsf,bshd->bhfd", kp, v)
    assert np.max(np.abs(_np(st_full[0]) - kv_ref)) <= 1e-3 * np.abs(kv_ref).max()
    assert np.max(np.abs(_np(st2[0]) - 0.5 * kv_ref)) <= 1e-3 * np.abs(kv_ref).max()
    ref, _, _ = lr.linear_attention(qp, np.repeat(kp, 2, axis=1),
                                    np.repeat(v.transpose(0, 2, 1, 3), 2, axis=1), True)
    assert np.max(np.abs(_np(full).transpose(0, 2, 1, 3) - ref)) <= 1e-4


def _split_planes(phi):
    """fp32 (B, H, S, Df) -> its bf16 (hi, lo) planes, as the kernels write them."""
    import torch
    hi = phi.to(torch.bfloat16)
    return torch.stack([hi, (phi - hi.float()).to(torch.bfloat16)])


@pytest.mark.parametrize("kernel,Dh,Df", [
    ("linear", 64, 64), ("linear", 36, 36),        # vectorised map, planes written directly
    ("linear", 6, 6),                              # scalar map: fp32 in the workspace, then split
    ("performer", 64, 256), ("performer", 32, 36),  # tensor-core map (36: a half-used 16-byte unit)
    ("performer", 64, 512)])                       # CUDA-core map, then split
def test_feature_map_planes_equal_split_fp32(cuda, kernel, Dh, Df):
    """The planes a map writes are exactly bf16(phi), bf16(phi - bf16(phi)) of
    its fp32 phi, and linear attention over them is bit-identical to the fp32
    call (the same planes reach the same kernels)."""
    import torch
    from enilnets_b200 import _native, kernels
    rng = np.random.RandomState(Dh * 7 + Df)
    B, S, H = 2, 133, 2
    x, xk = _t(rng.standard_normal((B, S, H, Dh))), _t(rng.standard_normal((B, S, H, Dh)))
    v = _t(rng.standard_normal((B, S, H, 40)))
    om = _t(lr.make_projection(Df, Dh, np.random.RandomState(Dh))) if kernel == "performer" \
        else None
    q32, _ = kernels.linear_feature_map(x, kernel, om)
    qpl, _ = kernels.linear_feature_map(x, kernel, om, planes=True)
    k32, st32 = kernels.linear_feature_map(xk, kernel, om, global_stab=True)
    kpl, stpl = kernels.linear_feature_map(xk, kernel, om, global_stab=True, planes=True)
    Dfp = (Df + 7) // 8 * 8
    assert tuple(qpl.shape) == (2, B, H, S, Dfp) and qpl.dtype == torch.bfloat16
    assert torch.equal(qpl[..., :Df], _split_planes(q32))
    assert torch.equal(kpl[..., :Df], _split_planes(k32))
    if st32 is not None:
        assert torch.equal(st32, stpl)
    o32 = kernels.linear_attention(q32, k32, v, causal=True)
    opl = kernels.linear_attention(qpl, kpl, v, causal=True, num_features=Df)
    torch_sync()
    _native.raise_on_device_error()
    assert torch.equal(o32, opl)


def test_linear_attention_planes_argument_errors(cuda):
    import torch
    from enilnets_b200 import kernels
    x = _t(np.random.RandomState(0).standard_normal((1, 16, 2, 32)))
    v = _t(np.random.RandomState(1).standard_normal((1, 16, 2, 32)))
    qpl, _ = kernels.linear_feature_map(x, "linear", planes=True)
    with pytest.raises(ValueError, match="num_features"):
        kernels.linear_attention(qpl, qpl, v, causal=True)
    with pytest.raises(ValueError, match="do not hold"):
        kernels.linear_attention(qpl, qpl, v, causal=True, num_features=20)
    assert not kernels.linear_planes_ok(160, 32) and kernels.linear_planes_ok(128, 1024)
