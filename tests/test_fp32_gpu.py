"""fp32 inputs (the split-bf16 tensor-core path of K1 and the fp32 decode of
K2) and head dims other than 64/128, against the float64 oracle on the same
inputs.

Tolerances: max abs error <= 1e-3 for fp32 inputs,
<= 2e-2 for bf16 inputs, on unit-variance activations."""
import numpy as np
import pytest

from oracle import attention_ref as ref

pytestmark = pytest.mark.gpu
TOL_F32 = 1e-3
TOL_BF16 = 2e-2


def _t(x, dtype):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    return t.to(dtype)


def _prefill(q, k, v, dtype, **kw):
    import torch
    from enilnets_b200 import _native, kernels
    lens = kw.pop("kv_valid_len", None)
    slopes = kw.pop("alibi", None)
    out, lse = kernels.attention_prefill(
        _t(q, dtype), _t(k, dtype), _t(v, dtype),
        kv_valid_len=None if lens is None else torch.tensor(lens, dtype=torch.int32).cuda(),
        alibi_slopes=None if slopes is None else torch.tensor(slopes, dtype=torch.float32).cuda(),
        out_dtype=torch.float32, return_lse=True, **kw)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    return out.cpu().numpy().astype(np.float64), lse.cpu().numpy().astype(np.float64)


def _check_prefill(q, k, v, dtype, tol, **kw):
    o, lse = _prefill(q, k, v, dtype, **dict(kw))
    kw_ref = dict(kw)
    oref, lref = ref.attention_ref(q, k, v, alibi=kw_ref.pop("alibi", None), **kw_ref)
    finite = np.isfinite(oref)
    assert np.array_equal(finite, np.isfinite(o)), "NaN pattern differs from the reference"
    err = float(np.max(np.abs(o[finite] - oref[finite]))) if finite.any() else 0.0
    assert err <= tol, f"max abs err {err:.3e} > {tol} for {kw}"
    lf = np.isfinite(lref)
    if kw.get("mask_mode", "exclude") == "exclude" and lf.any():
        assert np.max(np.abs(lse[lf] - lref[lf])) <= tol
    return err


def _inputs(seed, B, Sq, Skv, H, Hkv, D, bf16):
    q = ref.seeded_normal(seed, (B, Sq, H, D), bf16=bf16)
    k = ref.seeded_normal(seed + 1, (B, Skv, Hkv, D), bf16=bf16)
    v = ref.seeded_normal(seed + 2, (B, Skv, Hkv, D), bf16=bf16)
    return q, k, v


@pytest.mark.parametrize("D", [16, 32, 64, 96, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_fp32_prefill_shapes(cuda, D, causal):
    import torch
    errs = []
    for i, (B, Sq, Skv, H, Hkv) in enumerate([(1, 1, 1, 1, 1), (2, 77, 77, 2, 1),
                                               (1, 300, 300, 4, 2), (2, 129, 383, 2, 2)]):
        if causal and Sq != Skv:
            continue
        q, k, v = _inputs(100 * D + i, B, Sq, Skv, H, Hkv, D, bf16=False)
        errs.append(_check_prefill(q, k, v, torch.float32, TOL_F32, causal=causal))
    # The split path is far inside the bar; a regression to one bf16 product
    # would show up here long before it crossed 1e-3.
    assert max(errs) < 1e-4, errs


def test_fp32_prefill_masks(cuda):
    import torch
    B, S, H, Hkv, D = 3, 200, 4, 2, 64
    q, k, v = _inputs(7, B, S, S, H, Hkv, D, bf16=False)
    _check_prefill(q, k, v, torch.float32, TOL_F32, causal=True, window=50,
                   alibi=ref.alibi_slopes(H), q_pos0=20, k_pos0=20)
    _check_prefill(q, k, v, torch.float32, TOL_F32, causal=True, kv_valid_len=[200, 130, 1],
                   mask_mode="additive")
    # Fully masked rows under the additive rule (lengths 0): tier semantics.
    _check_prefill(q, k, v, torch.float32, TOL_F32, causal=False, kv_valid_len=[0, 64, 129],
                   mask_mode="additive")


def test_fp32_cross_attention_shape(cuda):
    """Config-4 layout at reduced size: non-causal, Sq != Skv, key padding."""
    import torch
    B, Sq, Skv, H, D = 2, 256, 512, 4, 64
    q, k, v = _inputs(11, B, Sq, Skv, H, H, D, bf16=False)
    _check_prefill(q, k, v, torch.float32, TOL_F32, kv_valid_len=[512, 300],
                   mask_mode="additive")


@pytest.mark.parametrize("D", [16, 32, 96])
def test_bf16_prefill_small_head_dims(cuda, D):
    import torch
    for causal in (False, True):
        q, k, v = _inputs(50 + D, 2, 190, 190, 4, 2, D, bf16=True)
        _check_prefill(q, k, v, torch.bfloat16, TOL_BF16, causal=causal)
        _check_prefill(q, k, v, torch.bfloat16, TOL_BF16, causal=causal,
                       kv_valid_len=[190, 77], mask_mode="additive")


def test_fp32_prefill_strided_qkv_views(cuda):
    """fp32 Q/K/V as head views of one fused projection output (B, S, 3E)."""
    import torch
    from enilnets_b200 import kernels
    B, S, H, D = 2, 150, 4, 32
    E = H * D
    qkv = np.random.RandomState(3).standard_normal((B, S, 3 * E)).astype(np.float32)
    t = torch.from_numpy(qkv).cuda()
    q = t[..., :E].unflatten(-1, (H, D))
    k = t[..., E:2 * E].unflatten(-1, (H, D))
    v = t[..., 2 * E:].unflatten(-1, (H, D))
    out = kernels.attention_prefill(q, k, v, causal=True, out_dtype=torch.float32)
    torch.cuda.synchronize()
    qn = qkv[..., :E].reshape(B, S, H, D).astype(np.float64)
    kn = qkv[..., E:2 * E].reshape(B, S, H, D).astype(np.float64)
    vn = qkv[..., 2 * E:].reshape(B, S, H, D).astype(np.float64)
    oref, _ = ref.attention_ref(qn, kn, vn, causal=True)
    assert np.max(np.abs(out.cpu().numpy() - oref)) <= TOL_F32


def test_fp32_prefill_rejects_missing_workspace(cuda):
    import ctypes
    import torch
    from enilnets_b200 import _native as nat
    q = torch.zeros((1, 8, 1, 64), dtype=torch.float32, device="cuda")
    o = torch.zeros_like(q)
    a = nat.PrefillArgs()
    a.q = a.k = a.v = q.data_ptr()
    a.o = o.data_ptr()
    a.batch = a.num_heads = a.num_kv_heads = 1
    a.seq_q = a.seq_kv = 8
    a.head_dim = 64
    a.q_stride_b = a.k_stride_b = a.v_stride_b = a.o_stride_b = 8 * 64
    a.q_stride_s = a.k_stride_s = a.v_stride_s = a.o_stride_s = 64
    a.q_stride_h = a.k_stride_h = a.v_stride_h = a.o_stride_h = 64
    a.in_dtype = a.out_dtype = nat.ENL_DTYPE_FP32
    a.scale = 0.125
    lib = nat.load()
    # (hi, lo) planes of q, k and v: 3 x (8 rows x 2 planes x 64 x 2 bytes)
    assert lib.enl_prefill_workspace_bytes(ctypes.byref(a)) == 3 * 8 * 2 * 64 * 2
    st = lib.enl_attn_prefill(ctypes.byref(a), None)
    assert st == nat.ENL_ERR_INVALID
    assert b"workspace" in lib.enl_last_error()


@pytest.mark.parametrize("D", [32, 128])
@pytest.mark.parametrize("G", [1, 4])
def test_fp32_decode(cuda, D, G):
    import torch
    from enilnets_b200 import _native, kernels
    B, Hkv, cap = 3, 2, 1500
    H = Hkv * G
    q = ref.seeded_normal(D + G, (B, H, D), bf16=False)
    K = ref.seeded_normal(D + G + 1, (B, Hkv, cap, D), bf16=False)
    V = ref.seeded_normal(D + G + 2, (B, Hkv, cap, D), bf16=False)
    for splits, kw in ((1, {}), (0, {}), (5, dict(window=300, alibi=ref.alibi_slopes(H)))):
        slopes = kw.get("alibi")
        o, lse = kernels.attention_decode(
            _t(q, torch.float32), _t(K, torch.float32), _t(V, torch.float32), slot_begin=3,
            slot_end=1400, pos_slot0=10, q_pos=1200, window=kw.get("window"),
            alibi_slopes=None if slopes is None else _t(slopes, torch.float32),
            n_splits=splits, out_dtype=torch.float32, return_lse=True)
        torch.cuda.synchronize()
        _native.raise_on_device_error()
        oref, lref = ref.decode_ref(q, K, V, slot_begin=3, slot_end=1400, pos_slot0=10,
                                    q_pos=1200, **kw)
        assert np.max(np.abs(o.cpu().numpy() - oref)) <= TOL_F32, (splits, kw)
        assert np.max(np.abs(lse.cpu().numpy() - lref)) <= TOL_F32, (splits, kw)
