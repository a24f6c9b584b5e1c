"""K2 decode, LSE merge, K3 append, cache gather and RoPE kernels through the
C ABI against the float64 oracle and the reference's golden vectors.
Integer/byte work (append, gather) must be bit-exact; floating point within
2e-2 max abs for bf16 inputs."""
import json

import numpy as np
import pytest

from oracle import attention_ref as ref

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _dev(x, dtype="bf16"):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    return t.to(torch.bfloat16) if dtype == "bf16" else t


def _np(t):
    return t.float().cpu().numpy().astype(np.float64)


def _decode(q, K, V, **kw):
    import torch
    from enilnets_b200 import kernels, _native
    slopes = kw.pop("alibi", None)
    out, lse = kernels.attention_decode(
        _dev(q), _dev(K), _dev(V),
        alibi_slopes=None if slopes is None else torch.tensor(slopes, dtype=torch.float32).cuda(),
        out_dtype=torch.float32, return_lse=True, **kw)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    return _np(out), _np(lse)


def test_golden_decode_cases_with_append(cuda, golden_dir):
    """Append the new token with K3, then decode with K2: equals the
    reference's _attention_step (nn/kvcache.py:123-214)."""
    import torch
    from enilnets_b200 import kernels
    from tests.test_oracle_golden import decode_case_inputs
    data = np.load(golden_dir / "kernel_decode.npz")
    meta = json.loads(str(data["meta"]))
    for i, c in enumerate(meta):
        Kc, Vc, q, new = decode_case_inputs(c)
        B, H, Hkv, D, ctx = c["B"], c["H"], c["Hkv"], c["D"], c["ctx"]
        cap = ctx + 64
        kc = torch.zeros((B, Hkv, cap, D), dtype=torch.bfloat16, device="cuda")
        vc = torch.zeros_like(kc)
        kc[:, :, :ctx] = _dev(Kc)
        vc[:, :, :ctx] = _dev(Vc)
        kernels.kv_append(kc, _dev(new), ctx)
        kernels.kv_append(vc, _dev(new), ctx)
        slopes = ref.alibi_slopes(H) if c["scheme"] == "alibi" else None
        out = kernels.attention_decode(
            _dev(q), kc, vc, slot_begin=0, slot_end=ctx + 1, pos_slot0=0, q_pos=ctx,
            window=c["window"], out_dtype=torch.float32,
            alibi_slopes=None if slopes is None else torch.tensor(slopes, dtype=torch.float32).cuda())
        torch.cuda.synchronize()
        y = data[f"y{i}"].astype(np.float64).reshape(B, H, D)
        err = np.max(np.abs(_np(out) - y))
        assert err <= TOL, f"case {c}: {err:.3e}"


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("G", [1, 2, 4, 8])
def test_random_decode_all_group_sizes(cuda, D, G):
    Hkv = 2
    H = Hkv * G
    B, ctx = 3, 1000
    q = ref.seeded_normal(D + G, (B, H, D))
    K = ref.seeded_normal(D + G + 1, (B, Hkv, ctx, D))
    V = ref.seeded_normal(D + G + 2, (B, Hkv, ctx, D))
    for splits in (1, 3, 0):
        o, lse = _decode(q, K, V, slot_begin=5, slot_end=997, pos_slot0=100, q_pos=1096,
                         n_splits=splits)
        oref, lref = ref.decode_ref(q, K, V, slot_begin=5, slot_end=997, pos_slot0=100,
                                    q_pos=1096)
        assert np.max(np.abs(o - oref)) <= TOL, splits
        assert np.max(np.abs(lse - lref)) <= 2e-2


def test_decode_alibi_window_and_causal_cut(cuda):
    B, H, Hkv, D, ctx = 2, 4, 4, 128, 700
    q = ref.seeded_normal(21, (B, H, D))
    K = ref.seeded_normal(22, (B, Hkv, ctx, D))
    V = ref.seeded_normal(23, (B, Hkv, ctx, D))
    slopes = ref.alibi_slopes(H)
    # query at position 500: slots after it are invisible even if live
    for kw in (dict(window=None, alibi=slopes), dict(window=37, alibi=None),
               dict(window=100, alibi=slopes)):
        o, _ = _decode(q, K, V, slot_begin=0, slot_end=ctx, pos_slot0=0, q_pos=500, **kw)
        oref, _ = ref.decode_ref(q, K, V, slot_begin=0, slot_end=ctx, pos_slot0=0, q_pos=500,
                                 **kw)
        assert np.max(np.abs(o - oref)) <= TOL, kw


def test_lse_merge_kernel(cuda):
    import torch
    from enilnets_b200 import kernels
    rng = np.random.RandomState(3)
    P, B, H, D = 5, 2, 3, 128
    po = rng.standard_normal((P, B, H, D))
    pl = rng.standard_normal((P, B, H)) * 3
    pl[2, 0, 1] = -np.inf  # a part that saw no key carries no weight
    out, lse = kernels.lse_merge(_dev(po, "f32"), _dev(pl, "f32"), out_dtype=torch.float32,
                                 return_lse=True)
    torch.cuda.synchronize()
    oref, lref = ref.lse_merge_ref(po, pl)
    np.testing.assert_allclose(_np(out), oref, atol=1e-5)
    np.testing.assert_allclose(_np(lse), lref, atol=1e-5)


def test_kv_append_and_gather_are_bit_exact(cuda):
    import torch
    from enilnets_b200 import kernels
    B, Hkv, cap, D = 3, 2, 40, 64
    rng = np.random.RandomState(4)
    cache = torch.from_numpy(rng.standard_normal((B, Hkv, cap, D)).astype(np.float32)).cuda()
    cache = cache.to(torch.bfloat16)
    src_full = torch.from_numpy(rng.standard_normal((B, 5, 3 * Hkv, D)).astype(np.float32))
    src_full = src_full.cuda().to(torch.bfloat16)
    src = src_full[:, :, Hkv:2 * Hkv]  # strided view, like a projection slice
    expect = cache.clone()
    expect[:, :, 17:22] = src.permute(0, 2, 1, 3)
    kernels.kv_append(cache, src, 17)
    torch.cuda.synchronize()
    assert torch.equal(cache, expect)
    index = torch.tensor([2, 2, 0, 1], dtype=torch.int64, device="cuda")
    dst = torch.zeros((4, Hkv, cap, D), dtype=torch.bfloat16, device="cuda")
    kernels.kv_gather(dst, cache, index, 3, 30)
    torch.cuda.synchronize()
    assert torch.equal(dst[:, :, 3:30], cache[index][:, :, 3:30])
    assert torch.count_nonzero(dst[:, :, :3]) == 0 and torch.count_nonzero(dst[:, :, 30:]) == 0


def test_kv_gather_bad_index_sets_device_error(cuda):
    import torch
    from enilnets_b200 import kernels, _native
    _native.device_error(clear=True)
    src = torch.zeros((2, 1, 8, 64), dtype=torch.bfloat16, device="cuda")
    dst = torch.zeros_like(src)
    kernels.kv_gather(dst, src, torch.tensor([0, 5], dtype=torch.int64, device="cuda"), 0, 8)
    code, info = _native.device_error(clear=True)
    assert code == 2 and info == 1


def test_append_rejects_capacity_overflow(cuda):
    import torch
    from enilnets_b200 import kernels
    cache = torch.zeros((1, 1, 8, 64), dtype=torch.bfloat16, device="cuda")
    src = torch.zeros((1, 3, 1, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="exceed capacity"):
        kernels.kv_append(cache, src, 6)


def test_rope_kernel_matches_reference_rotation(cuda):
    import torch
    from enilnets_b200 import kernels
    B, S, H, D = 2, 33, 3, 64
    x = ref.seeded_normal(5, (B, S, H, D))
    cos, sin = ref.rope_tables(100, D)
    t = _dev(x, "f32")
    kernels.rope_(t, _dev(cos, "f32"), _dev(sin, "f32"), 40)
    torch.cuda.synchronize()
    expect = ref.rope_rotate(x.transpose(0, 2, 1, 3), cos[40:73], sin[40:73]).transpose(0, 2, 1, 3)
    np.testing.assert_allclose(_np(t), expect, atol=1e-5)


def test_wait_timeout_is_reported_and_context_survives(cuda):
    """Failure-detection path of every kernel wait: a barrier that nothing
    arrives on runs out its (short) budget, the kernel records the timeout in
    the device error word and returns; the next launch works normally."""
    import torch
    from enilnets_b200 import _native, kernels
    lib = _native.load()
    _native.device_error(clear=True)
    _native.check(lib.enl_selftest_wait_timeout(2_000_000, None), "enl_selftest_wait_timeout")
    code, info = _native.device_error(clear=True)
    assert (code, info) == (1, 99)
    q = torch.randn((1, 64, 2, 64), device="cuda").to(torch.bfloat16)
    o = kernels.attention_prefill(q, q, q, causal=True)
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) == (0, 0)
    assert torch.isfinite(o.float()).all()
    with pytest.raises(ValueError):
        _native.check(lib.enl_selftest_wait_timeout(10 ** 9, None), "enl_selftest_wait_timeout")
