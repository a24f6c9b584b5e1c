"""K1 prefill kernel parity: the tcgen05 kernel through the C ABI against the
float64 oracle and the reference's golden vectors.

Tolerance (the north-star bar for bf16 inputs): max abs error <= 2e-2 against
the float64 result computed on the same bf16-rounded inputs."""
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


def _run(q, k, v, **kw):
    import torch
    from enilnets_b200 import kernels, _native
    lens = kw.pop("kv_valid_len", None)
    slopes = kw.pop("alibi", None)
    out, lse = kernels.attention_prefill(
        _dev(q), _dev(k), _dev(v),
        kv_valid_len=None if lens is None else torch.tensor(lens, dtype=torch.int32).cuda(),
        alibi_slopes=None if slopes is None else torch.tensor(slopes, dtype=torch.float32).cuda(),
        out_dtype=torch.float32, return_lse=True, **kw)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    return out.cpu().numpy().astype(np.float64), lse.cpu().numpy().astype(np.float64)


def _check(q, k, v, rows=None, **kw):
    kw_ref = dict(kw)
    o, lse = _run(q, k, v, **kw)
    oref, lref = ref.attention_ref(q, k, v, alibi=kw_ref.pop("alibi", None), **kw_ref)
    finite = np.isfinite(oref)
    assert np.array_equal(finite, np.isfinite(o)), "NaN pattern differs from the reference"
    err = np.max(np.abs(o[finite] - oref[finite])) if finite.any() else 0.0
    assert err <= TOL, f"max abs err {err:.3e} > {TOL} for {kw}"
    lf = np.isfinite(lref)
    if kw.get("mask_mode", "exclude") == "exclude":
        assert np.max(np.abs(lse[lf] - lref[lf])) <= 2e-2
    return err


def test_golden_prefill_cases(cuda, golden_dir):
    from tests.test_oracle_golden import prefill_case_inputs
    data = np.load(golden_dir / "kernel_prefill.npz")
    meta = json.loads(str(data["meta"]))
    for i, c in enumerate(meta):
        _, qkv = prefill_case_inputs(c)
        kw = dict(causal=c["causal"], window=c["window"])
        if c["kind"] == "nn":
            if c["scheme"] == "alibi":
                kw["alibi"] = ref.alibi_slopes(c["H"])
        else:
            kw["kv_valid_len"] = c["lengths"]
            kw["mask_mode"] = "additive"
        o, _ = _run(qkv, qkv, qkv, **kw)
        y = data[f"y{i}"].astype(np.float64)
        err = np.max(np.abs(o.reshape(y.shape) - y))
        assert err <= TOL, f"case {c}: max abs err {err:.3e}"


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_random_shapes_partial_tiles(cuda, D, causal):
    rng = np.random.RandomState(D + causal)
    for (B, Sq, Skv, H, Hkv) in [(1, 1, 1, 1, 1), (2, 77, 77, 2, 1), (1, 300, 300, 4, 2),
                                 (2, 129, 383, 2, 2)]:
        if causal and Sq != Skv:
            continue
        q = ref.seeded_normal(rng.randint(1 << 30), (B, Sq, H, D))
        k = ref.seeded_normal(rng.randint(1 << 30), (B, Skv, Hkv, D))
        v = ref.seeded_normal(rng.randint(1 << 30), (B, Skv, Hkv, D))
        _check(q, k, v, causal=causal)


def test_window_alibi_and_offsets(cuda):
    D = 64
    q = ref.seeded_normal(1, (2, 200, 4, D))
    k = ref.seeded_normal(2, (2, 260, 2, D))
    v = ref.seeded_normal(3, (2, 260, 2, D))
    slopes = ref.alibi_slopes(4)
    # multi-token cached step: queries at positions 60.., keys at 0.. (nn/kvcache.py:190-208)
    _check(q, k, v, causal=True, q_pos0=60, k_pos0=0)
    _check(q, k, v, causal=True, window=33, q_pos0=60, k_pos0=0, alibi=slopes)
    _check(q, k, v, causal=False, window=50, alibi=slopes)
    _check(q, k, v, causal=False, alibi=slopes, scale=0.05)


def test_key_padding_additive_semantics(cuda):
    D = 128
    q = ref.seeded_normal(4, (3, 260, 2, D))
    k = ref.seeded_normal(5, (3, 260, 2, D))
    v = ref.seeded_normal(6, (3, 260, 2, D))
    for causal in (False, True):
        for window in (None, 17):
            _check(q, k, v, causal=causal, window=window, kv_valid_len=[260, 100, 0],
                   mask_mode="additive")
            _check(q, k, v, causal=causal, window=window, kv_valid_len=[260, 100, 1],
                   mask_mode="exclude")


def test_garbage_in_padding_does_not_change_real_keys(cuda):
    # graph/sequence.py padding contract (reference test_enilnets.py:6791-6801).
    D = 64
    q = ref.seeded_normal(7, (2, 150, 2, D))
    k = ref.seeded_normal(8, (2, 150, 2, D))
    v = ref.seeded_normal(9, (2, 150, 2, D))
    lens = [150, 61]
    o1, _ = _run(q, k, v, kv_valid_len=lens, mask_mode="additive", causal=True)
    k2, v2 = k.copy(), v.copy()
    k2[1, 61:] = 999.0
    v2[1, 61:] = -999.0
    o2, _ = _run(q, k2, v2, kv_valid_len=lens, mask_mode="additive", causal=True)
    assert np.array_equal(o1, o2)


def test_query_zero_of_causal_stream_is_v0(cuda):
    q = ref.seeded_normal(10, (1, 130, 1, 64))
    k = ref.seeded_normal(11, (1, 130, 1, 64))
    v = ref.seeded_normal(12, (1, 130, 1, 64))
    o, _ = _run(q, k, v, causal=True)
    np.testing.assert_allclose(o[0, 0, 0], v[0, 0, 0], atol=1e-6)


def test_strided_projection_layout(cuda):
    """Q/K/V as head-split views of one (B, S, 3E) projection buffer."""
    import torch
    from enilnets_b200 import kernels
    B, S, H, D = 2, 140, 2, 64
    E = H * D
    x = ref.seeded_normal(13, (B, S, 3 * E))
    t = _dev(x)
    q = t[:, :, :E].view(B, S, H, D)
    k = t[:, :, E:2 * E].view(B, S, H, D)
    v = t[:, :, 2 * E:].view(B, S, H, D)
    out = torch.empty((B, S, H, D), dtype=torch.float32, device="cuda")
    kernels.attention_prefill(q, k, v, causal=True, out=out)
    torch.cuda.synchronize()
    xs = x.reshape(B, S, 3, H, D)
    oref, _ = ref.attention_ref(xs[:, :, 0], xs[:, :, 1], xs[:, :, 2], causal=True)
    assert np.max(np.abs(out.cpu().numpy() - oref)) <= TOL


def test_config2_shape_sampled_rows(cuda):
    """BASELINE config 2 at full size (B8 S4096 H16 D128, causal, key padding
    L~U[2048,4096]); the oracle checks a sample of rows in every batch."""
    import torch
    from enilnets_b200 import kernels
    B, S, H, D = 8, 4096, 16, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn((B, S, H, D), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((B, S, H, D), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((B, S, H, D), generator=g, device="cuda").to(torch.bfloat16)
    lens = np.random.RandomState(2).randint(2048, 4097, size=B)
    out = kernels.attention_prefill(q, k, v, causal=True, mask_mode="additive",
                                    kv_valid_len=torch.tensor(lens, dtype=torch.int32).cuda(),
                                    out_dtype=torch.float32)
    torch.cuda.synchronize()
    rows = np.array([0, 1, 127, 128, 1000, 2047, 2048, 3000, 4095])
    qh = q.float().cpu().numpy()
    kh = k.float().cpu().numpy()
    vh = v.float().cpu().numpy()
    oh = out.cpu().numpy()
    for b in range(B):
        for h in (0, 7, 15):
            for r in rows:
                o_r, _ = ref.attention_ref(qh[b:b + 1, r:r + 1, h:h + 1], kh[b:b + 1, :, h:h + 1],
                                           vh[b:b + 1, :, h:h + 1], causal=True, q_pos0=r,
                                           kv_valid_len=[lens[b]], mask_mode="additive")
                err = np.max(np.abs(o_r[0, 0, 0] - oh[b, r, h]))
                assert err <= TOL, (b, h, r, err)


def test_unit_list_computes_exactly_those_units(cuda):
    """K1 over a rank's (batch, head) units (sharding.contiguous_partition):
    listed units equal the full run bit for bit; the rows of other units are
    never written."""
    import torch
    from enilnets_b200 import kernels, _native
    B, S, H, D = 3, 300, 4, 128
    q, k, v = (_dev(ref.seeded_normal(70 + i, (B, S, H, D))) for i in range(3))
    lens = torch.tensor([300, 170, 41], dtype=torch.int32).cuda()
    full = kernels.attention_prefill(q, k, v, causal=True, kv_valid_len=lens,
                                     mask_mode="additive")
    units = [1, 6, 7, 11]
    out = torch.full_like(full, 7.0)
    kernels.attention_prefill(q, k, v, causal=True, kv_valid_len=lens, mask_mode="additive",
                              out=out, units=torch.tensor(units, dtype=torch.int32).cuda())
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    for u in range(B * H):
        b, h = divmod(u, H)
        if u in units:
            assert torch.equal(out[b, :, h], full[b, :, h]), f"unit {u}"
        else:
            assert bool((out[b, :, h] == 7.0).all()), f"unit {u} was written"
