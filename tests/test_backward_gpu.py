"""Attention backward (K5, enl_backward.cu) on the GPU.

dQ, dK, dV from the forward's LSE against the float64 oracle
(oracle/attention_ref.attention_backward_ref) on the bf16 values the kernels
read, and against the reference's own flash_attention_backward outputs
(tests/golden/flash_backward.npz). bf16 operands with fp32 accumulation:
max abs error <= 2e-2 relative to the gradient's largest magnitude (the
north-star bar for bf16 inputs)."""
import json

import numpy as np
import pytest

from oracle import attention_ref as ar

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _np(t):
    return t.float().cpu().numpy().astype(np.float64)


def _run(cuda, q, k, v, do, causal, window, slopes):
    import torch
    from enilnets_b200 import kernels, _native
    qt, kt, vt, dot = (torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
                       .to(torch.bfloat16) for a in (q, k, v, do))
    sl = torch.tensor(slopes, dtype=torch.float32, device=cuda) if slopes is not None else None
    o, lse = kernels.attention_prefill(qt, kt, vt, causal=causal, window=window,
                                       alibi_slopes=sl, out_dtype=torch.float32,
                                       return_lse=True)
    dq, dk, dv = kernels.attention_backward(qt, kt, vt, o, lse, dot, causal=causal,
                                            window=window, alibi_slopes=sl)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    return (qt, kt, vt, dot), (dq, dk, dv)


def _check(got, ref, what):
    for name, g, r in zip(("dq", "dk", "dv"), got, ref):
        err = np.max(np.abs(_np(g) - r))
        assert err <= TOL * max(1.0, np.abs(r).max()), (what, name, err, np.abs(r).max())


CASES = [
    # B, S, H, Hkv, D, causal, window, alibi
    (1, 128, 1, 1, 64, False, None, False),
    (2, 300, 2, 2, 64, True, None, False),
    (1, 517, 4, 2, 128, True, None, True),
    (1, 700, 2, 1, 128, False, 100, False),
    (2, 257, 3, 3, 32, False, None, True),
    (1, 1024, 2, 2, 128, True, 300, False),
    (1, 200, 8, 1, 16, True, None, False),
]


@pytest.mark.parametrize("B,S,H,Hkv,D,causal,window,alibi", CASES)
def test_backward_matches_oracle(cuda, B, S, H, Hkv, D, causal, window, alibi):
    rs = np.random.RandomState(S + D + H)
    q = rs.standard_normal((B, S, H, D))
    k = rs.standard_normal((B, S, Hkv, D))
    v = rs.standard_normal((B, S, Hkv, D))
    do = rs.standard_normal((B, S, H, D))
    slopes = ar.alibi_slopes(H) if alibi else None
    ins, got = _run(cuda, q, k, v, do, causal, window, slopes)
    qn, kn, vn, don = (_np(t) for t in ins)  # the values the kernels saw
    ref = ar.attention_backward_ref(qn, kn, vn, don, causal=causal, window=window,
                                    alibi=slopes)
    _check(got, ref, (B, S, H, Hkv, D, causal, window, alibi))


def test_backward_matches_reference(cuda, golden_dir):
    data = np.load(golden_dir / "flash_backward.npz")
    meta = json.loads(str(data["meta"]))
    for i, c in enumerate(meta):
        rs = np.random.RandomState(4000 + i)
        shape = (c["B"], c["H"], c["S"], c["Dh"])
        q, k, v, do = (rs.standard_normal(shape).transpose(0, 2, 1, 3) for _ in range(4))
        slopes = ar.alibi_slopes(c["H"]) if c["alibi"] else None
        _, got = _run(cuda, q, k, v, do, c["causal"], c["window"], slopes)
        ref = [data[f"{n}{i}"].transpose(0, 2, 1, 3).astype(np.float64)
               for n in ("dq", "dk", "dv")]
        # the reference ran on float64 inputs; the kernels read them as bf16
        for name, g, r in zip(("dq", "dk", "dv"), got, ref):
            err = np.max(np.abs(_np(g) - r))
            assert err <= 3 * TOL * max(1.0, np.abs(r).max()), (c, name, err)


def test_backward_cross_shapes_match_oracle(cuda):
    """Queries and keys of different lengths (positions both from 0), as a
    cross-attention layer would call it; GQA and ALiBi on."""
    rs = np.random.RandomState(11)
    B, Sq, Skv, H, Hkv, D = 2, 200, 333, 4, 2, 64
    q = rs.standard_normal((B, Sq, H, D))
    k = rs.standard_normal((B, Skv, Hkv, D))
    v = rs.standard_normal((B, Skv, Hkv, D))
    do = rs.standard_normal((B, Sq, H, D))
    slopes = ar.alibi_slopes(H)
    ins, got = _run(cuda, q, k, v, do, False, None, slopes)
    qn, kn, vn, don = (_np(t) for t in ins)
    ref = ar.attention_backward_ref(qn, kn, vn, don, causal=False, window=None, alibi=slopes)
    _check(got, ref, "cross")


def test_backward_strided_outputs_equal_contiguous(cuda):
    """Outputs written into views whose row strides are not multiples of four
    floats take the scalar epilogue; they equal the contiguous outputs."""
    import torch
    from enilnets_b200 import kernels
    rs = np.random.RandomState(12)
    B, S, H, D = 1, 300, 2, 128
    q, k, v, do = (torch.from_numpy(rs.standard_normal((B, S, H, D)).astype(np.float32))
                   .cuda().to(torch.bfloat16) for _ in range(4))
    o, lse = kernels.attention_prefill(q, k, v, causal=True, out_dtype=torch.float32,
                                       return_lse=True)
    ref = kernels.attention_backward(q, k, v, o, lse, do, causal=True)
    wide = [torch.full((B, S, H, D + 2), float("nan"), device=cuda) for _ in range(3)]
    views = tuple(w[..., :D] for w in wide)
    got = kernels.attention_backward(q, k, v, o, lse, do, causal=True, out=views)
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    torch.cuda.synchronize()


# fp32 operands (split-bf16, three MMAs per product): the reference's float32
# models at their own precision. Bar: 1e-3 relative to the gradient's largest
# magnitude (the north-star bar for fp32 inputs).
TOL32 = 1e-3
CASES32 = [
    # B, S, H, Hkv, D, causal, window, alibi
    (2, 300, 2, 2, 64, True, None, False),
    (2, 257, 3, 3, 32, False, None, True),
    (1, 200, 8, 1, 16, True, None, False),
    (1, 700, 2, 1, 64, False, 100, False),
    (2, 190, 4, 2, 40, True, None, True),
    (1, 129, 2, 2, 8, True, 5, True),
]


def _run32(cuda, q, k, v, do, causal, window, slopes):
    import torch
    from enilnets_b200 import kernels, _native
    qt, kt, vt, dot = (torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
                       for a in (q, k, v, do))
    sl = torch.tensor(slopes, dtype=torch.float32, device=cuda) if slopes is not None else None
    o, lse = kernels.attention_prefill(qt, kt, vt, causal=causal, window=window,
                                       alibi_slopes=sl, out_dtype=torch.float32,
                                       return_lse=True)
    dq, dk, dv = kernels.attention_backward(qt, kt, vt, o, lse, dot, causal=causal,
                                            window=window, alibi_slopes=sl)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    return (qt, kt, vt, dot), (dq, dk, dv)


@pytest.mark.parametrize("B,S,H,Hkv,D,causal,window,alibi", CASES32)
def test_backward_fp32_matches_oracle(cuda, B, S, H, Hkv, D, causal, window, alibi):
    rs = np.random.RandomState(7 * S + D + H)
    q = rs.standard_normal((B, S, H, D))
    k = rs.standard_normal((B, S, Hkv, D))
    v = rs.standard_normal((B, S, Hkv, D))
    do = rs.standard_normal((B, S, H, D))
    slopes = ar.alibi_slopes(H) if alibi else None
    ins, got = _run32(cuda, q, k, v, do, causal, window, slopes)
    qn, kn, vn, don = (_np(t) for t in ins)  # the fp32 values the kernels saw
    ref = ar.attention_backward_ref(qn, kn, vn, don, causal=causal, window=window,
                                    alibi=slopes)
    for name, g, r in zip(("dq", "dk", "dv"), got, ref):
        err = np.max(np.abs(_np(g) - r))
        assert err <= TOL32 * max(1.0, np.abs(r).max()), (name, err, np.abs(r).max())


def test_backward_fp32_matches_reference(cuda, golden_dir):
    """The reference's own flash_attention_backward outputs at head dims up to
    64, from fp32 copies of its float64 inputs, at the fp32 bar."""
    data = np.load(golden_dir / "flash_backward.npz")
    meta = json.loads(str(data["meta"]))
    ran = 0
    for i, c in enumerate(meta):
        if c["Dh"] > 64:
            continue
        rs = np.random.RandomState(4000 + i)
        shape = (c["B"], c["H"], c["S"], c["Dh"])
        q, k, v, do = (rs.standard_normal(shape).transpose(0, 2, 1, 3) for _ in range(4))
        slopes = ar.alibi_slopes(c["H"]) if c["alibi"] else None
        _, got = _run32(cuda, q, k, v, do, c["causal"], c["window"], slopes)
        ref = [data[f"{n}{i}"].transpose(0, 2, 1, 3).astype(np.float64)
               for n in ("dq", "dk", "dv")]
        for name, g, r in zip(("dq", "dk", "dv"), got, ref):
            err = np.max(np.abs(_np(g) - r))
            assert err <= TOL32 * max(1.0, np.abs(r).max()), (c, name, err)
        ran += 1
    assert ran == 9


def test_backward_fp32_rejects_wide_heads_and_mixed_dtypes(cuda):
    import torch
    from enilnets_b200 import kernels
    B, S, H, D = 1, 64, 1, 128
    x = torch.zeros((B, S, H, D), device=cuda)
    lse = torch.zeros((B, H, S), device=cuda)
    with pytest.raises(ValueError, match="head_dim <= 64"):
        kernels.attention_backward(x, x, x, x, lse, x)
    xb = x[..., :64].contiguous()
    with pytest.raises(ValueError, match="dout must be"):
        kernels.attention_backward(xb, xb, xb, xb, lse, xb.to(torch.bfloat16))


def test_backward_fp32_cross_shapes_and_strided_outputs(cuda):
    """fp32 operands with queries and keys of different lengths, GQA and
    ALiBi, at the fp32 bar; outputs written into strided views equal the
    contiguous ones bit for bit."""
    import torch
    from enilnets_b200 import kernels
    rs = np.random.RandomState(13)
    B, Sq, Skv, H, Hkv, D = 2, 200, 333, 4, 2, 48
    q = rs.standard_normal((B, Sq, H, D))
    k = rs.standard_normal((B, Skv, Hkv, D))
    v = rs.standard_normal((B, Skv, Hkv, D))
    do = rs.standard_normal((B, Sq, H, D))
    slopes = ar.alibi_slopes(H)
    ins, got = _run32(cuda, q, k, v, do, False, None, slopes)
    qn, kn, vn, don = (_np(t) for t in ins)
    ref = ar.attention_backward_ref(qn, kn, vn, don, causal=False, window=None, alibi=slopes)
    for name, g, r in zip(("dq", "dk", "dv"), got, ref):
        err = np.max(np.abs(_np(g) - r))
        assert err <= TOL32 * max(1.0, np.abs(r).max()), (name, err)
    qt, kt, vt, dot = ins
    sl = torch.tensor(slopes, dtype=torch.float32, device=cuda)
    o, lse = kernels.attention_prefill(qt, kt, vt, alibi_slopes=sl, out_dtype=torch.float32,
                                       return_lse=True)
    base = kernels.attention_backward(qt, kt, vt, o, lse, dot, alibi_slopes=sl)
    wide = [torch.full((B, S, Hh, D + 3), float("nan"), device=cuda)
            for S, Hh in ((Sq, H), (Skv, Hkv), (Skv, Hkv))]
    views = tuple(w[..., :D] for w in wide)
    strided = kernels.attention_backward(qt, kt, vt, o, lse, dot, alibi_slopes=sl, out=views)
    torch.cuda.synchronize()
    for a, b in zip(strided, base):
        assert torch.equal(a, b)
