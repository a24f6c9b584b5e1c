"""Block-sparse attention (K1's sparse mode, enl_sparse.cu masks) on the GPU.

- The device-built masks equal the oracle's visibility bit for bit, over
  every listed tile.
- The kernel against the float64 oracle (oracle/sparse_ref.py) on the same
  inputs: bf16 inputs within 2e-2, fp32 inputs (split-bf16 path) within
  1e-3, the north-star bars; patterns with block sizes below, equal to,
  above and not dividing the 128-key tile, ALiBi, GQA, cached-step positions.
- The reference's own outputs (tests/golden/sparse.npz): forward contexts,
  full layers and KV-cache stepping (one token at a time and 5 + 4), 1e-3.
"""
import json

import numpy as np
import pytest

import enilnets_b200 as enl
from enilnets_b200 import sparse as sp
from oracle import sparse_ref as sr
from oracle.attention_ref import alibi_slopes

pytestmark = pytest.mark.gpu
TOL_BF16, TOL_FP32 = 2e-2, 1e-3


def _np(t):
    return t.float().cpu().numpy().astype(np.float64)


def _check_device():
    import torch
    from enilnets_b200 import _native
    torch.cuda.synchronize()
    _native.raise_on_device_error()


MASK_CASES = [
    ({"block_size": 3, "local": 1, "global": 1, "random": 1}, 10, 10, 0, 0, False),
    ({"block_size": 16, "local": 2, "global": 1, "random": 2, "seed": 4}, 300, 300, 0, 0, False),
    ({"block_size": 64, "local": 1, "global": 1}, 700, 700, 0, 0, True),
    ({"block_size": 100, "local": 1, "random": 1}, 333, 333, 0, 0, True),
    ({"block_size": 1, "local": 5, "global": 2}, 200, 200, 0, 0, True),
    ({"block_size": 256, "local": 1}, 600, 600, 0, 0, True),
    ({"block_size": 3, "local": 1, "global": 1, "random": 1}, 1, 9, 8, 0, True),
    ({"block_size": 8, "local": 1, "global": 1}, 3, 40, 200, 163, True),
]


@pytest.mark.parametrize("pat,Sq,Skv,q0,k0,causal", MASK_CASES)
def test_masks_equal_oracle_visibility(cuda, pat, Sq, Skv, q0, k0, causal):
    spec = sp.normalize_pattern(pat)
    lay = sp.build_layout(spec, Sq, Skv, causal=causal, device=cuda, q_pos0=q0, k_pos0=k0)
    n_blocks = (k0 + Skv - 1) // spec["block_size"] + 1
    allow = sr.visibility(spec, np.arange(q0, q0 + Sq), np.arange(k0, k0 + Skv), causal,
                          n_blocks)
    masks = lay.masks[:lay.n_entries].cpu().numpy().view(np.uint64)
    ptr = lay.tile_ptr.cpu().numpy()
    kts = lay.tile_kt[:lay.n_entries].cpu().numpy()
    bits = ((masks[..., None] >> np.arange(64, dtype=np.uint64)) & np.uint64(1)).astype(bool)
    seen = np.zeros_like(allow)
    for t in range(ptr.size - 1):
        rows = slice(t * 128, min(Sq, t * 128 + 128))
        nr = rows.stop - rows.start
        for e in range(ptr[t], ptr[t + 1]):
            got = np.concatenate([bits[e, 0], bits[e, 1]], axis=1)  # (128 rows, 128 keys)
            k_lo = kts[e] * 128
            k_hi = min(Skv, k_lo + 128)
            assert np.array_equal(got[:nr, :k_hi - k_lo], allow[rows, k_lo:k_hi]), (t, e)
            assert not got[nr:].any() and not got[:, k_hi - k_lo:].any()
            seen[rows, k_lo:k_hi] |= got[:nr, :k_hi - k_lo]
    assert np.array_equal(seen, allow)  # nothing allowed lies outside the listed tiles
    _check_device()


KERNEL_CASES = [
    # pattern, S, D, H, Hkv, causal, alibi
    ({"block_size": 64, "local": 1, "global": 1, "random": 2}, 1000, 128, 4, 2, True, False),
    ({"block_size": 64, "local": 1, "global": 1, "random": 2}, 1000, 64, 2, 2, False, False),
    ({"block_size": 128, "local": 2, "global": 1}, 1300, 128, 2, 1, True, True),
    ({"block_size": 16, "local": 3, "random": 4, "seed": 2}, 517, 64, 4, 4, False, True),
    ({"block_size": 200, "local": 1, "global": 1}, 900, 128, 2, 2, True, False),
    ({"block_size": 7, "local": 2, "global": 3, "random": 3}, 450, 32, 3, 1, True, False),
    ({"block_size": 512, "local": 1}, 1536, 64, 2, 2, True, False),
]


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
@pytest.mark.parametrize("pat,S,D,H,Hkv,causal,alibi", KERNEL_CASES)
def test_sparse_kernel_matches_oracle(cuda, dtype, pat, S, D, H, Hkv, causal, alibi):
    import torch
    spec = sp.normalize_pattern(pat)
    rs = np.random.RandomState(S + D)
    q = rs.standard_normal((1, S, H, D)).astype(np.float32)
    k = rs.standard_normal((1, S, Hkv, D)).astype(np.float32)
    v = rs.standard_normal((1, S, Hkv, D)).astype(np.float32)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    qt, kt, vt = (torch.from_numpy(a).cuda().to(tdt) for a in (q, k, v))
    slopes = alibi_slopes(H) if alibi else None
    sl_t = torch.tensor(slopes, dtype=torch.float32, device=cuda) if alibi else None
    out = sp.attention(qt, kt, vt, spec, causal=causal, alibi_slopes=sl_t,
                       out_dtype=torch.float32)
    # the oracle sees the values the kernel saw
    qn, kn, vn = (_np(t).transpose(0, 2, 1, 3) for t in (qt, kt, vt))
    g = H // Hkv
    ref = sr.sparse_attention(qn, np.repeat(kn, g, axis=1), np.repeat(vn, g, axis=1), spec,
                              causal, slopes)
    err = np.max(np.abs(_np(out).transpose(0, 2, 1, 3) - ref))
    assert err <= (TOL_BF16 if dtype == "bf16" else TOL_FP32), err
    _check_device()


@pytest.mark.parametrize("q0,n,k0", [(700, 1, 0), (511, 1, 0), (600, 9, 0), (1000, 1, 389),
                                     (130, 130, 0)])
def test_sparse_step_positions_match_oracle(cuda, q0, n, k0):
    """Cached-step shape: queries [q0, q0 + n) against keys [k0, q0 + n) at
    absolute positions, as nn/kvcache.py:263-306 scores them."""
    import torch
    spec = sp.normalize_pattern({"block_size": 32, "local": 1, "global": 2, "random": 2,
                                 "seed": 1})
    H, D = 4, 64
    Skv = q0 + n - k0
    rs = np.random.RandomState(q0 + n)
    q = torch.from_numpy(rs.standard_normal((2, n, H, D)).astype(np.float32)).cuda()
    k = torch.from_numpy(rs.standard_normal((2, Skv, H, D)).astype(np.float32)).cuda()
    v = torch.from_numpy(rs.standard_normal((2, Skv, H, D)).astype(np.float32)).cuda()
    slopes = alibi_slopes(H)
    out = sp.attention(q, k, v, spec, causal=True, q_pos0=q0, k_pos0=k0,
                       alibi_slopes=torch.tensor(slopes, dtype=torch.float32, device=cuda),
                       out_dtype=torch.float32)
    ref = sr.sparse_step(_np(q).transpose(0, 2, 1, 3), _np(k).transpose(0, 2, 1, 3),
                         _np(v).transpose(0, 2, 1, 3), spec, np.arange(q0, q0 + n),
                         np.arange(k0, k0 + Skv), slopes)
    assert np.max(np.abs(_np(out).transpose(0, 2, 1, 3) - ref)) <= TOL_FP32
    _check_device()


def test_single_block_pattern_equals_dense_attention(cuda):
    """One block over the whole sequence selects everything: the sparse mode
    gives the dense kernel's result (test_enilnets.py:8190-8205). Non-causal,
    every half-tile takes the same path in both, so the results are equal;
    under a causal mask the sparse mode picks the unmasked path per 32-row
    warp rather than per 128-row tile, and that path draws one in four
    exponentials from a polynomial, so the two agree to bf16 rounding of P."""
    import torch
    from enilnets_b200 import kernels
    S, H, D = 700, 2, 128
    rs = np.random.RandomState(0)
    q, k, v = (torch.from_numpy(rs.standard_normal((2, S, H, D)).astype(np.float32))
               .cuda().to(torch.bfloat16) for _ in range(3))
    qn, kn, vn = (_np(t).transpose(0, 2, 1, 3) for t in (q, k, v))
    for causal in (False, True):
        spec = sp.normalize_pattern({"block_size": S})
        a = sp.attention(q, k, v, spec, causal=causal, out_dtype=torch.float32)
        b = kernels.attention_prefill(q, k, v, causal=causal, out_dtype=torch.float32)
        ref = sr.sparse_attention(qn, kn, vn, spec, causal)
        for out in (a, b):
            assert np.max(np.abs(_np(out).transpose(0, 2, 1, 3) - ref)) <= TOL_BF16
        # one bf16 ulp of a probability, in the rows with the fewest keys
        tol = 2e-3 if causal else 0.0
        assert torch.allclose(a, b, atol=tol, rtol=0), (causal, (a - b).abs().max().item())
    _check_device()


@pytest.fixture
def float64():
    enl.use_float64(True)
    yield
    enl.use_float64(False)


@pytest.fixture(scope="module")
def golden(golden_dir):
    data = np.load(golden_dir / "sparse.npz")
    return data, json.loads(str(data["meta"]))


def test_sparse_forward_matches_reference(cuda, golden):
    """The reference's sparse_attention_forward contexts (head dims the kernel
    takes: multiples of 8)."""
    import torch
    data, meta = golden
    n = 0
    for i, c in enumerate(meta["core"]):
        if c["Dh"] % 8:
            continue
        rs = np.random.RandomState(3100 + i)
        shape = (c["B"], c["H"], c["S"], c["Dh"])
        q, k, v = (torch.from_numpy(rs.standard_normal(shape).astype(np.float32))
                   .cuda().permute(0, 2, 1, 3) for _ in range(3))
        slopes = (torch.tensor(alibi_slopes(c["H"]), dtype=torch.float32, device=cuda)
                  if c["alibi"] else None)
        out = sp.attention(q, k, v, sp.normalize_pattern(c["pattern"]), causal=c["causal"],
                           alibi_slopes=slopes, out_dtype=torch.float32)
        err = np.max(np.abs(_np(out).transpose(0, 2, 1, 3) - data[f"core{i}_y"]))
        assert err <= TOL_FP32, (c, err)
        n += 1
    assert n >= 5
    _check_device()


def test_sparse_layers_match_reference(cuda, golden, float64):
    data, meta = golden
    for i, cfg in enumerate(meta["mha"]):
        enl.set_seed(3200 + i)
        m = enl.AttentionNet()
        m.add_multihead_attention(embed_dim=64, num_heads=4, **cfg)
        x = np.random.RandomState(3300 + i).standard_normal((2, 40, 64))
        err = float(np.max(np.abs(m.Forward(x, training=False) - data[f"mha{i}_y"])))
        assert err <= TOL_FP32, (cfg, err)


def test_sparse_kv_stepping_matches_reference(cuda, golden, float64):
    """One token at a time and a 5 + 4 split through the cache equal the
    reference's stepped outputs and its full Forward (test_enilnets.py:
    8252-8276)."""
    data, meta = golden
    for i, cfg in enumerate(meta["kv"]):
        enl.set_seed(3400 + i)
        m = enl.AttentionNet()
        m.add_embedding(vocab_size=13, embed_dim=32)
        if cfg["scheme"] == "absolute":
            m.add_positional_encoding(max_seq_len=16, learnable=False)
        m.add_multihead_attention(embed_dim=32, num_heads=4, causal=True,
                                  positional_scheme=cfg["scheme"],
                                  sparse_pattern=cfg["pattern"])
        m.add_dense(n_out=13, activation="linear")
        toks = np.random.RandomState(3500 + i).randint(0, 13, size=(2, 9))
        full = m.Forward(toks, training=False)
        assert np.max(np.abs(full - data[f"kv{i}_full"])) <= TOL_FP32, cfg
        c1 = enl.KVCache()
        one = np.concatenate([enl.cached_forward_step(m, toks[:, j:j + 1], c1)
                              for j in range(9)], axis=1)
        assert np.max(np.abs(one - data[f"kv{i}_one"])) <= TOL_FP32, cfg
        c2 = enl.KVCache()
        multi = np.concatenate([enl.cached_forward_step(m, toks[:, :5], c2),
                                enl.cached_forward_step(m, toks[:, 5:], c2)], axis=1)
        assert np.max(np.abs(multi - data[f"kv{i}_multi"])) <= TOL_FP32, cfg
    _check_device()
