"""Seeded random sweeps of the prefill (K1) and decode (K2) entry points
against the float64 oracle: head dims 8..128, GQA ratios, unequal query and
key lengths with position offsets, sliding windows, ALiBi, valid lengths
(including zero) under both mask rules, bf16 and fp32 inputs, split counts.
Each case is small; the sweep covers combinations the targeted tests do not.
Bars: bf16 inputs 2e-2 max abs error, fp32 inputs 1e-3;
rows without any visible key must be NaN exactly where the oracle's are."""
import numpy as np
import pytest

from oracle import attention_ref as ref

pytestmark = pytest.mark.gpu

HEAD_DIMS = (8, 16, 24, 32, 48, 64, 72, 96, 112, 128)


def _case(seed):
    rng = np.random.RandomState(seed)
    fp32 = bool(rng.rand() < 0.3)
    D = int(rng.choice(HEAD_DIMS))
    Hkv = int(rng.choice([1, 2, 3]))
    H = Hkv * int(rng.choice([1, 2, 4]))
    B = int(rng.randint(1, 4))
    Sq = int(rng.randint(1, 260))
    Skv = int(rng.randint(1, 260))
    causal = bool(rng.rand() < 0.5)
    # decode-style offsets: the queries are the last Sq positions of the keys
    q_pos0 = int(rng.randint(0, 64)) + max(0, Skv - Sq) if causal else int(rng.randint(0, 64))
    window = int(rng.randint(1, 80)) if rng.rand() < 0.3 else None
    alibi = ref.alibi_slopes(H) if rng.rand() < 0.3 else None
    mode = "additive" if rng.rand() < 0.5 else "exclude"
    lens = None
    if rng.rand() < 0.5:
        lens = [int(x) for x in rng.randint(0 if mode == "additive" else 1, Skv + 1, size=B)]
    return dict(fp32=fp32, D=D, H=H, Hkv=Hkv, B=B, Sq=Sq, Skv=Skv, causal=causal,
                q_pos0=q_pos0, window=window, alibi=alibi, mode=mode, lens=lens,
                seed=int(rng.randint(1 << 30)))


@pytest.mark.parametrize("block", range(6))
def test_prefill_random_sweep(cuda, block):
    import torch
    from enilnets_b200 import _native, kernels
    for seed in range(100 * block, 100 * block + 16):
        c = _case(seed)
        bf = not c["fp32"]
        q = ref.seeded_normal(c["seed"], (c["B"], c["Sq"], c["H"], c["D"]), bf16=bf)
        k = ref.seeded_normal(c["seed"] + 1, (c["B"], c["Skv"], c["Hkv"], c["D"]), bf16=bf)
        v = ref.seeded_normal(c["seed"] + 2, (c["B"], c["Skv"], c["Hkv"], c["D"]), bf16=bf)
        dt = torch.float32 if c["fp32"] else torch.bfloat16

        def dev(x):
            return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda().to(dt)

        out = kernels.attention_prefill(
            dev(q), dev(k), dev(v), causal=c["causal"], window=c["window"],
            kv_valid_len=None if c["lens"] is None else
            torch.tensor(c["lens"], dtype=torch.int32, device="cuda"),
            alibi_slopes=None if c["alibi"] is None else
            torch.tensor(c["alibi"], dtype=torch.float32, device="cuda"),
            q_pos0=c["q_pos0"], mask_mode=c["mode"], out_dtype=torch.float32)
        torch.cuda.synchronize()
        _native.raise_on_device_error()
        o = out.cpu().numpy().astype(np.float64)
        oref, _ = ref.attention_ref(q, k, v, causal=c["causal"], window=c["window"],
                                    kv_valid_len=c["lens"], alibi=c["alibi"],
                                    q_pos0=c["q_pos0"], mask_mode=c["mode"])
        finite = np.isfinite(oref)
        assert np.array_equal(finite, np.isfinite(o)), ("NaN pattern", seed, c)
        err = float(np.max(np.abs(o[finite] - oref[finite]))) if finite.any() else 0.0
        assert err <= (1e-3 if c["fp32"] else 2e-2), (seed, err, c)


@pytest.mark.parametrize("block", range(3))
def test_decode_random_sweep(cuda, block):
    import torch
    from enilnets_b200 import _native, kernels
    for seed in range(1000 + 50 * block, 1000 + 50 * block + 16):
        rng = np.random.RandomState(seed)
        D = int(rng.choice([64, 128]))
        Hkv = int(rng.choice([1, 2, 4]))
        H = Hkv * int(rng.choice([1, 2, 4, 8]))
        B = int(rng.randint(1, 5))
        cap = int(rng.randint(8, 1500))
        lo = int(rng.randint(0, cap))
        hi = int(rng.randint(lo, cap + 1))
        pos0 = int(rng.randint(0, 500))
        q_pos = pos0 + int(rng.randint(0, cap + 20))
        window = int(rng.randint(1, 300)) if rng.rand() < 0.3 else None
        alibi = ref.alibi_slopes(H) if rng.rand() < 0.3 else None
        splits = int(rng.choice([0, 1, 2, 5]))
        q = ref.seeded_normal(seed, (B, H, D))
        K = ref.seeded_normal(seed + 1, (B, Hkv, cap, D))
        V = ref.seeded_normal(seed + 2, (B, Hkv, cap, D))

        def dev(x):
            return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda().to(
                torch.bfloat16)

        o, lse = kernels.attention_decode(
            dev(q), dev(K), dev(V), slot_begin=lo, slot_end=hi, pos_slot0=pos0, q_pos=q_pos,
            window=window, alibi_slopes=None if alibi is None else
            torch.tensor(alibi, dtype=torch.float32, device="cuda"),
            out_dtype=torch.float32, return_lse=True, n_splits=splits)
        torch.cuda.synchronize()
        _native.raise_on_device_error()
        oref, lref = ref.decode_ref(q, K, V, slot_begin=lo, slot_end=hi, pos_slot0=pos0,
                                    q_pos=q_pos, window=window, alibi=alibi)
        on, ln = o.cpu().numpy().astype(np.float64), lse.cpu().numpy().astype(np.float64)
        finite = np.isfinite(oref)
        assert np.array_equal(finite, np.isfinite(on)), ("NaN pattern", seed)
        if finite.any():
            assert np.max(np.abs(on[finite] - oref[finite])) <= 2e-2, seed
        lf = np.isfinite(lref)
        assert np.array_equal(lf, np.isfinite(ln)), ("lse pattern", seed)
        if lf.any():
            assert np.max(np.abs(ln[lf] - lref[lf])) <= 2e-2, seed


@pytest.mark.parametrize("block", range(2))
def test_linear_random_sweep(cuda, block):
    """Feature map plus linear attention end to end (the layer's order: the
    maps write planes when the attention takes them), elu + 1 and Performer,
    head dims on both sides of the tensor-core limit (128), odd feature
    counts, GQA, causal and not: fp32 inputs at the 1e-4 kernel bar."""
    import torch
    from enilnets_b200 import _native, kernels
    from oracle import linear_ref as lr
    for seed in range(2000 + 50 * block, 2000 + 50 * block + 10):
        rng = np.random.RandomState(seed)
        kernel = "performer" if rng.rand() < 0.5 else "linear"
        Dh = int(rng.choice([8, 24, 32, 64, 96, 128, 160]))
        Df = int(rng.choice([36, 64, 128, 256])) if kernel == "performer" else Dh
        Hkv = int(rng.choice([1, 2]))
        H = Hkv * int(rng.choice([1, 2]))
        B, S = int(rng.randint(1, 3)), int(rng.randint(1, 300))
        causal = bool(rng.rand() < 0.6)
        D = Dh
        x_q = rng.standard_normal((B, S, H, Dh)) * 0.5
        x_k = rng.standard_normal((B, S, Hkv, Dh)) * 0.5
        v = rng.standard_normal((B, S, Hkv, D))
        omega = lr.make_projection(Df, Dh, np.random.RandomState(seed)) if kernel == "performer" \
            else None

        def dev(a):
            return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()

        om = dev(omega) if omega is not None else None
        planes = kernels.linear_planes_ok(D, Df)
        qp, _ = kernels.linear_feature_map(dev(x_q), kernel, om, planes=planes)
        kp, _ = kernels.linear_feature_map(dev(x_k), kernel, om, global_stab=True, planes=planes)
        out = kernels.linear_attention(qp, kp, dev(v), causal=causal, num_features=Df)
        torch.cuda.synchronize()
        _native.raise_on_device_error()
        fq = lr.feature_map(x_q.transpose(0, 2, 1, 3), kernel, omega, "row")
        fk = lr.feature_map(x_k.transpose(0, 2, 1, 3), kernel, omega, "global")
        G = H // Hkv
        oref, _, _ = lr.linear_attention(fq, np.repeat(fk, G, axis=1),
                                         np.repeat(v.transpose(0, 2, 1, 3), G, axis=1), causal)
        got = out.cpu().numpy().astype(np.float64).transpose(0, 2, 1, 3)
        err = float(np.max(np.abs(got - oref)))
        assert err <= 1e-4 * max(1.0, float(np.abs(oref).max())), (seed, kernel, Dh, Df, err)
