"""The linearized-attention oracle against the reference's own outputs
(tests/golden/linear_layers.npz, identity-weight layers so that the output is
the attention context of the input itself), plus the decode-step algebra:
a cached step sequence equals the full causal forward."""
import json

import numpy as np

from oracle import linear_ref as lr


def _heads(x, H):
    B, S, E = x.shape
    return x.reshape(B, S, H, E // H).transpose(0, 2, 1, 3)


def test_oracle_matches_reference_core(golden_dir):
    data = np.load(golden_dir / "linear_layers.npz", allow_pickle=False)
    meta = json.loads(str(data["meta"]))
    for i, cfg in enumerate(meta["core"]):
        x = np.random.RandomState(2100 + i).standard_normal((2, 21, cfg["embed_dim"]))
        H = cfg["num_heads"]
        xh = _heads(x, H)
        kernel = cfg["attention_kernel"]
        omega = data[f"core{i}_omega"] if kernel == "performer" else None
        qp = lr.feature_map(xh, kernel, omega, "row")
        kp = lr.feature_map(xh, kernel, omega, "global")
        ctx, _, _ = lr.linear_attention(qp, kp, xh, cfg["causal"])
        y = ctx.transpose(0, 2, 1, 3).reshape(x.shape)
        assert np.max(np.abs(y - data[f"core{i}_y"])) < 1e-10, cfg


def test_projection_shape_and_draw_order():
    rng = np.random.RandomState(7)
    w = lr.make_projection(24, 16, rng)
    assert w.shape == (24, 16)
    # two 16 x 16 orthogonal blocks, then the norm draws: the same seed again
    # gives the same matrix
    assert np.array_equal(w, lr.make_projection(24, 16, np.random.RandomState(7)))


def test_steps_equal_full_causal_forward():
    rng = np.random.RandomState(3)
    B, H, S, Dh = 2, 3, 11, 8
    x = rng.standard_normal((3, B, H, S, Dh))
    omega = lr.make_projection(32, Dh, np.random.RandomState(5))
    for kernel in ("linear", "performer"):
        qp = lr.feature_map(x[0], kernel, omega, "row")
        kp = lr.feature_map(x[1], kernel, omega, "global")
        full, _, _ = lr.linear_attention(qp, kp, x[2], True)
        state = None
        pieces = []
        for a, b in ((0, 4), (4, 5), (5, 9), (9, 11)):
            out, state = lr.linear_step(x[0][:, :, a:b], x[1][:, :, a:b], x[2][:, :, a:b],
                                        kernel, omega, state)
            pieces.append(out)
        stepped = np.concatenate(pieces, axis=2)
        # the key stabilizer is a common factor of numerator and denominator
        assert np.max(np.abs(stepped - full)) < 1e-9, kernel
