"""The attention layer's training path (enilnets_b200.training) against the
reference's own nn/backward.py:241-327 after Forward(training=True)
(tests/golden/mha_backward.npz): dx and the eight parameter gradients of
causal / windowed / ALiBi / RoPE / GQA / tiled layers rebuilt from the
reference's seeds (head dims 16 to 64). Both precisions run: "bf16" (bf16
attention operands, K1 forward with LSE, K5 backward) at 2e-2 and "fp32"
(the reference's float32 models: split-bf16 operands in both directions) at
1e-3, each relative to the gradient's largest magnitude, the north-star bars."""
import json

import numpy as np
import pytest

import enilnets_b200 as enl
from enilnets_b200 import training

pytestmark = pytest.mark.gpu
TOLS = {"bf16": 2e-2, "fp32": 1e-3}
NAMES = ("d_Wq", "d_bq", "d_Wk", "d_bk", "d_Wv", "d_bv", "d_Wo", "d_bo")


@pytest.fixture(params=["bf16", "fp32"])
def precision(request):
    enl.set_precision(request.param)
    yield request.param
    enl.set_precision("fp32")


def test_layer_backward_matches_reference(cuda, golden_dir, precision):
    TOL = TOLS[precision]
    data = np.load(golden_dir / "mha_backward.npz")
    meta = json.loads(str(data["meta"]))
    for i, cfg in enumerate(meta):
        enl.set_seed(4500 + i)
        m = enl.AttentionNet()
        m.add_multihead_attention(**cfg)
        rs = np.random.RandomState(4600 + i)
        x = rs.standard_normal((2, 37, cfg["embed_dim"]))
        dout = rs.standard_normal((2, 37, cfg["embed_dim"]))
        layer = m.layers[0]
        y, cache = training.multihead_attention_forward_train(layer, x)
        y_inf = m.Forward(x, training=False)
        assert np.max(np.abs(y - y_inf)) <= TOL * max(1.0, np.abs(y_inf).max()), cfg
        dx = training.multihead_attention_backward(dout, layer, cache)
        for name, got in [("dx", dx)] + [(n, layer[n]) for n in NAMES]:
            ref = data[f"{name}{i}"]
            err = float(np.max(np.abs(np.asarray(got) - ref)))
            scale = max(1.0, float(np.abs(ref).max()))
            if name.startswith("d_b"):
                # A bias gradient sums the same rows its weight gradient
                # contracts with x, and d_bk is exactly 0 (a key bias shifts
                # every score of a query row by one constant): its error
                # scale is the weight gradient's.
                scale = max(scale, float(np.abs(data[f"d_W{name[3:]}{i}"]).max()))
            assert err <= TOL * scale, (cfg, name, err)


def test_training_rejects_uncovered_layers(cuda):
    m = enl.AttentionNet()
    m.add_multihead_attention(embed_dim=16, num_heads=2, attention_kernel="linear")
    with pytest.raises(ValueError, match="softmax"):
        training.multihead_attention_forward_train(m.layers[0], np.zeros((1, 4, 16)))
    m = enl.AttentionNet()
    m.add_multihead_attention(embed_dim=16, num_heads=2, sparse_pattern={"block_size": 2})
    with pytest.raises(ValueError, match="sparse_pattern"):
        training.multihead_attention_forward_train(m.layers[0], np.zeros((1, 4, 16)))
