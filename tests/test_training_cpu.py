"""Host checks of the attention layer's training path (enilnets_b200.training):
layers the backward kernels do not cover are rejected before any device
work, with the option named."""
import numpy as np
import pytest

import enilnets_b200 as enl
from enilnets_b200 import training


@pytest.mark.parametrize("kwargs,match", [
    (dict(attention_kernel="linear"), "softmax"),
    (dict(attention_kernel="performer"), "softmax"),
    (dict(sparse_pattern={"block_size": 2}), "sparse_pattern"),
    (dict(dropout=0.1), "dropout"),
])
def test_uncovered_layers_are_rejected(kwargs, match):
    m = enl.AttentionNet()
    m.add_multihead_attention(embed_dim=16, num_heads=2, **kwargs)
    with pytest.raises(ValueError, match=match):
        training.multihead_attention_forward_train(m.layers[0], np.zeros((1, 4, 16)))
