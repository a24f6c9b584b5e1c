"""AttentionNet: a NeuralNet-compatible container whose Forward runs
transformer stacks on the B200 path.

It holds the same list of layer dicts as the reference's NeuralNet
(core/base.py:15-91, built by the same add_* builders, enilnets_b200.layers)
and executes the layer types a transformer uses -- embedding, positional
encoding, layernorm, dense (+ activations), dropout (inference no-op),
residual save/add, multihead_attention and cross_attention -- following
nn/forward.py:272-811. The attention layers run the hand-written kernels;
the rest is plain device tensor math. Any other layer type raises
ValueError naming it.
"""
from __future__ import annotations

import math

import numpy as np

from . import attention
from .backend import WEIGHTS, to_device, to_numpy
from .layers import BUILDERS

LEAKYRELU_ALPHA = 0.01   # core/constants.py:21
ELU_ALPHA = 1.0          # core/constants.py:22
SIGMOID_CLIP = 500.0     # core/constants.py:18


def activate(name: str, z, alpha=None, sigmoid_clip=None):
    """nn/activations.py:6-41 on device tensors."""
    import torch
    clip = SIGMOID_CLIP if sigmoid_clip is None else sigmoid_clip
    if name == "relu":
        return torch.clamp_min(z, 0)
    if name == "leakyrelu":
        a = LEAKYRELU_ALPHA if alpha is None else alpha
        return torch.where(z > 0, z, a * z)
    if name == "elu":
        a = ELU_ALPHA if alpha is None else alpha
        return torch.where(z > 0, z, a * (torch.exp(z) - 1))
    if name == "selu":
        return 1.0507009873554804934193349852946 * torch.where(
            z > 0, z, 1.6732632423543772848170429916717 * (torch.exp(z) - 1))
    if name == "gelu":
        return 0.5 * z * (1 + torch.tanh(math.sqrt(2 / math.pi) * (z + 0.044715 * z ** 3)))
    if name == "swish":
        return z / (1.0 + torch.exp(-z))
    if name == "mish":
        return z * torch.tanh(torch.log(1 + torch.exp(z)))
    if name == "sigmoid":
        return 1.0 / (1.0 + torch.exp(-torch.clamp(z, -clip, clip)))
    if name == "tanh":
        return torch.tanh(z)
    if name == "softmax":
        e = torch.exp(z - z.amax(dim=-1, keepdim=True))
        return e / e.sum(dim=-1, keepdim=True)
    if name == "softplus":
        return torch.log(1 + torch.exp(torch.clamp(z, -clip, clip)))
    if name == "linear":
        return z
    raise ValueError(f"Unknown activation: {name!r}")


def layernorm(x, layer):
    """Per-token LayerNorm over the last axis (nn/forward.py:207-255, 2-D/3-D)."""
    import torch
    eps = layer.get("epsilon", 1e-5)
    g = WEIGHTS.get(layer["gamma"], torch.float32)
    b = WEIGHTS.get(layer["beta"], torch.float32)
    mean = x.mean(dim=-1, keepdim=True)
    var = x.var(dim=-1, unbiased=False, keepdim=True)
    return g * ((x - mean) / torch.sqrt(var + eps)) + b


def dense(x, layer):
    """x @ W.T + b then the activation (nn/forward.py:317-321)."""
    import torch
    w = WEIGHTS.get(layer["weights"], torch.float32)
    z = x @ w.T + WEIGHTS.get(layer["bias"], torch.float32)
    return activate(layer["activation"], z, **layer.get("activation_params", {}))


def embed(tokens, layer):
    """Table lookup by integer token ids (nn/forward.py:414-419)."""
    import torch
    ids = to_device(np.asarray(tokens, dtype=np.int64), torch.int64)
    if ids.dim() == 1:
        ids = ids.reshape(-1, 1)
    return WEIGHTS.get(layer["weights"], torch.float32)[ids]


def positional_table(layer):
    import torch
    table = layer["weights"] if layer.get("_pos_type") == "learnable" else layer["pe"]
    return WEIGHTS.get(table, torch.float32)


def forward_device(model, inputs, training: bool = False):
    """Run model.layers on the device; returns (final output, outputs list)."""
    import torch
    layers = model.layers
    first = layers[0]["type"] if layers else None
    if first == "embedding":
        x = inputs
    else:
        x = to_device(inputs, torch.float32)
        if x.dim() == 1:
            x = x.reshape(1, -1)
    outputs = [x]
    for idx, layer in enumerate(layers):
        t = layer["type"]
        x = outputs[-1]
        if t == "embedding":
            x = embed(x, layer)
        elif t == "positional_encoding":
            x = x + positional_table(layer)[: x.shape[1]][None]
        elif t == "layernorm":
            x = layernorm(x, layer)
        elif t in ("dense", "sparse"):
            x = dense(x, layer)
        elif t == "dropout":
            if training and layer.get("rate", 0.0) > 0:
                raise ValueError("dropout at training=True is not supported by the B200 "
                                 "inference path")
        elif t == "residual_save":
            pass
        elif t == "residual_add":
            x = x + outputs[layer["save_index"]]
        elif t == "multihead_attention":
            attention.check_supported(layer, training)
            x = attention.self_attention(layer, x)
        elif t == "cross_attention":
            attention.check_supported(layer, training)
            src = outputs[layer["kv_source_index"] + 1]
            x = attention.cross_attention(layer, x, src)
        else:
            raise ValueError(f"layer type {t!r} (layer {idx}) is not supported by the B200 "
                             "attention path; it executes transformer stacks only.")
        outputs.append(x)
    return x, outputs


class AttentionNet:
    """Drop-in for NeuralNet on transformer stacks (core/base.py:15-91):
    same builders, same layer dicts, same Forward signature. Extra keyword
    arguments of the reference constructor (optimizer settings) are accepted
    and ignored -- this container runs inference only."""

    def __init__(self, *args, **kwargs) -> None:
        self.layers = []
        self.outputs = []
        self._last_width = None
        self._last_spatial = None
        self._last_spatial_1d = None
        self._residual_stack = []

    def Forward(self, inputs, training: bool = False, dropout_rate: float = 0.0):
        """nn/forward.py:272: returns the last layer's output as a NumPy
        array in the default working dtype; self.outputs keeps every layer's
        output (device tensors)."""
        out, self.outputs = forward_device(self, inputs, training)
        return to_numpy(out)

    def forward_device(self, inputs, training: bool = False):
        """Forward without the final device->host copy."""
        out, self.outputs = forward_device(self, inputs, training)
        return out


for _name, _fn in BUILDERS.items():
    setattr(AttentionNet, _name, _fn)
