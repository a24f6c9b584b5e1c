"""enilnets_b200: a B200-native (sm_100a) attention inference path behind the
Enilnets attention layer API.

The attention math runs in libenl_b200.so (hand-written tcgen05/TMA CUDA
kernels behind a plain C ABI, include/enl_attn.h); this package is the
Python host side that mirrors the reference's layer interface:

* builders with the reference signatures and weight draws
  (add_multihead_attention, add_cross_attention, add_transformer_block, ...)
* AttentionNet (alias NeuralNet): same layer dicts, Forward on the device
* KVCache / cached_forward_step: device-resident incremental decoding
* graph.MultiHeadAttention: key-padding-mask attention
* kernels: one tensor-level wrapper per C-ABI entry point
"""
__version__ = "0.2.0"

from .backend import (default_dtype, is_float64_enabled, precision, set_precision,  # noqa: F401
                      set_seed, use_float64)
from .graph import MultiHeadAttention, lengths_to_mask  # noqa: F401
from .kvcache import KVCache, cached_forward_step  # noqa: F401
from .layers import (add_cross_attention, add_multihead_attention,  # noqa: F401
                     add_transformer_block, init_weights)
from .network import AttentionNet  # noqa: F401
from .generation import TextGenerator  # noqa: F401

NeuralNet = AttentionNet
