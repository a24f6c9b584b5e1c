"""enilnets_b200: a B200-native (sm_100a) attention inference path behind the
Enilnets attention layer API.

The attention math runs in libenl_b200.so (hand-written tcgen05/TMA CUDA
kernels behind a plain C ABI, include/enl_attn.h); this package is the
Python host side that mirrors the reference's layer interface.
"""
__version__ = "0.1.0"
