"""enl_attn_decode_noalloc: the decode entry point for callers that cannot
allocate device memory (a host that owns all device memory and offers
plugins no allocation hook, or a token loop where a possibly-synchronising
cudaMalloc is not allowed). It keeps its split partials in a fixed scratch
array inside the library instead of a caller workspace.

This file sorts last so that a run stopping at the first failure has already
run every other test; it must also pass on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from oracle import attention_ref as ref

pytestmark = pytest.mark.gpu
TOL = 2e-2  # the tolerance the other bf16 decode tests use


def _noalloc_decode(q, kc, vc, out, *, slot_end, q_pos, n_splits, **override):
    """Call the new entry point straight through the C ABI (no workspace)."""
    import torch
    from enilnets_b200 import _native as nat
    B, H, D = q.shape
    a = nat.DecodeArgs()
    a.q, a.q_stride_b, a.q_stride_h = q.data_ptr(), q.stride(0), q.stride(1)
    a.k_cache, a.v_cache = kc.data_ptr(), vc.data_ptr()
    a.cache_stride_b, a.cache_stride_h, a.cache_stride_s = kc.stride(0), kc.stride(1), kc.stride(2)
    a.o, a.o_stride_b, a.o_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
    a.lse = None
    a.batch, a.num_heads, a.num_kv_heads, a.head_dim = B, H, kc.shape[1], D
    a.slot_begin, a.slot_end = 0, slot_end
    a.pos_slot0, a.q_pos = 0, q_pos
    a.window = -1
    a.alibi_slopes = None
    a.scale = 1.0 / np.sqrt(D)
    a.in_dtype, a.out_dtype = nat.ENL_DTYPE_BF16, nat.ENL_DTYPE_FP32
    a.n_splits = n_splits
    a.workspace, a.workspace_bytes = None, 0
    for name, value in override.items():
        setattr(a, name, value)
    status = nat.load().enl_attn_decode_noalloc(ctypes.byref(a),
                                                torch.cuda.current_stream().cuda_stream)
    nat.check(status, "enl_attn_decode_noalloc")


def _case(seed, B, H, Hkv, D, ctx):
    import torch
    cast = lambda x: torch.from_numpy(x.astype(np.float32)).cuda().to(torch.bfloat16)  # noqa
    q = cast(ref.seeded_normal(seed, (B, H, D)))
    kc = cast(ref.seeded_normal(seed + 1, (B, Hkv, ctx, D)))
    vc = cast(ref.seeded_normal(seed + 2, (B, Hkv, ctx, D)))
    return q, kc, vc


def test_noalloc_decode_matches_workspace_decode_twice_in_a_row():
    """Two calls in a row share (and overwrite) the scratch. Each must equal
    enl_attn_decode bit for bit (same kernel, same split count) and the
    float64 oracle within the bf16 bar."""
    import torch
    from enilnets_b200 import _native, kernels
    _native.load()
    cases = [dict(seed=31, B=4, H=8, Hkv=4, D=128, ctx=3000, n_splits=0),
             dict(seed=41, B=2, H=4, Hkv=4, D=64, ctx=1500, n_splits=5)]
    outs = []
    for c in cases:
        q, kc, vc = _case(c["seed"], c["B"], c["H"], c["Hkv"], c["D"], c["ctx"])
        out = torch.empty((c["B"], c["H"], c["D"]), dtype=torch.float32, device="cuda")
        _noalloc_decode(q, kc, vc, out, slot_end=c["ctx"], q_pos=c["ctx"] - 1,
                        n_splits=c["n_splits"])
        outs.append((c, q, kc, vc, out))
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    for c, q, kc, vc, out in outs:
        expect = kernels.attention_decode(q, kc, vc, slot_begin=0, slot_end=c["ctx"],
                                          pos_slot0=0, q_pos=c["ctx"] - 1,
                                          n_splits=c["n_splits"], out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert torch.equal(out, expect), \
            f"{c}: differs from enl_attn_decode by {(out - expect).abs().max().item():.3e}"
        oref, _ = ref.decode_ref(q.float().cpu().numpy(), kc.float().cpu().numpy(),
                                 vc.float().cpu().numpy(), slot_begin=0, slot_end=c["ctx"],
                                 pos_slot0=0, q_pos=c["ctx"] - 1)
        err = float(np.max(np.abs(out.cpu().numpy() - oref)))
        assert err <= TOL, f"{c}: max abs err {err:.3e} vs the float64 oracle"


def test_noalloc_decode_rejects_requests_beyond_its_scratch():
    import torch
    from enilnets_b200 import _native
    _native.load()
    q, kc, vc = _case(51, 8, 32, 32, 128, 64)
    out = torch.empty((8, 32, 128), dtype=torch.float32, device="cuda")
    # 64 splits x 8 x 32 x 129 floats = 8.5 MB > 4 MiB of scratch.
    with pytest.raises(ValueError, match="bytes of scratch"):
        _noalloc_decode(q, kc, vc, out, slot_end=64, q_pos=63, n_splits=64)
    # A bad size is reported as itself, not as an oversized scratch request.
    with pytest.raises(ValueError, match="must be >= 1"):
        _noalloc_decode(q, kc, vc, out, slot_end=64, q_pos=63, n_splits=8, batch=-1)
    # The bound is on the splits actually run: a query at slot 3 sees 4 keys,
    # which the decode runs as at most 4 splits, well inside the scratch.
    _noalloc_decode(q, kc, vc, out, slot_end=64, q_pos=3, n_splits=64)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
