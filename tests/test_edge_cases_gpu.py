"""Edge cases of the kernel entry points: empty batches and sequences (the
reference's NumPy code returns empty results for them and raises on a softmax
over no keys), empty key ranges in decode and merge, and the largest grid the
prefill accepts."""
import numpy as np
import pytest

from oracle import attention_ref as ref

pytestmark = pytest.mark.gpu


def _bf(shape, seed=0):
    import torch
    return torch.from_numpy(ref.seeded_normal(seed, shape)).to(torch.bfloat16).cuda()


def test_prefill_empty_batch_and_queries(cuda):
    import torch
    from enilnets_b200 import kernels
    for qs, ks in (((0, 64, 4, 64), (0, 64, 4, 64)), ((2, 0, 4, 64), (2, 64, 4, 64))):
        q = torch.zeros(qs, dtype=torch.bfloat16, device="cuda")
        k = torch.zeros(ks, dtype=torch.bfloat16, device="cuda")
        out, lse = kernels.attention_prefill(q, k, k, causal=False, return_lse=True)
        assert tuple(out.shape) == qs and lse.shape == (qs[0], qs[2], qs[1])
        assert out.numel() == 0


def test_prefill_over_no_keys_raises(cuda):
    import torch
    from enilnets_b200 import kernels
    q = _bf((1, 8, 2, 64))
    k = torch.zeros((1, 0, 2, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="no keys"):
        kernels.attention_prefill(q, k, k)


def test_prefill_largest_batch_times_heads(cuda):
    """batch x heads up to 65535 runs; one more is refused with the limit named."""
    import torch
    from enilnets_b200 import _native, kernels
    B, H, D = 4369, 15, 64  # 65535 (batch, head) units
    q, k, v = (_bf((B, 3, H, D), seed=s) for s in (1, 2, 3))
    out = kernels.attention_prefill(q, k, v, causal=True)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    for b in (0, 1234, B - 1):
        exp, _ = ref.attention_ref(q[b:b + 1].float().cpu().numpy(),
                                   k[b:b + 1].float().cpu().numpy(),
                                   v[b:b + 1].float().cpu().numpy(), causal=True)
        assert np.max(np.abs(out[b:b + 1].float().cpu().numpy() - exp)) <= 2e-2
    q2 = _bf((4096, 1, 16, D))
    with pytest.raises(ValueError, match="65535"):
        kernels.attention_prefill(q2, q2, q2)


def test_decode_empty_range_and_batch(cuda):
    import torch
    from enilnets_b200 import _native, kernels
    q = _bf((2, 4, 64))
    cache = _bf((2, 2, 32, 64), seed=5)
    out, lse = kernels.attention_decode(q, cache, cache, slot_begin=7, slot_end=7, pos_slot0=0,
                                        q_pos=6, out_dtype=torch.float32, return_lse=True)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    # No key: lse = -inf, and the output is NaN like the reference's softmax
    # over -inf scores (the oracle gives the same); a merge skips such parts.
    assert torch.isinf(lse).all() and (lse < 0).all()
    exp = ref.decode_ref(q.float().cpu().numpy(), cache.float().cpu().numpy(),
                         cache.float().cpu().numpy(), slot_begin=7, slot_end=7, pos_slot0=0,
                         q_pos=6)
    exp = exp[0] if isinstance(exp, tuple) else exp
    assert torch.isnan(out).all() and np.isnan(exp).all()
    e = kernels.attention_decode(q[:0], cache[:0], cache[:0], slot_begin=0, slot_end=8,
                                 pos_slot0=0, q_pos=8)
    assert tuple(e.shape) == (0, 4, 64)


def test_lse_merge_with_an_empty_partial(cuda):
    """A partial with lse = -inf (a shard holding no visible key) drops out of
    the merge; the result equals the other partials' merge."""
    import torch
    from enilnets_b200 import _native, kernels
    rng = np.random.RandomState(3)
    o = rng.standard_normal((3, 2, 4, 64)).astype(np.float32)
    lse = rng.standard_normal((3, 2, 4)).astype(np.float32)
    lse[1] = -np.inf
    o[1] = np.nan  # what a shard with no visible key outputs
    got = kernels.lse_merge(torch.from_numpy(o).cuda(), torch.from_numpy(lse).cuda(),
                            out_dtype=torch.float32)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    exp = ref.lse_merge_ref(o[[0, 2]], lse[[0, 2]])
    exp = exp[0] if isinstance(exp, tuple) else exp
    assert np.max(np.abs(got.cpu().numpy() - exp)) <= 1e-5


def test_linear_attention_and_feature_map_without_rows(cuda):
    import torch
    from enilnets_b200 import kernels
    x = torch.zeros((2, 0, 3, 32), dtype=torch.float32, device="cuda")
    phi, _ = kernels.linear_feature_map(x, "linear")
    assert tuple(phi.shape) == (2, 3, 0, 32)
    om = torch.rand((64, 32), device="cuda")
    floor = torch.full((2, 3), 1.5, device="cuda")
    _, stab = kernels.linear_feature_map(x, "performer", om, global_stab=True, stab_floor=floor)
    assert torch.equal(stab, floor)
    qp = torch.zeros((2, 3, 0, 32), dtype=torch.float32, device="cuda")
    v = torch.zeros((2, 0, 3, 16), dtype=torch.float32, device="cuda")
    kv = torch.rand((2, 3, 32, 16), device="cuda")
    ks = torch.rand((2, 3, 32), device="cuda")
    scale = torch.full((2, 3), 0.5, device="cuda")
    out, (kv2, ks2) = kernels.linear_attention(qp, qp, v, causal=True, state=(kv, ks),
                                               state_scale=scale, return_state=True)
    assert tuple(out.shape) == (2, 0, 3, 16)
    # No new rows: the returned sums are the carried state times its scale.
    assert torch.equal(kv2, kv * 0.5) and torch.equal(ks2, ks * 0.5)


def test_projection_and_backward_without_rows(cuda):
    import torch
    from enilnets_b200 import kernels
    x = torch.zeros((0, 64), dtype=torch.bfloat16, device="cuda")
    w = _bf((128, 64))
    y = kernels.project(x, w)
    assert tuple(y.shape) == (0, 128)
    q = torch.zeros((0, 16, 2, 64), dtype=torch.bfloat16, device="cuda")
    lse = torch.zeros((0, 2, 16), dtype=torch.float32, device="cuda")
    dq, dk, dv = kernels.attention_backward(q, q, q, q, lse, q, causal=True)
    assert dq.shape == q.shape and dk.numel() == 0 and dv.numel() == 0
