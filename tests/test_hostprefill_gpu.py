"""Prefill from pinned host buffers (enilnets_b200.hostprefill.HostPrefill):
the pipelined calls return exactly what the device-resident call returns,
whether or not the padded key/value rows were uploaded."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _host(rng, shape):
    import torch
    return torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(
        torch.bfloat16).pin_memory()


@pytest.mark.parametrize("lengths,window,mode", [
    ([300, 137, 5], None, "additive"),   # valid K/V rows only
    ([300, 137, 5], None, "exclude"),
    ([300, 0, 40], None, "additive"),    # a sequence with no real key: K/V move whole
    ([300, 137, 5], 64, "additive"),     # sliding window: K/V move whole
])
def test_host_prefill_equals_device_call(cuda, lengths, window, mode):
    import torch
    from enilnets_b200 import _native, kernels
    from enilnets_b200.hostprefill import HostPrefill
    B, S, H, D = 3, 300, 4, 64
    rng = np.random.RandomState(7)
    pipe = HostPrefill((B, S, H, D))
    calls = []
    for i in range(3):  # three pipelined calls, each with its own inputs and output
        hq, hk, hv = (_host(rng, (B, S, H, D)) for _ in range(3))
        hout = torch.empty((B, S, H, D), dtype=torch.bfloat16).pin_memory()
        pipe.submit(hq, hk, hv, hout, lengths, causal=True, window=window, mask_mode=mode)
        calls.append((hq, hk, hv, hout))
    pipe.synchronize()
    lens = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    for hq, hk, hv, hout in calls:
        ref = kernels.attention_prefill(hq.cuda(), hk.cuda(), hv.cuda(), causal=True,
                                        window=window, kv_valid_len=lens, mask_mode=mode)
        torch.cuda.synchronize()
        _native.raise_on_device_error()
        assert torch.equal(hout, ref.cpu())
    row = H * D * 2
    partial = window is None and min(lengths) >= 1
    kv = 2 * (sum(lengths) if partial else B * S) * row
    assert pipe.h2d_bytes == [B * S * row + kv + 4 * B] * 3
    assert pipe.d2h_bytes == [B * S * row] * 3


def test_host_prefill_fp32_inputs(cuda):
    """fp32 q/k/v (the split-bf16 path) with the partial K/V upload: equal to
    the device-resident call bit for bit."""
    import torch
    from enilnets_b200 import kernels
    from enilnets_b200.hostprefill import HostPrefill
    B, S, H, D = 2, 200, 2, 64
    rng = np.random.RandomState(11)
    lengths = [200, 61]
    host = [torch.from_numpy(rng.standard_normal((B, S, H, D)).astype(np.float32)).pin_memory()
            for _ in range(3)]
    hout = torch.empty((B, S, H, D), dtype=torch.float32).pin_memory()
    pipe = HostPrefill((B, S, H, D), dtype=torch.float32)
    pipe.submit(*host, hout, lengths, causal=True, mask_mode="additive")
    pipe.synchronize()
    ref = kernels.attention_prefill(*(t.cuda() for t in host), causal=True,
                                    kv_valid_len=torch.tensor(lengths, dtype=torch.int32,
                                                              device="cuda"),
                                    mask_mode="additive", out_dtype=torch.float32)
    assert torch.equal(hout, ref.cpu())


def test_host_prefill_rejects_unpinned_and_bad_lengths(cuda):
    import torch
    from enilnets_b200.hostprefill import HostPrefill
    pipe = HostPrefill((1, 8, 2, 16))
    t = torch.zeros((1, 8, 2, 16), dtype=torch.bfloat16)
    p = t.pin_memory()
    with pytest.raises(ValueError, match="pinned"):
        pipe.submit(t, p, p, p, [8])
    with pytest.raises(ValueError, match="kv_valid_len"):
        pipe.submit(p, p, p, p, [9])
