"""K6 projection GEMM (csrc/enl_gemm.cu) through the C ABI: y = x W^T + b
with the RoPE rotation fused into the epilogue, the projections of
nn/forward.py:428-430, :551 and :80-88.

References: a float64 product of the same (bf16-rounded) operands. Bars:
bf16 output 2^-8 relative rounding plus fp32 accumulation, held to
1e-2 x max |y|; fp32 output of bf16 inputs and the split-bf16 path (fp32
x and W) to 1e-4 x max |y|, well inside the north star's 1e-3 for fp32."""
import numpy as np
import pytest

from oracle import attention_ref as ref

pytestmark = pytest.mark.gpu


def _case(seed, M, N, K, fp32=False):
    rng = np.random.RandomState(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    if not fp32:
        x, w = ref.bf16_round(x), ref.bf16_round(w)
    return x, w, b


def _run(x, w, b, out_dtype, fp32_in=False, rope=None):
    import torch
    from enilnets_b200 import kernels, _native
    xd = torch.from_numpy(x).cuda()
    wd = torch.from_numpy(w).cuda()
    bd = None if b is None else torch.from_numpy(b).cuda()
    if fp32_in:
        hi, lo = kernels.split_bf16(wd)
        y = kernels.project(xd, hi, bd, w_lo=lo, out_dtype=out_dtype, rope=rope)
    else:
        y = kernels.project(xd.to(torch.bfloat16), wd.to(torch.bfloat16), bd,
                            out_dtype=out_dtype, rope=rope)
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    return y.float().cpu().numpy().astype(np.float64)


def _ref(x, w, b):
    y = x.astype(np.float64) @ w.astype(np.float64).T
    return y if b is None else y + b


SHAPES = [(256, 256, 64), (300, 392, 136), (64, 512, 2048), (1000, 768, 72), (4100, 1024, 512),
          (33, 8, 8)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_bf16_projection_matches_float64(cuda, M, N, K):
    import torch
    x, w, b = _case(M + N + K, M, N, K)
    yref = _ref(x, w, b)
    scale = np.max(np.abs(yref))
    y32 = _run(x, w, b, torch.float32)
    assert np.max(np.abs(y32 - yref)) <= 1e-4 * scale
    y16 = _run(x, w, b, torch.bfloat16)
    assert np.max(np.abs(y16 - yref)) <= 1e-2 * scale


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (300, 392, 136), (1000, 768, 200)])
def test_split_bf16_projection_meets_the_fp32_bar(cuda, M, N, K):
    import torch
    x, w, b = _case(7 * M + N, M, N, K, fp32=True)
    yref = _ref(x, w, b)
    y = _run(x, w, b, torch.float32, fp32_in=True)
    assert np.max(np.abs(y - yref)) <= 1e-4 * np.max(np.abs(yref))


def test_no_bias_and_strided_rows(cuda):
    import torch
    from enilnets_b200 import kernels
    x, w, _ = _case(5, 200, 256, 128)
    xd = torch.zeros((200, 192), dtype=torch.bfloat16, device="cuda")
    xd[:, :128] = torch.from_numpy(x).cuda().to(torch.bfloat16)
    out = torch.zeros((200, 264), dtype=torch.float32, device="cuda")
    kernels.project(xd[:, :128], torch.from_numpy(w).cuda().to(torch.bfloat16),
                    out=out[:, :256])
    torch.cuda.synchronize()
    y = out[:, :256].cpu().numpy()
    yref = _ref(x, w, None)
    assert np.max(np.abs(y - yref)) <= 1e-4 * np.max(np.abs(yref))
    assert float(out[:, 256:].abs().max()) == 0.0, "columns past N were written"


@pytest.mark.parametrize("D", [8, 16, 32, 64, 128])
@pytest.mark.parametrize("fp32_in", [False, True])
def test_fused_rope_matches_rotate_half(cuda, D, fp32_in):
    """Q and K columns rotated in the epilogue equal x W^T + b rotated by the
    oracle's rotate_half (nn/forward.py:80-88) at positions pos0 + r % S."""
    import torch
    H, Hkv, B, S, pos0 = 4, 2, 3, 70, 5
    N = (H + 2 * Hkv) * D
    K = 64
    x, w, b = _case(D + 100 * fp32_in, B * S, N, K, fp32=fp32_in)
    cos, sin = ref.rope_tables(pos0 + S + 3, D)
    tables = (torch.from_numpy(cos.astype(np.float32)).cuda(),
              torch.from_numpy(sin.astype(np.float32)).cuda())
    rot = (H + Hkv) * D
    y = _run(x, w, b, torch.float32, fp32_in=fp32_in,
             rope=(tables[0], tables[1], rot, D, S, pos0))
    yref = _ref(x, w, b).reshape(B, S, H + 2 * Hkv, D)
    c, s_ = cos[pos0:pos0 + S], sin[pos0:pos0 + S]
    qk = yref[:, :, :H + Hkv].transpose(0, 2, 1, 3)
    yref[:, :, :H + Hkv] = ref.rope_rotate(qk, c, s_).transpose(0, 2, 1, 3)
    yref = yref.reshape(B * S, N)
    assert np.max(np.abs(y - yref)) <= 1e-4 * np.max(np.abs(yref))


def test_projection_rejects_bad_arguments(cuda):
    import torch
    from enilnets_b200 import kernels
    x = torch.zeros((10, 12), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((16, 12), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="multiples of 8"):
        kernels.project(x, w)
    xf = torch.zeros((10, 16), dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError, match="w_lo"):
        kernels.project(xf, torch.zeros((16, 16), dtype=torch.bfloat16, device="cuda"))
