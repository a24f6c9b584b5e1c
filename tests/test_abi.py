"""C-ABI checks that need no GPU: the library loads, exports every function
include/enl_attn.h declares, the ctypes binding covers them all, the ctypes
struct layouts match the C compiler's, and argument validation rejects bad
calls before anything is launched."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from enilnets_b200 import _native

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "enl_attn.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(enl_\w+)\s*\(", text)))


def test_header_declares_the_expected_entry_points():
    names = declared_functions()
    for must in ("enl_attn_prefill", "enl_attn_prefill_sparse", "enl_sparse_build_masks",
                 "enl_attn_decode", "enl_kv_append", "enl_kv_gather",
                 "enl_lse_merge", "enl_rope_apply", "enl_last_error", "enl_device_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in enl_attn.h but not exported"
        assert name in _native.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.enl_abi_version() == _native.ABI_VERSION == 8


def test_nm_shows_c_linkage():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (enl_\w+)$", out, flags=re.M))
    assert set(declared_functions()) <= exported


def _c_offsets(struct, fields):
    src = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(){"]
    src.append(f'printf("%zu\\n", sizeof({struct}));')
    for f in fields:
        src.append(f'printf("%zu\\n", offsetof({struct}, {f}));')
    src.append("return 0;}")
    tmp = Path(subprocess.run(["mktemp", "-d"], capture_output=True, text=True).stdout.strip())
    c = tmp / "layout.c"
    c.write_text("\n".join(src))
    subprocess.run(["gcc", "-o", str(tmp / "layout"), str(c)], check=True)
    vals = [int(x) for x in subprocess.run([str(tmp / "layout")], capture_output=True,
                                           text=True, check=True).stdout.split()]
    return vals[0], vals[1:]


@pytest.mark.parametrize("cls,cname", [(_native.PrefillArgs, "enl_prefill_args"),
                                       (_native.DecodeArgs, "enl_decode_args")])
def test_ctypes_struct_layout_matches_c(cls, cname):
    fields = [f for f, _ in cls._fields_]
    size, offsets = _c_offsets(cname, fields)
    assert ctypes.sizeof(cls) == size
    for f, off in zip(fields, offsets):
        assert getattr(cls, f).offset == off, f


def test_validation_errors_raise_before_launch():
    """Argument errors come back as a status (ValueError in Python) without
    touching the device: NULL pointers and unsupported head dims."""
    lib = _native.load()
    a = _native.PrefillArgs()
    with pytest.raises(ValueError, match="non-NULL"):
        _native.check(lib.enl_attn_prefill(ctypes.byref(a), None), "enl_attn_prefill")
    a.q = a.k = a.v = a.o = 16
    a.batch = a.num_heads = a.num_kv_heads = a.seq_q = a.seq_kv = 1
    a.head_dim = 100
    with pytest.raises(ValueError, match="head_dim=100"):
        _native.check(lib.enl_attn_prefill(ctypes.byref(a), None), "enl_attn_prefill")
    a.head_dim = 64
    a.num_kv_heads = 3
    a.num_heads = 4
    with pytest.raises(ValueError, match="must divide"):
        _native.check(lib.enl_attn_prefill(ctypes.byref(a), None), "enl_attn_prefill")
    d = _native.DecodeArgs()
    with pytest.raises(ValueError):
        _native.check(lib.enl_attn_decode(ctypes.byref(d), None), "enl_attn_decode")
    with pytest.raises(ValueError, match="exceed capacity"):
        _native.check(lib.enl_kv_append(16, 0, 0, 0, 16, 0, 0, 0, 1, 1, 4, 64, 0, 6, 8, None),
                      "enl_kv_append")


def test_decode_split_heuristic():
    lib = _native.load()
    assert lib.enl_decode_auto_splits(64, 32, 8193) == 3
    assert lib.enl_decode_auto_splits(4, 32, 262145) == 37
    assert lib.enl_decode_auto_splits(1, 1, 10) == 1
    assert lib.enl_decode_workspace_bytes(2, 4, 128, 1) == 0
    assert lib.enl_decode_workspace_bytes(2, 4, 128, 3) == 3 * 2 * 4 * 129 * 4


def test_prefill_workspace_bytes_is_host_only_arithmetic():
    """fp32 prefill needs (hi, lo) bf16 planes of q, k and v, each padded to
    256 bytes; bf16 prefill needs none."""
    lib = _native.load()
    a = _native.PrefillArgs()
    a.batch, a.num_heads, a.num_kv_heads, a.seq_q, a.seq_kv, a.head_dim = 2, 8, 2, 100, 300, 40
    a.in_dtype = _native.ENL_DTYPE_BF16
    assert lib.enl_prefill_workspace_bytes(ctypes.byref(a)) == 0
    a.in_dtype = _native.ENL_DTYPE_FP32

    def planes(S, H):
        n = 2 * S * H * 2 * 40 * 2
        return (n + 255) // 256 * 256
    assert lib.enl_prefill_workspace_bytes(ctypes.byref(a)) == planes(100, 8) + 2 * planes(300, 2)


def test_backward_workspace_and_validation_are_host_only():
    """The backward's workspace is two fp32 rows per padded query, plus the
    bf16 (hi, lo) planes of q, k, v and dout for fp32 operands; fp32 operands
    past head dim 64 and unknown dtypes are rejected before any launch."""
    lib = _native.load()
    a = _native.BackwardArgs()
    a.batch, a.num_heads, a.num_kv_heads, a.seq_q, a.seq_kv, a.head_dim = 2, 4, 2, 100, 300, 32
    rows = (2 * 4 * 128 * 4 + 255) // 256 * 256
    a.in_dtype = _native.ENL_DTYPE_BF16
    assert lib.enl_backward_workspace_bytes(ctypes.byref(a)) == 2 * rows

    def planes(S, H):
        return (2 * S * H * 32 * 2 * 2 + 255) // 256 * 256
    a.in_dtype = _native.ENL_DTYPE_FP32
    assert lib.enl_backward_workspace_bytes(ctypes.byref(a)) == \
        2 * rows + 2 * planes(100, 4) + 2 * planes(300, 2)
    a.q = a.k = a.v = a.o = a.dout = a.lse = a.dq = a.dk = a.dv = 256
    a.head_dim = 128
    with pytest.raises(ValueError, match="head_dim <= 64"):
        _native.check(lib.enl_attn_backward(ctypes.byref(a), None), "enl_attn_backward")
    a.head_dim = 32
    a.in_dtype = 7
    with pytest.raises(ValueError, match="in_dtype=7"):
        _native.check(lib.enl_attn_backward(ctypes.byref(a), None), "enl_attn_backward")
    a.in_dtype = _native.ENL_DTYPE_FP32
    a.q_stride_b, a.q_stride_s, a.q_stride_h = 100 * 4 * 32, 4 * 32, 30  # not 16-byte in fp32
    with pytest.raises(ValueError, match="multiples of 16 bytes"):
        _native.check(lib.enl_attn_backward(ctypes.byref(a), None), "enl_attn_backward")


def test_linear_workspace_sizes():
    """Host-only arithmetic of enl_linear_workspace_bytes. Head dims up to 128
    take the tensor-core path: bf16 hi/lo planes of phi(Q) and phi(K)
    (row-major) and V' = [V | 1] transposed, the per-chunk
    states (128-row chunks) and their exclusive scan, each 256-byte aligned.
    Larger head dims take the CUDA-core pass, whose causal calls split into
    the segment count that best fills whole waves (one partial state each)."""
    lib = _native.load()

    def ws(B, H, Hkv, S, Df, D, causal):
        a = _native.LinearArgs()
        a.batch, a.num_heads, a.num_kv_heads, a.seq = B, H, Hkv, S
        a.num_features, a.head_dim, a.causal = Df, D, int(causal)
        return lib.enl_linear_workspace_bytes(ctypes.byref(a))

    def al(x):
        return (x + 255) // 256 * 256

    def tensor_path(B, H, Hkv, S, Df, D, causal):
        Dp, Dfp, Sp, nc = (D + 1 + 15) // 16 * 16, (Df + 7) // 8 * 8, (S + 7) // 8 * 8, \
            (S + 127) // 128
        return (al(2 * B * H * S * Dfp * 2) + al(2 * B * Hkv * S * Dfp * 2)
                + al(2 * B * Hkv * Dp * Sp * 2)
                + al(B * Hkv * nc * Df * Dp * 4) + al(2 * B * Hkv * nc * Dp * Dfp * 2))

    for args in [(4, 16, 16, 4096, 64, 64, True), (4, 16, 16, 4096, 256, 64, True),
                 (1, 2, 2, 1500, 64, 64, True), (4, 16, 16, 4096, 64, 64, False),
                 (2, 4, 1, 37, 100, 72, True), (1, 1, 1, 1, 8, 8, False)]:
        assert ws(*args) == tensor_path(*args), args

    def state(n, B, Hkv, Df, D):
        return n * B * Hkv * (Df * D + Df) * 4

    # head_dim 256 (CUDA-core pass): 512 CTAs per segment; 4 segments = 2048
    # CTAs, 98.8% of seven waves of 296
    assert ws(4, 16, 16, 4096, 64, 256, True) == state(4, 4, 16, 64, 256)
    assert ws(4, 16, 16, 4096, 64, 256, False) == 0
    assert ws(1, 2, 2, 255, 64, 256, True) == 0
