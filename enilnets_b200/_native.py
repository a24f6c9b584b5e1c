"""ctypes binding of libenl_b200.so (the C ABI declared in include/enl_attn.h).

There is no fallback: if the library is missing or cannot be loaded, every
entry point raises. Status codes map to the reference's error conventions:
argument problems raise ValueError (as the reference's layer builders do,
nn/layers.py:210-327), CUDA and device-side failures raise RuntimeError (as
core/backend.py:106-113 does for device problems).
"""
from __future__ import annotations

import ctypes
from ctypes import (POINTER, Structure, c_char_p, c_float, c_int32, c_int64, c_size_t,
                    c_void_p)
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libenl_b200.so"

ENL_OK = 0
ENL_ERR_INVALID = 1
ENL_ERR_UNSUPPORTED = 2
ENL_ERR_CUDA = 3
ENL_ERR_DEVICE = 4

ENL_DTYPE_BF16 = 0
ENL_DTYPE_FP32 = 1

ENL_MASK_EXCLUDE = 0
ENL_MASK_ADDITIVE = 1

DEVICE_ERRORS = {1: "an mbarrier wait exceeded its time budget",
                 2: "an index was out of range",
                 3: "a launch-time shape invariant was violated"}


ABI_VERSION = 8  # ENL_ABI_VERSION of include/enl_attn.h


class PrefillArgs(Structure):
    """Mirror of enl_prefill_args (field order and types match the header)."""
    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("o", c_void_p),
        ("lse", c_void_p),
        ("batch", c_int32), ("num_heads", c_int32), ("num_kv_heads", c_int32),
        ("seq_q", c_int32), ("seq_kv", c_int32), ("head_dim", c_int32),
        ("q_stride_b", c_int64), ("q_stride_s", c_int64), ("q_stride_h", c_int64),
        ("k_stride_b", c_int64), ("k_stride_s", c_int64), ("k_stride_h", c_int64),
        ("v_stride_b", c_int64), ("v_stride_s", c_int64), ("v_stride_h", c_int64),
        ("o_stride_b", c_int64), ("o_stride_s", c_int64), ("o_stride_h", c_int64),
        ("in_dtype", c_int32), ("out_dtype", c_int32),
        ("causal", c_int32), ("window", c_int32), ("mask_mode", c_int32),
        ("kv_valid_len", c_void_p), ("alibi_slopes", c_void_p),
        ("q_pos0", c_int64), ("k_pos0", c_int64),
        ("scale", c_float),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("kv_mask", c_void_p), ("kv_mask_stride_b", c_int64),
        ("units", c_void_p), ("n_units", c_int32),
    ]


class ProjectArgs(Structure):
    """Mirror of enl_project_args."""
    _fields_ = [
        ("x", c_void_p), ("x_stride_m", c_int64), ("x_dtype", c_int32),
        ("w", c_void_p), ("w_lo", c_void_p), ("w_stride_n", c_int64),
        ("bias", c_void_p),
        ("y", c_void_p), ("y_stride_m", c_int64), ("y_dtype", c_int32),
        ("M", c_int32), ("N", c_int32), ("K", c_int32),
        ("rope_cols", c_int32), ("rope_head_dim", c_int32), ("rope_seq", c_int32),
        ("rope_pos0", c_int64),
        ("rope_cos", c_void_p), ("rope_sin", c_void_p), ("rope_rows", c_int64),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
    ]


class DecodeArgs(Structure):
    """Mirror of enl_decode_args."""
    _fields_ = [
        ("q", c_void_p), ("q_stride_b", c_int64), ("q_stride_h", c_int64),
        ("k_cache", c_void_p), ("v_cache", c_void_p),
        ("cache_stride_b", c_int64), ("cache_stride_h", c_int64), ("cache_stride_s", c_int64),
        ("o", c_void_p), ("o_stride_b", c_int64), ("o_stride_h", c_int64),
        ("lse", c_void_p),
        ("batch", c_int32), ("num_heads", c_int32), ("num_kv_heads", c_int32),
        ("head_dim", c_int32),
        ("slot_begin", c_int32), ("slot_end", c_int32),
        ("pos_slot0", c_int64), ("q_pos", c_int64),
        ("window", c_int32), ("alibi_slopes", c_void_p), ("scale", c_float),
        ("in_dtype", c_int32), ("out_dtype", c_int32), ("n_splits", c_int32),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
    ]


class PhiArgs(Structure):
    """Mirror of enl_phi_args."""
    _fields_ = [
        ("x", c_void_p), ("x_stride_b", c_int64), ("x_stride_s", c_int64),
        ("x_stride_h", c_int64),
        ("batch", c_int32), ("seq", c_int32), ("num_heads", c_int32), ("head_dim", c_int32),
        ("in_dtype", c_int32), ("kernel", c_int32),
        ("omega", c_void_p), ("num_features", c_int32), ("global_stab", c_int32),
        ("stab_floor", c_void_p), ("stab", c_void_p), ("phi", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("phi_planes", c_void_p),
    ]


class LinearArgs(Structure):
    """Mirror of enl_linear_args."""
    _fields_ = [
        ("phi_q", c_void_p), ("phi_k", c_void_p),
        ("v", c_void_p), ("v_stride_b", c_int64), ("v_stride_s", c_int64),
        ("v_stride_h", c_int64), ("v_dtype", c_int32),
        ("o", c_void_p), ("o_stride_b", c_int64), ("o_stride_s", c_int64),
        ("o_stride_h", c_int64), ("out_dtype", c_int32),
        ("batch", c_int32), ("num_heads", c_int32), ("num_kv_heads", c_int32),
        ("seq", c_int32), ("num_features", c_int32), ("head_dim", c_int32),
        ("causal", c_int32),
        ("kv_in", c_void_p), ("ksum_in", c_void_p), ("state_scale", c_void_p),
        ("kv_out", c_void_p), ("ksum_out", c_void_p),
        ("eps", c_float),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("phi_q_planes", c_void_p), ("phi_k_planes", c_void_p),
    ]


ENL_PHI_LINEAR = 0
ENL_PHI_PERFORMER = 1


class BackwardArgs(Structure):
    """Mirror of enl_backward_args."""
    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("o", c_void_p), ("dout", c_void_p),
        ("lse", c_void_p), ("dq", c_void_p), ("dk", c_void_p), ("dv", c_void_p),
        ("batch", c_int32), ("num_heads", c_int32), ("num_kv_heads", c_int32),
        ("seq_q", c_int32), ("seq_kv", c_int32), ("head_dim", c_int32),
    ] + [(f"{t}_stride_{d}", c_int64) for t in ("q", "k", "v", "o", "do", "dq", "dk", "dv")
         for d in ("b", "s", "h")] + [
        ("o_dtype", c_int32), ("causal", c_int32), ("window", c_int32),
        ("alibi_slopes", c_void_p), ("scale", c_float),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("in_dtype", c_int32),
    ]


class SparseLayout(Structure):
    """Mirror of enl_sparse_layout."""
    _fields_ = [("tile_ptr", c_void_p), ("tile_kt", c_void_p), ("masks", c_void_p),
                ("n_entries", c_int32)]


class SparseMaskArgs(Structure):
    """Mirror of enl_sparse_mask_args."""
    _fields_ = [
        ("tile_ptr", c_void_p), ("tile_kt", c_void_p), ("masks", c_void_p),
        ("n_entries", c_int32),
        ("sel_ptr", c_void_p), ("sel_kb", c_void_p),
        ("n_qblocks", c_int32), ("n_sel", c_int32), ("qb0", c_int64),
        ("block_size", c_int32), ("seq_q", c_int32), ("seq_kv", c_int32),
        ("q_pos0", c_int64), ("k_pos0", c_int64), ("causal", c_int32),
    ]

# Exported symbol -> (argtypes, restype). Kept in sync with include/enl_attn.h
# (a CPU test checks every declared symbol is exported and bound here).
SIGNATURES = {
    "enl_attn_prefill": ([POINTER(PrefillArgs), c_void_p], c_int32),
    "enl_prefill_workspace_bytes": ([POINTER(PrefillArgs)], c_size_t),
    "enl_attn_decode": ([POINTER(DecodeArgs), c_void_p], c_int32),
    "enl_attn_decode_noalloc": ([POINTER(DecodeArgs), c_void_p], c_int32),
    "enl_decode_auto_splits": ([c_int32, c_int32, c_int32], c_int32),
    "enl_decode_workspace_bytes": ([c_int32, c_int32, c_int32, c_int32], c_size_t),
    "enl_lse_merge": ([c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p,
                       c_int64, c_int64, c_int32, c_void_p, c_void_p], c_int32),
    "enl_lse_merge_strided": ([c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int32, c_int32,
                               c_int32, c_void_p, c_int64, c_int64, c_int32, c_void_p, c_void_p],
                              c_int32),
    "enl_kv_append": ([c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64,
                       c_int64, c_int32, c_int32, c_int32, c_int32, c_int32, c_int64, c_int64,
                       c_void_p], c_int32),
    "enl_kv_gather": ([c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64,
                       c_int64, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32,
                       c_int32, c_void_p], c_int32),
    "enl_rope_apply": ([c_void_p, c_int64, c_int64, c_int64, c_int32, c_int32, c_int32,
                        c_int32, c_int32, c_void_p, c_void_p, c_int64, c_int64, c_void_p],
                       c_int32),
    "enl_linear_feature_map": ([POINTER(PhiArgs), c_void_p], c_int32),
    "enl_phi_workspace_bytes": ([POINTER(PhiArgs)], c_size_t),
    "enl_linear_attention": ([POINTER(LinearArgs), c_void_p], c_int32),
    "enl_linear_max_features": ([], c_int32),
    "enl_linear_planes_ok": ([c_int32, c_int32], c_int32),
    "enl_linear_workspace_bytes": ([POINTER(LinearArgs)], c_size_t),
    "enl_sparse_build_masks": ([POINTER(SparseMaskArgs), c_void_p], c_int32),
    "enl_attn_backward": ([POINTER(BackwardArgs), c_void_p], c_int32),
    "enl_backward_workspace_bytes": ([POINTER(BackwardArgs)], c_size_t),
    "enl_attn_prefill_sparse": ([POINTER(PrefillArgs), POINTER(SparseLayout), c_void_p],
                                c_int32),
    "enl_device_error": ([POINTER(c_int32), POINTER(c_int32), c_int32], c_int32),
    "enl_last_error": ([], c_char_p),
    "enl_abi_version": ([], c_int32),
    "enl_selftest_wait_timeout": ([c_int64, c_void_p], c_int32),
    "enl_project": ([POINTER(ProjectArgs), c_void_p], c_int32),
    "enl_project_workspace_bytes": ([POINTER(ProjectArgs)], c_size_t),
    "enl_split_bf16": ([c_void_p, c_int64, c_int64, c_int32, c_void_p, c_void_p, c_void_p],
                       c_int32),
    "enl_selftest_exp2": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_void_p], c_int32),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load the library once; raise a clear error when it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH.name} is not built (expected at {LIB_PATH}). Build it with "
            "`python -m enilnets_b200.build`; there is no CPU fallback for the attention path.")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (argtypes, restype) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    if lib.enl_abi_version() != ABI_VERSION:
        raise RuntimeError(
            f"{LIB_PATH.name} has ABI version {lib.enl_abi_version()}, these bindings expect "
            f"{ABI_VERSION}: rebuild it with `python -m enilnets_b200.build --force`.")
    _lib = lib
    return lib


def last_error() -> str:
    msg = load().enl_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    """Raise the reference-style exception for a non-zero ABI status."""
    if status == ENL_OK:
        return
    msg = f"{what}: {last_error()}"
    if status in (ENL_ERR_INVALID, ENL_ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(msg)


def device_error(clear: bool = True) -> tuple[int, int]:
    """(code, info) of the device error word; synchronises the device."""
    code, info = c_int32(0), c_int32(0)
    check(load().enl_device_error(ctypes.byref(code), ctypes.byref(info), int(clear)),
          "enl_device_error")
    return code.value, info.value


def raise_on_device_error() -> None:
    code, info = device_error(clear=True)
    if code:
        raise RuntimeError(
            f"enilnets_b200 kernel reported device error {code} "
            f"({DEVICE_ERRORS.get(code, 'unknown')}), info={info}")
