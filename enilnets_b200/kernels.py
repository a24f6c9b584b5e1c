"""Tensor-level wrappers over the C ABI: one Python function per entry point.

Tensors are torch CUDA tensors (device memory and streams are plumbing; the
math runs in libenl_b200.so). Every function launches on the current torch
stream and returns without synchronising, like the ABI itself.

Shapes follow the reference's head-split convention
(nn/forward.py:433-435): queries (B, S, H, D) and keys/values (B, S, Hkv, D)
as strided views of the projection outputs, KV caches (B, Hkv, S, D)
(nn/kvcache.py:27-30).
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _native as nat

_DTYPES = {torch.bfloat16: nat.ENL_DTYPE_BF16, torch.float32: nat.ENL_DTYPE_FP32}
_MASK_MODES = {"exclude": nat.ENL_MASK_EXCLUDE, "additive": nat.ENL_MASK_ADDITIVE}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _require_cuda(name: str, t: torch.Tensor, dtype=None, last_contiguous=True) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (got {type(t).__name__})")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype} (got {t.dtype})")
    if last_contiguous and t.stride(-1) != 1:
        raise ValueError(f"{name} must have a contiguous last (head) dimension")


def attention_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                      causal: bool = False, window: Optional[int] = None,
                      kv_valid_len: Optional[torch.Tensor] = None,
                      alibi_slopes: Optional[torch.Tensor] = None,
                      q_pos0: int = 0, k_pos0: int = 0, mask_mode: str = "exclude",
                      scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                      out_dtype: torch.dtype = torch.bfloat16,
                      return_lse: bool = False, sparse=None,
                      kv_mask: Optional[torch.Tensor] = None,
                      units: Optional[torch.Tensor] = None):
    """softmax(q k^T * scale + alibi + mask) v via the K1 tcgen05 kernel.

    q: (B, Sq, H, D); k, v: (B, Skv, Hkv, D); all bf16, or all fp32 (the
    split-bf16 path: three bf16 MMAs per product, about 2^-16 relative
    error). H % Hkv == 0 and query head h reads kv head h // (H // Hkv)
    (nn/forward.py:165-171).
    kv_valid_len: int32 (B,) -- keys [0, len_b) are real (graph/sequence.py:23-29).
    kv_mask: int64 (B, W), W >= ceil(Skv / 64) -- any key-padding mask as
    packed bits (pack_key_mask): bit c of word w set = key 64 w + c is real
    (graph/sequence.py:162-168 accepts any boolean mask, not only prefixes).
    mask_mode: "exclude" (-inf, the nn/ path) or "additive" (-1e9 per violated
    mask term, graph/sequence.py:162-176).
    units: int32 (n,) device list of the (batch, head) units b * H + h to
    compute (a rank's share of sharding.partition_units); rows of other
    units are left untouched. None = all.
    sparse: a block-sparse layout (enilnets_b200.sparse.SparseLayout) built for
    these Sq, Skv, q_pos0 and k_pos0; it is then the whole mask (causal only
    picks the ALiBi distance), nn/sparse_attention.py:96-142.
    Returns out (B, Sq, H, D) [and lse (B, H, Sq) fp32].
    """
    if q.dtype not in _DTYPES:
        raise ValueError(f"q must be bfloat16 or float32 (got {q.dtype})")
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda(name, t, q.dtype)
        if t.dim() != 4:
            raise ValueError(f"{name} must be 4-D (batch, seq, heads, head_dim)")
    B, Sq, H, D = q.shape
    Bk, Skv, Hkv, Dk = k.shape
    if tuple(v.shape) != (Bk, Skv, Hkv, Dk) or Bk != B or Dk != D:
        raise ValueError(f"shape mismatch: q {tuple(q.shape)}, k {tuple(k.shape)}, "
                         f"v {tuple(v.shape)}")
    if mask_mode not in _MASK_MODES:
        raise ValueError(f"mask_mode must be one of {sorted(_MASK_MODES)}, got {mask_mode!r}")
    if out is None:
        out = torch.empty((B, Sq, H, D), device=q.device, dtype=out_dtype)
    _require_cuda("out", out)
    if tuple(out.shape) != (B, Sq, H, D) or out.dtype not in _DTYPES:
        raise ValueError(f"out must be ({B}, {Sq}, {H}, {D}) bf16/fp32")
    lse = torch.empty((B, H, Sq), device=q.device, dtype=torch.float32) if return_lse else None
    if Skv == 0 and B * Sq > 0:
        # A softmax over no keys: the reference's reduction over an empty key
        # axis raises too.
        raise ValueError("attention over no keys (seq_kv = 0)")
    if B == 0 or Sq == 0:
        # Nothing to compute: the reference returns the empty result as well.
        return (out, lse) if return_lse else out
    if kv_valid_len is not None:
        _require_cuda("kv_valid_len", kv_valid_len, torch.int32, last_contiguous=False)
        if tuple(kv_valid_len.shape) != (B,) or not kv_valid_len.is_contiguous():
            raise ValueError(f"kv_valid_len must be a contiguous int32 ({B},) tensor")
    if alibi_slopes is not None:
        _require_cuda("alibi_slopes", alibi_slopes, torch.float32, last_contiguous=False)
        if tuple(alibi_slopes.shape) != (H,) or not alibi_slopes.is_contiguous():
            raise ValueError(f"alibi_slopes must be a contiguous float32 ({H},) tensor")
    if kv_mask is not None:
        _require_cuda("kv_mask", kv_mask, torch.int64)
        if kv_mask.dim() != 2 or kv_mask.shape[0] != B or kv_mask.shape[1] * 64 < Skv:
            raise ValueError(f"kv_mask must be int64 ({B}, >= {(Skv + 63) // 64}) packed words, "
                             f"got {tuple(kv_mask.shape)}")
        if sparse is not None:
            raise ValueError("kv_mask cannot be combined with a sparse layout")
    a = nat.PrefillArgs()
    a.q, a.k, a.v, a.o, a.lse = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), _ptr(lse)
    a.batch, a.num_heads, a.num_kv_heads = B, H, Hkv
    a.seq_q, a.seq_kv, a.head_dim = Sq, Skv, D
    a.q_stride_b, a.q_stride_s, a.q_stride_h = q.stride(0), q.stride(1), q.stride(2)
    a.k_stride_b, a.k_stride_s, a.k_stride_h = k.stride(0), k.stride(1), k.stride(2)
    a.v_stride_b, a.v_stride_s, a.v_stride_h = v.stride(0), v.stride(1), v.stride(2)
    a.o_stride_b, a.o_stride_s, a.o_stride_h = out.stride(0), out.stride(1), out.stride(2)
    a.in_dtype = _DTYPES[q.dtype]
    a.out_dtype = _DTYPES[out.dtype]
    a.causal = int(bool(causal))
    a.window = -1 if window is None else int(window)
    a.mask_mode = _MASK_MODES[mask_mode]
    a.kv_valid_len = _ptr(kv_valid_len)
    a.alibi_slopes = _ptr(alibi_slopes)
    a.q_pos0, a.k_pos0 = int(q_pos0), int(k_pos0)
    a.scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    if kv_mask is not None:
        a.kv_mask, a.kv_mask_stride_b = kv_mask.data_ptr(), kv_mask.stride(0)
    if units is not None:
        _require_cuda("units", units, torch.int32, last_contiguous=False)
        if units.dim() != 1 or not units.is_contiguous():
            raise ValueError("units must be a contiguous int32 1-D tensor")
        a.units, a.n_units = units.data_ptr(), units.numel()
    lib = nat.load()
    ws = None
    need = int(lib.enl_prefill_workspace_bytes(ctypes.byref(a)))
    if need > 0:
        # Stream-ordered by torch's caching allocator, freed after the launch.
        ws = torch.empty(need, dtype=torch.uint8, device=q.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), need
    if sparse is None:
        nat.check(lib.enl_attn_prefill(ctypes.byref(a), _stream()), "enl_attn_prefill")
    else:
        if (sparse.seq_q, sparse.seq_kv, sparse.q_pos0, sparse.k_pos0) != (Sq, Skv, int(q_pos0),
                                                                           int(k_pos0)):
            raise ValueError(
                f"sparse layout is for seq_q={sparse.seq_q} seq_kv={sparse.seq_kv} "
                f"q_pos0={sparse.q_pos0} k_pos0={sparse.k_pos0}, not {Sq}, {Skv}, {q_pos0}, "
                f"{k_pos0}")
        for name in ("tile_ptr", "tile_kt", "masks"):
            if getattr(sparse, name).device != q.device:
                raise ValueError(f"sparse layout {name} is on {getattr(sparse, name).device}, "
                                 f"not {q.device}")
        nat.check(lib.enl_attn_prefill_sparse(ctypes.byref(a), ctypes.byref(sparse.native()),
                                              _stream()), "enl_attn_prefill_sparse")
    return (out, lse) if return_lse else out


def split_bf16(w: torch.Tensor):
    """fp32 (rows, cols) -> contiguous bf16 planes (hi, lo), hi = bf16(w),
    lo = bf16(w - hi): the weight operand of project() for fp32 inputs."""
    _require_cuda("w", w, torch.float32)
    if w.dim() != 2:
        raise ValueError("w must be 2-D (rows, cols)")
    rows, cols = w.shape
    hi = torch.empty((rows, cols), dtype=torch.bfloat16, device=w.device)
    lo = torch.empty_like(hi)
    nat.check(nat.load().enl_split_bf16(w.data_ptr(), w.stride(0), rows, cols, hi.data_ptr(),
                                        lo.data_ptr(), _stream()), "enl_split_bf16")
    return hi, lo


def project(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None, *,
            w_lo: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
            out_dtype: Optional[torch.dtype] = None, rope=None) -> torch.Tensor:
    """y = x @ w.T + bias on the K6 tcgen05 GEMM (nn/forward.py:428-430, :551).

    x: (..., K) bf16, or fp32 with w_lo given (the split-bf16 path: w = the hi
    plane, w_lo the lo plane from split_bf16). w: (N, K) bf16. bias: fp32 (N,).
    rope: optional (cos, sin, rot_cols, head_dim, seq, pos0): rotate-half RoPE
    (nn/forward.py:80-88) fused into the epilogue on columns < rot_cols, heads
    of head_dim columns, row r of x at position pos0 + (r % seq); cos/sin fp32
    (rows, head_dim / 2) tables. Returns y (..., N), out_dtype (default: x's).
    """
    _require_cuda("x", x)
    _require_cuda("w", w, torch.bfloat16)
    if x.dtype not in _DTYPES:
        raise ValueError(f"x must be bfloat16 or float32 (got {x.dtype})")
    if w.dim() != 2 or x.shape[-1] != w.shape[1]:
        raise ValueError(f"shape mismatch: x {tuple(x.shape)}, w {tuple(w.shape)}")
    lead = x.shape[:-1]
    K, N = w.shape[1], w.shape[0]
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    out_dtype = out_dtype or x.dtype
    if out is None:
        out = torch.empty(lead + (N,), dtype=out_dtype, device=x.device)
    _require_cuda("out", out)
    y2 = out.view(-1, N)
    a = nat.ProjectArgs()
    a.x, a.x_stride_m, a.x_dtype = x2.data_ptr(), x2.stride(0), _DTYPES[x.dtype]
    a.w, a.w_stride_n = w.data_ptr(), w.stride(0)
    if w_lo is not None:
        _require_cuda("w_lo", w_lo, torch.bfloat16)
        if w_lo.shape != w.shape or w_lo.stride() != w.stride():
            raise ValueError("w_lo must match w's shape and strides")
        a.w_lo = w_lo.data_ptr()
    if bias is not None:
        _require_cuda("bias", bias, torch.float32, last_contiguous=False)
        if tuple(bias.shape) != (N,) or not bias.is_contiguous():
            raise ValueError(f"bias must be a contiguous float32 ({N},) tensor")
        a.bias = bias.data_ptr()
    a.y, a.y_stride_m, a.y_dtype = y2.data_ptr(), y2.stride(0), _DTYPES[out.dtype]
    a.M, a.N, a.K = M, N, K
    if rope is not None:
        cos, sin, cols, hd, seq, pos0 = rope
        for name, t in (("cos", cos), ("sin", sin)):
            _require_cuda(name, t, torch.float32)
            if not t.is_contiguous() or t.dim() != 2 or t.shape[1] != hd // 2:
                raise ValueError(f"rope {name} must be a contiguous fp32 (rows, {hd // 2}) table")
        a.rope_cols, a.rope_head_dim, a.rope_seq, a.rope_pos0 = int(cols), int(hd), int(seq), \
            int(pos0)
        a.rope_cos, a.rope_sin, a.rope_rows = cos.data_ptr(), sin.data_ptr(), cos.shape[0]
    lib = nat.load()
    need = int(lib.enl_project_workspace_bytes(ctypes.byref(a)))
    ws = None
    if need > 0:
        ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), need
    nat.check(lib.enl_project(ctypes.byref(a), _stream()), "enl_project")
    return out


def attention_backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor,
                       lse: torch.Tensor, dout: torch.Tensor, *, causal: bool = False,
                       window: Optional[int] = None,
                       alibi_slopes: Optional[torch.Tensor] = None,
                       scale: Optional[float] = None, out=None):
    """dQ, dK, dV of attention_prefill (K5, nn/flash_attention.py:83-114).

    q: (B, Sq, H, D), k, v: (B, Skv, Hkv, D), dout like o: one dtype, bf16
    (the forward's operands) or fp32 (split into bf16 hi/lo planes, three
    MMAs per product, as attention_prefill does for fp32; D <= 64); o: the
    forward output, bf16 or fp32; lse: (B, H, Sq) fp32 from
    attention_prefill(..., return_lse=True). Returns fp32 dq (B, Sq, H, D) and
    dk, dv (B, Skv, Hkv, D), dk/dv summed over each kv head's query heads;
    out=(dq, dk, dv) writes into given fp32 views of those shapes instead
    (any strides with a contiguous head dim).
    """
    in_dt = q.dtype if isinstance(q, torch.Tensor) else None
    if in_dt not in _DTYPES:
        raise ValueError(f"q must be bfloat16 or float32 (got {in_dt})")
    for name, t in (("q", q), ("k", k), ("v", v), ("dout", dout)):
        _require_cuda(name, t, in_dt)
        if t.dim() != 4:
            raise ValueError(f"{name} must be 4-D (batch, seq, heads, head_dim)")
    _require_cuda("o", o)
    if o.dtype not in _DTYPES:
        raise ValueError(f"o must be bfloat16 or float32 (got {o.dtype})")
    B, Sq, H, D = q.shape
    Bk, Skv, Hkv, Dk = k.shape
    if tuple(v.shape) != (Bk, Skv, Hkv, Dk) or Bk != B or Dk != D:
        raise ValueError(f"shape mismatch: q {tuple(q.shape)}, k {tuple(k.shape)}, "
                         f"v {tuple(v.shape)}")
    if tuple(o.shape) != (B, Sq, H, D) or tuple(dout.shape) != (B, Sq, H, D):
        raise ValueError(f"o and dout must be {(B, Sq, H, D)}")
    _require_cuda("lse", lse, torch.float32, last_contiguous=False)
    if tuple(lse.shape) != (B, H, Sq) or not lse.is_contiguous():
        raise ValueError(f"lse must be a contiguous float32 {(B, H, Sq)} tensor")
    if alibi_slopes is not None:
        _require_cuda("alibi_slopes", alibi_slopes, torch.float32, last_contiguous=False)
        if tuple(alibi_slopes.shape) != (H,) or not alibi_slopes.is_contiguous():
            raise ValueError(f"alibi_slopes must be a contiguous float32 ({H},) tensor")
    if out is None:
        dq = torch.empty((B, Sq, H, D), device=q.device, dtype=torch.float32)
        dk = torch.empty((B, Skv, Hkv, D), device=q.device, dtype=torch.float32)
        dv = torch.empty((B, Skv, Hkv, D), device=q.device, dtype=torch.float32)
    else:
        dq, dk, dv = out
        for name, t, shape in (("dq", dq, (B, Sq, H, D)), ("dk", dk, (B, Skv, Hkv, D)),
                               ("dv", dv, (B, Skv, Hkv, D))):
            _require_cuda(name, t, torch.float32)
            if tuple(t.shape) != shape:
                raise ValueError(f"{name} must be {shape}, got {tuple(t.shape)}")
    if B == 0 or Sq == 0 or Skv == 0:
        # No (query, key) pair: every gradient is zero (empty when B == 0).
        for t in (dq, dk, dv):
            t.zero_()
        return dq, dk, dv
    a = nat.BackwardArgs()
    a.q, a.k, a.v, a.o, a.dout = (t.data_ptr() for t in (q, k, v, o, dout))
    a.lse, a.dq, a.dk, a.dv = lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    a.batch, a.num_heads, a.num_kv_heads = B, H, Hkv
    a.seq_q, a.seq_kv, a.head_dim = Sq, Skv, D
    for name, t in (("q", q), ("k", k), ("v", v), ("o", o), ("do", dout), ("dq", dq),
                    ("dk", dk), ("dv", dv)):
        setattr(a, f"{name}_stride_b", t.stride(0))
        setattr(a, f"{name}_stride_s", t.stride(1))
        setattr(a, f"{name}_stride_h", t.stride(2))
    a.o_dtype = _DTYPES[o.dtype]
    a.in_dtype = _DTYPES[in_dt]
    a.causal = int(bool(causal))
    a.window = -1 if window is None else int(window)
    a.alibi_slopes = _ptr(alibi_slopes)
    a.scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    lib = nat.load()
    need = int(lib.enl_backward_workspace_bytes(ctypes.byref(a)))
    ws = torch.empty(need, dtype=torch.uint8, device=q.device)
    a.workspace, a.workspace_bytes = ws.data_ptr(), need
    nat.check(lib.enl_attn_backward(ctypes.byref(a), _stream()), "enl_attn_backward")
    return dq, dk, dv


def sparse_build_masks(tile_ptr: torch.Tensor, tile_kt: torch.Tensor, masks: torch.Tensor,
                       sel_ptr: torch.Tensor, sel_kb: torch.Tensor, *, qb0: int,
                       block_size: int, seq_q: int, seq_kv: int, q_pos0: int, k_pos0: int,
                       causal: bool) -> None:
    """Fill a block-sparse layout's column masks on the device from the
    per-query-block selection (nn/sparse_attention.py:48-84, :130-134)."""
    for name, t, dt in (("tile_ptr", tile_ptr, torch.int32), ("tile_kt", tile_kt, torch.int32),
                        ("masks", masks, torch.int64), ("sel_ptr", sel_ptr, torch.int32),
                        ("sel_kb", sel_kb, torch.int32)):
        _require_cuda(name, t, dt, last_contiguous=False)
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    n_entries = tile_kt.numel()
    if masks.numel() != n_entries * 256:
        raise ValueError(f"masks must hold {n_entries} x 2 x 128 words, got {masks.numel()}")
    a = nat.SparseMaskArgs()
    a.tile_ptr, a.tile_kt, a.masks = tile_ptr.data_ptr(), tile_kt.data_ptr(), masks.data_ptr()
    a.n_entries = n_entries
    a.sel_ptr, a.sel_kb = sel_ptr.data_ptr(), sel_kb.data_ptr()
    a.n_qblocks, a.n_sel, a.qb0 = sel_ptr.numel() - 1, sel_kb.numel(), int(qb0)
    a.block_size, a.seq_q, a.seq_kv = int(block_size), int(seq_q), int(seq_kv)
    a.q_pos0, a.k_pos0, a.causal = int(q_pos0), int(k_pos0), int(bool(causal))
    nat.check(nat.load().enl_sparse_build_masks(ctypes.byref(a), _stream()),
              "enl_sparse_build_masks")


def key_mask_words(mask):
    """Boolean (B, S) key-padding mask (True = real token) -> host int64
    (B, ceil(S / 64)) words, bit c of word w = key 64 w + c, as the
    prefill's kv_mask takes it."""
    import numpy as np
    m = np.ascontiguousarray(np.asarray(mask, dtype=bool))
    if m.ndim != 2:
        raise ValueError(f"key mask must be (batch, seq), got shape {m.shape}")
    B, S = m.shape
    W = max(1, (S + 63) // 64)
    padded = np.zeros((B, W * 64), dtype=bool)
    padded[:, :S] = m
    words = np.packbits(padded.reshape(B, W, 8, 8), axis=-1, bitorder="little")
    return words.reshape(B, W * 8).view("<i8").copy()


def pack_key_mask(mask, device) -> torch.Tensor:
    """key_mask_words(mask) as a device tensor."""
    return torch.from_numpy(key_mask_words(mask)).to(device)


_workspaces: dict = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Split-partial scratch of attention_decode and linear_attention, one per
    (device, stream): calls on one stream run in order and may share it;
    calls on different streams get their own, so they never race. A buffer
    that grows is replaced under the same stream it was allocated on, so
    torch's stream-ordered allocator reuses the old one only after the
    kernels queued before it."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (index, torch.cuda.current_stream(index).cuda_stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def decode_workspace_bytes(batch: int, num_heads: int, head_dim: int, n_splits: int) -> int:
    return int(nat.load().enl_decode_workspace_bytes(batch, num_heads, head_dim, n_splits))


def decode_auto_splits(batch: int, num_kv_heads: int, n_slots: int) -> int:
    return int(nat.load().enl_decode_auto_splits(batch, num_kv_heads, max(1, n_slots)))


def attention_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, *,
                     slot_begin: int, slot_end: int, pos_slot0: int, q_pos: int,
                     window: Optional[int] = None,
                     alibi_slopes: Optional[torch.Tensor] = None,
                     scale: Optional[float] = None, n_splits: int = 0,
                     out: Optional[torch.Tensor] = None,
                     out_dtype: torch.dtype = torch.bfloat16,
                     workspace: Optional[torch.Tensor] = None,
                     return_lse: bool = False, lse_out: Optional[torch.Tensor] = None):
    """One-token decode via the K2 split-KV kernel.

    q: (B, H, D); k_cache/v_cache: (B, Hkv, capacity, D) with equal strides,
    all bf16 or all fp32; live slots [slot_begin, slot_end), slot s at absolute position
    pos_slot0 + s; the query sits at q_pos (keys after it are invisible).
    Returns out (B, H, D) [and lse (B, H) fp32].
    """
    if q.dtype not in _DTYPES:
        raise ValueError(f"q must be bfloat16 or float32 (got {q.dtype})")
    _require_cuda("q", q, q.dtype)
    _require_cuda("k_cache", k_cache, q.dtype)
    _require_cuda("v_cache", v_cache, q.dtype)
    if q.dim() != 3 or k_cache.dim() != 4:
        raise ValueError("q must be (B, H, D) and caches (B, Hkv, capacity, D)")
    if k_cache.shape != v_cache.shape or k_cache.stride() != v_cache.stride():
        raise ValueError("k_cache and v_cache must have the same shape and strides")
    B, H, D = q.shape
    Bc, Hkv, cap, Dc = k_cache.shape
    if Bc != B or Dc != D:
        raise ValueError(f"shape mismatch: q {tuple(q.shape)} vs cache {tuple(k_cache.shape)}")
    if not (0 <= slot_begin <= slot_end <= cap):
        raise ValueError(f"slot range [{slot_begin}, {slot_end}) outside capacity {cap}")
    if out is None:
        out = torch.empty((B, H, D), device=q.device, dtype=out_dtype)
    _require_cuda("out", out)
    if tuple(out.shape) != (B, H, D) or out.dtype not in _DTYPES:
        raise ValueError(f"out must be ({B}, {H}, {D}) bf16/fp32")
    lse = torch.empty((B, H), device=q.device, dtype=torch.float32) if return_lse else None
    if lse_out is not None:
        _require_cuda("lse_out", lse_out, torch.float32, last_contiguous=False)
        if tuple(lse_out.shape) != (B, H) or lse_out.stride() != (H, 1):
            raise ValueError(f"lse_out must be a contiguous float32 ({B}, {H}) tensor")
        lse = lse_out
    if alibi_slopes is not None:
        _require_cuda("alibi_slopes", alibi_slopes, torch.float32, last_contiguous=False)
    if B == 0:
        return (out, lse) if (return_lse or lse_out is not None) else out
    n_slots = max(1, slot_end - slot_begin)
    splits = n_splits if n_splits > 0 else decode_auto_splits(B, Hkv, n_slots)
    need = decode_workspace_bytes(B, H, D, splits)
    if workspace is None and need > 0:
        workspace = _workspace(q.device, need)
    a = nat.DecodeArgs()
    a.q, a.q_stride_b, a.q_stride_h = q.data_ptr(), q.stride(0), q.stride(1)
    a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    a.cache_stride_b, a.cache_stride_h, a.cache_stride_s = (k_cache.stride(0), k_cache.stride(1),
                                                            k_cache.stride(2))
    a.o, a.o_stride_b, a.o_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
    a.lse = _ptr(lse)
    a.batch, a.num_heads, a.num_kv_heads, a.head_dim = B, H, Hkv, D
    a.slot_begin, a.slot_end = int(slot_begin), int(slot_end)
    a.pos_slot0, a.q_pos = int(pos_slot0), int(q_pos)
    a.window = -1 if window is None else int(window)
    a.alibi_slopes = _ptr(alibi_slopes)
    a.scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    a.in_dtype, a.out_dtype = _DTYPES[q.dtype], _DTYPES[out.dtype]
    a.n_splits = int(splits)
    a.workspace = _ptr(workspace)
    a.workspace_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    nat.check(nat.load().enl_attn_decode(ctypes.byref(a), _stream()), "enl_attn_decode")
    return (out, lse) if (return_lse or lse_out is not None) else out


def lse_merge(part_o: torch.Tensor, part_lse: torch.Tensor, *,
              out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.bfloat16,
              return_lse: bool = False):
    """Merge (n_parts, B, H, D) fp32 partials by their (n_parts, B, H) LSEs.
    Each part must be contiguous; the parts may sit any distance apart (a
    gathered buffer of packed [out | lse] parts is merged in place)."""
    _require_cuda("part_o", part_o, torch.float32)
    _require_cuda("part_lse", part_lse, torch.float32, last_contiguous=False)
    P, B, H, D = part_o.shape
    if tuple(part_lse.shape) != (P, B, H):
        raise ValueError("part_lse must be (n_parts, B, H)")
    if part_o[0].stride() != (H * D, D, 1) or part_lse[0].stride() != (H, 1):
        raise ValueError("each part of part_o / part_lse must be contiguous")
    if out is None:
        out = torch.empty((B, H, D), device=part_o.device, dtype=out_dtype)
    lse = torch.empty((B, H), device=part_o.device, dtype=torch.float32) if return_lse else None
    nat.check(nat.load().enl_lse_merge_strided(
        part_o.data_ptr(), part_o.stride(0), part_lse.data_ptr(), part_lse.stride(0), P, B, H,
        D, out.data_ptr(), out.stride(0), out.stride(1), _DTYPES[out.dtype], _ptr(lse),
        _stream()), "enl_lse_merge_strided")
    return (out, lse) if return_lse else out


def kv_append(cache: torch.Tensor, src: torch.Tensor, slot0: int) -> None:
    """cache[b, h, slot0 + t] = src[b, t, h] for a (B, Hkv, cap, D) cache and a
    (B, n_new, Hkv, D) source (the head-split projection output)."""
    _require_cuda("cache", cache)
    _require_cuda("src", src)
    if cache.dtype != src.dtype or cache.dtype not in _DTYPES:
        raise ValueError("cache and src must share a bf16/fp32 dtype")
    B, Hkv, cap, D = cache.shape
    Bs, n_new, Hs, Ds = src.shape
    if (Bs, Hs, Ds) != (B, Hkv, D):
        raise ValueError(f"src {tuple(src.shape)} does not match cache {tuple(cache.shape)}")
    nat.check(nat.load().enl_kv_append(cache.data_ptr(), cache.stride(0), cache.stride(1),
                                       cache.stride(2), src.data_ptr(), src.stride(0),
                                       src.stride(1), src.stride(2), B, Hkv, n_new, D,
                                       _DTYPES[cache.dtype], int(slot0), cap, _stream()),
              "enl_kv_append")


def kv_gather(dst: torch.Tensor, src: torch.Tensor, index: torch.Tensor, slot_begin: int,
              slot_end: int) -> None:
    """dst[i, :, s] = src[index[i], :, s] for s in [slot_begin, slot_end)."""
    _require_cuda("dst", dst)
    _require_cuda("src", src)
    _require_cuda("index", index, torch.int64, last_contiguous=False)
    if dst.dtype != src.dtype or dst.shape[1:] != src.shape[1:]:
        raise ValueError("dst and src must agree in dtype and (Hkv, cap, D)")
    if tuple(index.shape) != (dst.shape[0],) or not index.is_contiguous():
        raise ValueError("index must be a contiguous int64 (B_out,) tensor")
    nat.check(nat.load().enl_kv_gather(dst.data_ptr(), dst.stride(0), dst.stride(1),
                                       dst.stride(2), src.data_ptr(), src.stride(0),
                                       src.stride(1), src.stride(2), index.data_ptr(),
                                       dst.shape[0], src.shape[0], src.shape[1], int(slot_begin),
                                       int(slot_end), src.shape[3], _DTYPES[src.dtype],
                                       _stream()),
              "enl_kv_gather")


def rope_(x: torch.Tensor, cos_table: torch.Tensor, sin_table: torch.Tensor,
          row0: int) -> torch.Tensor:
    """Rotate x (B, S, H, D) in place; sequence row s uses table row row0 + s."""
    _require_cuda("x", x)
    _require_cuda("cos_table", cos_table, torch.float32)
    _require_cuda("sin_table", sin_table, torch.float32)
    B, S, H, D = x.shape
    if cos_table.shape != sin_table.shape or cos_table.shape[1] != D // 2:
        raise ValueError("cos/sin tables must both be (rows, head_dim/2)")
    nat.check(nat.load().enl_rope_apply(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2), B, S,
                                        H, D, _DTYPES[x.dtype], cos_table.data_ptr(),
                                        sin_table.data_ptr(), int(row0), cos_table.shape[0],
                                        _stream()),
              "enl_rope_apply")
    return x


_PHI_KERNELS = {"linear": nat.ENL_PHI_LINEAR, "performer": nat.ENL_PHI_PERFORMER}


def linear_planes_ok(head_dim: int, num_features: int) -> bool:
    """Whether linear_attention takes phi planes for these sizes (its
    tensor-core path)."""
    return bool(nat.load().enl_linear_planes_ok(int(head_dim), int(num_features)))


def linear_feature_map(x: torch.Tensor, kernel: str, omega: Optional[torch.Tensor] = None, *,
                       global_stab: bool = False, stab_floor: Optional[torch.Tensor] = None,
                       planes: bool = False):
    """phi(x) of the linearized attention kernels (nn/attention_kernels.py:58-74).

    x: (B, S, H, Dh) bf16/fp32 head view. kernel "linear" (elu + 1) or
    "performer" with omega (Df, Dh) fp32. Returns (phi (B, H, S, Df) fp32,
    stab (B, H) fp32 or None): with global_stab (keys) one stabilizer per
    (b, h), the max of w.x' over every row and stab_floor; otherwise (queries)
    each row's own max. With planes, phi comes back as its bf16 hi/lo planes
    (2, B, H, S, Dfp), Dfp = Df rounded up to 8, hi = bf16(phi) and
    lo = bf16(phi - hi): the operand layout linear_attention reads on its
    tensor-core path."""
    if kernel not in _PHI_KERNELS:
        raise ValueError(f"Unknown attention feature map: {kernel!r}")
    _require_cuda("x", x)
    if x.dtype not in _DTYPES or x.dim() != 4:
        raise ValueError("x must be a 4-D bf16 or fp32 tensor (batch, seq, heads, head_dim)")
    B, S, H, Dh = x.shape
    performer = kernel == "performer"
    if performer:
        _require_cuda("omega", omega, torch.float32)
        if omega.dim() != 2 or omega.shape[1] != Dh or not omega.is_contiguous():
            raise ValueError(f"omega must be a contiguous (num_features, {Dh}) fp32 tensor")
    Df = omega.shape[0] if performer else Dh
    if B * S == 0:
        # No rows: an empty map; a key stabilizer stays at its floor (-inf
        # without one), as a carried decode state expects.
        phi = torch.empty((2, B, H, S, (Df + 7) // 8 * 8) if planes else (B, H, S, Df),
                          device=x.device, dtype=torch.bfloat16 if planes else torch.float32)
        stab = None
        if performer and global_stab:
            stab = stab_floor.reshape(B, H).clone().float() if stab_floor is not None else \
                torch.full((B, H), -math.inf, device=x.device, dtype=torch.float32)
        return phi, stab
    if planes:
        phi = torch.empty((2, B, H, S, (Df + 7) // 8 * 8), device=x.device, dtype=torch.bfloat16)
    else:
        phi = torch.empty((B, H, S, Df), device=x.device, dtype=torch.float32)
    stab = None
    if performer and global_stab:
        stab = torch.empty((B, H), device=x.device, dtype=torch.float32)
        if stab_floor is not None:
            _require_cuda("stab_floor", stab_floor, torch.float32, last_contiguous=False)
            stab_floor = stab_floor.reshape(B, H).contiguous()
    a = nat.PhiArgs()
    a.x = x.data_ptr()
    a.x_stride_b, a.x_stride_s, a.x_stride_h = x.stride(0), x.stride(1), x.stride(2)
    a.batch, a.seq, a.num_heads, a.head_dim = B, S, H, Dh
    a.in_dtype = _DTYPES[x.dtype]
    a.kernel = _PHI_KERNELS[kernel]
    a.omega = _ptr(omega) if performer else None
    a.num_features = Df if performer else 0
    a.global_stab = int(performer and global_stab)
    a.stab_floor = _ptr(stab_floor) if stab is not None else None
    a.stab = _ptr(stab)
    if planes:
        a.phi, a.phi_planes = None, phi.data_ptr()
    else:
        a.phi = phi.data_ptr()
    lib = nat.load()
    need = int(lib.enl_phi_workspace_bytes(ctypes.byref(a)))
    ws = None
    if need > 0:
        ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), need
    nat.check(lib.enl_linear_feature_map(ctypes.byref(a), _stream()), "enl_linear_feature_map")
    return phi, stab


def linear_attention(phi_q: torch.Tensor, phi_k: torch.Tensor, v: torch.Tensor, *,
                     causal: bool, state=None, state_scale: Optional[torch.Tensor] = None,
                     return_state: bool = False, out_dtype: torch.dtype = torch.float32,
                     eps: float = 1e-20, num_features: Optional[int] = None):
    """Linear attention over feature-mapped queries/keys
    (nn/attention_kernels.py:119-143). phi_q (B, H, S, Df), phi_k (B, Hkv, S, Df)
    fp32, or both as the bf16 planes linear_feature_map(planes=True) returns
    (2, B, H, S, Dfp) / (2, B, Hkv, S, Dfp) with num_features=Df (sizes where
    linear_planes_ok holds); v (B, S, Hkv, D) bf16/fp32 head view. Causal:
    prefix sums, starting from state = (kv (B, Hkv, Df, D), ksum (B, Hkv, Df))
    times state_scale (B, Hkv) when given; with return_state the sums after the
    last row are returned too. Returns out (B, S, H, D) [, (kv, ksum)]."""
    planes = phi_q.dim() == 5
    for name, t in (("phi_q", phi_q), ("phi_k", phi_k)):
        if planes:
            _require_cuda(name, t, torch.bfloat16)
            if t.dim() != 5 or t.shape[0] != 2 or not t.is_contiguous():
                raise ValueError(f"{name} planes must be a contiguous (2, B, H, S, Dfp) bf16 tensor")
        else:
            _require_cuda(name, t, torch.float32)
            if t.dim() != 4 or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous 4-D fp32 tensor")
    _require_cuda("v", v)
    if v.dtype not in _DTYPES or v.dim() != 4:
        raise ValueError("v must be a 4-D bf16 or fp32 tensor (batch, seq, kv_heads, head_dim)")
    if planes:
        if num_features is None:
            raise ValueError("phi planes need num_features")
        B, H, S, Dfp = phi_q.shape[1:]
        _, _, Hkv, Sk, Dfpk = phi_k.shape
        Df, Dfk = int(num_features), int(num_features)
        if Dfp != (Df + 7) // 8 * 8 or Dfpk != Dfp:
            raise ValueError(f"phi planes of width {Dfp}/{Dfpk} do not hold {Df} features")
    else:
        B, H, S, Df = phi_q.shape
        _, Hkv, Sk, Dfk = phi_k.shape
    D = v.shape[3]
    if planes and not linear_planes_ok(D, Df):
        raise ValueError(f"phi planes need linear_planes_ok({D}, {Df})")
    if (phi_k.shape[-4], Sk, Dfk) != (B, S, Df) or tuple(v.shape[:3]) != (B, S, Hkv):
        raise ValueError(f"shape mismatch: phi_q {tuple(phi_q.shape)}, phi_k "
                         f"{tuple(phi_k.shape)}, v {tuple(v.shape)}")
    if (state is not None or return_state) and not causal:
        raise ValueError("a carried state needs causal attention")
    out = torch.empty((B, S, H, D), device=phi_q.device, dtype=out_dtype)
    new_state = None
    if return_state:
        new_state = (torch.empty((B, Hkv, Df, D), device=phi_q.device, dtype=torch.float32),
                     torch.empty((B, Hkv, Df), device=phi_q.device, dtype=torch.float32))
    if state is not None:
        for name, t, shape in (("kv", state[0], (B, Hkv, Df, D)), ("ksum", state[1], (B, Hkv, Df))):
            _require_cuda(name, t, torch.float32)
            if tuple(t.shape) != shape or not t.is_contiguous():
                raise ValueError(f"state {name} must be a contiguous fp32 {shape} tensor")
        if state_scale is not None:
            _require_cuda("state_scale", state_scale, torch.float32, last_contiguous=False)
            state_scale = state_scale.reshape(B, Hkv).contiguous()
    if B == 0 or S == 0:
        # No rows: the output is empty and the sums after the last row are
        # the carried state (times its scale), or zero.
        if new_state is not None:
            if state is None:
                new_state[0].zero_()
                new_state[1].zero_()
            else:
                sc = state_scale if state_scale is not None else \
                    torch.ones((B, Hkv), device=phi_q.device, dtype=torch.float32)
                torch.mul(state[0], sc[:, :, None, None], out=new_state[0])
                torch.mul(state[1], sc[:, :, None], out=new_state[1])
        return (out, new_state) if return_state else out
    a = nat.LinearArgs()
    if planes:
        a.phi_q_planes, a.phi_k_planes = phi_q.data_ptr(), phi_k.data_ptr()
    else:
        a.phi_q, a.phi_k = phi_q.data_ptr(), phi_k.data_ptr()
    a.v = v.data_ptr()
    a.v_stride_b, a.v_stride_s, a.v_stride_h = v.stride(0), v.stride(1), v.stride(2)
    a.v_dtype = _DTYPES[v.dtype]
    a.o = out.data_ptr()
    a.o_stride_b, a.o_stride_s, a.o_stride_h = out.stride(0), out.stride(1), out.stride(2)
    a.out_dtype = _DTYPES[out_dtype]
    a.batch, a.num_heads, a.num_kv_heads, a.seq = B, H, Hkv, S
    a.num_features, a.head_dim = Df, D
    a.causal = int(bool(causal))
    a.kv_in = _ptr(state[0]) if state is not None else None
    a.ksum_in = _ptr(state[1]) if state is not None else None
    a.state_scale = _ptr(state_scale) if state is not None else None
    a.kv_out = _ptr(new_state[0]) if new_state is not None else None
    a.ksum_out = _ptr(new_state[1]) if new_state is not None else None
    a.eps = float(eps)
    lib = nat.load()
    ws_bytes = lib.enl_linear_workspace_bytes(ctypes.byref(a))
    if ws_bytes:
        ws = _workspace(phi_q.device, ws_bytes)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws_bytes
    nat.check(lib.enl_linear_attention(ctypes.byref(a), _stream()), "enl_linear_attention")
    return (out, new_state) if return_state else out
