"""Prefill from host memory: attention over pinned host q/k/v with the output
returned to pinned host memory, pipelined across calls.

The reference computes its attention where its arrays live, in host memory
(graph/sequence.py:159-183, nn/forward.py:525-551). A caller that keeps its
activations on the host pays a PCIe round trip per call; this class hides
what it can of it and moves no byte the kernel does not need:

* Two device slots, a copy-in stream, the compute stream and a copy-out
  stream. Call i + 1's upload runs while call i computes and call i - 1's
  output comes down (PCIe is full duplex). Events order each slot's reuse.
* Key/value rows past a sequence's valid length are not uploaded when no
  row can see them: without a sliding window and with every valid length
  >= 1, each query row has an unmasked key (key 0 for causal rows, all
  valid keys otherwise), so padded keys carry no weight under either mask
  rule. Rows [0, L_b) of sequence b go up as one copy per tensor; the rest of
  each device slot is zeroed once, so the kernel's partial last key tile
  reads finite values. Otherwise K and V move whole. One consequence: a
  non-finite value in a padded host row is never read, where the reference
  (and the device-resident call) would carry a NaN in a padded V row into
  the output through 0 * NaN.
* Queries (padded query rows still see every real key) and the output move
  whole.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from . import kernels


class HostPrefill:
    """Pipelined attention_prefill over pinned host buffers of one shape.

    shape: (B, S, H, D) of q, k, v and the output (self-attention shapes;
    Hkv = H). submit() enqueues one call and returns; synchronize() waits for
    every submitted call, after which the host outputs hold their results.
    h2d_bytes / d2h_bytes count the bytes each call moved."""

    def __init__(self, shape: Sequence[int], dtype: torch.dtype = torch.bfloat16,
                 device: Optional[torch.device] = None, slots: int = 2):
        if len(shape) != 4:
            raise ValueError("shape must be (batch, seq, heads, head_dim)")
        self.shape = tuple(int(x) for x in shape)
        self.dtype = dtype
        self.device = torch.device(device) if device is not None else \
            torch.device("cuda", torch.cuda.current_device())
        if self.device.type != "cuda":
            raise ValueError("HostPrefill needs a CUDA device")
        B = self.shape[0]
        self._in = [tuple(torch.zeros(self.shape, dtype=dtype, device=self.device)
                          for _ in range(3)) for _ in range(slots)]
        self._out = [torch.empty(self.shape, dtype=dtype, device=self.device)
                     for _ in range(slots)]
        self._len_h = [torch.zeros(B, dtype=torch.int32).pin_memory() for _ in range(slots)]
        self._len_d = [torch.zeros(B, dtype=torch.int32, device=self.device)
                       for _ in range(slots)]
        self._s_in, self._s_cmp, self._s_out = (torch.cuda.Stream(device=self.device)
                                                for _ in range(3))
        self._ev_in, self._ev_cmp, self._ev_out = (
            [torch.cuda.Event() for _ in range(slots)] for _ in range(3))
        self._used = [False] * slots
        self._n = 0
        self.h2d_bytes: List[int] = []
        self.d2h_bytes: List[int] = []

    def _check(self, name: str, t: torch.Tensor) -> None:
        if t.device.type != "cpu" or not t.is_pinned():
            raise ValueError(f"{name} must be a pinned host tensor")
        if tuple(t.shape) != self.shape or t.dtype != self.dtype or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous {self.dtype} tensor of shape "
                             f"{self.shape}, got {t.dtype} {tuple(t.shape)}")

    def submit(self, hq: torch.Tensor, hk: torch.Tensor, hv: torch.Tensor, hout: torch.Tensor,
               kv_valid_len: Sequence[int], *, causal: bool = False,
               window: Optional[int] = None, mask_mode: str = "exclude",
               units: Optional[torch.Tensor] = None, **kw) -> None:
        """Enqueue attention_prefill(q, k, v) for host q/k/v into host hout.
        kv_valid_len: B host ints, keys [0, len_b) of sequence b are real. The
        host buffers must stay untouched until synchronize(). Other keyword
        arguments go to kernels.attention_prefill."""
        for name, t in (("q", hq), ("k", hk), ("v", hv), ("out", hout)):
            self._check(name, t)
        B, S, H, D = self.shape
        lens = [int(x) for x in kv_valid_len]
        if len(lens) != B or min(lens) < 0 or max(lens) > S:
            raise ValueError(f"kv_valid_len must hold {B} lengths in [0, {S}]")
        partial = window is None and min(lens) >= 1
        slot = self._n % len(self._in)
        dq, dk, dv = self._in[slot]
        row_bytes = H * D * hq.element_size()
        if self._used[slot]:
            # The host writes the slot's pinned lengths below: its previous
            # upload of them must have run (one call back in the pipeline).
            self._ev_in[slot].synchronize()
        self._len_h[slot].copy_(torch.tensor(lens, dtype=torch.int32))
        with torch.cuda.stream(self._s_in):
            if self._used[slot]:
                self._s_in.wait_event(self._ev_cmp[slot])  # the slot's last call read its inputs
            self._len_d[slot].copy_(self._len_h[slot], non_blocking=True)
            dq.copy_(hq, non_blocking=True)
            if partial:
                for b, L in enumerate(lens):
                    dk[b, :L].copy_(hk[b, :L], non_blocking=True)
                    dv[b, :L].copy_(hv[b, :L], non_blocking=True)
                kv_bytes = 2 * sum(lens) * row_bytes
            else:
                dk.copy_(hk, non_blocking=True)
                dv.copy_(hv, non_blocking=True)
                kv_bytes = 2 * B * S * row_bytes
            self._ev_in[slot].record(self._s_in)
        with torch.cuda.stream(self._s_cmp):
            self._s_cmp.wait_event(self._ev_in[slot])
            if self._used[slot]:
                self._s_cmp.wait_event(self._ev_out[slot])  # its last output is on the host
            kernels.attention_prefill(dq, dk, dv, causal=causal, window=window,
                                      kv_valid_len=self._len_d[slot], mask_mode=mask_mode,
                                      out=self._out[slot], out_dtype=self.dtype, units=units,
                                      **kw)
            self._ev_cmp[slot].record(self._s_cmp)
        with torch.cuda.stream(self._s_out):
            self._s_out.wait_event(self._ev_cmp[slot])
            hout.copy_(self._out[slot], non_blocking=True)
            self._ev_out[slot].record(self._s_out)
        self._used[slot] = True
        self._n += 1
        self.h2d_bytes.append(B * S * row_bytes + kv_bytes + 4 * B)
        self.d2h_bytes.append(B * S * row_bytes)

    def wait_on(self, stream: torch.cuda.Stream) -> None:
        """Make the pipeline's streams wait for `stream` (e.g. a timing event
        recorded on it) before their next work."""
        for s in (self._s_in, self._s_cmp, self._s_out):
            s.wait_stream(stream)

    def join(self, stream: torch.cuda.Stream) -> None:
        """Make `stream` wait for every submitted call (their outputs on the host)."""
        stream.wait_stream(self._s_in)
        stream.wait_stream(self._s_cmp)
        stream.wait_stream(self._s_out)

    def synchronize(self) -> None:
        for s in (self._s_in, self._s_cmp, self._s_out):
            s.synchronize()
