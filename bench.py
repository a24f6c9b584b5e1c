"""Benchmark of the B200 attention inference path (one JSON line on rank 0).

Headline: causal self-attention prefill, per GPU batch 8 x
seq 4096 x 16 heads x head_dim 128, bf16 in / fp32 accumulate, per-sequence
key padding with valid lengths ~U[2048, 4096] -> TFLOP/s of useful attention
FLOPs (4 * D * H * sum_b P_b, P_b = L(L+1)/2 + (S - L) * L). Weak scaling:
every rank runs its own batch of 8 sequences (partitioned by batch x head, no
collective); value = all ranks' FLOPs / max-over-ranks device time.

Also measured in the same run (sub-objects of the line):
  decode_cfg3  -- KV-cache decode B64 H32 D128 ctx 8192, 128 steps with a
                  K3 append each step (HBM GB/s, tokens/s), batch rows split
                  across ranks.
  longctx_cfg5 -- split-KV decode B4 H32 D128 over a 262144-token cache
                  sharded by sequence across ranks; per-GPU (out, LSE)
                  partials all-gathered over NCCL and LSE-merged.
  cross_cfg4   -- cross-attention prefill, decoder B16 x 1024 queries against
                  2048 memory keys, H16 D64, non-causal, memory key padding
                  L~U[1024, 2048], bf16 (per-GPU batch 16, no collective).
  layer_cfg2   -- the whole graph.MultiHeadAttention layer on config 2 in
                  bf16 precision (fused QKV GEMM, K1, output GEMM).
  layer_cfg1   -- config 1 (B4 S256 E256 H8, causal, float32) through the
                  NumPy-facing Forward on the fp32 split-bf16 path.
  sparse_attention -- sparse_pattern (block-sparse, K1's sparse mode), B4
                  S16384 H16 D128 causal bf16, beside the dense causal kernel
  backward     -- dQ, dK, dV (K5) of the causal B4 S4096 H16 D128 bf16 forward
  linear_attention -- the attention_kernel="linear" and "performer" options
                  (feature maps + causal linear attention, K4), B4 S4096 H16
                  D64 per GPU, fp32 on the CUDA cores.

Run: python bench.py [--gpus N --steps K --warmup W] [--impl reference]
Multi-GPU: torchrun --nproc-per-node N bench.py --gpus N ...
"""
from __future__ import annotations

import argparse
import json
import math
import os
import platform
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "attn prefill TFLOP/s (causal, key-padded, bf16)"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

CFG2 = dict(B=8, S=4096, H=16, D=128, lo=2048, hi=4096)
CFG3 = dict(B=64, H=32, D=128, ctx=8192, steps=128)
CFG5 = dict(B=4, H=32, D=128, ctx=262144, steps=16)
CFG4 = dict(B=16, Sq=1024, Skv=2048, H=16, D=64, lo=1024, hi=2048)


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def cfg2_lengths(rank: int):
    import numpy as np
    return np.random.RandomState(2 + rank).randint(CFG2["lo"], CFG2["hi"] + 1, size=CFG2["B"])


def cfg2_flops(lengths) -> float:
    S, H, D = CFG2["S"], CFG2["H"], CFG2["D"]
    pairs = sum(L * (L + 1) / 2 + (S - L) * L for L in (int(x) for x in lengths))
    return 4.0 * D * H * pairs


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples taken while the timed
    region runs (20 ms period)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.samples = []
        self.proc = None
        self.windows = []
        self._thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20", "-i", str(self.device_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), line.strip()))

    def mark(self, t0, t1):
        self.windows.append((t0, t1))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self):
        def parse(line):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                return None
            try:
                return dict(sm=float(parts[1]), smax=float(parts[2]),
                            hw=parts[5], hwt=parts[6], swt=parts[7], pcap=parts[8])
            except ValueError:
                return None
        inside = [parse(l) for t, l in self.samples
                  if any(a - 0.05 <= t <= b + 0.05 for a, b in self.windows)]
        inside = [s for s in inside if s]
        if not inside:
            inside = [s for s in (parse(l) for _, l in self.samples) if s]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = set()
        for s in inside:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
                if s[key].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s["sm"] for s in inside),
                "sm_max_mhz": max(s["smax"] for s in inside),
                "reasons": sorted(reasons), "samples": len(inside)}


# ------------------------------------------------------------ dist helpers
class Dist:
    def __init__(self, n_gpus: int):
        import torch
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != n_gpus:
            raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={self.world}")
        torch.cuda.set_device(self.local_rank)
        self.device = torch.device("cuda", self.local_rank)
        self.pg = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=self.device)
            self.pg = dist

    def barrier(self):
        import torch
        torch.cuda.synchronize()
        if self.pg:
            self.pg.barrier()
        torch.cuda.synchronize()

    def max(self, value: float) -> float:
        import torch
        if not self.pg:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, value: float) -> float:
        import torch
        if not self.pg:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.barrier()
            self.pg.destroy_process_group()


def timed(dist: Dist, clocks: ClockSampler, fn, steps: int) -> float:
    """Run fn() `steps` times between CUDA events on the current stream,
    bracketed by barrier + synchronize; return max-over-ranks milliseconds."""
    import torch
    dist.barrier()
    t0 = time.time()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    t1 = time.time()
    dist.barrier()
    clocks.mark(t0, t1)
    return dist.max(start.elapsed_time(end))


# ------------------------------------------------------------- workloads
def bench_prefill(dist: Dist, clocks: ClockSampler, steps: int, warmup: int, batch: int = 0,
                  e2e_on: bool = True):
    import torch
    from enilnets_b200 import kernels, _native
    B, S, H, D = batch or CFG2["B"], CFG2["S"], CFG2["H"], CFG2["D"]
    g = torch.Generator(device=dist.device).manual_seed(1000 + dist.rank)
    q, k, v = (torch.randn((B, S, H, D), generator=g, device=dist.device).to(torch.bfloat16)
               for _ in range(3))
    lengths = cfg2_lengths(dist.rank)[:B]
    lens = torch.tensor(lengths, dtype=torch.int32, device=dist.device)
    out = torch.empty((B, S, H, D), dtype=torch.bfloat16, device=dist.device)

    def step():
        kernels.attention_prefill(q, k, v, causal=True, kv_valid_len=lens,
                                  mask_mode="additive", out=out)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    ms = timed(dist, clocks, step, steps)
    flops_rank = cfg2_flops(lengths)
    flops_total = dist.sum(flops_rank)
    ms_step = ms / steps
    value = flops_total / (ms_step * 1e-3) / 1e12

    if not e2e_on:
        return dict(value=value, ms_step=ms_step, flops_rank=flops_rank, flops_total=flops_total,
                    e2e=None, lengths=[int(x) for x in lengths], per_launch_ms=ms_step)
    # End to end through the same public call: every step copies its inputs
    # from pinned host memory and reads its output back. Consecutive steps
    # overlap (PCIe is full duplex): two device input/output sets on separate
    # copy streams, so step i + 1's inputs go up while step i computes and
    # step i - 1's output comes down. Events order each slot's reuse.
    # The pinned buffers are allocated and first touched on the GPU's own
    # NUMA node (enilnets_b200.hostmem): with eight ranks copying at once,
    # buffers on the far socket make the socket link the bottleneck.
    from enilnets_b200 import hostmem
    with hostmem.local_to(dist.local_rank) as host_cpus:
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        hout = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
        for h in hout:
            h.zero_()
    dev_in = [tuple(torch.empty_like(t) for t in (q, k, v)) for _ in range(2)]
    dev_out = [torch.empty_like(out) for _ in range(2)]
    s_in, s_cmp, s_out = (torch.cuda.Stream(device=dist.device) for _ in range(3))
    ev_in, ev_cmp, ev_out = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))
    used = [False, False]

    def e2e_step(i):
        slot = i % 2
        dq, dk, dv = dev_in[slot]
        with torch.cuda.stream(s_in):
            if used[slot]:
                s_in.wait_event(ev_cmp[slot])  # the slot's previous kernel read its inputs
            dq.copy_(hq, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            ev_in[slot].record(s_in)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(ev_in[slot])
            if used[slot]:
                s_cmp.wait_event(ev_out[slot])  # the slot's previous output is on the host
            kernels.attention_prefill(dq, dk, dv, causal=True, kv_valid_len=lens,
                                      mask_mode="additive", out=dev_out[slot])
            ev_cmp[slot].record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_cmp[slot])
            hout[slot].copy_(dev_out[slot], non_blocking=True)
            ev_out[slot].record(s_out)
        used[slot] = True

    e2e_steps = max(4, min(steps, 20))
    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream()
    dist.barrier()
    t0 = time.time()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(cur)
    for s_ in (s_in, s_cmp, s_out):
        s_.wait_stream(cur)
    for i in range(e2e_steps):
        e2e_step(i)
    cur.wait_stream(s_out)
    end.record(cur)
    torch.cuda.synchronize()
    clocks.mark(t0, time.time())
    dist.barrier()
    ms_e2e = dist.max(start.elapsed_time(end)) / e2e_steps
    h2d = 3 * q.numel() * q.element_size()
    d2h = out.numel() * out.element_size()
    e2e = {"value": flops_total / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
           "ms_per_step": ms_e2e, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "pinned_host_memory": (f"GPU-local NUMA node ({len(host_cpus)} CPUs)" if host_cpus
                                  else "unbound (NVML gave no CPU affinity)")}
    return dict(value=value, ms_step=ms_step, flops_rank=flops_rank, flops_total=flops_total,
                e2e=e2e, lengths=[int(x) for x in lengths], per_launch_ms=ms_step)


def bench_decode_cfg3(dist: Dist, clocks: ClockSampler, warmup: int, batch: int = 0):
    """Batch rows split across ranks (64 / N per GPU)."""
    import torch
    from enilnets_b200 import kernels, _native
    from enilnets_b200 import sharding
    Btot, H, D, ctx, T = batch or CFG3["B"], CFG3["H"], CFG3["D"], CFG3["ctx"], CFG3["steps"]
    b0, b1 = sharding.batch_shard(Btot, dist.world, dist.rank)
    B = b1 - b0
    if B == 0:
        return {"skipped": f"batch {Btot} has no rows for rank {dist.rank}"}
    cap = ctx + T
    g = torch.Generator(device=dist.device).manual_seed(3 + dist.rank)
    kc = torch.empty((B, H, cap, D), dtype=torch.bfloat16, device=dist.device)
    vc = torch.empty_like(kc)
    kc[:, :, :ctx].normal_(generator=g)
    vc[:, :, :ctx].normal_(generator=g)
    qs = torch.randn((T, B, H, D), generator=g, device=dist.device).to(torch.bfloat16)
    kn = torch.randn((T, B, 1, H, D), generator=g, device=dist.device).to(torch.bfloat16)
    vn = torch.randn((T, B, 1, H, D), generator=g, device=dist.device).to(torch.bfloat16)
    out = torch.empty((B, H, D), dtype=torch.bfloat16, device=dist.device)
    state = {"t": 0}

    def step():
        t = state["t"]
        kernels.kv_append(kc, kn[t], ctx + t)
        kernels.kv_append(vc, vn[t], ctx + t)
        kernels.attention_decode(qs[t], kc, vc, slot_begin=0, slot_end=ctx + t + 1,
                                 pos_slot0=0, q_pos=ctx + t, out=out)
        state["t"] = (t + 1) % T

    for _ in range(max(warmup, 3)):
        step()
    state["t"] = 0
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    # Decode-only timing of the same kernel on a fixed context, for the roofline.
    ms_all = timed(dist, clocks, step, T)
    bytes_rank = 0
    for t in range(T):
        n = ctx + t + 1
        bytes_rank += 2 * B * H * D * 2 * n + 2 * B * H * D * 2 + 2 * B * H * D * 2
    bytes_total = dist.sum(bytes_rank)
    gbs = bytes_total / (ms_all * 1e-3) / 1e9
    state["t"] = 0
    ms_dec = timed(dist, clocks, lambda: kernels.attention_decode(
        qs[0], kc, vc, slot_begin=0, slot_end=ctx + 1, pos_slot0=0, q_pos=ctx, out=out), T)
    dec_bytes = 2 * B * H * D * 2 * (ctx + 1) + 2 * B * H * D * 2
    dec_gbs = dist.sum(dec_bytes) / (ms_dec / T * 1e-3) / 1e9
    return {"GB_s": gbs, "tokens_s": Btot * T / (ms_all * 1e-3), "ms_per_step": ms_all / T,
            "decode_kernel_GB_s": dec_gbs, "decode_kernel_ms": ms_dec / T,
            "splits": kernels.decode_auto_splits(B, H, ctx + 1),
            "config": f"B{Btot} H{H} D{D} ctx {ctx}+{T} steps, append each step, "
                      f"{B} rows per GPU"}


def bench_longctx_cfg5(dist: Dist, clocks: ClockSampler, warmup: int):
    """Sequence-sharded split-KV decode with an NCCL all-gather of (out, LSE)."""
    import torch
    from enilnets_b200 import kernels, sharding, _native
    B, H, D, ctx, T = CFG5["B"], CFG5["H"], CFG5["D"], CFG5["ctx"], CFG5["steps"]
    N = dist.world
    k0, k1 = sharding.kv_shard_range(ctx, N, dist.rank)
    shard = k1 - k0
    tail = dist.rank == N - 1
    cap = shard + (T if tail else 0)
    g = torch.Generator(device=dist.device).manual_seed(5 + dist.rank)
    kc = torch.empty((B, H, cap, D), dtype=torch.bfloat16, device=dist.device)
    vc = torch.empty_like(kc)
    kc[:, :, :shard].normal_(generator=g)
    vc[:, :, :shard].normal_(generator=g)
    gq = torch.Generator(device=dist.device).manual_seed(55)  # same query on every rank
    qs = torch.randn((T, B, H, D), generator=gq, device=dist.device).to(torch.bfloat16)
    kn = torch.randn((T, B, 1, H, D), generator=gq, device=dist.device).to(torch.bfloat16)
    vn = torch.randn((T, B, 1, H, D), generator=gq, device=dist.device).to(torch.bfloat16)
    out = torch.empty((B, H, D), dtype=torch.bfloat16, device=dist.device)
    decode = sharding.SequenceShardedDecode()  # local split-KV decode, NCCL gather, LSE merge
    state = {"t": 0}

    def step():
        t = state["t"]
        pos = ctx + t
        if tail:
            kernels.kv_append(kc, kn[t], shard + t)
            kernels.kv_append(vc, vn[t], shard + t)
        n_live = shard + (t + 1 if tail else 0)
        decode(qs[t], kc, vc, slot_begin=0, slot_end=n_live, pos_slot0=k0, q_pos=pos, out=out)
        state["t"] = (t + 1) % T

    for _ in range(max(warmup, 3)):
        step()
    state["t"] = 0
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    ms = timed(dist, clocks, step, T)
    bytes_total = sum(2 * B * H * D * 2 * (ctx + t + 1) for t in range(T))
    return {"GB_s": bytes_total / (ms * 1e-3) / 1e9, "tokens_s": B * T / (ms * 1e-3),
            "ms_per_step": ms / T, "shard_tokens_per_gpu": shard,
            "collective": "none" if N == 1 else "ncclAllGather of fp32 (out, LSE) + LSE merge"}


def bench_cross_cfg4(dist: Dist, clocks: ClockSampler, warmup: int, steps: int = 50):
    """Cross-attention core: per-GPU batch 16, memory key padding."""
    import numpy as np
    import torch
    from enilnets_b200 import kernels, _native
    B, Sq, Skv, H, D = CFG4["B"], CFG4["Sq"], CFG4["Skv"], CFG4["H"], CFG4["D"]
    g = torch.Generator(device=dist.device).manual_seed(4000 + dist.rank)
    q = torch.randn((B, Sq, H, D), generator=g, device=dist.device).to(torch.bfloat16)
    k, v = (torch.randn((B, Skv, H, D), generator=g, device=dist.device).to(torch.bfloat16)
            for _ in range(2))
    lengths = np.random.RandomState(4 + dist.rank).randint(CFG4["lo"], CFG4["hi"] + 1, size=B)
    lens = torch.tensor(lengths, dtype=torch.int32, device=dist.device)
    out = torch.empty_like(q)

    def step():
        kernels.attention_prefill(q, k, v, causal=False, kv_valid_len=lens,
                                  mask_mode="additive", out=out)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    ms = timed(dist, clocks, step, steps) / steps
    flops = 4.0 * D * H * Sq * float(lengths.sum())
    return {"TFLOP_s": dist.sum(flops) / (ms * 1e-3) / 1e12, "ms_per_step": ms,
            "config": f"B{B}/GPU Sq{Sq} Skv{Skv} H{H} D{D} non-causal, memory key padding "
                      f"L~U[{CFG4['lo']},{CFG4['hi']}], bf16"}


FP32_CORE_TFLOPS = 148 * 128 * 2 * 1.965e-3  # nominal fp32 FMA TFLOP/s of the CUDA cores


def bench_linear(dist: Dist, clocks: ClockSampler, warmup: int, steps: int = 10):
    """Linearized attention (attention_kernel "linear" and "performer"):
    feature maps plus causal linear attention on device fp32 head views, per
    GPU B4 S4096 H16 D64 (Performer with 256 features). FLOPs count the
    reference's reassociated form, 4 S Df D per query head, plus the
    Performer projections (2 S Dh Df for queries, twice that for keys: the
    stabilizer pass and the map)."""
    import torch
    from enilnets_b200 import kernels, _native
    B, S, H, D, Df = 4, 4096, 16, 64, 256
    g = torch.Generator(device=dist.device).manual_seed(6000 + dist.rank)
    qkv = torch.randn((B, S, 3 * H * D), generator=g, device=dist.device) * 0.5
    q, k, v = (qkv[..., i * H * D:(i + 1) * H * D].unflatten(-1, (H, D)) for i in range(3))
    omega = torch.randn((Df, D), generator=g, device=dist.device)
    res = {}
    for kernel in ("linear", "performer"):
        om = omega if kernel == "performer" else None
        nf = Df if kernel == "performer" else D

        def step():
            qp, _ = kernels.linear_feature_map(q, kernel, om)
            kp, _ = kernels.linear_feature_map(k, kernel, om, global_stab=True)
            kernels.linear_attention(qp, kp, v, causal=True)

        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        _native.raise_on_device_error()
        ms = timed(dist, clocks, step, steps) / steps
        flops = 4.0 * S * nf * D * B * H
        if kernel == "performer":
            flops += 3 * 2.0 * S * D * Df * B * H
        tf = dist.sum(flops) / (ms * 1e-3) / 1e12
        res[kernel] = {"ms_per_step": ms, "TFLOP_s": tf,
                       "frac_of_fp32_core_peak_per_gpu": tf / dist.world / FP32_CORE_TFLOPS,
                       "tokens_s": dist.sum(B * S) / (ms * 1e-3)}
    res["config"] = (f"B{B}/GPU S{S} H{H} D{D} causal, fp32 arithmetic on CUDA cores; performer "
                     f"with {Df} features; peak = nominal {FP32_CORE_TFLOPS:.1f} TFLOP/s fp32")
    return res


def bench_backward(dist: Dist, clocks: ClockSampler, warmup: int, steps: int = 10,
                   batch: int = 0):
    """Attention backward (K5): dQ, dK, dV of the causal cfg2-shaped forward
    (B4 S4096 H16 D128 per GPU, bf16, no padding) from its LSE. FLOPs follow
    the usual convention for a flash backward, 10 D per allowed pair (five
    GEMMs); the kernels issue 14 D (S and dP are recomputed in the dQ pass),
    reported as tensor_TFLOP_s."""
    import torch
    from enilnets_b200 import kernels, _native
    B, S, H, D = batch or 4, 4096, 16, 128
    g = torch.Generator(device=dist.device).manual_seed(8000 + dist.rank)
    q, k, v, do = (torch.randn((B, S, H, D), generator=g, device=dist.device)
                   .to(torch.bfloat16) for _ in range(4))
    o, lse = kernels.attention_prefill(q, k, v, causal=True, out_dtype=torch.bfloat16,
                                       return_lse=True)

    def step():
        kernels.attention_backward(q, k, v, o, lse, do, causal=True)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    ms = timed(dist, clocks, step, steps) / steps
    pairs = B * H * S * (S + 1) / 2
    tf = dist.sum(10.0 * D * pairs) / (ms * 1e-3) / 1e12
    peak = float(load_peaks()[0]["bf16_tflops"])
    return {"ms_per_step": ms, "TFLOP_s": tf, "frac_of_bf16_peak_per_gpu": tf / dist.world / peak,
            "tensor_TFLOP_s": tf * 1.4,
            "config": f"B{B}/GPU S{S} H{H} D{D} causal bf16; dQ, dK, dV (fp32) from dO and LSE"}


SPARSE_PATTERNS = {
    "bs128": {"block_size": 128, "local": 2, "global": 1, "random": 2},
    "bs64": {"block_size": 64, "local": 3, "global": 2, "random": 3},
}


def bench_sparse(dist: Dist, clocks: ClockSampler, warmup: int, steps: int = 10,
                 batch: int = 0):
    """Block-sparse attention (sparse_pattern, local + global + random blocks)
    on K1's sparse mode, per GPU B4 S16384 H16 D128 causal bf16, next to the
    dense causal kernel on the same inputs. FLOPs count the pairs the pattern
    allows (4 D per pair); tile_fill is that over the visited 128 x 128
    tiles' area."""
    import torch
    from enilnets_b200 import kernels, _native, sparse
    B, S, H, D = batch or 4, 16384, 16, 128
    g = torch.Generator(device=dist.device).manual_seed(7000 + dist.rank)
    q, k, v = (torch.randn((B, S, H, D), generator=g, device=dist.device).to(torch.bfloat16)
               for _ in range(3))
    peak = float(load_peaks()[0]["bf16_tflops"])

    def run(step):
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        _native.raise_on_device_error()
        return timed(dist, clocks, step, steps) / steps

    dense_ms = run(lambda: kernels.attention_prefill(q, k, v, causal=True))
    res = {"dense_causal_ms": dense_ms}
    for name, pat in SPARSE_PATTERNS.items():
        spec = sparse.normalize_pattern(pat)
        lay = sparse.build_layout(spec, S, S, causal=True, device=q.device)
        ms = run(lambda: sparse.attention(q, k, v, spec, causal=True))
        tf = dist.sum(4.0 * D * lay.pairs * B * H) / (ms * 1e-3) / 1e12
        res[name] = {"pattern": pat, "ms_per_step": ms, "TFLOP_s": tf,
                     "frac_of_bf16_peak_per_gpu": tf / dist.world / peak,
                     "speedup_vs_dense_causal": dense_ms / ms,
                     "allowed_fraction_of_causal": lay.pairs / (S * (S + 1) / 2),
                     "tile_fill": lay.pairs / (lay.n_entries * 128.0 * 128.0)}
    res["config"] = f"B{B}/GPU S{S} H{H} D{D} causal bf16; FLOPs over allowed pairs"
    return res


def bench_layer_cfg2(dist: Dist, clocks: ClockSampler, warmup: int, steps: int = 10):
    """graph.MultiHeadAttention(2048, 16, causal) forward with key padding on
    device-resident x, bf16 precision: QKV GEMM + K1 + output GEMM."""
    import numpy as np
    import torch
    import enilnets_b200 as enl
    from enilnets_b200 import _native
    from enilnets_b200.graph import MultiHeadAttention, lengths_to_mask
    B, S, H, D = CFG2["B"], CFG2["S"], CFG2["H"], CFG2["D"]
    E = H * D
    enl.set_precision("bf16")
    try:
        enl.set_seed(0)
        layer = MultiHeadAttention(E, H, causal=True)
        g = torch.Generator(device=dist.device).manual_seed(2000 + dist.rank)
        x = torch.randn((B, S, E), generator=g, device=dist.device)
        lengths = cfg2_lengths(dist.rank)
        mask = lengths_to_mask(lengths, S)

        def step():
            layer.forward_device(x, key_padding_mask=mask)

        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        _native.raise_on_device_error()
        ms = timed(dist, clocks, step, steps) / steps
    finally:
        enl.set_precision("fp32")
    proj = 2.0 * B * S * E * (3 * E) + 2.0 * B * S * E * E
    attn = cfg2_flops(lengths)
    return {"TFLOP_s": dist.sum(proj + attn) / (ms * 1e-3) / 1e12, "ms_per_step": ms,
            "attention_share_of_flops": attn / (proj + attn),
            "config": "graph.MultiHeadAttention(2048, 16, causal) forward, x (8, 4096, 2048) "
                      "on device, key padding as config 2, bf16 precision"}


def bench_layer_cfg1(dist: Dist, warmup: int, steps: int = 20):
    """Config 1 through the NumPy-facing API (host array in, host array out),
    fp32 precision; host wall time per Forward, max over ranks."""
    import numpy as np
    import torch
    import enilnets_b200 as enl
    enl.set_seed(0)
    m = enl.AttentionNet()
    m.add_multihead_attention(embed_dim=256, num_heads=8, causal=True)
    x = np.random.RandomState(1).standard_normal((4, 256, 256))
    for _ in range(warmup):
        m.Forward(x)
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        m.Forward(x)
    torch.cuda.synchronize()
    ms = dist.max((time.perf_counter() - t0) * 1e3 / steps)
    return {"ms_per_forward": ms, "precision": "fp32 (split-bf16 attention, fp32 GEMMs)",
            "config": "set_seed(0), add_multihead_attention(256, 8, causal=True), "
                      "x (4, 256, 256) float NumPy in/out"}


# ------------------------------------------------------------- CPU baseline
def cpu_sample_tflops(heads: int = 16, repeats: int = 1):
    """The reference's streaming softmax (oracle port of
    nn/flash_attention.py:42-80, float64, block 512) on one full-length
    causal sequence x `heads` heads of config 2; useful causal FLOPs / s."""
    import numpy as np
    from oracle.attention_ref import flash_attention_ref
    S, D = CFG2["S"], CFG2["D"]
    rng = np.random.RandomState(0)
    Q, K, V = (rng.standard_normal((1, heads, S, D)) for _ in range(3))
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        flash_attention_ref(Q, K, V, 512, causal=True)
        times.append(time.perf_counter() - t0)
    flops = 4.0 * D * heads * S * (S + 1) / 2
    t = statistics.mean(times)
    return flops / t / 1e12, t, f"1 sequence x {heads} heads, S={S}, D={D}, causal, float64"


def cpu_info():
    model = platform.processor()
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return model, os.cpu_count()


def arm_config(n_gpus: int) -> dict:
    """The headline workload's config, shared by both arms."""
    return {"workload": "cfg2 causal prefill B8/GPU S4096 H16 D128, key padding L~U[2048,4096]",
            "global_batch": CFG2["B"] * n_gpus, "seq_len": CFG2["S"],
            "parallelism": f"batch x head over {n_gpus} GPU(s), no collective",
            "l2": "inputs 402 MB per GPU > 126 MB L2 (no flush needed)"}


def run_reference(args):
    """--impl reference: the reference algorithm (NumPy float64 port) on the
    host cores, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    model, cores = cpu_info()
    for _ in range(args.warmup):
        cpu_sample_tflops(heads=2)
    vals = []
    t_total = 0.0
    for _ in range(args.steps):
        v, t, sample = cpu_sample_tflops(heads=2)
        vals.append(v)
        t_total += t
    value = statistics.mean(vals)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000 * t_total / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {**arm_config(args.gpus), "cpu": model,
                       "reference_sample": "the reference's streaming softmax on a bounded "
                                           "sample of the workload, scaled by useful FLOPs"},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--skip-sub", action="store_true", help="headline only")
    ap.add_argument("--only", choices=["all", "prefill", "decode", "longctx", "cross", "layer",
                                       "linear", "sparse", "backward"],
                    default="all",
                    help="profiling: run one workload")
    ap.add_argument("--batch", type=int, default=0,
                    help="profiling: batch override for prefill, sparse and backward")
    ap.add_argument("--decode-batch", type=int, default=0,
                    help="profiling: cfg3 decode batch override")
    ap.add_argument("--no-e2e", action="store_true", help="profiling: skip the e2e leg")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)

    import torch
    from enilnets_b200 import _native
    _native.load()
    dist = Dist(args.gpus)
    clocks = ClockSampler(dist.local_rank)
    clocks.start()
    try:
        if args.only != "all":
            res = {}
            if args.only == "prefill":
                res = bench_prefill(dist, clocks, args.steps, args.warmup, args.batch,
                                    e2e_on=False)
            elif args.only == "decode":
                res = bench_decode_cfg3(dist, clocks, args.warmup, args.decode_batch)
            elif args.only == "cross":
                res = bench_cross_cfg4(dist, clocks, args.warmup)
            elif args.only == "linear":
                res = bench_linear(dist, clocks, args.warmup)
            elif args.only == "sparse":
                res = bench_sparse(dist, clocks, args.warmup, batch=args.batch)
            elif args.only == "backward":
                res = bench_backward(dist, clocks, args.warmup, batch=args.batch)
            elif args.only == "layer":
                res = {"layer_cfg2": bench_layer_cfg2(dist, clocks, args.warmup),
                       "layer_cfg1": bench_layer_cfg1(dist, args.warmup)}
            else:
                res = bench_longctx_cfg5(dist, clocks, args.warmup)
            if dist.rank == 0:
                print(json.dumps({"profiling_only": args.only, **res}))
            dist.close()
            return 0
        pre = bench_prefill(dist, clocks, args.steps, args.warmup, args.batch,
                            e2e_on=not args.no_e2e)
        sub = {}
        if not args.skip_sub:
            sub["decode_cfg3"] = bench_decode_cfg3(dist, clocks, args.warmup, args.decode_batch)
            sub["longctx_cfg5"] = bench_longctx_cfg5(dist, clocks, args.warmup)
            sub["cross_cfg4"] = bench_cross_cfg4(dist, clocks, args.warmup)
            sub["linear_attention"] = bench_linear(dist, clocks, args.warmup)
            sub["sparse_attention"] = bench_sparse(dist, clocks, args.warmup)
            sub["backward"] = bench_backward(dist, clocks, args.warmup)
            sub["layer_cfg2"] = bench_layer_cfg2(dist, clocks, args.warmup)
            sub["layer_cfg1"] = bench_layer_cfg1(dist, args.warmup)
    finally:
        clocks.stop()
    peaks, peak_kind = load_peaks()
    if dist.rank == 0:
        achieved = pre["flops_rank"] / (pre["per_launch_ms"] * 1e-3) / 1e12
        peak = float(peaks["bf16_tflops"])
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "traffic": None,
                    "peak_source": f"{peak_kind} bf16 burst (MEASURED_PEAKS.json)"
                    if peak_kind == "measured" else "fallback 1590 TFLOP/s"}
        prof = REPO / "profiles" / "prefill_traffic.json"
        if prof.exists():
            roofline["traffic"] = json.loads(prof.read_text()).get("bytes_per_launch")
        hbm = float(peaks["hbm_gbs"])
        if "cross_cfg4" in sub:
            sub["cross_cfg4"]["frac_of_bf16_peak_per_gpu"] = \
                sub["cross_cfg4"]["TFLOP_s"] / dist.world / peak
        for key in ("decode_cfg3", "longctx_cfg5"):
            if key in sub and "GB_s" in sub[key]:
                per_gpu = sub[key]["GB_s"] / dist.world
                sub[key]["frac_of_hbm_per_gpu"] = per_gpu / hbm
        if "decode_cfg3" in sub and "decode_kernel_GB_s" in sub["decode_cfg3"]:
            sub["decode_cfg3"]["decode_kernel_frac_of_hbm"] = \
                sub["decode_cfg3"]["decode_kernel_GB_s"] / dist.world / hbm
        cpu = None
        if not args.no_cpu_baseline:
            model, cores = cpu_info()
            v, t, sample = cpu_sample_tflops(heads=16)
            cpu = {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                   "sample": sample + f" ({t:.1f} s, numpy/BLAS on all host threads, {model})"}
        line = {
            "metric": METRIC, "value": pre["value"], "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": pre["ms_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic N(0,1) activations, seeded",
            "config": {**arm_config(args.gpus), "lengths_rank0": pre["lengths"]},
            "e2e": pre["e2e"],
            "roofline": roofline,
            "cpu_baseline": cpu,
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
            **sub,
        }
        print(json.dumps(line))
    dist.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
