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


def cfg2_lengths(rank: int, n: int = 0):
    """Valid lengths ~U[2048, 4096] of config 2 from seed 2 + rank (n values,
    default one per-GPU batch)."""
    import numpy as np
    return np.random.RandomState(2 + rank).randint(CFG2["lo"], CFG2["hi"] + 1,
                                                   size=n or CFG2["B"])


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


def timed_graph(dist: Dist, clocks: ClockSampler, steps_fn, n_steps: int):
    """Capture `steps_fn` (which issues n_steps decode steps) as one CUDA
    graph and time one replay (max over ranks); returns ms per step. The
    graph removes the host's per-launch cost from steps of a fraction of a
    millisecond; the kernels it replays are the eager steps' kernels."""
    import torch
    g = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        steps_fn()
    torch.cuda.synchronize()
    g.replay()  # warm replay
    torch.cuda.synchronize()
    ms = timed(dist, clocks, g.replay, 1) / n_steps
    del g
    torch.cuda.synchronize()
    return ms


# ------------------------------------------------------------- workloads
def prefill_partition(world: int, rank: int, batch: int = 0):
    """This rank's share of the global cfg2 batch (8 sequences per GPU, valid
    lengths ~U[2048, 4096] from one seed): cost-balanced contiguous
    (batch, head) units. Returns (global units, first row, end row, global
    lengths)."""
    from enilnets_b200 import sharding
    S, H = CFG2["S"], CFG2["H"]
    Bg = (batch or CFG2["B"]) * world
    lengths = cfg2_lengths(0, Bg)
    costs = sharding.prefill_unit_costs(lengths, S, H)
    units = sharding.contiguous_partition(costs, world)[rank]
    return units, units[0] // H, units[-1] // H + 1, lengths


def bench_prefill(dist: Dist, clocks: ClockSampler, steps: int, warmup: int, batch: int = 0,
                  e2e_on: bool = True, e2e_policy: str = "local"):
    """Weak scaling: a global batch of 8 sequences per GPU, partitioned into
    cost-balanced contiguous (batch, head) units (sharding.contiguous_partition);
    each rank holds only the sequences its units touch and K1 runs exactly
    its units. Sequence b's q/k/v come from seed 1000 + b on every rank."""
    import torch
    from enilnets_b200 import kernels, _native
    S, H, D = CFG2["S"], CFG2["H"], CFG2["D"]
    units, b_lo, b_hi, lengths_g = prefill_partition(dist.world, dist.rank, batch)
    B = b_hi - b_lo
    q, k, v = (torch.empty((B, S, H, D), dtype=torch.bfloat16, device=dist.device)
               for _ in range(3))
    for i in range(B):
        g = torch.Generator(device=dist.device).manual_seed(1000 + b_lo + i)
        for t in (q, k, v):
            t[i] = torch.randn((S, H, D), generator=g, device=dist.device).to(torch.bfloat16)
    lengths = lengths_g[b_lo:b_hi]
    lens = torch.tensor(lengths, dtype=torch.int32, device=dist.device)
    out = torch.empty((B, S, H, D), dtype=torch.bfloat16, device=dist.device)
    local = [u - b_lo * H for u in units]
    unit_t = None if local == list(range(B * H)) else \
        torch.tensor(local, dtype=torch.int32, device=dist.device)

    def step():
        kernels.attention_prefill(q, k, v, causal=True, kv_valid_len=lens,
                                  mask_mode="additive", out=out, units=unit_t)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    ms = timed(dist, clocks, step, steps)
    from enilnets_b200 import sharding
    costs = sharding.prefill_unit_costs(lengths_g, S, H)
    flops_rank = 4.0 * D * sum(costs[u] for u in units)
    flops_total = dist.sum(flops_rank)
    ms_step = ms / steps
    value = flops_total / (ms_step * 1e-3) / 1e12

    info = dict(value=value, ms_step=ms_step, flops_rank=flops_rank, flops_total=flops_total,
                lengths=[int(x) for x in lengths], per_launch_ms=ms_step,
                rows=[b_lo, b_hi], n_units=len(units), e2e=None)
    if not e2e_on:
        return info
    # End to end through the same public call: every step copies its inputs
    # from pinned host memory and reads its output back. Consecutive steps
    # overlap (PCIe is full duplex): two device input/output sets on separate
    # copy streams, so step i + 1's inputs go up while step i computes and
    # step i - 1's output comes down. Events order each slot's reuse.
    info["e2e"] = run_e2e(dist, clocks, q, k, v, out, lens, unit_t, steps, flops_total,
                          e2e_policy)
    return info


def run_e2e(dist: Dist, clocks: ClockSampler, q, k, v, out, lens, unit_t, steps: int,
            flops_total: float, policy: str = "local"):
    """The e2e leg of the headline through the host-buffer API
    (hostprefill.HostPrefill): host q/k/v in, host output back, every step,
    pipelined across steps. Key/value rows past each sequence's valid length
    are not uploaded (no row can see them under this mask), so the upload is
    the queries plus the valid K/V rows. policy "local" first-touches the
    pinned buffers on the CPUs NVML reports as local to the GPU; "spread" on
    NUMA node rank % nodes. At N > 1 the leg runs twice: rank 0 alone (the
    other ranks idle), then every rank at once, so that the line shows what
    concurrent copies cost."""
    import torch
    from enilnets_b200 import hostmem
    from enilnets_b200.hostprefill import HostPrefill
    cpus = hostmem.spread_cpus(dist.rank) if policy == "spread" else None
    with hostmem.local_to(dist.local_rank, cpus) as host_cpus:
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        hout = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        hout.zero_()
    lengths = [int(x) for x in lens.cpu()]
    pipe = HostPrefill(tuple(q.shape), dtype=q.dtype, device=q.device)

    def e2e_step():
        pipe.submit(hq, hk, hv, hout, lengths, causal=True, mask_mode="additive", units=unit_t)

    e2e_steps = max(4, min(steps, 20))
    for _ in range(2):
        e2e_step()
    pipe.synchronize()
    # The pipeline's output equals the device-resident call's (on the rank's
    # own units: rows of other units are left untouched by both).
    got = hout.to(out.device)
    if unit_t is None:
        check = bool(torch.equal(got, out))
    else:
        H = q.shape[2]
        check = all(bool(torch.equal(got[u // H, :, u % H], out[u // H, :, u % H]))
                    for u in unit_t.cpu().tolist())

    def leg(active: bool) -> float:
        cur = torch.cuda.current_stream()
        dist.barrier()
        ms = 0.0
        if active:
            t0 = time.time()
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record(cur)
            pipe.wait_on(cur)
            for _ in range(e2e_steps):
                e2e_step()
            pipe.join(cur)
            end.record(cur)
            torch.cuda.synchronize()
            clocks.mark(t0, time.time())
            ms = start.elapsed_time(end) / e2e_steps
        dist.barrier()
        return dist.max(ms)

    alone = leg(dist.rank == 0) if dist.world > 1 else None
    ms_e2e = leg(True)
    h2d = pipe.h2d_bytes[-1]
    d2h = pipe.d2h_bytes[-1]
    place = (f"{policy}: {len(host_cpus)} CPUs ({min(host_cpus)}-{max(host_cpus)})" if host_cpus
             else f"{policy}: unbound (no CPU set available)")
    e2e = {"value": flops_total / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
           "ms_per_step": ms_e2e, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "h2d_bytes_dense_inputs": 3 * q.numel() * q.element_size(),
           "api": "hostprefill.HostPrefill.submit (pinned host q/k/v/out, valid K/V rows only)",
           "output_equals_device_call": check,
           "h2d_GB_s_per_rank": h2d / (ms_e2e * 1e-3) / 1e9,
           "d2h_GB_s_per_rank": d2h / (ms_e2e * 1e-3) / 1e9,
           "pinned_host_memory": place, "numa_nodes": len(hostmem.numa_nodes())}
    if alone is not None:
        e2e["rank0_alone_ms_per_step"] = alone
        e2e["rank0_alone_h2d_GB_s"] = h2d / (alone * 1e-3) / 1e9
        e2e["host_copy_GB_s_all_ranks"] = dist.world * (h2d + d2h) / (ms_e2e * 1e-3) / 1e9
    return e2e


def bench_decode_cfg3(dist: Dist, clocks: ClockSampler, warmup: int, batch: int = 0):
    """Batch rows split across ranks (64 / N per GPU). K and V live in one
    (2, B, H, capacity, D) allocation, so one K3 launch appends both."""
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
    kv = torch.empty((2, B, H, cap, D), dtype=torch.bfloat16, device=dist.device)
    kc, vc = kv[0], kv[1]
    kc[:, :, :ctx].normal_(generator=g)
    vc[:, :, :ctx].normal_(generator=g)
    qs = torch.randn((T, B, H, D), generator=g, device=dist.device).to(torch.bfloat16)
    new = torch.randn((T, 2, B, 1, H, D), generator=g, device=dist.device).to(torch.bfloat16)
    kv_rows = kv.view(2 * B, H, cap, D)  # K rows then V rows: one append covers both
    out = torch.empty((B, H, D), dtype=torch.bfloat16, device=dist.device)
    state = {"t": 0}

    def step():
        t = state["t"]
        kernels.kv_append(kv_rows, new[t].view(2 * B, 1, H, D), ctx + t)
        kernels.attention_decode(qs[t], kc, vc, slot_begin=0, slot_end=ctx + t + 1,
                                 pos_slot0=0, q_pos=ctx + t, out=out)
        state["t"] = (t + 1) % T

    for _ in range(max(warmup, 3)):
        step()
    state["t"] = 0
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    ms_eager = timed(dist, clocks, step, T)
    state["t"] = 0

    def all_steps():
        for _ in range(T):
            step()

    ms_all = timed_graph(dist, clocks, all_steps, T) * T
    state["t"] = 0
    _native.raise_on_device_error()
    bytes_rank = 0
    for t in range(T):
        n = ctx + t + 1
        bytes_rank += 2 * B * H * D * 2 * n + 2 * B * H * D * 2 + 2 * B * H * D * 2
    bytes_total = dist.sum(bytes_rank)
    gbs = bytes_total / (ms_all * 1e-3) / 1e9
    state["t"] = 0
    # Decode-only timing of the same kernel on a fixed context, for the roofline.
    ms_dec = timed(dist, clocks, lambda: kernels.attention_decode(
        qs[0], kc, vc, slot_begin=0, slot_end=ctx + 1, pos_slot0=0, q_pos=ctx, out=out), T)
    dec_bytes = 2 * B * H * D * 2 * (ctx + 1) + 2 * B * H * D * 2
    dec_gbs = dist.sum(dec_bytes) / (ms_dec / T * 1e-3) / 1e9
    return {"GB_s": gbs, "tokens_s": Btot * T / (ms_all * 1e-3), "ms_per_step": ms_all / T,
            "eager_ms_per_step": ms_eager / T,
            "decode_kernel_GB_s": dec_gbs, "decode_kernel_ms": ms_dec / T,
            "splits": kernels.decode_auto_splits(B, H, ctx + 1),
            "config": f"B{Btot} H{H} D{D} ctx {ctx}+{T} steps, one K+V append each step, "
                      f"{B} rows per GPU; the {T} steps replayed from one CUDA graph"}


def _cfg5_shard(dist: "Dist", rank: int, B: int, H: int, D: int, ctx: int, T: int):
    """Rank `rank`'s cfg5 cache shard on this device, generated exactly as
    that rank generates it (same seed, same calls), and its slot range."""
    import torch
    from enilnets_b200 import sharding
    k0, k1 = sharding.kv_shard_range(ctx, dist.world, rank)
    shard = k1 - k0
    cap = shard + (T if rank == dist.world - 1 else 0)
    g = torch.Generator(device=dist.device).manual_seed(5 + rank)
    kc = torch.empty((B, H, cap, D), dtype=torch.bfloat16, device=dist.device)
    vc = torch.empty_like(kc)
    kc[:, :, :shard].normal_(generator=g)
    vc[:, :, :shard].normal_(generator=g)
    return kc, vc, k0, shard


def bench_longctx_cfg5(dist: Dist, clocks: ClockSampler, warmup: int):
    """Sequence-sharded split-KV decode with an NCCL all-gather of (out, LSE).
    After the timed steps: a split of the step into its parts, and a check of
    the NCCL-merged output against the float64 oracle on sampled (b, h)."""
    import numpy as np
    import torch
    from enilnets_b200 import kernels, sharding, _native
    from oracle.attention_ref import decode_ref
    B, H, D, ctx, T = CFG5["B"], CFG5["H"], CFG5["D"], CFG5["ctx"], CFG5["steps"]
    N = dist.world
    tail = dist.rank == N - 1
    kc, vc, k0, shard = _cfg5_shard(dist, dist.rank, B, H, D, ctx, T)
    gq = torch.Generator(device=dist.device).manual_seed(55)  # same query on every rank
    qs = torch.randn((T, B, H, D), generator=gq, device=dist.device).to(torch.bfloat16)
    kn = torch.randn((T, B, 1, H, D), generator=gq, device=dist.device).to(torch.bfloat16)
    vn = torch.randn((T, B, 1, H, D), generator=gq, device=dist.device).to(torch.bfloat16)
    out = torch.empty((B, H, D), dtype=torch.bfloat16, device=dist.device)
    decode = sharding.SequenceShardedDecode()  # local split-KV decode, NCCL gather, LSE merge
    state = {"t": 0}

    def n_live(t):
        return shard + (t + 1 if tail else 0)

    def step():
        t = state["t"]
        pos = ctx + t
        if tail:
            kernels.kv_append(kc, kn[t], shard + t)
            kernels.kv_append(vc, vn[t], shard + t)
        decode(qs[t], kc, vc, slot_begin=0, slot_end=n_live(t), pos_slot0=k0, q_pos=pos,
               out=out)
        state["t"] = (t + 1) % T

    for _ in range(max(warmup, 3)):
        step()
    state["t"] = 0
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    ms_eager = timed(dist, clocks, step, T)
    state["t"] = 0

    def all_steps():
        for _ in range(T):
            step()

    ms = timed_graph(dist, clocks, all_steps, T) * T
    state["t"] = 0
    _native.raise_on_device_error()
    bytes_total = sum(2 * B * H * D * 2 * (ctx + t + 1) for t in range(T))
    res = {"GB_s": bytes_total / (ms * 1e-3) / 1e9, "tokens_s": B * T / (ms * 1e-3),
           "ms_per_step": ms / T, "eager_ms_per_step": ms_eager / T,
           "shard_tokens_per_gpu": shard,
           "collective": "none" if N == 1 else "ncclAllGather of fp32 (out, LSE) + LSE merge",
           "steps": f"the {T} steps replayed from one CUDA graph (collectives included)"}

    # The step's parts, each timed alone over T repetitions (max over ranks).
    t_last = T - 1
    o_loc, lse_loc = kernels.attention_decode(
        qs[t_last], kc, vc, slot_begin=0, slot_end=n_live(t_last), pos_slot0=k0,
        q_pos=ctx + t_last, out_dtype=torch.float32, return_lse=True)
    parts = {"local_decode_ms": timed(dist, clocks, lambda: kernels.attention_decode(
        qs[t_last], kc, vc, slot_begin=0, slot_end=n_live(t_last), pos_slot0=k0,
        q_pos=ctx + t_last, out=o_loc, return_lse=True), T) / T}
    if N > 1:
        packed = sharding.pack_partials(o_loc, lse_loc)
        parts["all_gather_ms"] = timed(dist, clocks,
                                       lambda: sharding.gather_partials(packed), T) / T
        po, pl = sharding.split_partials(sharding.gather_partials(packed))
        parts["merge_ms"] = timed(dist, clocks, lambda: kernels.lse_merge(po, pl, out=out), T) / T
    res["step_parts"] = parts

    # Correctness across ranks: one more step (t = 0, its tail token already
    # in place) through the NCCL path, then rank 0 rebuilds every rank's
    # shard from its seed and compares sampled (b, h) with the oracle.
    state["t"] = 0
    step()
    torch.cuda.synchronize()
    _native.raise_on_device_error()
    if dist.rank == 0:
        pairs = [(0, 0), (1, 17), (B - 1, H - 1)]
        keys = {p: [] for p in pairs}
        vals = {p: [] for p in pairs}
        for r in range(N):
            kr, vr, _, sr = _cfg5_shard(dist, r, B, H, D, ctx, T)
            live = sr
            if r == N - 1:  # the tail's slot sr holds token 0 of the appended ones
                kr[:, :, sr:sr + T] = kn[:, :, 0].permute(1, 2, 0, 3)
                vr[:, :, sr:sr + T] = vn[:, :, 0].permute(1, 2, 0, 3)
                live = sr + 1
            for (b, h) in pairs:
                keys[(b, h)].append(kr[b, h, :live].float().cpu().numpy())
                vals[(b, h)].append(vr[b, h, :live].float().cpu().numpy())
            del kr, vr
        got = out.float().cpu().numpy()
        q0 = qs[0].float().cpu().numpy()
        err = 0.0
        for (b, h) in pairs:
            K = np.concatenate(keys[(b, h)])[None, None]
            V = np.concatenate(vals[(b, h)])[None, None]
            o_ref, _ = decode_ref(q0[b:b + 1, h:h + 1], K, V, slot_begin=0,
                                  slot_end=K.shape[2], pos_slot0=0, q_pos=ctx)
            err = max(err, float(np.max(np.abs(got[b, h] - o_ref[0, 0]))))
        res["check"] = {"max_abs_err": err, "pairs": [list(p) for p in pairs],
                        "against": "float64 oracle over all ranks' shards (rebuilt from seeds)"}
    return res


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


def bench_linear(dist: Dist, clocks: ClockSampler, warmup: int, steps: int = 10):
    """Linearized attention (attention_kernel "linear" and "performer"):
    feature maps plus causal linear attention on device fp32 head views, per
    GPU B4 S4096 H16 D64 (Performer with 256 features), as the layer runs them
    (attention.linearized): the maps write phi as the bf16 hi/lo planes the
    tensor-core attention reads. ms_fp32_phi times the same work through fp32
    phi (the separate-call form). FLOPs count the reference's reassociated
    form, 4 S Df D per query head, plus the Performer projections (2 S Dh Df
    for queries, twice that for keys: the stabilizer pass and the map)."""
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
        planes = kernels.linear_planes_ok(D, nf)

        def step(pl=planes):
            qp, _ = kernels.linear_feature_map(q, kernel, om, planes=pl)
            kp, _ = kernels.linear_feature_map(k, kernel, om, global_stab=True, planes=pl)
            kernels.linear_attention(qp, kp, v, causal=True, num_features=nf)

        times = {}
        for pl in (False, planes):
            for _ in range(warmup):
                step(pl)
            torch.cuda.synchronize()
            _native.raise_on_device_error()
            times[pl] = timed(dist, clocks, lambda: step(pl), steps) / steps
        ms = times[planes]
        flops = 4.0 * S * nf * D * B * H
        if kernel == "performer":
            flops += 3 * 2.0 * S * D * Df * B * H
        tf = dist.sum(flops) / (ms * 1e-3) / 1e12
        res[kernel] = {"ms_per_step": ms, "TFLOP_s": tf, "ms_fp32_phi": times[False],
                       "phi_planes": planes, "tokens_s": dist.sum(B * S) / (ms * 1e-3)}
    res["config"] = (f"B{B}/GPU S{S} H{H} D{D} causal, fp32 inputs and outputs, split-bf16 "
                     f"tcgen05 contractions (fp32-level accuracy); performer with {Df} features")
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
    out = {"ms_per_step": ms, "TFLOP_s": tf, "frac_of_bf16_peak_per_gpu": tf / dist.world / peak,
           "tensor_TFLOP_s": tf * 1.4,
           "config": f"B{B}/GPU S{S} H{H} D{D} causal bf16; dQ, dK, dV (fp32) from dO and LSE"}
    # fp32 operands (split-bf16, three MMAs per product) at head dim 64, the
    # widest the split mode takes, beside bf16 operands on the same shape.
    D32 = 64
    for name, dt in (("fp32_d64", torch.float32), ("bf16_d64", torch.bfloat16)):
        q, k, v, do = (torch.randn((B, S, H, D32), generator=g, device=dist.device).to(dt)
                       for _ in range(4))
        o, lse = kernels.attention_prefill(q, k, v, causal=True, out_dtype=torch.float32,
                                           return_lse=True)

        def step32():
            kernels.attention_backward(q, k, v, o, lse, do, causal=True)

        for _ in range(warmup):
            step32()
        torch.cuda.synchronize()
        _native.raise_on_device_error()
        ms32 = timed(dist, clocks, step32, steps) / steps
        out[name] = {"ms_per_step": ms32,
                     "TFLOP_s": dist.sum(10.0 * D32 * pairs) / (ms32 * 1e-3) / 1e12,
                     "config": f"B{B}/GPU S{S} H{H} D{D32} causal, {str(dt)[6:]} operands"}
        del q, k, v, do, o, lse
    return out


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


def bench_projections(dist: Dist, clocks: ClockSampler, warmup: int, steps: int = 20):
    """The cfg2 layer's projections on K6 (tcgen05 CTA pairs): the fused QKV
    GEMM (M = 8 x 4096, N = 3 x 2048, K = 2048) and the output GEMM (N = 2048),
    bf16 in / bf16 out with bias, and the QKV GEMM with RoPE fused on the Q/K
    columns; cuBLAS (torch.nn.functional.linear) on the same operands for
    reference. Inputs 134 MB > L2."""
    import torch
    import torch.nn.functional as F
    from enilnets_b200 import kernels, _native
    from enilnets_b200.attention import rope_tables
    M, E, H, D = CFG2["B"] * CFG2["S"], 2048, 16, 128
    g = torch.Generator(device=dist.device).manual_seed(9000 + dist.rank)
    x = torch.randn((M, E), generator=g, device=dist.device).to(torch.bfloat16)
    peak = float(load_peaks()[0]["bf16_tflops"])
    res = {}
    for name, N in (("qkv", 3 * E), ("o", E)):
        w = (torch.randn((N, E), generator=g, device=dist.device) / E ** 0.5).to(torch.bfloat16)
        b = torch.randn(N, generator=g, device=dist.device)
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dist.device)
        fl = 2.0 * M * N * E

        def run(fn):
            for _ in range(warmup):
                fn()
            torch.cuda.synchronize()
            _native.raise_on_device_error()
            return timed(dist, clocks, fn, steps) / steps

        ms = run(lambda: kernels.project(x, w, b, out=out))
        bb = b.to(torch.bfloat16)
        ms_cublas = run(lambda: F.linear(x, w, bb))
        tf = dist.sum(fl) / (ms * 1e-3) / 1e12
        res[name] = {"ms": ms, "TFLOP_s": tf, "frac_of_bf16_peak_per_gpu": tf / dist.world / peak,
                     "cublas_ms": ms_cublas,
                     "cublas_TFLOP_s": dist.sum(fl) / (ms_cublas * 1e-3) / 1e12,
                     "shape": [M, N, E]}
        if name == "qkv":
            cos, sin = rope_tables(CFG2["S"], D)
            ms_r = run(lambda: kernels.project(x, w, b, out=out,
                                               rope=(cos, sin, 2 * E, D, CFG2["S"], 0)))
            res["qkv_rope"] = {"ms": ms_r, "TFLOP_s": dist.sum(fl) / (ms_r * 1e-3) / 1e12}
    res["config"] = "x (32768, 2048) bf16, W (N, 2048) bf16, fp32 bias, bf16 out"
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
CPU_SAMPLE_HEADS = 2  # one full-length causal sequence x 2 heads of config 2 per sample


def host_blas_threads() -> int:
    """Give NumPy's BLAS every host thread. torchrun sets OMP_NUM_THREADS=1
    for its workers, which would otherwise leave the CPU baseline on one
    core; returns the thread count BLAS reports afterwards."""
    cores = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info, threadpool_limits
        threadpool_limits(limits=cores, user_api="blas")
        counts = [i["num_threads"] for i in threadpool_info() if i["user_api"] == "blas"]
        return max(counts) if counts else cores
    except ImportError:
        return cores


def cpu_sample_tflops(heads: int = CPU_SAMPLE_HEADS, repeats: int = 1):
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


def cpu_sample_desc(model: str, threads: int) -> str:
    return (f"the reference's streaming softmax (nn/flash_attention.py:42-80, float64, block "
            f"512) on 1 full-length causal sequence x {CPU_SAMPLE_HEADS} heads of config 2 per "
            f"sample, scaled by useful FLOPs; NumPy/OpenBLAS with {threads} threads on {model}")


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


def decode_summary(sub: dict, world: int, hbm: float) -> dict:
    """Compact record of the two decode workloads at this GPU count, last on
    the line so that it survives a truncated tail: HBM GB/s (all GPUs),
    fraction of the measured per-GPU copy bandwidth, tokens/s, the cfg5
    step's parts and its multi-rank check."""
    out = {"n_gpus": world, "hbm_peak_gbs": hbm}
    c3 = sub.get("decode_cfg3", {})
    if "GB_s" in c3:
        out["cfg3"] = {"GB_s": round(c3["GB_s"], 1),
                       "frac_per_gpu": round(c3["GB_s"] / world / hbm, 4),
                       "tokens_s": round(c3["tokens_s"], 1),
                       "ms_step": round(c3["ms_per_step"], 4),
                       "eager_ms_step": round(c3["eager_ms_per_step"], 4),
                       "kernel_frac_per_gpu": round(c3["decode_kernel_GB_s"] / world / hbm, 4)}
    c5 = sub.get("longctx_cfg5", {})
    if "GB_s" in c5:
        out["cfg5"] = {"GB_s": round(c5["GB_s"], 1),
                       "frac_per_gpu": round(c5["GB_s"] / world / hbm, 4),
                       "tokens_s": round(c5["tokens_s"], 1),
                       "ms_step": round(c5["ms_per_step"], 4),
                       "eager_ms_step": round(c5["eager_ms_per_step"], 4),
                       "parts_ms": {k: round(v, 4) for k, v in c5.get("step_parts", {}).items()},
                       "max_abs_err": c5.get("check", {}).get("max_abs_err")}
    return out


def arm_config(n_gpus: int) -> dict:
    """The headline workload's config, shared by both arms."""
    return {"workload": "cfg2 causal prefill B8/GPU S4096 H16 D128, key padding L~U[2048,4096]",
            "global_batch": CFG2["B"] * n_gpus, "seq_len": CFG2["S"],
            "parallelism": f"batch x head over {n_gpus} GPU(s): cost-balanced contiguous "
                           "(batch, head) units per GPU, no collective",
            "l2": "inputs 402 MB per GPU > 126 MB L2 (no flush needed)"}


def run_reference(args):
    """--impl reference: the reference algorithm (NumPy float64 port) on the
    host cores, rank 0 only, BLAS on every host thread."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    model, _ = cpu_info()
    threads = host_blas_threads()
    for _ in range(args.warmup):
        cpu_sample_tflops()
    vals = []
    t_total = 0.0
    for _ in range(args.steps):
        v, t, _ = cpu_sample_tflops()
        vals.append(v)
        t_total += t
    value = statistics.mean(vals)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000 * t_total / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": arm_config(args.gpus),
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads,
                             "kind": "port", "sample": cpu_sample_desc(model, threads)},
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
                                       "linear", "sparse", "backward", "e2e", "gemm"],
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
            elif args.only == "gemm":
                res = bench_projections(dist, clocks, args.warmup)
            elif args.only == "e2e":
                res = {pol: bench_prefill(dist, clocks, args.steps, args.warmup, args.batch,
                                          e2e_policy=pol)["e2e"] for pol in ("local", "spread")}
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
        if not args.no_cpu_baseline and dist.world == 1:
            model, _ = cpu_info()
            threads = host_blas_threads()
            cpu_sample_tflops()  # warm-up
            v, t, _ = cpu_sample_tflops(repeats=8)
            cpu = {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                   "sample": cpu_sample_desc(model, threads) + f"; 8 samples, {8 * t:.1f} s"}
        line = {
            "metric": METRIC, "value": pre["value"], "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": pre["ms_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic N(0,1) activations, seeded",
            "config": arm_config(args.gpus),
            "prefill_rank0": {"rows": pre["rows"], "n_units": pre["n_units"],
                              "lengths": pre["lengths"]},
            "e2e": pre["e2e"],
            "roofline": roofline,
            "cpu_baseline": cpu,
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
            **sub,
        }
        line["decode"] = decode_summary(sub, dist.world, hbm)
        print(json.dumps(line))
    dist.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
