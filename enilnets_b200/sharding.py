"""Work partitioning over the GPUs of one node, one process per GPU.

Two shapes of sharding cover the attention path:

* Prefill (K1) shards by independent (batch, head) units, with no
  collective. Key padding makes the units unequal: a causal row of valid
  length L has L(L+1)/2 + (S - L) * L visible (query, key) pairs (padded
  query rows still see all L real keys, the graph layer's rule,
  graph/sequence.py:159-183). The units are balanced by that cost, either
  with the longest-processing-time rule (partition_units, any units) or as
  cost-balanced contiguous ranges (contiguous_partition), so that a rank's
  inputs are a run of consecutive sequences; K1 then runs exactly the
  rank's units (the units argument of kernels.attention_prefill).
* Long-context decode (K2) shards the KV sequence into contiguous slot
  ranges. Each rank runs the split-KV decode on its range and produces a
  normalised partial (out, lse). The partials are all-gathered (NCCL on GPUs,
  gloo in the CPU tests) and merged by log-sum-exp (enl_lse_merge). This is
  the only exchange step on the path.

The reference has no multi-device path. Its attention runs in one process
(nn/forward.py:525-551, nn/kvcache.py:198-213).
"""
from __future__ import annotations

import heapq
from typing import Callable, List, Optional, Sequence, Tuple


# ------------------------------------------------------------------ prefill
def causal_pairs(length: int, seq: int, causal: bool = True) -> int:
    """Visible (query, key) pairs of one head of one padded sequence."""
    length = max(0, min(int(length), int(seq)))
    if not causal:
        return seq * length
    return length * (length + 1) // 2 + (seq - length) * length


def prefill_unit_costs(lengths: Sequence[int], seq: int, num_heads: int,
                       causal: bool = True) -> List[int]:
    """Cost of every (batch, head) unit, unit index b * num_heads + h."""
    out = []
    for L in lengths:
        c = causal_pairs(L, seq, causal)
        out.extend([c] * num_heads)
    return out


def partition_units(costs: Sequence[int], world: int) -> List[List[int]]:
    """Longest-processing-time partition of units over `world` ranks.

    Units go heaviest first to the currently lightest rank (ties to the
    lower rank), and each rank's list is returned in ascending unit order.
    The result is deterministic, so every rank computes the same partition
    without communicating. The largest rank load is at most 4/3 of the
    optimum.
    """
    if world < 1:
        raise ValueError(f"world must be >= 1, got {world}")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0, r) for r in range(world)]
    parts: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    return [sorted(p) for p in parts]


def contiguous_partition(costs: Sequence[int], world: int) -> List[List[int]]:
    """Cost-balanced partition of units into `world` contiguous index ranges.

    Units are taken in index order (for (batch, head) units: batch-major,
    so a rank's units cover a run of consecutive sequences and its inputs
    are those sequences only). Unit i goes to the rank whose share of the
    total cost contains the unit's cost midpoint, so every rank's load is
    within one unit's cost of total / world. Deterministic: every rank
    computes the same partition without communicating."""
    if world < 1:
        raise ValueError(f"world must be >= 1, got {world}")
    total = float(sum(costs))
    parts: List[List[int]] = [[] for _ in range(world)]
    acc = 0.0
    for i, c in enumerate(costs):
        mid = acc + c / 2.0
        r = min(world - 1, int(mid * world / total)) if total > 0 else i * world // len(costs)
        parts[r].append(i)
        acc += c
    return parts


def batch_shard(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous batch rows [start, end) of `rank`, sizes differing by at
    most one (decode of independent rows, config-3 style)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


# --------------------------------------------------------- long-context KV
def kv_shard_range(ctx: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous KV positions [start, end) held by `rank`, sizes differing
    by at most one. Ranks hold consecutive ranges in rank order."""
    return batch_shard(ctx, world, rank)


def pack_partials(o, lse):
    """(B, H, D) fp32 out and (B, H) fp32 lse -> one (B, H, D + 1) buffer,
    so that a single collective moves both."""
    import torch
    return torch.cat([o.float(), lse.float().unsqueeze(-1)], dim=-1).contiguous()


def gather_partials(packed, group=None):
    """All-gather every rank's packed partials -> (world, B, H, D + 1), in
    rank order. Uses all_gather_into_tensor where the backend has it (NCCL),
    else a list all_gather (gloo)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(packed.shape), dtype=packed.dtype, device=packed.device)
    if packed.is_cuda:
        dist.all_gather_into_tensor(out, packed, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), packed, group=group)
    return out


def split_partials(gathered):
    """(world, B, H, D + 1) -> contiguous (world, B, H, D) out and
    (world, B, H) lse."""
    return gathered[..., :-1].contiguous(), gathered[..., -1].contiguous()


class SequenceShardedDecode:
    """One decode step over a KV cache sharded by sequence across ranks.

    Each rank holds the slots of its contiguous position range. A call runs
    the local split-KV decode, all-gathers the (out, lse) partials and
    merges them. Every rank returns the full (B, H, D) output. A rank whose
    range holds no visible key contributes lse = -inf, which carries no
    weight in the merge.

    `local` and `merge` default to the CUDA kernels (kernels.attention_decode,
    kernels.lse_merge). They are parameters so that the partition and gather
    logic can be exercised on CPU ranks.
    """

    def __init__(self, group=None, local: Optional[Callable] = None,
                 merge: Optional[Callable] = None):
        self.group = group
        self._local = local
        self._merge = merge
        self._bufs = {}  # (shape, device) -> (packed, gathered) for the CUDA path

    def _cuda_step(self, q, k_cache, v_cache, out, out_dtype, **kw):
        """The CUDA path: K2 writes its (out, lse) straight into one packed
        fp32 buffer [out (B*H*D) | lse (B*H)], a single all_gather_into_tensor
        moves it, and the merge reads the gathered parts in place."""
        import torch
        import torch.distributed as dist
        from . import kernels
        B, H, D = q.shape
        world = dist.get_world_size(self.group)
        key = (B, H, D, world, q.device)
        if key not in self._bufs:
            n = B * H * (D + 1)
            self._bufs[key] = (torch.empty(n, dtype=torch.float32, device=q.device),
                               torch.empty((world, n), dtype=torch.float32, device=q.device))
        packed, gathered = self._bufs[key]
        kernels.attention_decode(q, k_cache, v_cache, out=packed[:B * H * D].view(B, H, D),
                                 lse_out=packed[B * H * D:].view(B, H), **kw)
        dist.all_gather_into_tensor(gathered, packed, group=self.group)
        part_o = gathered[:, :B * H * D].unflatten(1, (B, H, D))
        part_lse = gathered[:, B * H * D:].unflatten(1, (B, H))
        return kernels.lse_merge(part_o, part_lse, out=out, out_dtype=out_dtype or torch.bfloat16)

    def __call__(self, q, k_cache, v_cache, *, slot_begin: int, slot_end: int,
                 pos_slot0: int, q_pos: int, window=None, alibi_slopes=None, scale=None,
                 out=None, out_dtype=None):
        import torch
        import torch.distributed as dist
        if self._local is None and self._merge is None and q.is_cuda and dist.is_initialized():
            return self._cuda_step(q, k_cache, v_cache, out, out_dtype, slot_begin=slot_begin,
                                   slot_end=slot_end, pos_slot0=pos_slot0, q_pos=q_pos,
                                   window=window, alibi_slopes=alibi_slopes, scale=scale)
        if self._local is None:
            from . import kernels
            o, lse = kernels.attention_decode(
                q, k_cache, v_cache, slot_begin=slot_begin, slot_end=slot_end,
                pos_slot0=pos_slot0, q_pos=q_pos, window=window, alibi_slopes=alibi_slopes,
                scale=scale, out_dtype=torch.float32, return_lse=True)
        else:
            o, lse = self._local(q, k_cache, v_cache, slot_begin=slot_begin, slot_end=slot_end,
                                 pos_slot0=pos_slot0, q_pos=q_pos, window=window,
                                 alibi_slopes=alibi_slopes, scale=scale)
        import torch.distributed as dist
        if not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return o if out is None else out.copy_(o)
        part_o, part_lse = split_partials(gather_partials(pack_partials(o, lse), self.group))
        if self._merge is not None:
            return self._merge(part_o, part_lse, out=out)
        from . import kernels
        return kernels.lse_merge(part_o, part_lse, out=out,
                                 out_dtype=out_dtype or torch.bfloat16)
