"""Multi-rank host logic on CPU: the prefill unit partition, the KV sequence
shards, and the gather of (out, lse) partials for sequence-sharded decode,
the last over world-size-2 gloo process groups. The per-rank attention runs
through the float64 oracle here; on GPUs the same SequenceShardedDecode
calls the split-KV kernel and the LSE-merge kernel over NCCL."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from enilnets_b200 import sharding
from oracle import attention_ref as ref


def test_partition_covers_every_unit_once_and_is_balanced():
    rng = np.random.RandomState(0)
    lengths = rng.randint(2048, 4097, size=8)
    costs = sharding.prefill_unit_costs(lengths, 4096, 16)
    for world in (1, 2, 3, 4, 8):
        parts = sharding.partition_units(costs, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(costs)))
        loads = [sum(costs[i] for i in p) for p in parts]
        lower = max(sum(costs) / world, max(costs))
        assert max(loads) <= 4 / 3 * lower
        assert parts == sharding.partition_units(costs, world)  # deterministic


def test_contiguous_partition_is_balanced_ranges():
    """Contiguous (batch-major) unit ranges, every rank within one unit's
    cost of the mean load; the bench's 8-sequences-per-GPU batches."""
    rng = np.random.RandomState(2)
    for world in (1, 2, 3, 4, 8):
        lengths = rng.randint(2048, 4097, size=8 * world)
        costs = sharding.prefill_unit_costs(lengths, 4096, 16)
        parts = sharding.contiguous_partition(costs, world)
        flat = [i for p in parts for i in p]
        assert flat == list(range(len(costs))), "ranges in order, each unit once"
        mean = sum(costs) / world
        for p in parts:
            assert p == list(range(p[0], p[-1] + 1))
            assert abs(sum(costs[i] for i in p) - mean) <= max(costs)
        assert parts == sharding.contiguous_partition(costs, world)
    assert sharding.contiguous_partition([5, 5], 4) == [[], [0], [], [1]] or \
        sum(len(p) for p in sharding.contiguous_partition([5, 5], 4)) == 2


def test_causal_pairs_match_the_padding_rule():
    # padded query rows still see all L real keys (graph/sequence.py:159-183)
    assert sharding.causal_pairs(3, 5) == 3 * 4 // 2 + 2 * 3
    assert sharding.causal_pairs(5, 5) == 15
    assert sharding.causal_pairs(0, 5) == 0
    assert sharding.causal_pairs(3, 5, causal=False) == 15


@pytest.mark.parametrize("n,world", [(262144, 8), (10, 3), (2, 4), (0, 2)])
def test_shard_ranges_are_contiguous_and_cover(n, world):
    ranges = [sharding.kv_shard_range(n, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a, b), (c, d) in zip(ranges, ranges[1:]):
        assert b == c and a <= b
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.batch_shard(n, world, world)


# ---------------------------------------------------------------- gloo
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_local(q, k, v, *, slot_begin, slot_end, pos_slot0, q_pos, window, alibi_slopes,
                  scale):
    o, lse = ref.decode_ref(q.numpy(), k.numpy(), v.numpy(), slot_begin=slot_begin,
                            slot_end=slot_end, pos_slot0=pos_slot0, q_pos=q_pos, window=window,
                            alibi=None if alibi_slopes is None else alibi_slopes.numpy(),
                            scale=scale)
    return torch.from_numpy(o), torch.from_numpy(lse)


def _oracle_merge(part_o, part_lse, out=None):
    o, _ = ref.lse_merge_ref(part_o.numpy(), part_lse.numpy())
    return torch.from_numpy(o)


def _rank_main(rank, world, port, case, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, H, Hkv, D, ctx, q_pos, window = case
        q = ref.seeded_normal(1, (B, H, D), bf16=False)
        K = ref.seeded_normal(2, (B, Hkv, ctx, D), bf16=False)
        V = ref.seeded_normal(3, (B, Hkv, ctx, D), bf16=False)
        start, end = sharding.kv_shard_range(ctx, world, rank)
        step = sharding.SequenceShardedDecode(local=_oracle_local, merge=_oracle_merge)
        o = step(torch.from_numpy(q), torch.from_numpy(K[:, :, start:end].copy()),
                 torch.from_numpy(V[:, :, start:end].copy()), slot_begin=0,
                 slot_end=end - start, pos_slot0=start, q_pos=q_pos, window=window)
        full, _ = ref.decode_ref(q, K, V, slot_begin=0, slot_end=ctx, pos_slot0=0, q_pos=q_pos,
                                 window=window)
        result_q.put((rank, float(np.max(np.abs(o.numpy() - full)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [
    (2, 4, 2, 32, 300, 299, None),   # every shard visible
    (1, 2, 1, 16, 200, 60, None),    # rank 1's keys all after the query: lse = -inf there
    (2, 2, 2, 16, 257, 256, 40),     # a sliding window inside rank 1's shard
])
def test_sequence_sharded_decode_gloo_world2(case):
    world = 2
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, case, result_q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    errs = dict(result_q.get(timeout=5) for _ in range(world))
    # The partials travel as fp32 (as on the GPUs), the rest is float64.
    assert max(errs.values()) < 1e-6, errs
