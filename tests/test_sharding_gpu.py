"""SequenceShardedDecode's CUDA path on one GPU: K2 writes (out, lse) into
the packed all-gather buffer, NCCL all_gather_into_tensor moves it, and the
strided LSE merge reads the gathered parts in place (the path every rank of
config 5 runs). With one rank the merge of a single part is exact, so the
result equals the plain decode bit for bit; both are held to the float64
oracle at the bf16 bar."""
import os
import socket

import numpy as np
import pytest

from oracle import attention_ref as ref

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sequence_sharded_decode_over_nccl(cuda):
    import torch
    import torch.distributed as dist
    from enilnets_b200 import _native, kernels, sharding
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = str(_free_port())
    created = not dist.is_initialized()
    if created:
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    try:
        B, H, Hkv, D, ctx = 2, 8, 4, 128, 3000
        cast = lambda x: torch.from_numpy(x.astype(np.float32)).cuda().to(torch.bfloat16)  # noqa
        q = ref.seeded_normal(91, (B, H, D))
        kc = ref.seeded_normal(92, (B, Hkv, ctx, D))
        vc = ref.seeded_normal(93, (B, Hkv, ctx, D))
        qd, kd, vd = cast(q), cast(kc), cast(vc)
        dec = sharding.SequenceShardedDecode()
        outs = []
        for _ in range(2):  # the packed buffers are reused across steps
            outs.append(dec(qd, kd, vd, slot_begin=0, slot_end=ctx, pos_slot0=0, q_pos=ctx - 1,
                            out_dtype=torch.float32))
        plain = kernels.attention_decode(qd, kd, vd, slot_begin=0, slot_end=ctx, pos_slot0=0,
                                         q_pos=ctx - 1, out_dtype=torch.float32)
        torch.cuda.synchronize()
        _native.raise_on_device_error()
        for o in outs:
            assert torch.equal(o, plain)
        oref, _ = ref.decode_ref(q, kc, vc, slot_begin=0, slot_end=ctx, pos_slot0=0,
                                 q_pos=ctx - 1)
        assert float(np.max(np.abs(outs[0].cpu().numpy() - oref))) <= 2e-2
    finally:
        if created:
            dist.destroy_process_group()
