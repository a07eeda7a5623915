"""Expert parallelism on B200s: two NCCL ranks (skipped with fewer than 2 GPUs).

Each rank keeps half the experts of a thinker-shaped layer (128 experts,
intermediate 768, hidden 2048, top-8) and dispatches its own tokens. Because
every received pair is computed by the same grouped kernels and the combine
sums slots in slot order, each rank's output must equal, bit for bit, the
single-GPU layer (all experts on one device) on that rank's tokens.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

E, I, H, K = 128, 768, 2048, 8


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from mstar_accelerators_b200.moe import ThinkerMoEB200, route
        from mstar_accelerators_b200.moe_ep import ExpertParallelMoE
        g = torch.Generator().manual_seed(5)
        w1 = (torch.randn((E, 2 * I, H), generator=g) * 0.02).to(torch.bfloat16).cuda()
        w2 = (torch.randn((E, H, I), generator=g) * 0.02).to(torch.bfloat16).cuda()
        wr = (torch.randn((E, H), generator=g) * 0.02).to(torch.bfloat16).cuda()
        gx = torch.Generator().manual_seed(50 + rank)
        T = 96 + 32 * rank
        x = torch.randn((T, H), generator=gx).to(torch.bfloat16).cuda()
        w, ids = route(x, wr, top_k=K)
        layer = ExpertParallelMoE.b200(w1, w2, experts=E, top_k=K, capacity=512)
        got = layer(x, w, ids)
        whole = ThinkerMoEB200(w1, w2, fmt="bf16", top_k=K, max_tokens=T)
        ref = whole(x, w, ids)
        torch.cuda.synchronize()
        results[rank] = bool(torch.equal(got, ref))
        whole.close()
    finally:
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_expert_parallel_equals_single_gpu():
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        mp.start_processes(_worker, args=(world, _port(), results), nprocs=world, join=True, start_method="spawn")
        assert dict(results) == {0: True, 1: True}
