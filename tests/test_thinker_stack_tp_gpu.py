"""The thinker stack tensor-parallel (attention by heads, o_proj row-parallel through the
peer-memory reduction) and expert-parallel (experts split over the ranks, the slot-order
combine over peer memory) on two B200s, against the oracle composition
(oracle/thinker_oracle.ThinkerStackOracle) and the single-GPU stack (skipped with fewer
than 2 GPUs).

Two geometries: 8 query / 2 KV heads (each rank holds one whole GQA group) and 4 query /
1 KV head (the KV head is computed on both ranks, the config-5 layout at W = 8). Prefill of
3 sequences x 70 tokens, then 4 decode steps teacher-forced with the oracle's tokens, the
decode step replayed as one captured CUDA graph. Both ranks must return identical logits;
logits are held to the oracle as the single-GPU stack is (5e-2 of the largest |logit|,
mean 1e-2; greedy tokens same or reciprocal top-5), and to the single-GPU stack within
the same bounds (o_proj's partial folds are summed in rank order, so the two are not
bit-identical)."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, results, heads):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from mstar_accelerators_b200.thinker_stack import ThinkerStackB200, ThinkerStackConfig, head_weights, \
            layer_weights
        from mstar_accelerators_b200.thinker_stack_tp import ThinkerStackTP
        from oracle.thinker_oracle import ThinkerStackOracle
        from oracle.whisper_oracle import greedy_agrees
        qh, kh = heads
        cfg = ThinkerStackConfig(hidden=256, layers=2, q_heads=qh, kv_heads=kh, experts=16, top_k=4,
                                 moe_intermediate=128, vocab=1000)
        layers = [layer_weights(cfg, i, seed=3) for i in range(cfg.layers)]
        tp = ThinkerStackTP(cfg, max_seqs=3, max_len=80, seed=3, experts="q8_0", gemm_rows=256,
                            weights=lambda i: layers[i])
        one = ThinkerStackB200(cfg, max_seqs=3, max_len=80, seed=3, experts="q8_0", gemm_rows=256,
                               weights=lambda i: layers[i])
        ref = ThinkerStackOracle(cfg, [{k: v.cpu() for k, v in L.items()} for L in layers],
                                 {k: v.cpu() for k, v in head_weights(cfg, seed=3).items()}, experts="q8_0")
        tokens = np.random.default_rng(4).integers(0, cfg.vocab, (3, 70))
        errors = []

        def check(got, want, single):
            gl, gt = got[0].cpu().numpy(), got[1].cpu().numpy()
            rl, rt = want
            scale = np.abs(rl).max()
            d = np.abs(gl - rl)
            errors.append(("oracle", float(d.max() / scale), float(d.mean() / scale)))
            d1 = np.abs(gl - single[0].cpu().numpy())
            errors.append(("single", float(d1.max() / scale), float(d1.mean() / scale)))
            agree = all(greedy_agrees(int(gt[b]), rl[b], int(rt[b]), gl[b]) for b in range(len(gt)))
            others = [torch.empty_like(got[0]) for _ in range(world)]
            dist.all_gather(others, got[0].contiguous())
            same = all(torch.equal(o, got[0]) for o in others)
            errors.append(("agree", agree, same))
            return rt

        t = torch.from_numpy(tokens).cuda()
        nxt = check(tp.prefill(t), ref.prefill(tokens), one.prefill(t))
        for _ in range(4):
            nt = torch.from_numpy(nxt).cuda()
            got = tp.decode(nt, graph=True)
            got = (got[0].clone(), got[1].clone())
            nxt = check(got, ref.decode(nxt), one.decode(nt))
        torch.cuda.synchronize()
        results[rank] = (errors, int(tp.status.item()), tp.expert_status(), int(one.status.item()))
        tp.close()
        one.close()
    finally:
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("heads", [(8, 2), (4, 1)])
def test_tensor_expert_parallel_stack(heads):
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        mp.start_processes(_worker, args=(world, _port(), results, heads), nprocs=world, join=True,
                           start_method="spawn")
        for rank in range(world):
            errors, st, est, st1 = results[rank]
            assert st == 0 and est == 0 and st1 == 0, (rank, st, est, st1)
            for kind, a, b in errors:
                if kind == "agree":
                    assert a and b, (rank, errors)
                else:
                    assert a <= 5e-2 and b <= 1e-2, (rank, kind, a, b)
