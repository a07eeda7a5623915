"""Expert-parallel dispatch / combine logic on CPU: two gloo ranks.

ExpertParallelMoE's host logic (ordering of the (token, slot) pairs by owning
rank, count exchange, the three all_to_all exchanges, the reversed return and
the slot-ordered combine) is exercised with the oracle as the local expert
computation (oracle/moe_oracle.py, top-1 per received pair) and a numpy
slot-ordered combine. Every rank's output must equal, bit for bit, the
single-process oracle layer over all experts for that rank's tokens. Includes a
rank whose tokens all route to the other rank's experts, and a rank with no
tokens at all in the step (it still takes every collective step and serves the
other rank's pairs).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe_oracle as M

E, I, H, K = 16, 64, 128, 4


def _weights():
    g = torch.Generator().manual_seed(11)
    w1 = (torch.randn((E, 2 * I, H), generator=g) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn((E, H, I), generator=g) * 0.05).to(torch.bfloat16)
    return w1, w2


def _tokens(rank):
    g = torch.Generator().manual_seed(100 + rank)
    T = 9 + 4 * rank
    x = torch.randn((T, H), generator=g).to(torch.bfloat16)
    w = torch.rand((T, K), generator=g)
    w = w / w.sum(-1, keepdim=True)
    if rank == 0:
        ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)])
    else:  # every pair of this rank goes to rank 0's experts
        ids = torch.stack([torch.randperm(E // 2, generator=g)[:K] for _ in range(T)])
    return x, w.float(), ids.to(torch.int32)


def _worker(rank, world, port, results, empty_rank=-1):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mstar_accelerators_b200.moe_ep import ExpertParallelMoE, owned_experts
        w1, w2 = _weights()
        own = owned_experts(E, world, rank)
        w1f, w2f = w1.float().numpy(), w2.float().numpy()

        def local(rows, weights, ids):
            if rows.shape[0] == 0:
                return rows.new_empty((0, H))
            y = M.experts_bf16(rows.float().numpy(), w1f[own.start:own.stop], w2f[own.start:own.stop],
                               weights.numpy()[:, None], ids.numpy()[:, None])
            return torch.from_numpy(y).to(torch.bfloat16)

        def combine(y, rows, k):
            yf = y.float().numpy()
            r = rows.numpy().reshape(-1, k)
            out = np.zeros((r.shape[0], H), np.float32)
            for s in range(k):
                out = (out + yf[r[:, s]]).astype(np.float32)
            return torch.from_numpy(M.bf16(out)).to(torch.bfloat16)

        layer = ExpertParallelMoE(local, combine, experts=E, top_k=K)
        x, w, ids = _tokens(rank)
        if rank == empty_rank:  # this step routes no tokens from this rank; it still serves its experts
            x, w, ids = x[:0], w[:0], ids[:0]
        got = layer(x, w, ids).float().numpy()
        if x.shape[0]:
            ref = M.experts_bf16(x.float().numpy(), w1f, w2f, w.numpy(), ids.numpy())
        else:
            ref = np.zeros((0, H), np.float32)
        results[rank] = bool(got.shape == ref.shape and np.array_equal(got, ref))
    finally:
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_parallel_matches_single_process_oracle():
    world = 2
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_worker, args=(world, _port(), results), nprocs=world, join=True)
        assert dict(results) == {0: True, 1: True}


def test_a_rank_with_no_tokens_still_serves_its_experts():
    world = 2
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_worker, args=(world, _port(), results, 1), nprocs=world, join=True)
        assert dict(results) == {0: True, 1: True}


def test_b200_combine_of_no_tokens_launches_nothing():
    from mstar_accelerators_b200.moe_ep import b200_combine
    out = b200_combine(None)(torch.empty((0, H), dtype=torch.bfloat16), torch.empty(0, dtype=torch.int32), K)
    assert out.shape == (0, H) and out.dtype == torch.bfloat16


def test_owned_experts_split():
    from mstar_accelerators_b200.moe_ep import owned_experts
    assert owned_experts(128, 8, 3) == range(48, 64)
    with pytest.raises(ValueError):
        owned_experts(10, 4, 0)


def _bad_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mstar_accelerators_b200.moe_ep import ExpertParallelMoE
        layer = ExpertParallelMoE(lambda r, w, i: r, lambda y, rows, k: y, experts=E, top_k=K)
        x, w, ids = _tokens(rank)
        if rank == 1:
            ids[2, 1] = E + 3                       # one invalid id on one rank only
        try:
            layer(x, w, ids)
            results[rank] = "no error"
        except ValueError as err:
            results[rank] = "raised" if "expert id" in str(err) else str(err)
    finally:
        dist.destroy_process_group()


def test_an_invalid_id_on_one_rank_stops_every_rank():
    world = 2
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_bad_worker, args=(world, _port(), results), nprocs=world, join=True)
        assert dict(results) == {0: "raised", 1: "raised"}
