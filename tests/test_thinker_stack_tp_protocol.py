"""Host logic of the tensor / expert-parallel thinker stack on the CPU: the head and expert
shard plan, the owner row ranges, and (two gloo ranks) one layer computed from each rank's
shards with the exchanges of thinker_stack_tp -- the o_proj partials summed in rank order by
each row's owner, the expert rows read from the rank holding each slot's expert and summed
in slot order -- equal to the unsharded layer (torch float64 stand-ins for the kernels)."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mstar_accelerators_b200.thinker_stack import ThinkerStackConfig
from mstar_accelerators_b200.thinker_stack_tp import owner_rows, shard_plan


@pytest.mark.parametrize("heads,world", [((32, 4), 1), ((32, 4), 2), ((32, 4), 4), ((32, 4), 8), ((8, 2), 2),
                                         ((4, 1), 2), ((16, 4), 8)])
def test_shard_plan_covers_heads_and_experts(heads, world):
    cfg = ThinkerStackConfig(q_heads=heads[0], kv_heads=heads[1], experts=128)
    group = cfg.q_heads // cfg.kv_heads
    q_seen, e_seen = [], []
    for r in range(world):
        q0, qn, k0, kn, e0, en = shard_plan(cfg, world, r)
        q_seen += range(q0, q0 + qn)
        e_seen += range(e0, e0 + en)
        for q in range(q0, q0 + qn):        # every held query head reads a held KV head,
            assert k0 <= q // group < k0 + kn
            # at the same position of the local GQA fold [kv_heads, group', D]
            assert (q - q0) // (qn // kn) == q // group - k0
    assert q_seen == list(range(cfg.q_heads)) and e_seen == list(range(cfg.experts))


def test_shard_plan_refuses_uneven_splits():
    with pytest.raises(ValueError):
        shard_plan(ThinkerStackConfig(q_heads=32, kv_heads=4, experts=128), 3, 0)
    with pytest.raises(ValueError):
        shard_plan(ThinkerStackConfig(q_heads=24, kv_heads=6, experts=128), 4, 0)   # 6 heads per rank, groups of 4


@pytest.mark.parametrize("rows,world", [(0, 2), (1, 8), (32, 8), (35, 4), (32768, 8), (7, 3)])
def test_owner_rows_partition(rows, world):
    seen = []
    for r in range(world):
        row0, owned = owner_rows(rows, world, r)
        seen += range(row0, row0 + owned)
    assert seen == list(range(rows))


def _layer_half(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        cfg = ThinkerStackConfig(hidden=64, q_heads=8, kv_heads=2, head_dim=16, experts=8, top_k=3)
        g = torch.Generator().manual_seed(5)
        T, H, D = 11, cfg.hidden, cfg.head_dim
        x = torch.randn(T, H, generator=g, dtype=torch.float64)
        att = torch.randn(T, cfg.q_heads * D, generator=g, dtype=torch.float64)
        o = torch.randn(H, cfg.q_heads * D, generator=g, dtype=torch.float64)
        ids = torch.stack([torch.randperm(cfg.experts, generator=g)[:cfg.top_k] for _ in range(T)]).int()
        wts = torch.rand(T, cfg.top_k, generator=g, dtype=torch.float64)
        experts = torch.randn(cfg.experts, H, H, generator=g, dtype=torch.float64)
        q0, qn, k0, kn, e0, en = shard_plan(cfg, world, rank)
        # o_proj row-parallel: this rank's partial from its heads' columns
        part = att[:, q0 * D:(q0 + qn) * D] @ o[:, q0 * D:(q0 + qn) * D].T
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)                  # stands for the peer-visible partial buffers
        row0, owned = owner_rows(T, world, rank)
        new = x[row0:row0 + owned].clone()
        s = parts[0][row0:row0 + owned].clone()
        for p in range(1, world):
            s += parts[p][row0:row0 + owned]
        new += s
        # expert-parallel: this rank's expert rows for its held pairs and their row index
        y, inv = [], torch.full((T * cfg.top_k,), -1, dtype=torch.int32)
        for i, e in enumerate(ids.view(-1).tolist()):
            if e0 <= e < e0 + en:
                inv[i] = len(y)
                y.append(wts.view(-1)[i] * (experts[e] @ x[i // cfg.top_k]))
        y = torch.stack(y) if y else torch.zeros(0, H, dtype=torch.float64)
        ys = [None] * world
        invs = [torch.empty_like(inv) for _ in range(world)]
        dist.all_gather_object(ys, y)
        dist.all_gather(invs, inv)
        comb = torch.zeros(owned, H, dtype=torch.float64)
        for j, t in enumerate(range(row0, row0 + owned)):
            for s_ in range(cfg.top_k):
                e = int(ids[t, s_])
                p = e // en
                comb[j] += ys[p][int(invs[p][t * cfg.top_k + s_])]
        full_o = x + att @ o.T
        full_moe = torch.stack([sum(wts[t, s_] * (experts[int(ids[t, s_])] @ x[t]) for s_ in range(cfg.top_k))
                                for t in range(T)])
        out[rank] = (float((new - full_o[row0:row0 + owned]).abs().max()) if owned else 0.0,
                     float((comb - full_moe[row0:row0 + owned]).abs().max()) if owned else 0.0)
    finally:
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_layer_exchanges_equal_the_unsharded_layer():
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        out = manager.dict()
        mp.start_processes(_layer_half, args=(world, _port(), out), nprocs=world, join=True, start_method="spawn")
        for r in range(world):
            assert out[r][0] < 1e-9 and out[r][1] < 1e-9, out[r]
