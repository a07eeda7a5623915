"""The tensor-parallel encoder's data flow with two gloo ranks on the CPU (no GPU): each
rank holds only its shard (mstar_accelerators_b200.encoder_tp.shard_weights) and runs one
encoder layer's contractions through the oracle's Q8_0 mul_mat; the exchange follows the
B200 protocol: row-parallel partials gathered to the owner of each row range
(owner_split), summed in rank order, bias added once, then the owned rows all-gathered.

  * column-parallel QKV by heads (head_split) and fc1 by FFN columns reassemble the
    single-process outputs bit for bit (each output column is the same block dots);
  * row-parallel out_proj / fc2 equal the single-process product up to the fp32 order
    of the two ranks' block sums (<= 1e-5 of the largest |output|), every rank ends with
    the same rows, and the bias is counted once.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mstar_accelerators_b200.encoder import EncoderConfig, synthetic_weights
        from mstar_accelerators_b200.encoder_tp import head_split, owner_split, shard_weights
        from oracle import oracle as O
        cfg = EncoderConfig(mels=80, width=256, heads=4, layers=1, positions=40)
        full = synthetic_weights(cfg, seed=5)
        mine = shard_weights(full, cfg, world, rank)
        p = "encoder.layers.0."
        rng = np.random.default_rng(9)
        M = 2 * cfg.positions                            # two utterances
        x = rng.standard_normal((M, cfg.width)).astype(np.float32)
        h = rng.standard_normal((M, cfg.ffn)).astype(np.float32)
        f = lambda t: t.contiguous().numpy().astype(np.float32)

        # column parallel: my heads' q|k|v and my fc1 columns, all-gathered in rank order
        qkv = np.concatenate([O.mul_mat(O.pack_weights(f(mine[p + f"self_attn.{n}_proj.weight"])), x)
                              for n in "qkv"], 1)
        sizes = [3 * c * (cfg.width // cfg.heads) for c in head_split(cfg.heads, world)]
        gathered = [torch.zeros((M, s_), dtype=torch.float32) for s_ in sizes]
        dist.all_gather(gathered, torch.from_numpy(qkv))
        ref_qkv = {n: O.mul_mat(O.pack_weights(f(full[p + f"self_attn.{n}_proj.weight"])), x) for n in "qkv"}
        hd = cfg.width // cfg.heads
        col = 0
        ok_cols = True
        for r, g in enumerate(gathered):
            c = head_split(cfg.heads, world)[r] * hd
            for j, n in enumerate("qkv"):
                ok_cols &= np.array_equal(g.numpy()[:, j * c:(j + 1) * c], ref_qkv[n][:, col:col + c])
            col += c

        # row parallel fc2: my K shard's partial of every row, reduced by the rows' owners
        ffn_shard = cfg.ffn // world
        partial = O.mul_mat(O.pack_weights(f(mine[p + "fc2.weight"])), h[:, rank * ffn_shard:(rank + 1) * ffn_shard])
        every = [torch.zeros_like(torch.from_numpy(partial)) for _ in range(world)]
        dist.all_gather(every, torch.from_numpy(partial))
        own = owner_split(M, world)
        r0, r1 = rank * own, min(M, (rank + 1) * own)
        acc = every[0].numpy()[r0:r1].copy()
        for r in range(1, world):
            acc = (acc + every[r].numpy()[r0:r1]).astype(np.float32)
        acc = (acc + f(mine[p + "fc2.bias"])).astype(np.float32)
        pad = np.zeros((own, cfg.width), np.float32)
        pad[:r1 - r0] = acc
        rows = [torch.zeros((own, cfg.width)) for _ in range(world)]
        dist.all_gather(rows, torch.from_numpy(pad))
        out = torch.cat(rows).numpy()[:M]
        ref = (O.mul_mat(O.pack_weights(f(full[p + "fc2.weight"])), h) + f(full[p + "fc2.bias"])).astype(np.float32)
        results[rank] = (bool(ok_cols), float(np.abs(out - ref).max() / np.abs(ref).max()), out.tobytes())
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_follow_the_row_and_column_splits():
    world = 2
    with mp.get_context("spawn").Manager() as manager:
        results = manager.dict()
        mp.start_processes(_worker, args=(world, _port(), results), nprocs=world, join=True, start_method="spawn")
        same = results[0][2] == results[1][2]
        for r in range(world):
            ok_cols, rel, _ = results[r]
            assert ok_cols, r
            assert rel <= 1e-5, (r, rel)
        assert same
