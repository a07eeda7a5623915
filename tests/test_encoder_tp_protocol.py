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


# --------------------------------------------------------------------------------------
# The pushed reduction (linear_gemm_push + tp_reduce_recv) with two gloo ranks: a model of
# the CTA-pair GEMM epilogue's walk (256 x 256 pair tiles; per CTA 4 TMEM lane quarters of
# 32 rows x 4 column groups of two 32-column blocks; one arrival per warp and tile on the
# owner's counter of its 32 rows) delivers every rank's partial product into the owners'
# receive slots; the owners check the arrival counts the kernel waits for
# (world * 4 * ceil(N / 256) per 32-row group, none elsewhere), that every element of
# every slot was written exactly once and nothing outside the owned rows, and that the
# rank-order sum of the slots equals the pulled reduction bit for bit.

def _push_walk(M, N, owner_rows):
    """(row_base, rows, nc, owner) stores and (owner, group) arrivals of one rank's epilogue."""
    stores, arrivals = [], []
    for m0 in range(0, M, 256):
        for n0 in range(0, N, 256):
            for cta in range(2):
                for q in range(4):
                    row_base = m0 + cta * 128 + 32 * q
                    for cg in range(4):
                        if row_base >= M:
                            continue
                        owner = row_base // owner_rows
                        for c in (2 * cg, 2 * cg + 1):
                            nc = n0 + 32 * c
                            if nc < N:
                                stores.append((row_base, min(32, M - row_base), nc, owner))
                        arrivals.append((owner, (row_base - owner * owner_rows) // 32))
    return stores, arrivals


def _push_worker(rank, world, port, results, M, N):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mstar_accelerators_b200.encoder_tp import owner_split
        from oracle import oracle as O
        K = 64 * world
        rng = np.random.default_rng(11)
        w = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
        x = rng.standard_normal((M, K)).astype(np.float32)
        ks = K // world
        partial = O.mul_mat(O.pack_weights(np.ascontiguousarray(w[:, rank * ks:(rank + 1) * ks])),
                            np.ascontiguousarray(x[:, rank * ks:(rank + 1) * ks]))
        owner_rows = -(-owner_split(M, world) // 32) * 32
        assert owner_rows * world >= M
        # this rank's outgoing slot rows for every owner, with a write count per element
        out = np.zeros((world, owner_rows, N), np.float32)
        writes = np.zeros((world, owner_rows, N), np.int32)
        counts = np.zeros((world, owner_rows // 32), np.int32)
        stores, arrivals = _push_walk(M, N, owner_rows)
        for row_base, rows, nc, owner in stores:
            lr = row_base - owner * owner_rows
            assert 0 <= owner < world and lr + rows <= owner_rows
            out[owner, lr:lr + rows, nc:nc + 32] = partial[row_base:row_base + rows, nc:nc + 32]
            writes[owner, lr:lr + rows, nc:nc + 32] += 1
        for owner, g in arrivals:
            counts[owner, g] += 1
        # the stores and arrivals reach the owners (the NVLink stores of the GEMM epilogue)
        every = [torch.zeros((world, owner_rows, N)) for _ in range(world)]
        dist.all_gather(every, torch.from_numpy(out))
        every_w = [torch.zeros((world, owner_rows, N), dtype=torch.int32) for _ in range(world)]
        dist.all_gather(every_w, torch.from_numpy(writes))
        every_c = [torch.zeros((world, owner_rows // 32), dtype=torch.int32) for _ in range(world)]
        dist.all_gather(every_c, torch.from_numpy(counts))
        recv = np.stack([every[s][rank].numpy() for s in range(world)])          # [slot][owner_rows][N]
        wcount = np.stack([every_w[s][rank].numpy() for s in range(world)])
        arrived = sum(every_c[s][rank].numpy() for s in range(world))
        row0 = rank * owner_rows
        owned = max(0, min(M, row0 + owner_rows) - row0)
        expect = world * 4 * -(-N // 256)
        groups = -(-owned // 32)
        ok_arrivals = bool((arrived[:groups] == expect).all() and (arrived[groups:] == 0).all())
        ok_writes = bool((wcount[:, :owned] == 1).all() and (wcount[:, owned:] == 0).all())
        acc = recv[0, :owned].copy()
        for s in range(1, world):
            acc = (acc + recv[s, :owned]).astype(np.float32)
        # the pulled reduction: every rank's whole partial, rank order
        full = [torch.zeros((M, N)) for _ in range(world)]
        dist.all_gather(full, torch.from_numpy(partial))
        pulled = full[0].numpy()[row0:row0 + owned].copy()
        for s in range(1, world):
            pulled = (pulled + full[s].numpy()[row0:row0 + owned]).astype(np.float32)
        results[rank] = (ok_arrivals, ok_writes, bool(np.array_equal(acc, pulled)), owned)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M,N", [(3000, 384), (7500, 384), (3000, 1280), (1500, 160)])
def test_pushed_partials_reach_every_owner_once(M, N):
    """M = utterances x 1500 (ragged owner ranges, a last pair tile half past M); N = the tiny
    and large-v3 widths and one below a whole 256-column tile."""
    world = 2
    with mp.get_context("spawn").Manager() as manager:
        results = manager.dict()
        mp.start_processes(_push_worker, args=(world, _port(), results, M, N), nprocs=world, join=True,
                           start_method="spawn")
        assert sum(results[r][3] for r in range(world)) == M
        for r in range(world):
            ok_arrivals, ok_writes, same, _ = results[r]
            assert ok_arrivals and ok_writes and same, (r, results[r])


@pytest.mark.parametrize("world", [1, 3, 4, 8])
def test_push_arrival_counts_at_the_large_encoder_shape(world):
    """The arrival count each owner's 32-row groups wait for, at the Whisper-large-v3 shape
    (24,000 rows, width 1280) over 1..8 ranks: every rank's epilogue walk gives every owned
    group exactly 4 * ceil(1280 / 256) = 20 arrivals and no group outside the owned rows any."""
    from mstar_accelerators_b200.encoder_tp import owner_split
    M, N = 24000, 1280
    owner_rows = -(-owner_split(M, world) // 32) * 32
    _, arrivals = _push_walk(M, N, owner_rows)
    counts = np.zeros((world, owner_rows // 32), np.int64)
    for owner, g in arrivals:
        counts[owner, g] += 1
    for o in range(world):
        owned = max(0, min(M, (o + 1) * owner_rows) - o * owner_rows)
        groups = -(-owned // 32)
        assert (counts[o, :groups] == 20).all() and (counts[o, groups:] == 0).all(), o
