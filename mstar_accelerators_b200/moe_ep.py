"""Expert parallelism for the thinker MoE layer over torch.distributed (NCCL).

Each of the W ranks holds experts [r*E/W, (r+1)*E/W) (16 of 128 at W = 8) and
the full routing of its own tokens. One forward:

  1. dispatch: the (token, slot) pairs are ordered by owning rank (stable, so
     slot order inside a rank is kept; on B200 one counting-sort CTA and one
     row-copy launch, mstar_b200_moe_dispatch); send counts and an invalid-id flag are
     exchanged with one all_to_all and read on the host in the call's one
     synchronisation (the split sizes of the next collectives; an invalid id on
     any rank makes every rank raise there); token rows (bf16) and the (local
     expert id, routing weight) pairs travel with two all_to_all_single;
  2. every rank runs its local experts on the received pairs as a top-1 MoE
     whose routing weight is the pair's weight, so each returned row is
     y_s = bf16((mid . w_down) * w_s) exactly as in down_vector_reduce
     (thinker_moe.py:51-83);
  3. combine: the rows go back with the reversed splits and every token sums
     its slots in slot order in fp32, then rounds to bf16 (moe_sum_reduce,
     thinker_moe.py:75-81; mstar_b200_moe_combine).

Results are therefore bit-identical to the single-GPU layer on the same
inputs. Every rank takes the same collective steps in the same order, also
with zero pairs for a peer. The local expert computation is a callable so the
host logic is testable on CPU with gloo.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

LocalExperts = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]
Combine = Callable[[torch.Tensor, torch.Tensor, int], torch.Tensor]
# (x, topk_weights, topk_ids, top_k, experts, ranks) -> meta int64 [2W], rows [P, H],
# pairs int32 [P, 2], inverse int32 [P] (the send-side plan; mstar_b200_moe_dispatch)
Dispatch = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, int, int, int],
                    tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]]


def torch_dispatch(x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor, top_k: int, experts: int,
                   ranks: int):
    """The send-side plan in torch operations (the host-logic tests on CPU ranks):
    pairs grouped by owning rank clamp(floor(id / per), 0, W - 1), pair order
    inside a rank; meta [W][2] = (pairs for rank d, 1 if any id is outside
    [0, experts)); rows = x[pair / k], pairs = (local id, weight bits) and inverse
    = each pair's send position."""
    per = experts // ranks
    ids = topk_ids.reshape(-1).long()
    bad = ((ids < 0) | (ids >= experts)).any().to(torch.int64).reshape(1)
    dest = torch.div(ids, per, rounding_mode="floor").clamp_(0, ranks - 1)
    order = torch.sort(dest, stable=True).indices          # send position -> pair index
    counts = torch.bincount(dest, minlength=ranks)
    meta = torch.stack([counts, bad.expand(ranks)], dim=1).reshape(-1).contiguous()
    rows = x[order // top_k].contiguous()
    local_ids = (ids[order] - dest[order] * per).to(torch.int32)
    weights = topk_weights.reshape(-1)[order].to(torch.float32)
    pairs = torch.stack([local_ids, weights.view(torch.int32)], dim=1).contiguous()
    inverse = torch.empty_like(order)
    inverse[order] = torch.arange(order.numel(), device=order.device)
    return meta, rows, pairs, inverse.to(torch.int32)


def owned_experts(experts: int, world: int, rank: int) -> range:
    if experts % world:
        raise ValueError("experts must divide evenly over the ranks")
    per = experts // world
    return range(rank * per, (rank + 1) * per)


class ExpertParallelMoE:
    """One thinker MoE layer sharded by experts over ``group``."""

    def __init__(self, local_experts: LocalExperts, combine: Combine, *, experts: int, top_k: int, group=None,
                 dispatch: Dispatch = torch_dispatch):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.experts, self.top_k = experts, top_k
        self.owned = owned_experts(experts, self.world, self.rank)
        self.local = local_experts
        self.combine = combine
        self.dispatch = dispatch

    @classmethod
    def b200(cls, w1: torch.Tensor, w2: torch.Tensor, *, experts: int, top_k: int = 8, group=None,
             capacity: int = 65536) -> "ExpertParallelMoE":
        """The B200 layer: w1 [E, 2I, H] / w2 [E, H, I] bf16 (the full layer, on this
        rank's device); this rank keeps its experts. ``capacity`` bounds the pairs
        one local launch takes (larger receptions run in chunks)."""
        from . import native
        from .moe import ThinkerMoEB200
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        own = owned_experts(experts, world, rank)
        local = ThinkerMoEB200(w1[own.start:own.stop].contiguous(), w2[own.start:own.stop].contiguous(), fmt="bf16",
                               top_k=1, max_tokens=capacity)
        lib = native.require_capability()
        return cls(b200_local_experts(local, capacity), b200_combine(lib), experts=experts, top_k=top_k, group=group,
                   dispatch=b200_dispatch(lib))

    def _exchange(self, send: torch.Tensor, send_counts: list[int], recv_counts: list[int]) -> torch.Tensor:
        recv = send.new_empty((sum(recv_counts),) + tuple(send.shape[1:]))
        dist.all_to_all_single(recv, send, output_split_sizes=recv_counts, input_split_sizes=send_counts,
                               group=self.group)
        return recv

    def __call__(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
        """x [T, H] bf16, topk_weights [T, k] fp32, topk_ids [T, k] -> [T, H] bf16."""
        k = self.top_k
        meta, rows, pairs, inverse = self.dispatch(x, topk_weights, topk_ids, k, self.experts, self.world)
        # one exchange of (count, invalid-id flag) per peer and one host synchronisation: the split
        # sizes of the next collectives, and an invalid id on any rank stops every rank here
        recv_meta = torch.empty_like(meta)
        dist.all_to_all_single(recv_meta, meta, group=self.group)
        host = torch.stack([meta, recv_meta]).cpu().view(2, self.world, 2)
        if int(host[1, :, 1].max()) != 0:
            raise ValueError("expert id outside [0, experts)")
        send_counts, recv_counts = host[0, :, 0].tolist(), host[1, :, 0].tolist()
        r_rows = self._exchange(rows, send_counts, recv_counts)
        r_pairs = self._exchange(pairs, send_counts, recv_counts)  # (local expert id, weight bits)
        r_ids = r_pairs[:, 0].contiguous()
        r_w = r_pairs[:, 1].contiguous().view(torch.float32)
        y_local = self.local(r_rows, r_w, r_ids)               # [received, H] bf16, one row per pair
        y_back = self._exchange(y_local.contiguous(), recv_counts, send_counts)
        return self.combine(y_back, inverse, k)


def b200_local_experts(moe, capacity: int) -> LocalExperts:
    """Adapter: a top-1 ThinkerMoEB200 holding this rank's experts, run over the
    received pairs (local expert id, routing weight) in chunks of ``capacity``."""
    def run(rows, weights, ids):
        out = rows.new_empty((rows.shape[0], rows.shape[1]))
        for p0 in range(0, rows.shape[0], capacity):
            p1 = min(p0 + capacity, rows.shape[0])
            moe(rows[p0:p1], weights[p0:p1].view(-1, 1), ids[p0:p1].view(-1, 1), out=out[p0:p1])
        return out
    return run


def b200_dispatch(lib) -> Dispatch:
    """The send-side plan on the device (mstar_b200_moe_dispatch): one counting-sort
    CTA and one row-copy launch, no host synchronisation."""
    from .linear import _stream
    from .native import check, error_buffer

    def run(x, topk_weights, topk_ids, top_k, experts, ranks):
        T, H = x.shape
        P = T * top_k
        dev = x.device
        ids = topk_ids.reshape(-1)
        if ids.dtype != torch.int32:  # ids outside int32 stay outside [0, experts)
            ids = ids.clamp(-1, experts).to(torch.int32)
        ids = ids.contiguous()
        w = topk_weights.reshape(-1).to(torch.float32).contiguous()
        xc = x.contiguous()
        meta = torch.empty(2 * ranks, dtype=torch.int64, device=dev)
        rows = torch.empty((P, H), dtype=torch.bfloat16, device=dev)
        pairs = torch.empty((P, 2), dtype=torch.int32, device=dev)
        inverse = torch.empty(P, dtype=torch.int32, device=dev)
        e = error_buffer()
        ptr = (lambda t: t.data_ptr() if t.numel() else None)
        check(lib.mstar_b200_moe_dispatch(ptr(xc), T, H, ptr(w), ptr(ids), top_k, experts, ranks, meta.data_ptr(),
                                          ptr(rows), ptr(pairs), ptr(inverse), _stream(dev), e, len(e)), e,
              "B200 MoE dispatch")
        return meta, rows, pairs, inverse
    return run


def b200_combine(lib) -> Combine:
    from .linear import _stream
    from .native import check, error_buffer

    def run(y, rows, top_k):
        T = rows.numel() // top_k
        out = torch.empty((T, y.shape[1]), dtype=torch.bfloat16, device=rows.device)
        if T == 0:  # a rank that routed no tokens this step: nothing to sum
            return out
        e = error_buffer()
        check(lib.mstar_b200_moe_combine(y.data_ptr() if y.numel() else rows.data_ptr(), y.shape[0],
                                         rows.contiguous().data_ptr(), T, top_k, y.shape[1], out.data_ptr(),
                                         _stream(rows.device), e, len(e)), e, "B200 MoE combine")
        return out
    return run
