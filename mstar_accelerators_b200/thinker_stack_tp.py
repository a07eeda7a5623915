"""The thinker stack with attention tensor-parallel and the MoE expert-parallel over
the GPUs of one node (one process per GPU; torch.distributed for rendezvous and the
peer mappings of symmetric memory; the data path is this library's kernels over
NVLink peer memory, no NCCL in a step).

Layout of one layer on W ranks (the reference's thinker layer,
implementations/qwen3_omni/amd/thinker_model.py:106-148):
  * the bf16 residual stream x [T, hidden] is replicated: every rank holds it in a
    peer-visible buffer, and the owner of a row (rows split into W ranges) writes
    each new version of it into every rank's copy;
  * the fused QKV is column-parallel by heads: rank r holds query heads
    [r Hq/W, (r+1) Hq/W) and the KV heads those query heads read (GQA groups of
    Hq/Hkv); with more ranks than KV heads a KV head is computed on every rank of
    its group (replicated x2 at W = 8 for 32 / 4 heads). The QK-norm / RoPE / KV
    write and attention run on the held heads only, over a KV cache of the held
    heads;
  * o_proj is row-parallel (K = the held heads' 128-wide columns): the partial
    product goes to this rank's peer-visible buffer, a bounded peer barrier, then
    mstar_b200_thinker_reduce (owners sum the W partials in rank order and store
    bf16(x + bf16(sum)) into every rank's x), a second barrier;
  * the MoE is expert-parallel: E/W experts per rank. Every rank routes all T rows
    (identical inputs, identical ids), runs its own experts' (token, slot) pairs
    into its peer-visible expert-output rows (mstar_b200_moe_run_experts), a
    barrier, then mstar_b200_thinker_combine (owners read each slot's row from the
    rank holding its expert, sum in slot order, store bf16(x + bf16(sum)) into
    every rank's x), a barrier. The expert rows and the slot order are those of one
    GPU, so the MoE half of the layer is bit-identical to the single-GPU stack;
    o_proj's rank-order sum of partial folds is not (one GPU folds all of K).
  * the final RMSNorm and lm_head readout run on every rank (replicated), so every
    rank returns the same logits and tokens.
Per layer: two row exchanges (o_proj, MoE) and four barriers; bytes on NVLink per
rank and exchange: about (W-1)/W of the owned rows' partials (fp32) or slot rows
(bf16) in, and the owned new rows (bf16) to W-1 peers out.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import native
from .linear import _stream
from .moe import route
from .native import check, error_buffer
from .thinker_stack import ThinkerStackB200, ThinkerStackConfig


def shard_plan(cfg: ThinkerStackConfig, world: int, rank: int):
    """(q0, q_heads, k0, kv_heads, e0, experts) held by ``rank`` of ``world``."""
    if cfg.q_heads % world or cfg.experts % world or cfg.q_heads % cfg.kv_heads:
        raise ValueError("query heads and experts must split evenly over the ranks")
    group = cfg.q_heads // cfg.kv_heads
    qn = cfg.q_heads // world
    q0 = rank * qn
    if qn % group == 0:
        k0, kn = q0 // group, qn // group
    elif group % qn == 0:
        k0, kn = q0 // group, 1
    else:
        raise ValueError("a rank's query heads must cover whole GQA groups or lie inside one")
    en = cfg.experts // world
    return q0, qn, k0, kn, rank * en, en


def owner_rows(rows: int, world: int, rank: int) -> tuple[int, int]:
    """(row0, owned) of ``rank``'s owner range; ranges of ceil(rows / world) rows."""
    per = -(-rows // world)
    row0 = min(rows, rank * per)
    return row0, max(0, min(rows, row0 + per) - row0)


class ThinkerStackTP(ThinkerStackB200):
    """This rank's part of the thinker stack for up to ``max_seqs`` sequences of ``max_len``
    positions; ``max_tokens`` bounds the rows of one prefill (default max_seqs * max_len)."""

    def __init__(self, cfg: ThinkerStackConfig = ThinkerStackConfig(), *, group=None, max_seqs: int = 32,
                 max_len: int = 1152, max_tokens: int | None = None, **kwargs):
        import torch.distributed._symmetric_memory as symm
        self.lib = native.require_capability()
        self.group = group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        dev = torch.device("cuda", torch.cuda.current_device())
        super().__init__(cfg, max_seqs=max_seqs, max_len=max_len, device=dev, **kwargs)
        H, k = cfg.hidden, cfg.top_k
        self.max_tokens = int(max_tokens or max_seqs * max_len)
        rows = self.max_tokens
        self.ids = torch.zeros(rows * k, dtype=torch.int32, device=dev)
        self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
        pg = group if group is not None else dist.group.WORLD
        if hasattr(symm, "is_symm_mem_enabled_for_group") and not symm.is_symm_mem_enabled_for_group(pg.group_name):
            symm.enable_symm_mem_for_group(pg.group_name)
        self.part = symm.empty(rows * H, dtype=torch.float32, device=dev)
        self.x = symm.empty(rows * H, dtype=torch.bfloat16, device=dev)
        self.y = symm.empty(rows * k * H, dtype=torch.bfloat16, device=dev)
        self.inv = symm.empty(rows * k, dtype=torch.int32, device=dev)
        self.flags = symm.empty(self.world, dtype=torch.int32, device=dev)
        self.flags.zero_()
        torch.cuda.synchronize()
        self._h = [symm.rendezvous(t, pg) for t in (self.part, self.x, self.y, self.inv, self.flags)]

        def ptrs(h):
            return torch.tensor(h.buffer_ptrs, dtype=torch.int64, device=dev)

        self.part_ptrs, self.x_ptrs, self.y_ptrs, self.inv_ptrs, self.flag_ptrs = (ptrs(h) for h in self._h)
        dist.barrier(group=group)

    def _shard_plan(self):
        return shard_plan(self.cfg, self.world, self.rank)

    # ------------------------------------------------------------------ exchanges
    def _barrier(self):
        e = error_buffer()
        check(self.lib.mstar_b200_tp_barrier(self.flag_ptrs.data_ptr(), self.flags.data_ptr(), self.rank, self.world,
                                             self.counter.data_ptr(), self.status.data_ptr(), _stream(self.device),
                                             e, len(e)), e, "B200 TP barrier")

    def _embed(self, tokens: torch.Tensor) -> torch.Tensor:
        tokens = tokens.reshape(-1)
        T = tokens.shape[0]
        if T > self.max_tokens:
            raise ValueError("more rows than the prepared exchange buffers hold")
        x = self.x[:T * self.cfg.hidden].view(T, self.cfg.hidden)
        torch.index_select(self.embed, 0, tokens, out=x)
        return x

    # Buffer hazards between ranks: the barrier after each partial product (or expert
    # run) comes after every rank has read x for that half-layer's RMSNorm and written
    # its partial (expert rows), so owners may read partials and overwrite x; the
    # barrier after each reduction (combine) publishes the new x before anyone reads
    # it, and comes before any rank overwrites its partial (expert) buffer again.
    def _attention_out(self, L, att: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        T, H = x.shape[0], self.cfg.hidden
        self._o_proj(L, att, out=self.part[:T * H].view(T, H))
        self._barrier()
        row0, owned = owner_rows(T, self.world, self.rank)
        e = error_buffer()
        check(self.lib.mstar_b200_thinker_reduce(self.part_ptrs.data_ptr(), self.x_ptrs.data_ptr(), self.rank,
                                                 self.world, owned, H, row0, _stream(self.device), e, len(e)),
              e, "B200 thinker reduction")
        self._barrier()
        return x

    def _moe_residual(self, L, h: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        T, H, k = h.shape[0], cfg.hidden, cfg.top_k
        for r0 in range(0, T, self.gemm_rows):
            part = h[r0:r0 + self.gemm_rows]
            n = part.shape[0]
            w, ids = route(part, L["router"], top_k=k)
            self.ids[r0 * k:(r0 + n) * k].copy_(ids.view(-1))
            L["moe"].run_experts(part, w, ids, expert0=self.e0, experts_total=cfg.experts, y=self.y,
                                 row_base=r0 * k, inv=self.inv[r0 * k:(r0 + n) * k])
        self._barrier()
        row0, owned = owner_rows(T, self.world, self.rank)
        e = error_buffer()
        check(self.lib.mstar_b200_thinker_combine(self.y_ptrs.data_ptr(), self.inv_ptrs.data_ptr(),
                                                  self.max_tokens * k, self.ids.data_ptr(), self.local_experts,
                                                  cfg.experts, k, self.x_ptrs.data_ptr(), self.rank, self.world,
                                                  owned, H, row0, self.status.data_ptr(), _stream(self.device),
                                                  e, len(e)), e, "B200 thinker combine")
        self._barrier()
        return x

    def expert_status(self) -> int:
        """OR of the held experts' status words (bit value 4: an expert id outside the table)."""
        v = 0
        for L in self.layers:
            v |= int(L["moe"].status.item())
        return v
