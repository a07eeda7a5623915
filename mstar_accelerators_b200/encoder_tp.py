"""Tensor-parallel Whisper encoder over the GPUs of one node (one process per
GPU, torch.distributed for rendezvous and the peer mappings of symmetric
memory; the data path is this library's kernels over NVLink peer memory).

Layout (the reference's TP pattern, accelerations/whisper/cpu_tp2/
decoder_all_reduce.py:64-90 and weights.py:26-67, extended to the whole
encoder block):
  * the convolution stems run replicated (1-2 % of the work);
  * QKV is column-parallel by heads (an uneven split when the heads do not
    divide, e.g. 20 heads over 8 ranks), attention runs on the local heads;
  * out_proj is row-parallel (its K = the local heads' columns); rows are split
    into W owner ranges (whole 32-row groups);
  * the row-parallel GEMM's epilogue stores each partial tile straight into
    the owner's receive slot over NVLink and raises the owner's arrival counter
    of those 32 rows (the reduction fused into the GEMM: the transfer runs under
    the GEMM's MMAs, and no barrier separates the GEMM from the reduction);
    each owner waits per 32-row group for every rank's arrivals, sums the slots
    in rank order, adds the bias once, then the residual (x = x + (sum + b)),
    LayerNorms and Q8_0-stages the new rows straight into every rank's staged
    operand (the all-gather of the next column-parallel GEMM), and a barrier
    publishes them;
  * fc1 is column-parallel (bias + GELU + Q8_0-staged output local), fc2
    row-parallel with the same fused reduction, whose staging applies the next
    layer's first LayerNorm;
  * the final LayerNorm runs on each owner's rows; ``forward`` all-gathers the
    rows (NCCL) so every rank returns the full encoder states.
Two earlier forms stay selectable (``reduction``): "pull" (each rank's GEMM writes
its partial locally, a barrier, then each owner pulls the W partials of its rows
with peer loads) and "multicast" (after the barrier the owner reads each row's
sum over all ranks with NVSwitch multimem loads that add in the switch). Where the
platform binds the staged operand to a multicast object and there are at least
four ranks, the staged rows are written once through the multicast address.
Q8_0 blocks lie along K and every shard boundary is a multiple of 32, so each
rank's weights are exactly sub-blocks of the single-GPU weights.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import native
from .encoder import EncoderConfig, conv_k_padded
from .linear import BlockLinear, _stream, layer_norm, stage_conv, stage_rows
from .native import check, error_buffer


MULTICAST_FROM_RANKS = 4   # ranks from which the automatic choice reduces through NVSwitch multicast


def head_split(heads: int, world: int) -> list[int]:
    """Heads per rank: as even as possible, the first ranks take the remainder."""
    return [heads // world + (1 if r < heads % world else 0) for r in range(world)]


def owner_split(rows: int, world: int) -> int:
    """Rows per owner range (the last range may be shorter)."""
    return -(-rows // world)


def shard_weights(weights: dict, cfg: EncoderConfig, world: int, rank: int) -> dict:
    """This rank's slices of one encoder's weights (fp32 tensors, reference names)."""
    if cfg.ffn % (32 * world):
        raise ValueError("the FFN width must split into whole Q8_0 blocks")
    counts = head_split(cfg.heads, world)
    if counts[rank] == 0:
        raise ValueError("more ranks than heads")
    hd = cfg.width // cfg.heads
    c0, c1 = sum(counts[:rank]) * hd, sum(counts[:rank + 1]) * hd
    f = cfg.ffn // world
    f0, f1 = rank * f, (rank + 1) * f
    out = {k: v for k, v in weights.items() if not k.startswith("encoder.layers.")}
    for i in range(cfg.layers):
        p = f"encoder.layers.{i}."
        for n in ("self_attn_layer_norm", "final_layer_norm"):
            out[p + n + ".weight"] = weights[p + n + ".weight"]
            out[p + n + ".bias"] = weights[p + n + ".bias"]
        for n in "qkv":
            out[p + f"self_attn.{n}_proj.weight"] = weights[p + f"self_attn.{n}_proj.weight"][c0:c1]
            b = weights.get(p + f"self_attn.{n}_proj.bias")
            out[p + f"self_attn.{n}_proj.bias"] = (b if b is not None else torch.zeros(cfg.width))[c0:c1]
        out[p + "self_attn.out_proj.weight"] = weights[p + "self_attn.out_proj.weight"][:, c0:c1]
        out[p + "self_attn.out_proj.bias"] = weights[p + "self_attn.out_proj.bias"]
        out[p + "fc1.weight"] = weights[p + "fc1.weight"][f0:f1]
        out[p + "fc1.bias"] = weights[p + "fc1.bias"][f0:f1]
        out[p + "fc2.weight"] = weights[p + "fc2.weight"][:, f0:f1]
        out[p + "fc2.bias"] = weights[p + "fc2.bias"]
    return out


class WhisperEncoderTP:
    """This rank's part of a tensor-parallel encoder for up to ``max_batch`` utterances."""

    def __init__(self, weights: dict, cfg: EncoderConfig, *, max_batch: int = 1, group=None, rounding: str = "arm",
                 reduction: str = "push"):
        """reduction: "push" (the default: partial tiles stored into the owners' receive slots
        by the GEMM epilogue, per-32-row arrival counters, no barrier before the reduction);
        "pull" (local partials, a peer barrier, owners pull with peer loads); "multicast"
        (local partials, a barrier, owners read the sums with NVSwitch multimem loads; raises
        ValueError where the platform has no multicast object). Measured on 2 B200s
        (large-v3 shape, batch 16, before the push form): pull 32.3 ms per forward, multicast
        39.8 ms."""
        import torch.distributed._symmetric_memory as symm
        self.lib = native.require_capability()
        self.group = group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.cfg, self.max_batch, self.rounding = cfg, max_batch, rounding
        dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        W = {k: v.detach().to(device=dev, dtype=torch.float32).contiguous()
             for k, v in shard_weights(weights, cfg, self.world, self.rank).items()}
        d = cfg.width
        self.heads_local = head_split(cfg.heads, self.world)[self.rank]
        self.d_local = self.heads_local * (d // cfg.heads)
        self.f_local = cfg.ffn // self.world
        self.k1, self.k2 = conv_k_padded(cfg.mels), conv_k_padded(d)

        def conv(name, channels, kp):
            w = W[name + ".weight"].reshape(d, 3 * channels)
            if kp > 3 * channels:
                w = torch.cat([w, torch.zeros((d, kp - 3 * channels), device=dev)], dim=1)
            lin = BlockLinear(w.contiguous(), bias=W[name + ".bias"])
            lin.prepare_gemm(64)
            return lin

        self.conv1 = conv("encoder.conv1", cfg.mels, self.k1)
        self.conv2 = conv("encoder.conv2", d, self.k2)
        self.positions = W["encoder.embed_positions.weight"]
        self.layers = []
        for i in range(cfg.layers):
            p = f"encoder.layers.{i}."
            L = {
                "ln1": (W[p + "self_attn_layer_norm.weight"], W[p + "self_attn_layer_norm.bias"], cfg.eps),
                "ln2": (W[p + "final_layer_norm.weight"], W[p + "final_layer_norm.bias"], cfg.eps),
                "qkv": BlockLinear(torch.cat([W[p + f"self_attn.{n}_proj.weight"] for n in "qkv"]),
                                   bias=torch.cat([W[p + f"self_attn.{n}_proj.bias"] for n in "qkv"])),
                "out": BlockLinear(W[p + "self_attn.out_proj.weight"].contiguous()),
                "out_b": W[p + "self_attn.out_proj.bias"],
                "fc1": BlockLinear(W[p + "fc1.weight"], bias=W[p + "fc1.bias"]),
                "fc2": BlockLinear(W[p + "fc2.weight"].contiguous()),
                "fc2_b": W[p + "fc2.bias"],
            }
            for k in ("qkv", "out", "fc1", "fc2"):
                L[k].prepare_gemm(64)
            self.layers.append(L)
        self.final_norm = (W["encoder.layer_norm.weight"], W["encoder.layer_norm.bias"], cfg.eps)

        # buffers
        T, P = cfg.positions, cfg.padded_keys
        M = max_batch * T
        if reduction not in ("push", "pull", "multicast"):
            raise ValueError("reduction must be 'push', 'pull' or 'multicast'")
        self.reduction = reduction
        self.owner_rows_max = owner_split(M, self.world)
        # pushed partials: owner ranges of whole 32-row groups (a group never spans two owners)
        self.push_rows_max = -(-self.owner_rows_max // 32) * 32
        self.staged = torch.empty(max(2 * M * self.k1, M * self.k2), dtype=torch.float16, device=dev)
        self.conv_out = torch.empty((2 * M, d), dtype=torch.float32, device=dev)
        self.x_full = torch.empty((M, d), dtype=torch.float32, device=dev)
        self.x_own = torch.empty((self.push_rows_max, d), dtype=torch.float32, device=dev)
        self.qkv16 = torch.zeros((max_batch, P, 3 * self.d_local), dtype=torch.float16, device=dev)
        self.att_staged = torch.empty((M, self.d_local), dtype=torch.float16, device=dev)
        self.hidden16 = torch.empty((M, self.f_local), dtype=torch.float16, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
        # symmetric (peer-mapped) buffers: partial products, the all-gathered staged LayerNorm rows, flags
        pg = group if group is not None else dist.group.WORLD
        if hasattr(symm, "is_symm_mem_enabled_for_group") and not symm.is_symm_mem_enabled_for_group(pg.group_name):
            symm.enable_symm_mem_for_group(pg.group_name)
        # partials: [M][d] local (pull / multicast) or the receive slots [world][push_rows][d] (push)
        part_rows = self.world * self.push_rows_max if reduction == "push" else M
        self.part = symm.empty(part_rows * d, dtype=torch.float32, device=dev)
        self.ln_staged = symm.empty(M * d, dtype=torch.float16, device=dev)
        self.flags = symm.empty(self.world, dtype=torch.int32, device=dev)
        self.arrivals = symm.empty(self.push_rows_max // 32 + 1, dtype=torch.int32, device=dev)
        self.flags.zero_()
        self.arrivals.zero_()
        torch.cuda.synchronize()
        pg = group if group is not None else dist.group.WORLD
        self._h = [symm.rendezvous(t, pg) for t in (self.part, self.ln_staged, self.flags, self.arrivals)]
        def ptrs(h):
            return torch.tensor(h.buffer_ptrs, dtype=torch.int64, device=dev)
        self.part_ptrs, self.staged_ptrs, self.flag_ptrs, self.arrival_ptrs = (ptrs(h) for h in self._h)
        mc = [int(getattr(h, "multicast_ptr", 0) or 0) for h in self._h[:2]]
        # every rank must take the same path: an all-reduce of what each rank can do
        avail = torch.tensor([1 if self.world > 1 and mc[0] else 0, 1 if self.world > 1 and mc[1] else 0],
                             dtype=torch.int32, device=dev)
        dist.all_reduce(avail, op=dist.ReduceOp.MIN, group=group)
        if reduction == "multicast" and not bool(avail[0].item() and avail[1].item()):
            raise ValueError("the symmetric buffers have no multicast object on this platform")
        self.multicast = reduction == "multicast"
        # the staged rows of the pushed form go through the multicast address from four ranks up
        self.mc_staged_rows = reduction == "push" and bool(avail[1].item()) and self.world >= MULTICAST_FROM_RANKS
        self.mc_part, self.mc_staged = mc
        dist.barrier(group=group)

    # ------------------------------------------------------------------ pieces
    def _barrier(self):
        e = error_buffer()
        check(self.lib.mstar_b200_tp_barrier(self.flag_ptrs.data_ptr(), self.flags.data_ptr(), self.rank, self.world,
                                             self.counter.data_ptr(), self.status.data_ptr(), _stream(self.device),
                                             e, len(e)), e, "B200 TP barrier")

    def _partial(self, lin: BlockLinear, staged: torch.Tensor, owner_rows: int):
        """Row-parallel partial product: pushed into the owners' receive slots, or [M][width]
        fp32 into this rank's peer-visible buffer followed by the barrier the pull needs."""
        if self.reduction == "push":
            lin.gemm_push(staged, recv_ptrs=self.part_ptrs, flag_ptrs=self.arrival_ptrs, world=self.world,
                          rank=self.rank, owner_rows=owner_rows, status=self.status)
            return
        lin.gemm(staged, out=self.part[:staged.shape[0] * lin.rows].view(-1, lin.rows), bias=False,
                 rounding=self.rounding, status=self.status)
        self._barrier()

    def _reduce(self, owner_rows: int, owned: int, bias: torch.Tensor, norm):
        lw, lb, eps = (norm[0].data_ptr(), norm[1].data_ptr(), float(norm[2])) if norm else (None, None, 0.0)
        e = error_buffer()
        if self.reduction == "push":
            staged = (None, self.mc_staged) if self.mc_staged_rows else (self.staged_ptrs.data_ptr(), None)
            check(self.lib.mstar_b200_tp_reduce_recv(self.part.data_ptr(), self.arrivals.data_ptr(), self.world,
                                                     owned, owner_rows, self.cfg.width, bias.data_ptr(),
                                                     self.x_own.data_ptr(), lw, lb, eps,
                                                     staged[0] if norm else None, staged[1] if norm else None,
                                                     self.rank * owner_rows, native.ROUNDING[self.rounding],
                                                     self.status.data_ptr(), _stream(self.device), e, len(e)),
                  e, "B200 TP reduce")
            return
        if self.multicast:
            check(self.lib.mstar_b200_tp_reduce_multicast(self.mc_part, self.world, owned, self.cfg.width,
                                                          bias.data_ptr(), self.x_own.data_ptr(), lw, lb, eps,
                                                          self.mc_staged if norm else None, self.rank * owner_rows,
                                                          native.ROUNDING[self.rounding], self.status.data_ptr(),
                                                          _stream(self.device), e, len(e)), e, "B200 TP reduce")
            return
        check(self.lib.mstar_b200_tp_reduce(self.part_ptrs.data_ptr(), self.world, owned, self.cfg.width,
                                            bias.data_ptr(), self.x_own.data_ptr(), lw, lb, eps,
                                            self.staged_ptrs.data_ptr() if norm else None, self.rank * owner_rows,
                                            native.ROUNDING[self.rounding], self.status.data_ptr(),
                                            _stream(self.device), e, len(e)), e, "B200 TP reduce")

    # ------------------------------------------------------------------ forward
    # Buffer hazards between ranks. Pull / multicast: the barrier after each partial
    # GEMM (every partial is complete, and every rank has finished the GEMMs that read
    # ln_staged, before any owner reads partials or writes staged rows). Push: an owner
    # finishes a 32-row group only after every rank's arrivals for it, and a rank's
    # pushing GEMM starts after its own GEMMs that read ln_staged, so no staged row is
    # overwritten while a rank still reads it. Both: the barrier after each reduction
    # (the staged rows are complete before the next column-parallel GEMM reads them, and
    # every owner has consumed the partials and cleared its counters before any rank
    # writes partials again).
    def forward(self, mel: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """mel fp32 [batch, mels, 2 * positions] (the same on every rank) ->
        encoder_states fp32 [batch, positions, width] on every rank (into ``out`` when given)."""
        cfg, r = self.cfg, self.rounding
        B = mel.shape[0]
        if B > self.max_batch or mel.shape[1:] != (cfg.mels, 2 * cfg.positions):
            raise ValueError("mel must be fp32 [batch <= max_batch, mels, 2 * positions]")
        d, T, P, H = cfg.width, cfg.positions, cfg.padded_keys, self.heads_local
        M = B * T
        own_rows = owner_split(M, self.world)
        if self.reduction == "push":
            own_rows = -(-own_rows // 32) * 32
        row0 = self.rank * own_rows
        owned = max(0, min(M, row0 + own_rows) - row0)
        st = self.status
        # replicated stems: every rank has the full x and stages LayerNorm 1 itself
        a = stage_conv(mel, time_major=False, stride=1, k_padded=self.k1, rounding=r,
                       out=self.staged[:2 * M * self.k1].view(2 * M, self.k1), status=st)
        self.conv1.gemm(a, out=self.conv_out[:2 * M], gelu="tanh", rounding=r, status=st)
        a = stage_conv(self.conv_out[:2 * M].view(B, 2 * T, d), time_major=True, stride=2, k_padded=self.k2,
                       rounding=r, out=self.staged[:M * self.k2].view(M, self.k2), status=st)
        x = self.x_full[:M]
        self.conv2.gemm(a, out=x, gelu="tanh", residual=self.positions, residual_period=T, rounding=r, status=st)
        self.x_own[:owned].copy_(x[row0:row0 + owned])
        ln_staged = self.ln_staged[:M * d].view(M, d)
        stage_rows(x, norm=self.layers[0]["ln1"], rounding=r, out=ln_staged, status=st)
        qkv = self.qkv16[:B]
        hd = d // cfg.heads
        for i, L in enumerate(self.layers):
            L["qkv"].gemm(ln_staged, out=qkv, out_format="f16", segments=(T, P), rounding=r, status=st)
            dl = self.d_local
            q = qkv[:, :T, :dl].unflatten(-1, (H, hd)).transpose(1, 2)
            k = qkv[:, :, dl:2 * dl].unflatten(-1, (H, hd)).transpose(1, 2)
            v = qkv[:, :, 2 * dl:].unflatten(-1, (H, hd)).transpose(1, 2)
            att = F.scaled_dot_product_attention(q, k, v, scale=hd ** -0.5).transpose(1, 2).reshape(M, dl)
            sa = stage_rows(att, rounding=r, out=self.att_staged[:M], status=st)
            self._partial(L["out"], sa, own_rows)
            self._reduce(own_rows, owned, L["out_b"], L["ln2"])
            self._barrier()
            h = L["fc1"].gemm(ln_staged, out=self.hidden16[:M], out_format="staged", gelu="tanh", rounding=r,
                              status=st)
            self._partial(L["fc2"], h, own_rows)
            nxt = self.layers[i + 1]["ln1"] if i + 1 < len(self.layers) else None
            self._reduce(own_rows, owned, L["fc2_b"], nxt)
            self._barrier()
        w, b, eps = self.final_norm
        states = torch.zeros((own_rows * self.world, d), dtype=torch.float32, device=self.device)
        mine = torch.zeros((own_rows, d), dtype=torch.float32, device=self.device)
        if owned:
            layer_norm(self.x_own[:owned], w, b, eps, out=mine[:owned])
        dist.all_gather_into_tensor(states, mine, group=self.group)
        if out is not None:
            out.view(M, d).copy_(states[:M])
            return out
        return states[:M].view(B, T, d)

    __call__ = forward

    def launches_per_forward(self) -> int:
        """This library's kernel launches in one forward: the replicated stems (two stagings,
        two GEMMs), the first LayerNorm staging, per layer two column-parallel GEMMs, the
        attention staging, two row-parallel partial GEMMs, two reductions and two peer
        barriers (four with the pulled forms), then the final LayerNorm. The attention, the
        row copy and the closing all-gather are torch / NCCL."""
        return 4 + 1 + (9 if self.reduction == "push" else 11) * len(self.layers) + 1

    def close(self):
        for lin in [self.conv1, self.conv2] + [L[k] for L in self.layers for k in ("qkv", "out", "fc1", "fc2")]:
            lin.close()
