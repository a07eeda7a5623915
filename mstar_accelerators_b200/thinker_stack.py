"""Qwen3-Omni thinker decoder stack on B200 with Q8_0 linears (the 48-layer workload).

The layer is the reference's thinker layer (implementations/qwen3_omni/amd/
thinker_model.py:106-148, transformers' Qwen3OmniMoeThinkerTextDecoderLayer):
    h = RMSNorm(x); q, k, v = Wq h, Wk h, Wv h
    q, k = QK-RMSNorm + RoPE(q, k); K/V appended to the cache
    x = x + Wo attention(q, K, V)              (GQA, causal)
    h = RMSNorm(x); x = x + MoE(h)             (router top-8, SwiGLU experts, slot-order combine)
and the stack ends with the final RMSNorm and the lm_head with greedy argmax.
Every linear is this library's block-quantized contraction: the fused QKV and o_proj
as Q8_0 (split-K GEMV for <= 32 rows, bit-exact with ggml's generic order; the
tcgen05 GEMM for prefill rows), the experts as the grouped tcgen05 MoE kernels
(Q8_0 or bf16 experts), lm_head as the one-launch tile readout (GEMV + argmax).
QK-RMSNorm + RoPE + the KV write are one launch (mstar_b200_qknorm_rope). RMSNorm,
the embedding lookup and attention (torch SDPA over the bf16 cache, GQA) are torch,
as the reference leaves them to its runtime. Text-only positions: the MRoPE sections
all take the same position, so the prepared cos / sin rows are the plain rotary ones
(theta 1e6). bf16 residual stream, as transformers runs the layer.

One process, one GPU (tensor / expert parallelism 1): the weights of the 48 Q8_0
layers (~31 GB, ~60 GB with the experts' fp16 GEMM operands) fit one B200.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import native
from .linear import BlockLinear, _stream, pack, stage_heads
from .moe import ThinkerMoEB200, route
from .native import check, error_buffer
from .thinker import qknorm_rope


@dataclass(frozen=True)
class ThinkerStackConfig:
    hidden: int = 2048
    layers: int = 48
    q_heads: int = 32
    kv_heads: int = 4
    head_dim: int = 128
    experts: int = 128
    top_k: int = 8
    moe_intermediate: int = 768
    vocab: int = 151936
    rope_theta: float = 1e6
    eps: float = 1e-6


def layer_weights(cfg: ThinkerStackConfig, layer: int, seed: int = 1, device="cuda") -> dict:
    """Seeded random weights of one layer, bf16: matrices N(0, 0.02), norm weights 1 + N(0, 0.02)."""
    g = torch.Generator(device=device).manual_seed(seed * 1000 + layer)
    H, D, E, I = cfg.hidden, cfg.head_dim, cfg.experts, cfg.moe_intermediate

    def n(*shape, one=False):
        t = torch.randn(shape, generator=g, device=device) * 0.02
        return (t + 1.0 if one else t).to(torch.bfloat16)

    return {"ln1": n(H, one=True), "q": n(cfg.q_heads * D, H), "k": n(cfg.kv_heads * D, H), "v": n(cfg.kv_heads * D, H),
            "q_norm": n(D, one=True), "k_norm": n(D, one=True), "o": n(H, cfg.q_heads * D), "ln2": n(H, one=True),
            "router": n(E, H), "w1": n(E, 2 * I, H), "w2": n(E, H, I)}


def head_weights(cfg: ThinkerStackConfig, seed: int = 1, device="cuda") -> dict:
    g = torch.Generator(device=device).manual_seed(seed * 1000 + 999)
    return {"embed": (torch.randn((cfg.vocab, cfg.hidden), generator=g, device=device) * 0.02).to(torch.bfloat16),
            "norm": (1.0 + torch.randn(cfg.hidden, generator=g, device=device) * 0.02).to(torch.bfloat16),
            "lm_head": (torch.randn((cfg.vocab, cfg.hidden), generator=g, device=device) * 0.02).to(torch.bfloat16)}


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, *, f32: bool = False) -> torch.Tensor:
    """transformers' Qwen3OmniMoeThinkerTextRMSNorm (fp32 normalisation, bf16 before the weight)
    in one launch (mstar_b200_rms_norm): bf16 x [rows, width] -> bf16 rows, or with f32 the
    same values as fp32 (the Q8_0 linears' input)."""
    lib = native.require_capability()
    x = x.contiguous()
    rows, width = x.shape
    out = torch.empty_like(x)
    out32 = torch.empty((rows, width), dtype=torch.float32, device=x.device) if f32 else None
    e = error_buffer()
    check(lib.mstar_b200_rms_norm(x.data_ptr(), width, rows, width, w.contiguous().data_ptr(), float(eps),
                                  out.data_ptr(), width, out32.data_ptr() if f32 else None, width,
                                  _stream(x.device), e, len(e)), e, "B200 RMSNorm")
    return out32 if f32 else out


def residual_add(x: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """x + v.to(bf16) in bf16 (torch's residual add of a projection computed in fp32) in one
    launch (mstar_b200_residual_add_bf16): bf16 x, fp32 v of the same shape -> new bf16 tensor."""
    lib = native.require_capability()
    x, v = x.contiguous(), v.contiguous()
    out = torch.empty_like(x)
    e = error_buffer()
    check(lib.mstar_b200_residual_add_bf16(x.data_ptr(), v.data_ptr(), x.numel(), out.data_ptr(), _stream(x.device),
                                           e, len(e)), e, "B200 residual add")
    return out


def rotary(positions: torch.Tensor, cfg: ThinkerStackConfig):
    """Prepared cos / sin rows [T, head_dim] (bf16) of the plain rotary embedding."""
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, cfg.head_dim, 2, device=positions.device, dtype=torch.float32)
                                    / cfg.head_dim))
    f = positions.float()[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


class ThinkerStackB200:
    """The thinker stack for up to ``max_seqs`` sequences of ``max_len`` positions on one GPU."""

    def __init__(self, cfg: ThinkerStackConfig = ThinkerStackConfig(), *, max_seqs: int = 32, max_len: int = 1152,
                 seed: int = 1, experts: str = "q8_0", gemm_rows: int = 4096, weights=None, device="cuda"):
        self.cfg, self.max_seqs, self.max_len = cfg, max_seqs, max_len
        self.device = torch.device(device)
        self.gemm_rows = gemm_rows
        self.experts_fmt = experts
        D = cfg.head_dim
        # heads and experts held by this process: [q0, q0 + q_heads), [k0, k0 + kv_heads), [e0, e0 + local_experts)
        self.q0, self.q_heads, self.k0, self.kv_heads, self.e0, self.local_experts = self._shard_plan()
        self.layers = []
        for i in range(cfg.layers):
            w = weights(i) if weights is not None else layer_weights(cfg, i, seed, self.device)
            self.layers.append(self._build_layer(w))
            del w
        hw = head_weights(cfg, seed, self.device)
        self.embed, self.final_norm = hw["embed"], hw["norm"]
        self.lm_head = BlockLinear(hw["lm_head"].float().contiguous(), fmt="q8_0")
        self.lm_head.prepare_readout()
        slots = max_seqs * max_len
        self.k_cache = [torch.zeros((slots, self.kv_heads, D), dtype=torch.bfloat16, device=self.device)
                        for _ in range(cfg.layers)]
        self.v_cache = [torch.zeros_like(c) for c in self.k_cache]
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.length = 0
        self.graph = None
        self._graph_rows = 0

    def _shard_plan(self):
        """(q0, q_heads, k0, kv_heads, e0, experts) held here: everything on one GPU."""
        c = self.cfg
        return 0, c.q_heads, 0, c.kv_heads, 0, c.experts

    def _build_layer(self, w: dict) -> dict:
        """One layer's device state from its full bf16 weights: the held heads' rows of the fused QKV,
        the held heads' columns of o_proj, the held experts."""
        cfg, D, H, I = self.cfg, self.cfg.head_dim, self.cfg.hidden, self.cfg.moe_intermediate
        q = w["q"][self.q0 * D:(self.q0 + self.q_heads) * D]
        k = w["k"][self.k0 * D:(self.k0 + self.kv_heads) * D]
        v = w["v"][self.k0 * D:(self.k0 + self.kv_heads) * D]
        qkv = BlockLinear(torch.cat([q, k, v]).float().contiguous(), fmt="q8_0")
        o = BlockLinear(w["o"][:, self.q0 * D:(self.q0 + self.q_heads) * D].float().contiguous(), fmt="q8_0")
        qkv.prepare_gemm(self.gemm_rows)
        o.prepare_gemm(self.gemm_rows)
        e0, en = self.e0, self.local_experts
        if self.experts_fmt == "q8_0":
            b1 = pack(w["w1"][e0:e0 + en].float().reshape(-1, H), "q8_0", preround=False).reshape(en, 2 * I, -1)
            b2 = pack(w["w2"][e0:e0 + en].float().reshape(-1, I), "q8_0", preround=False).reshape(en, H, -1)
            moe = ThinkerMoEB200(b1, b2, fmt="q8_0", top_k=cfg.top_k, max_tokens=self.gemm_rows, intermediate=I,
                                 hidden=H)
            del b1, b2
        else:
            moe = ThinkerMoEB200(w["w1"][e0:e0 + en].contiguous(), w["w2"][e0:e0 + en].contiguous(), fmt="bf16",
                                 top_k=cfg.top_k, max_tokens=self.gemm_rows)
        return {"ln1": w["ln1"], "ln2": w["ln2"], "q_norm": w["q_norm"], "k_norm": w["k_norm"],
                "router": w["router"].contiguous(), "qkv": qkv, "o": o, "moe": moe}

    # ------------------------------------------------------------------ pieces
    def _linear(self, lin: BlockLinear, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        x = x.float().contiguous()
        if out is None:
            out = torch.empty((x.shape[0], lin.rows), dtype=torch.float32, device=x.device)
        step = self.gemm_rows if x.shape[0] >= 64 else max(x.shape[0], 1)
        for r0 in range(0, x.shape[0], step):
            lin(x[r0:r0 + step], out=out[r0:r0 + step])
        return out

    def _moe(self, L, h: torch.Tensor) -> torch.Tensor:
        if h.shape[0] <= self.gemm_rows:   # one chunk: the layer's output as it comes
            w, ids = route(h, L["router"], top_k=self.cfg.top_k)
            return L["moe"](h, w, ids)
        out = torch.empty_like(h)
        for r0 in range(0, h.shape[0], self.gemm_rows):
            part = h[r0:r0 + self.gemm_rows]
            w, ids = route(part, L["router"], top_k=self.cfg.top_k)
            out[r0:r0 + self.gemm_rows] = L["moe"](part, w, ids)
        return out

    def _embed(self, tokens: torch.Tensor) -> torch.Tensor:
        return self.embed[tokens.reshape(-1)]

    def _o_proj(self, L, att: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """o_proj (fp32) of the attention output: decode rows [T, heads * D] go through the linear
        as they are; the prefill's [S, heads, n, D] is staged for the GEMM in one pass (the same
        bytes the linear stages from the transposed fp32 rows, without writing those out)."""
        lin = L["o"]
        if att.ndim == 2:
            return self._linear(lin, att, out=out)
        S, Hq, n, D = att.shape
        T = S * n
        if out is None:
            out = torch.empty((T, lin.rows), dtype=torch.float32, device=att.device)
        if T < 64 or (T % self.gemm_rows and T % self.gemm_rows < 64):
            # a short (last) chunk takes the linear's GEMV path on the fp32 rows, as _linear does
            return self._linear(lin, att.transpose(1, 2).reshape(T, Hq * D), out=out)
        staged = stage_heads(att, status=self.status)
        for r0 in range(0, T, self.gemm_rows):
            r1 = min(T, r0 + self.gemm_rows)
            lin.gemm(staged[r0:r1], out=out[r0:r1], bias=False, status=self.status)
        return out

    def _attention_out(self, L, att: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        """x + o_proj(att) in bf16."""
        return residual_add(x, self._o_proj(L, att))

    def _moe_residual(self, L, h: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        """x + MoE(h) in bf16."""
        return x + self._moe(L, h)

    def _positions(self, S: int, n: int, pos: torch.Tensor):
        """What every layer of a step shares, computed once per step: the rotary tables of the
        positions, each new row's KV-cache slot and (decode) the additive mask over the cache."""
        cos, sin = rotary(pos, self.cfg)
        slots = torch.arange(S, device=pos.device).repeat_interleave(n) * self.max_len + pos
        mask = None
        if n == 1:
            mask = torch.where(torch.arange(self.max_len, device=pos.device)[None, :] <= pos[:, None], 0.0,
                               float("-inf")).to(torch.bfloat16).view(S, 1, 1, self.max_len)
        return cos, sin, slots, mask

    def _layer(self, i: int, x: torch.Tensor, S: int, n: int, start, shared) -> torch.Tensor:
        """x [S * n, H] bf16: n new positions of each of S sequences; shared: _positions() of
        their positions. The attention output reaches _attention_out as [S * n, heads * D] rows
        (decode) or as [S, heads, n, D] (prefill). Prefill (start == 0, n > 1): causal attention over the n positions.
        Decode (n == 1): every query attends to the cache up to its own position through a
        fixed-length view of the whole cache and an additive mask, so the step's shapes never
        change (one CUDA graph replays it)."""
        cfg, L = self.cfg, self.layers[i]
        D, Hq, Hk = cfg.head_dim, self.q_heads, self.kv_heads
        T = S * n
        cos, sin, slots, mask = shared
        h = rms_norm(x, L["ln1"], cfg.eps, f32=True)
        qkv = self._linear(L["qkv"], h)   # fp32; the prologue rounds q / k / v to bf16 as it reads them
        q = qkv[:, :Hq * D].view(T, Hq, D)
        k = qkv[:, Hq * D:(Hq + Hk) * D].view(T, Hk, D)
        v = qkv[:, (Hq + Hk) * D:].view(T, Hk, D)
        q, _ = qknorm_rope(q, k, L["q_norm"], L["k_norm"], cos, sin, eps=cfg.eps, v=v, k_cache=self.k_cache[i],
                           v_cache=self.v_cache[i], slots=slots, status=self.status)
        if n == 1:
            kk = self.k_cache[i].view(self.max_seqs, self.max_len, Hk, D)[:S].transpose(1, 2)
            vv = self.v_cache[i].view(self.max_seqs, self.max_len, Hk, D)[:S].transpose(1, 2)
            # the query heads of one KV head as that head's query rows: [S, Hk, Hq / Hk, D]
            qq = q.view(S, Hk, Hq // Hk, D)
            att = F.scaled_dot_product_attention(qq, kk, vv, attn_mask=mask, scale=D ** -0.5)
            att = att.reshape(T, Hq * D)
        else:
            ctx = start + n
            kk = self.k_cache[i].view(self.max_seqs, self.max_len, Hk, D)[:S, :ctx].transpose(1, 2)
            vv = self.v_cache[i].view(self.max_seqs, self.max_len, Hk, D)[:S, :ctx].transpose(1, 2)
            qq = q.view(S, n, Hq, D).transpose(1, 2)
            if start == 0:
                att = F.scaled_dot_product_attention(qq, kk, vv, is_causal=True, scale=D ** -0.5, enable_gqa=True)
            else:
                m = torch.ones((n, ctx), dtype=torch.bool, device=x.device).tril(ctx - n)
                att = F.scaled_dot_product_attention(qq, kk, vv, attn_mask=m, scale=D ** -0.5, enable_gqa=True)
        x = self._attention_out(L, att, x)
        h = rms_norm(x, L["ln2"], cfg.eps)
        return self._moe_residual(L, h, x)

    def _readout(self, last: torch.Tensor):
        h = rms_norm(last, self.final_norm, self.cfg.eps, f32=True)
        logits = torch.empty((h.shape[0], self.cfg.vocab), dtype=torch.float32, device=h.device)
        tokens = torch.empty(h.shape[0], dtype=torch.int64, device=h.device)
        self.lm_head.readout(h, logits=logits, token=tokens, status=self.status)
        return logits, tokens

    # ------------------------------------------------------------------ walks
    def prefill(self, tokens: torch.Tensor):
        """tokens [S, n] -> (logits [S, vocab] of each last position, greedy next tokens [S])."""
        S, n = tokens.shape
        if S > self.max_seqs or n > self.max_len:
            raise ValueError("prompt exceeds the prepared capacity")
        x = self._embed(tokens)
        pos = torch.arange(n, device=self.device).repeat(S)
        shared = self._positions(S, n, pos)
        for i in range(self.cfg.layers):
            x = self._layer(i, x, S, n, 0, shared)
        self.length, self.seqs = n, S
        self.graph = None
        return self._readout(x.view(S, n, -1)[:, -1])

    def _decode_step(self, tokens: torch.Tensor, pos: torch.Tensor):
        x = self._embed(tokens)
        shared = self._positions(tokens.shape[0], 1, pos)
        for i in range(self.cfg.layers):
            x = self._layer(i, x, tokens.shape[0], 1, None, shared)
        return self._readout(x)

    def decode(self, tokens: torch.Tensor, *, graph: bool = False):
        """tokens [S] at the next position of every sequence -> (logits [S, vocab], next tokens [S]).
        graph=True replays the whole step (48 layers and the readout) as one captured CUDA graph,
        captured on the first such call after a prefill."""
        S = tokens.shape[0]
        if self.length >= self.max_len:
            raise ValueError("sequence capacity exhausted")
        if not graph:
            pos = torch.full((S,), self.length, dtype=torch.int64, device=self.device)
            out = self._decode_step(tokens.reshape(-1), pos)
            self.length += 1
            return out
        if getattr(self, "graph", None) is None or self._graph_rows != S:
            self._tok = torch.zeros(S, dtype=torch.int64, device=self.device)
            self._pos = torch.zeros(S, dtype=torch.int64, device=self.device)
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):   # warm-up outside capture (handles, attention plans)
                self._pos.fill_(self.length)
                self._decode_step(self._tok, self._pos)
            torch.cuda.current_stream().wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._graph_out = self._decode_step(self._tok, self._pos)
            self._graph_rows = S
        self._tok.copy_(tokens.reshape(-1))
        self._pos.fill_(self.length)
        self.graph.replay()
        self.length += 1
        return self._graph_out

    def close(self) -> None:
        self.graph = None
        for L in self.layers:
            L["qkv"].close()
            L["o"].close()
            L["moe"].close()
        self.lm_head.close()
