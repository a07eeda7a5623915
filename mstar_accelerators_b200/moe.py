"""Qwen3-Omni thinker MoE on B200 (torch-facing wrappers of the C ABI).

``ThinkerMoEB200`` is the experts backend of the reference's
``SmallTokenThinkerMoE`` (implementations/qwen3_omni/amd/thinker_moe.py:104-188):
``backend(hidden_states, topk_weights, topk_ids)`` with the layer's w1
[E, 2I, H] / w2 [E, H, I] prepared once, for every token count up to
``max_tokens`` (the reference handles only 1, 2, 4, 8 rows and defers the rest).
``route`` mirrors ``ConsistentBF16Router.forward`` (router_consistency.py:54-62).
"""
from __future__ import annotations

import torch

from . import native
from .linear import _stream
from .native import check, error_buffer


def route(x: torch.Tensor, router_weight: torch.Tensor, top_k: int = 8, renormalize: bool = True,
          logits: torch.Tensor | None = None):
    """bf16 x [T, H], router weight [E, H] -> (topk weights fp32 [T, k], topk ids int32 [T, k])."""
    lib = native.require_capability()
    if x.dtype != torch.bfloat16 or router_weight.dtype != torch.bfloat16:
        raise ValueError("the router takes bf16 activations and weights")
    x = x.reshape(-1, x.shape[-1]).contiguous()
    w = router_weight.contiguous()
    T, H = x.shape
    E = w.shape[0]
    weights = torch.empty((T, top_k), dtype=torch.float32, device=x.device)
    ids = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
    if logits is None:
        logits = torch.empty((T, E), dtype=torch.float32, device=x.device)
    e = error_buffer()
    check(lib.mstar_b200_moe_route(x.data_ptr(), T, H, w.data_ptr(), E, top_k, int(renormalize), logits.data_ptr(),
                                   weights.data_ptr(), ids.data_ptr(), _stream(x.device), e, len(e)),
          e, "B200 MoE router")
    return weights, ids


class ThinkerMoEB200:
    """One MoE layer's experts on the current device (bf16 or Q8_0 weights)."""

    def __init__(self, w1: torch.Tensor, w2: torch.Tensor, *, fmt: str = "bf16", top_k: int = 8,
                 max_tokens: int = 4096, intermediate: int | None = None, hidden: int | None = None,
                 rounding: str = "arm"):
        self.lib = native.require_capability()
        self.fmt, self.top_k, self.max_tokens, self.rounding = fmt, top_k, max_tokens, rounding
        if fmt == "bf16":
            if w1.dtype != torch.bfloat16 or w2.dtype != torch.bfloat16:
                raise ValueError("bf16 experts need bf16 w1/w2")
            E, two_i, H = w1.shape
            I = two_i // 2
        elif fmt == "q8_0":
            if intermediate is None or hidden is None:
                raise ValueError("Q8_0 experts need the intermediate and hidden sizes")
            E, I, H = w1.shape[0], intermediate, hidden
        else:
            raise ValueError("experts are bf16 or q8_0")
        self.E, self.I, self.H = E, I, H
        w1 = w1.contiguous()
        w2 = w2.contiguous()
        e = error_buffer()
        torch.cuda.current_stream(w1.device).synchronize()
        handle = self.lib.mstar_b200_moe_create(native.FORMATS[fmt], w1.data_ptr(), w1.numel() * w1.element_size(),
                                                w2.data_ptr(), w2.numel() * w2.element_size(), E, I, H, top_k,
                                                max_tokens, e, len(e))
        if not handle:
            raise native.NativeError("B200 MoE preparation: " + e.value.decode(errors="replace"))
        self.handle = handle
        self.status = torch.zeros(1, dtype=torch.int32, device=w1.device)

    def __call__(self, hidden_states: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        x = hidden_states.reshape(-1, self.H)
        if x.dtype != torch.bfloat16:
            raise ValueError("MoE activations are bf16")
        x = x.contiguous()
        w = topk_weights.to(torch.float32).contiguous()
        ids = topk_ids.to(torch.int32).contiguous()
        if out is None:
            out = torch.empty_like(x)
        e = error_buffer()
        check(self.lib.mstar_b200_moe_run(self.handle, x.data_ptr(), x.shape[0], w.data_ptr(), ids.data_ptr(),
                                          out.data_ptr(), self.status.data_ptr(), native.ROUNDING[self.rounding],
                                          _stream(x.device), e, len(e)), e, "B200 MoE")
        return out.view(hidden_states.shape)

    def run_experts(self, hidden_states: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor, *,
                    expert0: int, experts_total: int, y: torch.Tensor, row_base: int, inv: torch.Tensor) -> None:
        """The held experts [expert0, expert0 + E) of experts_total, without the combine: each held
        (token, slot) pair's routed row goes to y (bf16 [rows, H]) at row_base + its permuted
        position and inv[token * top_k + slot] (int32) names that row, or -1 (another rank's expert)."""
        x = hidden_states.reshape(-1, self.H)
        if x.dtype != torch.bfloat16 or y.dtype != torch.bfloat16 or inv.dtype != torch.int32:
            raise ValueError("bf16 activations and outputs, int32 row indices expected")
        x = x.contiguous()
        w = topk_weights.to(torch.float32).contiguous()
        ids = topk_ids.to(torch.int32).contiguous()
        if inv.numel() < x.shape[0] * self.top_k or not inv.is_contiguous() or not y.is_contiguous():
            raise ValueError("inv needs tokens * top_k contiguous entries")
        e = error_buffer()
        check(self.lib.mstar_b200_moe_run_experts(self.handle, x.data_ptr(), x.shape[0], w.data_ptr(), ids.data_ptr(),
                                                  int(expert0), int(experts_total), y.data_ptr(), y.numel() // self.H,
                                                  int(row_base), inv.data_ptr(), self.status.data_ptr(),
                                                  native.ROUNDING[self.rounding], _stream(x.device), e, len(e)),
              e, "B200 MoE experts")

    def close(self):
        if getattr(self, "handle", None):
            e = error_buffer()
            check(self.lib.mstar_b200_moe_close(self.handle, e, len(e)), e, "B200 MoE close")
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ThinkerExpertsBackend:
    """``experts_backend`` of one thinker MoE layer: the role SmallTokenThinkerMoE
    plays on gfx942 (thinker_moe.py:104-188, installed by select_expert_kernels,
    qwen3_omni/amd/moe.py:6-22), for every token count. Called like the
    reference backends, ``backend(hidden_states, w1, w2, topk_weights, topk_ids,
    *, skip_invalid=False)``, with the layer's own gate_up_proj [E, 2I, H] and
    down_proj [E, H, I]; the B200 layout is prepared once from those tensors.
    Calls with more than ``max_tokens`` rows run in row chunks (tokens are
    independent). Ids outside [0, E) add nothing, with or without skip_invalid.
    """

    def __init__(self, w1: torch.Tensor, w2: torch.Tensor, *, top_k: int = 8, max_tokens: int = 2048):
        self._weights = (w1.data_ptr(), w2.data_ptr())
        self.max_tokens = max_tokens
        self.moe = ThinkerMoEB200(w1.detach(), w2.detach(), fmt="bf16", top_k=top_k, max_tokens=max_tokens)

    def __call__(self, hidden_states, w1, w2, topk_weights, topk_ids, *, skip_invalid=False):
        if (w1.data_ptr(), w2.data_ptr()) != self._weights:
            raise ValueError("this experts backend was prepared for other expert weights")
        x = hidden_states.reshape(-1, hidden_states.shape[-1])
        if x.shape[0] <= self.max_tokens:
            return self.moe(x, topk_weights, topk_ids).view(hidden_states.shape)
        out = torch.empty_like(x)
        for t0 in range(0, x.shape[0], self.max_tokens):
            t1 = min(t0 + self.max_tokens, x.shape[0])
            self.moe(x[t0:t1], topk_weights[t0:t1], topk_ids[t0:t1], out=out[t0:t1])
        return out.view(hidden_states.shape)

    def close(self):
        self.moe.close()


def install_thinker_experts(module, *, experts: int = 128, intermediate: int = 768, hidden: int = 2048,
                            top_k: int = 8, max_tokens: int = 2048) -> int:
    """Give every thinker MoE layer under ``module`` (a child with an
    ``experts_backend`` and ``experts.gate_up_proj`` [E, 2I, H] / ``experts.down_proj``
    [E, H, I] of the thinker geometry, MoEProblem(128, 768, 2048, 8)) a
    ThinkerExpertsBackend; returns how many were installed."""
    count = 0
    for child in module.modules():
        if not hasattr(child, "experts_backend"):
            continue
        bank = getattr(child, "experts", None)
        w1, w2 = getattr(bank, "gate_up_proj", None), getattr(bank, "down_proj", None)
        if w1 is None or w2 is None:
            continue
        if tuple(w1.shape) != (experts, 2 * intermediate, hidden) or tuple(w2.shape) != (experts, hidden, intermediate):
            continue
        if w1.dtype != torch.bfloat16 or w2.dtype != torch.bfloat16 or w1.device.type != "cuda":
            continue
        child.experts_backend = ThinkerExpertsBackend(w1, w2, top_k=top_k, max_tokens=max_tokens)
        count += 1
    return count
