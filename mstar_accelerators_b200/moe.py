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
