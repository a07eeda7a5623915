"""Qwen3-Omni thinker attention-prologue linears on B200 as Q8_0 contractions.

The thinker's attention prologue (implementations/qwen3_omni/amd/thinker_model.py:106-148,
thinker_attention.py:108-143; transformers' Qwen3OmniMoeThinkerTextAttention) projects
x [T, 2048] to q [T, 4096] and k / v [T, 512] (GQA 32 / 4 heads of 128), and o_proj
maps the attended rows [T, 4096] back to [T, 2048]; lm_head is [151936, 2048]. With the
linears in Q8_0 (the 48-layer stack workload) each projection is ggml_mul_mat(Q8_0 W,
x): the activations are quantized to Q8_0 per row and the per-block integer dots are
rescaled in ggml's generic order — for up to 32 rows at a time the split-K decode
GEMV, or for lm_head the tile GEMV (the readout kernel without its argmax), both
bit-exact; the tcgen05 GEMM on fp16(q * d) operands for prefill-sized calls.

``Q8LinearB200`` is a drop-in for an ``nn.Linear``; ``install_thinker_attention_linears``
swaps the plain ``nn.Linear`` projections (q_proj, k_proj, v_proj, qkv_proj, o_proj and
lm_head) of a thinker module for it and returns how many it replaced. Tensor-parallel
linears (which own a collective) are not plain ``nn.Linear`` and are left alone.
``qknorm_rope`` is the next step of the prologue in one launch: per-head QK RMSNorm, the
prepared MRoPE rotation and the KV-cache write, with the bf16 rounding points of the
reference's fused op (qknorm_rope.py:9-53).
"""
from __future__ import annotations

import torch
from torch import nn

from .linear import BlockLinear

PROJECTIONS = ("q_proj", "k_proj", "v_proj", "qkv_proj", "o_proj", "lm_head")
GEMM_ROWS = 4096  # rows per tcgen05 GEMM call (the handle's activation buffer)
TILE_ROWS = 16384  # outputs from which the decode rows use the tile GEMV (lm_head) instead of the split GEMV


class Q8LinearB200(nn.Module):
    """y = ggml_mul_mat(Q8_0(W), x) (+ bias) with the sm_100a kernels; x [..., K] in any float dtype,
    y in x's dtype. Weights are packed once (fp16 pre-round, Q8_0) from the given linear."""

    def __init__(self, linear: nn.Linear, *, rounding: str = "arm", gemm_rows: int = GEMM_ROWS):
        super().__init__()
        w = linear.weight.detach()
        if w.device.type != "cuda":
            raise ValueError("the B200 linear needs a CUDA weight")
        self.in_features, self.out_features = int(w.shape[1]), int(w.shape[0])
        if self.in_features % 32:
            raise ValueError("Q8_0 needs an input width that is a multiple of 32")
        bias = linear.bias.detach().float() if linear.bias is not None else None
        self.lin = BlockLinear(w.float().contiguous(), fmt="q8_0", bias=bias)
        if self.out_features >= TILE_ROWS:  # vocabulary-sized: decode rows run on the tile GEMV
            self.lin.prepare_readout()
        self.rounding = rounding
        self.gemm_rows = int(gemm_rows)
        self._gemm_ready = False

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features)
        if x2.dtype != torch.float32 or not x2.is_contiguous():
            x2 = x2.float().contiguous()
        rows = x2.shape[0]
        out = torch.empty((rows, self.out_features), dtype=torch.float32, device=x2.device)
        if rows >= 64 and not self._gemm_ready:
            self.lin.prepare_gemm(self.gemm_rows)
            self._gemm_ready = True
        for r0 in range(0, rows, self.gemm_rows if rows >= 64 else max(rows, 1)):
            r1 = min(rows, r0 + self.gemm_rows)
            self.lin(x2[r0:r1], out=out[r0:r1], rounding=self.rounding)
        return out.to(x.dtype).reshape(*lead, self.out_features)

    def close(self) -> None:
        self.lin.close()


def qknorm_rope(q: torch.Tensor, k: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                cos: torch.Tensor, sin: torch.Tensor, *, eps: float = 1e-6, round_products: bool = True,
                v: torch.Tensor | None = None, k_cache: torch.Tensor | None = None,
                v_cache: torch.Tensor | None = None, slots: torch.Tensor | None = None,
                status: torch.Tensor | None = None):
    """The thinker's QK RMSNorm + prepared MRoPE (+ KV write) in one launch (the reference's
    fused op, qknorm_rope.py:9-53). q [T, Hq, 128], k / v [T, Hkv, 128], weights [128], cos / sin
    [T, 128], all bf16; or q / k / v fp32 (the projection's output, rounded to bf16 as they are
    read). Returns (q_out [T, Hq, 128], k_cache); without a cache the normed, roped k comes back
    as a fresh [T, Hkv, 128] tensor. slots [T] int64 picks each token's cache row."""
    from . import native
    from .linear import _stream
    from .native import check, error_buffer
    lib = native.require_capability()
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    f32 = q.dtype == torch.float32
    rows = (q, k) + ((v,) if v is not None else ())
    for t in rows + (q_weight, k_weight, cos, sin):
        want = torch.float32 if f32 and any(t is r for r in rows) else torch.bfloat16
        if t.dtype != want or not t.is_cuda or t.stride(-1) != 1:
            raise ValueError("CUDA tensors with unit last stride expected: q / k / v all bf16 or all fp32, "
                             "weights and cos / sin bf16")
    out_q = torch.empty((T, Hq, D), dtype=torch.bfloat16, device=q.device)
    if k_cache is None:
        k_cache = torch.empty((T, Hkv, D), dtype=torch.bfloat16, device=q.device)
    slot_stride = k_cache.stride(0)
    if v is not None and (v_cache is None or v_cache.stride(0) != slot_stride):
        raise ValueError("v needs a v_cache laid out like k_cache")
    if slots is not None and (slots.dtype != torch.int64 or slots.shape != (T,)):
        raise ValueError("slots must be int64 [T]")
    st = status if status is not None else torch.zeros(1, dtype=torch.int32, device=q.device)
    e = error_buffer()
    op = lib.mstar_b200_qknorm_rope_f32 if f32 else lib.mstar_b200_qknorm_rope
    check(op(
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1),
        v.data_ptr() if v is not None else None, v.stride(0) if v is not None else 0,
        v.stride(1) if v is not None else 0, q_weight.data_ptr(), k_weight.data_ptr(), cos.data_ptr(), cos.stride(0),
        sin.data_ptr(), sin.stride(0), T, Hq, Hkv, D, float(eps), int(round_products), out_q.data_ptr(),
        k_cache.data_ptr(), v_cache.data_ptr() if v is not None else None, slot_stride,
        slots.data_ptr() if slots is not None else None, k_cache.shape[0], st.data_ptr(), _stream(q.device),
        e, len(e)), e, "B200 QK norm / RoPE")
    return out_q, k_cache


def thinker_linear_targets(module: nn.Module) -> list[tuple[nn.Module, str, nn.Linear]]:
    """(parent, attribute, linear) for every plain nn.Linear projection under module."""
    found = []
    for parent in module.modules():
        for name in PROJECTIONS:
            child = getattr(parent, name, None)
            if type(child) is nn.Linear and child.in_features % 32 == 0:
                found.append((parent, name, child))
    return found


def install_thinker_attention_linears(module: nn.Module, *, rounding: str = "arm", lm_head: bool = True,
                                      gemm_rows: int = GEMM_ROWS) -> int:
    """Replace the thinker's plain nn.Linear projections with Q8LinearB200; returns the count."""
    count = 0
    for parent, name, linear in thinker_linear_targets(module):
        if name == "lm_head" and not lm_head:
            continue
        setattr(parent, name, Q8LinearB200(linear, rounding=rounding, gemm_rows=gemm_rows))
        count += 1
    return count
