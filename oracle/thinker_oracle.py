"""ORACLE — test infrastructure only.

CPU restatement of the reference's fused Thinker Q/K RMSNorm + prepared MRoPE op
(implementations/qwen3_omni/amd/qknorm_rope.py:9-53) with its bf16 boundaries and no
fused multiply-add: per token and head of 128,
    x = fp32(bf16 row); r = 1 / sqrt(sum(x * x) / 128 + eps)   (fp32 steps)
    n = bf16((x * r) * w)
    rot[d] = -n[d + 64] (d < 64), n[d - 64] (d >= 64)
    a = n * cos, b = rot * sin, each rounded to bf16 when round_products
    y = bf16(a + b)
The fp32 squares are summed exactly (float64) and rounded once, so the oracle has no
summation order of its own; an implementation with another order can differ by one
bf16 step where a value lands on a rounding boundary.
"""
from __future__ import annotations

import numpy as np

from .moe_oracle import bf16


def qknorm_rope(q, k, qw, kw, cos, sin, eps=1e-6, round_products=True):
    """q [T, Hq, 128], k [T, Hkv, 128], qw / kw [128], cos / sin [T, 128] (float32 holding bf16
    values) -> (q_out, k_out), float32 holding bf16 values."""
    f32 = np.float32

    def one(x, w):
        x = np.asarray(x, np.float32)
        sq = (x * x).astype(np.float32)
        ss = sq.astype(np.float64).sum(-1, keepdims=True).astype(np.float32)
        r = (f32(1.0) / np.sqrt((ss / f32(128.0)).astype(np.float32) + f32(eps))).astype(np.float32)
        n = bf16(((x * r).astype(np.float32) * np.asarray(w, np.float32)).astype(np.float32))
        rot = np.concatenate([-n[..., 64:], n[..., :64]], axis=-1)
        c = np.asarray(cos, np.float32)[:, None, :]
        s = np.asarray(sin, np.float32)[:, None, :]
        a = (n * c).astype(np.float32)
        b = (rot * s).astype(np.float32)
        if round_products:
            a, b = bf16(a), bf16(b)
        return bf16((a + b).astype(np.float32))

    return one(q, qw), one(k, kw)
