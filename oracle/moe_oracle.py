"""ORACLE — test infrastructure only.

CPU restatement of the reference's thinker MoE semantics:
  router  ConsistentBF16Router.forward (implementations/qwen3_omni/amd/
          router_consistency.py:54-62): logits = bf16(x . Wr^T), softmax in fp32,
          top-k, w /= sum(w) when renormalising.
  experts gate_up_vector / down_vector_reduce (thinker_moe.py:17-83):
          g = bf16(x . w_gate); u = bf16(x . w_up); act = bf16(g * sigmoid(g));
          mid = bf16(act * u); y_s = bf16((mid . w_down) * w_s);
          out = bf16(sum_s fp32(y_s)) in slot order.
Dot products are accumulated in float64 and rounded once to float32 (the
reference's fp32 accumulation order is unspecified; reorder-level differences
are what the GPU tests allow). The Q8_0 variant replaces every dot with the
ggml generic-order Q8_0 mul_mat of oracle.mul_mat on the Q8_0-quantized
activation (x, then mid).
"""
from __future__ import annotations

import numpy as np

from . import oracle as O


def bf16(x) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest even), returned as float32."""
    a = np.ascontiguousarray(x, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(a), a, out).astype(np.float32)


def route(x_bf16: np.ndarray, wr_bf16: np.ndarray, top_k: int, renormalize: bool = True):
    logits = bf16((x_bf16.astype(np.float64) @ wr_bf16.astype(np.float64).T).astype(np.float32))
    m = logits.max(-1, keepdims=True)
    e = np.exp((logits - m).astype(np.float32))
    p = (e / e.sum(-1, keepdims=True)).astype(np.float32)
    ids = np.argsort(-p, axis=-1, kind="stable")[:, :top_k]
    w = np.take_along_axis(p, ids, -1)
    if renormalize:
        w = (w / w.sum(-1, keepdims=True)).astype(np.float32)
    return w.astype(np.float32), ids.astype(np.int32), p


def experts_bf16(x, w1, w2, topk_w, topk_ids):
    """x [T, H], w1 [E, 2I, H], w2 [E, H, I] (float32 holding bf16 values)."""
    T, H = x.shape
    I = w1.shape[1] // 2
    k = topk_ids.shape[1]
    out = np.zeros((T, H), np.float32)
    for t in range(T):
        acc = np.zeros(H, np.float32)
        for s in range(k):
            e = int(topk_ids[t, s])
            g = bf16((w1[e, :I].astype(np.float64) @ x[t]).astype(np.float32))
            u = bf16((w1[e, I:].astype(np.float64) @ x[t]).astype(np.float32))
            act = bf16((g * (1.0 / (1.0 + np.exp(-g.astype(np.float64))))).astype(np.float32))
            mid = bf16(act * u)
            y = (w2[e].astype(np.float64) @ mid).astype(np.float32)
            acc = (acc + bf16((y * topk_w[t, s]).astype(np.float32))).astype(np.float32)
        out[t] = bf16(acc)
    return out


def experts_q8(x, w1_blocks, w2_blocks, topk_w, topk_ids, I, H, mode="arm"):
    """Q8_0 composition: w1_blocks [E][2I][H/32*34], w2_blocks [E][H][I/32*34]."""
    T = x.shape[0]
    k = topk_ids.shape[1]
    out = np.zeros((T, H), np.float32)
    for t in range(T):
        acc = np.zeros(H, np.float32)
        for s in range(k):
            e = int(topk_ids[t, s])
            gu = O.mul_mat(w1_blocks[e], x[t:t + 1], "q8_0", mode=mode)[0]
            g, u = bf16(gu[:I]), bf16(gu[I:])
            act = bf16((g * (1.0 / (1.0 + np.exp(-g.astype(np.float64))))).astype(np.float32))
            mid = bf16(act * u)
            y = O.mul_mat(w2_blocks[e], mid[None], "q8_0", mode=mode)[0]
            acc = (acc + bf16((y * topk_w[t, s]).astype(np.float32))).astype(np.float32)
        out[t] = bf16(acc)
    return out
