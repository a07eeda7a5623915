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


def _groups(topk_ids: np.ndarray):
    """(expert, token indices, slot indices) for every expert that has pairs, pairs in token order."""
    T, k = topk_ids.shape
    flat = topk_ids.reshape(-1).astype(np.int64)
    order = np.argsort(flat, kind="stable")
    for e in np.unique(flat):
        sel = order[flat[order] == e]
        yield int(e), sel // k, sel % k


def _swiglu(g, u):
    act = bf16((g * (1.0 / (1.0 + np.exp(-g.astype(np.float64))))).astype(np.float32))
    return bf16(act * u)


def experts_bf16(x, w1, w2, topk_w, topk_ids):
    """x [T, H], w1 [E, 2I, H], w2 [E, H, I] (float32 holding bf16 values).

    The pairs of one expert are contracted together (float64 products, one rounding to
    float32 per output, as the per-pair dot would give); every bf16 rounding point is
    the reference's (thinker_moe.py:17-83) and the slots are summed in slot order."""
    T, H = x.shape
    I = w1.shape[1] // 2
    k = topk_ids.shape[1]
    y = np.zeros((T, k, H), np.float32)
    for e, tok, slot in _groups(topk_ids):
        xe = x[tok].astype(np.float64)
        g = bf16((xe @ w1[e, :I].astype(np.float64).T).astype(np.float32))
        u = bf16((xe @ w1[e, I:].astype(np.float64).T).astype(np.float32))
        mid = _swiglu(g, u)
        ye = (mid.astype(np.float64) @ w2[e].astype(np.float64).T).astype(np.float32)
        y[tok, slot] = bf16((ye * topk_w[tok, slot][:, None]).astype(np.float32))
    acc = np.zeros((T, H), np.float32)
    for s in range(k):  # moe_sum_reduce: fp32 sum in slot order (thinker_moe.py:75-81)
        acc = (acc + y[:, s]).astype(np.float32)
    return bf16(acc)


def experts_bf16_hf(x, w1, w2, topk_w, topk_ids):
    """The rounding points of transformers' eager Qwen3OmniMoeThinkerTextExperts.forward
    (the reference's HF oracle, testing/models/qwen3_omni_hf.py:16-53): the down projection
    is rounded to bf16 before the routing weight multiplies it in fp32, that product is
    rounded to bf16, and the pairs are added into a bf16 output expert by expert
    (index_add_ in ascending expert order, one bf16 rounding per add)."""
    T, H = x.shape
    I = w1.shape[1] // 2
    out = np.zeros((T, H), np.float32)
    for e, tok, slot in _groups(topk_ids):
        xe = x[tok].astype(np.float64)
        g = bf16((xe @ w1[e, :I].astype(np.float64).T).astype(np.float32))
        u = bf16((xe @ w1[e, I:].astype(np.float64).T).astype(np.float32))
        mid = _swiglu(g, u)
        ye = bf16((mid.astype(np.float64) @ w2[e].astype(np.float64).T).astype(np.float32))
        contrib = bf16((ye * topk_w[tok, slot][:, None]).astype(np.float32))
        for i, t in enumerate(tok):   # index_add_ visits the pairs of one expert in token order
            out[t] = bf16(out[t] + contrib[i])
    return out


def experts_q8(x, w1_blocks, w2_blocks, topk_w, topk_ids, I, H, mode="arm"):
    """Q8_0 composition: w1_blocks [E][2I][H/32*34], w2_blocks [E][H][I/32*34]; every dot is
    the ggml generic-order Q8_0 mul_mat of its Q8_0-quantized activation row (x, then mid)."""
    T = x.shape[0]
    k = topk_ids.shape[1]
    y = np.zeros((T, k, H), np.float32)
    for e, tok, slot in _groups(topk_ids):
        gu = O.mul_mat(w1_blocks[e], x[tok], "q8_0", mode=mode)
        mid = _swiglu(bf16(gu[:, :I]), bf16(gu[:, I:]))
        ye = O.mul_mat(w2_blocks[e], mid, "q8_0", mode=mode)
        y[tok, slot] = bf16((ye * topk_w[tok, slot][:, None]).astype(np.float32))
    acc = np.zeros((T, H), np.float32)
    for s in range(k):
        acc = (acc + y[:, s]).astype(np.float32)
    return bf16(acc)
