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

import math

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


# ----------------------------------------------------------------------------- the stack
def rms_norm(x, w, eps):
    """transformers' Qwen3OmniMoeThinkerTextRMSNorm on bf16 values: fp32 normalisation, bf16
    before the bf16 weight product."""
    x = np.asarray(x, np.float32)
    var = (x.astype(np.float64) ** 2).mean(-1, keepdims=True).astype(np.float32)
    h = bf16((x * (np.float32(1.0) / np.sqrt(var + np.float32(eps)))).astype(np.float32))
    return bf16((np.asarray(w, np.float32) * h).astype(np.float32))


def rotary(positions, head_dim, theta):
    inv = (1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))).astype(np.float32)
    f = (np.asarray(positions, np.float32)[:, None] * inv[None, :]).astype(np.float32)
    emb = np.concatenate([f, f], -1)
    return bf16(np.cos(emb)), bf16(np.sin(emb))


class ThinkerStackOracle:
    """The thinker layer stack of mstar_accelerators_b200.thinker_stack, composed from the
    oracle's pieces: Q8_0 generic-order mul_mat for the fused QKV, o_proj and lm_head
    (ARM activation rounding), the fused QK-norm / RoPE restatement above, float64
    softmax attention over the bf16 cache (GQA, causal), the MoE oracle's router and
    Q8_0 / bf16 experts, bf16 residual adds, suppression-free first-index argmax."""

    def __init__(self, cfg, layers: list, head: dict, experts: str = "q8_0"):
        from . import moe_oracle as MO
        from . import oracle as O
        self.O, self.MO = O, MO
        self.cfg, self.experts = cfg, experts
        f = lambda t: np.asarray(t.float().cpu().numpy() if hasattr(t, "float") else t, np.float32)
        self.L = []
        for w in layers:
            qkv = np.concatenate([f(w["q"]), f(w["k"]), f(w["v"])], 0)
            d = {"ln1": f(w["ln1"]), "ln2": f(w["ln2"]), "q_norm": f(w["q_norm"]), "k_norm": f(w["k_norm"]),
                 "router": f(w["router"]), "qkv": O.pack_weights(qkv), "o": O.pack_weights(f(w["o"]))}
            if experts == "q8_0":
                H, I = cfg.hidden, cfg.moe_intermediate
                d["w1"] = O.pack_weights(f(w["w1"]).reshape(-1, H), preround=False).reshape(cfg.experts, 2 * I, -1)
                d["w2"] = O.pack_weights(f(w["w2"]).reshape(-1, I), preround=False).reshape(cfg.experts, H, -1)
            else:
                d["w1"], d["w2"] = f(w["w1"]), f(w["w2"])
            self.L.append(d)
        self.embed, self.norm = f(head["embed"]), f(head["norm"])
        self.lm_head = O.pack_weights(f(head["lm_head"]))
        self.k = [None] * cfg.layers
        self.v = [None] * cfg.layers

    def _attend(self, q, K, V, start):
        cfg = self.cfg
        S, n, Hq, D = q.shape
        rep = Hq // cfg.kv_heads
        out = np.zeros((S, n, Hq, D), np.float32)
        for s in range(S):
            for h in range(Hq):
                kk, vv = K[s, :, h // rep].astype(np.float64), V[s, :, h // rep].astype(np.float64)
                sc = q[s, :, h].astype(np.float64) @ kk.T / math.sqrt(D)
                for i in range(n):
                    sc[i, start + i + 1:] = -np.inf
                p = np.exp(sc - sc.max(-1, keepdims=True))
                out[s, :, h] = (p @ vv / p.sum(-1, keepdims=True)).astype(np.float32)
        return bf16(out)

    def _layer(self, i, x, S, n, start):
        cfg, L, O, MO = self.cfg, self.L[i], self.O, self.MO
        D, Hq, Hk = cfg.head_dim, cfg.q_heads, cfg.kv_heads
        T = S * n
        h = rms_norm(x, L["ln1"], cfg.eps)
        qkv = bf16(O.mul_mat(L["qkv"], h, "q8_0"))
        q = qkv[:, :Hq * D].reshape(T, Hq, D)
        k = qkv[:, Hq * D:(Hq + Hk) * D].reshape(T, Hk, D)
        v = qkv[:, (Hq + Hk) * D:].reshape(T, Hk, D)
        pos = np.tile(np.arange(start, start + n), S)
        cos, sin = rotary(pos, D, cfg.rope_theta)
        q, k = qknorm_rope(q, k, L["q_norm"], L["k_norm"], cos, sin, eps=cfg.eps)
        k, v = k.reshape(S, n, Hk, D), v.reshape(S, n, Hk, D)
        self.k[i] = k if start == 0 else np.concatenate([self.k[i], k], 1)
        self.v[i] = v if start == 0 else np.concatenate([self.v[i], v], 1)
        att = self._attend(q.reshape(S, n, Hq, D), self.k[i], self.v[i], start).reshape(T, Hq * D)
        x = bf16(x + bf16(O.mul_mat(L["o"], att, "q8_0")))
        h = rms_norm(x, L["ln2"], cfg.eps)
        w, ids, _ = MO.route(h, L["router"], cfg.top_k)
        if self.experts == "q8_0":
            y = MO.experts_q8(h, L["w1"], L["w2"], w, ids, cfg.moe_intermediate, cfg.hidden)
        else:
            y = MO.experts_bf16(h, L["w1"], L["w2"], w, ids)
        return bf16(x + y)

    def _readout(self, last):
        h = rms_norm(last, self.norm, self.cfg.eps)
        logits = self.O.mul_mat(self.lm_head, h, "q8_0")
        return logits, logits.argmax(-1)

    def prefill(self, tokens):
        S, n = tokens.shape
        x = self.embed[np.asarray(tokens).reshape(-1)]
        for i in range(self.cfg.layers):
            x = self._layer(i, x, S, n, 0)
        self.length = n
        return self._readout(x.reshape(S, n, -1)[:, -1])

    def decode(self, tokens):
        x = self.embed[np.asarray(tokens).reshape(-1)]
        for i in range(self.cfg.layers):
            x = self._layer(i, x, len(tokens), 1, self.length)
        self.length += 1
        return self._readout(x)
