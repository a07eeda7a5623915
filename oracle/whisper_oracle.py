"""ORACLE — test infrastructure only.

CPU restatement of the reference's Q8_0 Whisper decoder graph
(backends/cpu_ggml/decoder.cpp:489-600 Graph::build, run() :655-697) composed
from the oracle's block-quantized ops: every linear is ggml mul_mat of Q8_0
weights (generic block order) plus bias; LayerNorm is ggml_norm + mul + add
(ggml-cpu/ops.cpp:4094-4137); attention is fp32 over fp16-stored K/V with scale
1/sqrt(64) (decoder.cpp:504-511, the F16 plain storage encoding); GELU is the
stock fp16-table form (decoder.cpp:580); the readout is Q4_0 (or Q8_0) mul_mat
of the final-LayerNorm output, suppression, and the first-index / NaN-first
argmax (decoder.cpp:583-588, 686-696). Parity of the pieces is pinned in
tests/test_oracle.py; the GPU decoder is compared against this composition.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O


def _ln(x, w, b, eps):
    mean = x.mean(-1, keepdims=True, dtype=np.float64).astype(np.float32)
    y = (x - mean).astype(np.float32)
    var = (y.astype(np.float64) ** 2).mean(-1, keepdims=True).astype(np.float32)
    return ((y * (np.float32(1.0) / np.sqrt(var + np.float32(eps)))) * w + b).astype(np.float32)


class WhisperDecoderOracle:
    def __init__(self, weights: dict, cfg, batch: int = 1, readout_format: str = "q4_0", rounding: str = "arm",
                 suppressed: dict | None = None):
        self.cfg, self.B, self.mode = cfg, batch, rounding
        self.W = {k: np.ascontiguousarray(v.detach().cpu().numpy() if hasattr(v, "detach") else v, np.float32)
                  for k, v in weights.items()}
        self.blocks = {}
        for k, v in self.W.items():
            if v.ndim == 2 and "embed" not in k:
                self.blocks[k] = O.pack_weights(v, "q8_0")
        self.fmt = readout_format
        self.head = O.pack_weights(self.W["decoder.embed_tokens.weight"], readout_format)
        self.suppressed = suppressed or {"prefill": [], "decode": []}
        d = cfg.d_model
        self.k = [np.zeros((batch, cfg.target, d), np.float32) for _ in range(cfg.layers)]
        self.v = [np.zeros((batch, cfg.target, d), np.float32) for _ in range(cfg.layers)]
        self.ck = self.cv = None

    def _lin(self, name, x, bias=True):
        out = O.mul_mat(self.blocks[name + ".weight"], x, "q8_0", mode=self.mode)
        b = self.W.get(name + ".bias")
        if bias and b is not None:
            out = (out + b).astype(np.float32)
        return out

    def _att(self, q, K, V, lens):
        # q [nq, d]; K/V [T, d] fp16-rounded; query i sees keys [0, lens[i]); fp32 scores,
        # softmax and weighted sum per head (all heads of a query at once)
        cfg = self.cfg
        H, hd = cfg.heads, cfg.d_model // cfg.heads
        out = np.zeros_like(q)
        Kh = K.reshape(K.shape[0], H, hd)
        Vh = V.reshape(V.shape[0], H, hd)
        scale = np.float32(1.0 / np.sqrt(hd))
        for i in range(q.shape[0]):
            n = int(lens[i])
            s = np.einsum("thd,hd->ht", Kh[:n], q[i].reshape(H, hd)).astype(np.float32) * scale
            p = np.exp(s - s.max(-1, keepdims=True)).astype(np.float32)
            o = np.einsum("ht,thd->hd", p, Vh[:n]).astype(np.float32) / p.sum(-1, keepdims=True)
            out[i] = o.reshape(-1)
        return out

    def set_cross(self, enc):
        cfg = self.cfg
        enc = np.asarray(enc, np.float32).reshape(-1, cfg.source, cfg.d_model)
        self.ck, self.cv = [], []
        for i in range(cfg.layers):
            p = f"decoder.layers.{i}.encoder_attn."
            kk = [O.fp16_round(self._lin(p + "k_proj", e)) for e in enc]
            vv = [O.fp16_round(self._lin(p + "v_proj", e)) for e in enc]
            self.ck.append(np.stack(kk))
            self.cv.append(np.stack(vv))

    def forward(self, tokens, positions, walk):
        """tokens/positions [B, nq]; returns (masked logits of each sequence's last query, tokens)."""
        cfg, W = self.cfg, self.W
        tokens = np.asarray(tokens).reshape(self.B, -1)
        positions = np.asarray(positions).reshape(self.B, -1)
        nq = tokens.shape[1]
        x = (W["decoder.embed_tokens.weight"][tokens] + W["decoder.embed_positions.weight"][positions]).astype(
            np.float32).reshape(-1, cfg.d_model)
        for i in range(cfg.layers):
            p = f"decoder.layers.{i}."
            n = _ln(x, W[p + "self_attn_layer_norm.weight"], W[p + "self_attn_layer_norm.bias"], cfg.eps)
            q = self._lin(p + "self_attn.q_proj", n)
            k = self._lin(p + "self_attn.k_proj", n)
            v = self._lin(p + "self_attn.v_proj", n)
            att = np.zeros_like(x)
            for b in range(self.B):
                rows = slice(b * nq, (b + 1) * nq)
                self.k[i][b, positions[b]] = O.fp16_round(k[rows])
                self.v[i][b, positions[b]] = O.fp16_round(v[rows])
                att[rows] = self._att(q[rows], self.k[i][b], self.v[i][b], positions[b] + 1)
            x = (x + self._lin(p + "self_attn.out_proj", att)).astype(np.float32)
            n = _ln(x, W[p + "encoder_attn_layer_norm.weight"], W[p + "encoder_attn_layer_norm.bias"], cfg.eps)
            q = self._lin(p + "encoder_attn.q_proj", n)
            for b in range(self.B):
                rows = slice(b * nq, (b + 1) * nq)
                s = 0 if self.ck[i].shape[0] == 1 else b
                att[rows] = self._att(q[rows], self.ck[i][s], self.cv[i][s], [cfg.source] * nq)
            x = (x + self._lin(p + "encoder_attn.out_proj", att)).astype(np.float32)
            n = _ln(x, W[p + "final_layer_norm.weight"], W[p + "final_layer_norm.bias"], cfg.eps)
            hcur = O.gelu_ggml(self._lin(p + "fc1", n))
            x = (x + self._lin(p + "fc2", hcur)).astype(np.float32)
        last = x.reshape(self.B, nq, -1)[:, -1]
        n = _ln(last, W["decoder.layer_norm.weight"], W["decoder.layer_norm.bias"], cfg.eps)
        logits = O.mul_mat(self.head, n, self.fmt, mode=self.mode)
        out, toks = [], []
        for b in range(self.B):
            masked, tok = O.argmax(logits[b], self.suppressed.get(walk, []))
            out.append(masked)
            toks.append(tok)
        return np.stack(out), np.array(toks, np.int64)


def greedy_agrees(token: int, logits_ref: np.ndarray, token_ref: int, logits_got: np.ndarray, k: int = 5) -> bool:
    """The reference harness's greedy policy (testing/generation.py:25-57): the
    same token, or each side's token inside the other side's top-k."""
    if token == token_ref:
        return True
    top_ref = np.argsort(-logits_ref)[:k]
    top_got = np.argsort(-logits_got)[:k]
    return token in top_ref and token_ref in top_got
