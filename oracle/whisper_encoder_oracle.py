"""ORACLE — test infrastructure only.

CPU composition of the reference's stock-Q8 Whisper encoder graph
(backends/cpu_ggml/encoder.cpp:400-754) from the C oracle's Q8_0 pieces:
  conv i   convolution_q8 (encoder.cpp:45-52): ggml_im2col (kernel 3, pad 1,
           column = channel * 3 + tap) zero-padded to a multiple of 32 columns
           (encoder.cpp:551), mul_mat with the Q8_0 kernel matrix packed from the
           fp16-rounded weights with zero added columns (encoder.cpp:620-634),
           + bias, ggml GELU (encoder.cpp:672, activation() at :327-329);
           conv1's output is transposed to channel rows for conv2 (encoder.cpp:675)
  x        = conv2 output + embed_positions (encoder.cpp:689)
  layer    n = norm_affine(x) (encoder_norm_affine, :117-142); all = mul_mat(qkv, n);
           q = all_q + b_q, k = fp16(all_k + b_k), v = fp16(all_v + b_v), K/V
           zero-padded to a multiple of 256 rows (qkv_scatter, :202-234);
           attention over the padded keys with scale 1/sqrt(d) (:371-388);
           x = x + (mul_mat(out, a) + b) (encoder_bias_residual, :146-166);
           n = norm_affine(x); h = gelu(mul_mat(fc1, n) + b1) (:91-112);
           x = x + (mul_mat(fc2, h) + b2)
  output   norm_affine(x) (:725)
mul_mat is oracle.mul_mat (generic ggml order, activations quantized with the
selected rounding). LayerNorm follows ggml_compute_forward_norm_f32
(ggml-cpu/ops.cpp:4094-4137) with float64 sums. Attention is evaluated in
float64 from fp16 q, k, v (ggml's CPU flash kernel converts Q to fp16 and
accumulates in its own order; attention is not a block-quantized contraction,
so it is compared by tolerance like everything after the first LayerNorm).
"""
from __future__ import annotations

import numpy as np

from . import oracle as O


def _k_padded(channels: int) -> int:
    return -(-3 * channels // 32) * 32


def layer_norm(x, w, b, eps=1e-5):
    x = np.asarray(x, np.float32)
    n = x.shape[-1]
    mean = (x.astype(np.float64).sum(-1, keepdims=True).astype(np.float32) / np.float32(n)).astype(np.float32)
    y = (x - mean).astype(np.float32)
    var = ((y.astype(np.float64) ** 2).sum(-1, keepdims=True) / n).astype(np.float32)
    scale = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    return (((y * scale).astype(np.float32) * w).astype(np.float32) + b).astype(np.float32)


def im2col(src_ct, stride, k_padded):
    """Channel-major [C, T] fp32 -> columns [T_out, k_padded] (kernel 3, pad 1)."""
    C, T = src_ct.shape
    t_out = (T - 1) // stride + 1
    padded = np.zeros((C, T + 2), np.float32)
    padded[:, 1:T + 1] = src_ct
    cols = np.zeros((t_out, k_padded), np.float32)
    for tap in range(3):
        cols[:, tap:3 * C:3] = padded[:, tap:tap + stride * t_out:stride][:, :t_out].T
    return cols


class WhisperEncoderOracle:
    def __init__(self, weights: dict, cfg, mode: str = "arm"):
        self.cfg, self.mode = cfg, mode
        W = {k: np.asarray(v, np.float32) for k, v in weights.items()}
        self.W = W
        d = cfg.width

        def conv(name, channels):
            kp = _k_padded(channels)
            w = np.zeros((d, kp), np.float32)
            w[:, :3 * channels] = W[name + ".weight"].reshape(d, 3 * channels)
            return O.pack_weights(w), W[name + ".bias"], kp

        self.conv1 = conv("encoder.conv1", cfg.mels)
        self.conv2 = conv("encoder.conv2", d)
        self.layers = []
        for i in range(cfg.layers):
            p = f"encoder.layers.{i}."
            qkv = np.concatenate([W[p + f"self_attn.{n}_proj.weight"] for n in "qkv"], 0)
            self.layers.append({
                "qkv": O.pack_weights(qkv),
                "qkv_b": [W[p + f"self_attn.{n}_proj.bias"] for n in "qkv"],
                "out": O.pack_weights(W[p + "self_attn.out_proj.weight"]), "out_b": W[p + "self_attn.out_proj.bias"],
                "fc1": O.pack_weights(W[p + "fc1.weight"]), "fc1_b": W[p + "fc1.bias"],
                "fc2": O.pack_weights(W[p + "fc2.weight"]), "fc2_b": W[p + "fc2.bias"],
                "ln1": (W[p + "self_attn_layer_norm.weight"], W[p + "self_attn_layer_norm.bias"]),
                "ln2": (W[p + "final_layer_norm.weight"], W[p + "final_layer_norm.bias"]),
            })

    def mm(self, blocks, x):
        return O.mul_mat(blocks, np.ascontiguousarray(x, np.float32), "q8_0", mode=self.mode)

    def attention(self, q, k, v):
        cfg = self.cfg
        T, d = q.shape
        H, hd = cfg.heads, d // cfg.heads
        P = -(-T // 256) * 256
        qh = q.astype(np.float16).astype(np.float64).reshape(T, H, hd).transpose(1, 0, 2)
        kp = np.zeros((P, d), np.float64)
        vp = np.zeros((P, d), np.float64)
        kp[:T], vp[:T] = k, v
        kh = kp.reshape(P, H, hd).transpose(1, 0, 2)
        vh = vp.reshape(P, H, hd).transpose(1, 0, 2)
        s = (qh @ kh.transpose(0, 2, 1)) / np.sqrt(hd)
        s -= s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        return (p @ vh).transpose(1, 0, 2).reshape(T, d).astype(np.float32)

    def forward_one(self, mel):
        """mel [mels, 2 * positions] -> encoder_states [positions, width] (fp32)."""
        cfg = self.cfg
        (b1, bias1, k1), (b2, bias2, k2) = self.conv1, self.conv2
        y = O.gelu_ggml(self.mm(b1, im2col(np.asarray(mel, np.float32), 1, k1)) + bias1)
        y = O.gelu_ggml(self.mm(b2, im2col(np.ascontiguousarray(y.T), 2, k2)) + bias2)
        x = (y + self.W["encoder.embed_positions.weight"]).astype(np.float32)
        d = cfg.width
        for L in self.layers:
            n = layer_norm(x, *L["ln1"], cfg.eps)
            a = self.mm(L["qkv"], n)
            qb, kb, vb = L["qkv_b"]
            q = (a[:, :d] + qb).astype(np.float32)
            k = O.fp16_round(a[:, d:2 * d] + kb)
            v = O.fp16_round(a[:, 2 * d:] + vb)
            att = self.attention(q, k, v)
            x = (x + (self.mm(L["out"], att) + L["out_b"]).astype(np.float32)).astype(np.float32)
            n = layer_norm(x, *L["ln2"], cfg.eps)
            h = O.gelu_ggml((self.mm(L["fc1"], n) + L["fc1_b"]).astype(np.float32))
            x = (x + (self.mm(L["fc2"], h) + L["fc2_b"]).astype(np.float32)).astype(np.float32)
        return layer_norm(x, self.W["encoder.layer_norm.weight"], self.W["encoder.layer_norm.bias"], cfg.eps)

    def forward(self, mel_batch):
        return np.stack([self.forward_one(m) for m in np.asarray(mel_batch, np.float32)])
