"""ORACLE-side CPU baseline — benchmark infrastructure only.

Times the reference's own CPU arithmetic for a Whisper encoder on a bounded
sample: ONE utterance (``positions`` rows) through the two convolution stems,
``sample_layers`` of the identical pre-LN layers and the final LayerNorm.

  * every block-quantized contraction (the two im2col convolutions, fused QKV,
    out_proj, fc1, fc2) runs through the reference's vendored ggml x86 kernels
    compiled into ``_ref`` (``quantize_row_q8_0`` + ``ggml_vec_dot_q8_0_q8_0``,
    arch/x86/quants.c:302-350 and :1372, driven by ``ref_mul_mat`` over every
    host thread), the arithmetic ``ggml_compute_forward_mul_mat`` performs on an
    x86 host (ggml-cpu.c:1255; x86 has no Q8_0 repack, repack.cpp:5105-5115);
  * LayerNorm follows ggml_compute_forward_norm_f32 with float64 sums
    (whisper_encoder_oracle.layer_norm), GELU is ggml's fp16 table
    (ggml-cpu/vec.h:963-1013, one lookup per element), and attention runs in
    torch fp32 on the host over the keys zero-padded to a multiple of 256
    (encoder.cpp:202-234, 371-388).

The graph is the reference's stock-Q8 encoder (backends/cpu_ggml/encoder.cpp:
400-754); its own Q8 entry points refuse on x86 (``*_q8_capability`` is 0
without the ARM repack), so the same graph is composed here from those kernels.

Every layer has the same shapes, so the time of a whole ``layers``-deep forward
is t(stems) + t(sampled layers) * layers / sample_layers + t(final norm); the
result is reported as tokens (positions) per second per layer stack.
"""
from __future__ import annotations

import time

import numpy as np

from . import oracle as O
from .whisper_encoder_oracle import _k_padded, im2col, layer_norm


def gelu_table() -> np.ndarray:
    """ggml's GELU over every fp16 input, as fp32 values indexed by fp16 bits."""
    h = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32)
    return O.gelu_ggml(np.nan_to_num(h, nan=0.0, posinf=10.0, neginf=-10.0))


class CpuEncoderSample:
    """One utterance of a Whisper encoder of width ``width`` on the host cores."""

    def __init__(self, *, mels: int, width: int, heads: int, layers: int, positions: int = 1500,
                 sample_layers: int = 2, seed: int = 1, threads: int = 0):
        import torch
        if O.ref_lib() is None:
            O.build()
        if O.ref_lib() is None:
            raise RuntimeError("the reference ggml kernels (oracle/_ref) are not built")
        self.threads = threads or O.cpu_cores()
        torch.set_num_threads(self.threads)
        self.mels, self.width, self.heads, self.layers, self.positions = mels, width, heads, layers, positions
        self.sample_layers = min(sample_layers, layers)
        rng = np.random.default_rng(seed)
        d, f = width, 4 * width

        def mat(n, k):
            return O.pack_weights((rng.standard_normal((n, k)) * 0.02).astype(np.float32))

        def vec(n, one=False):
            return ((1.0 if one else 0.0) + rng.standard_normal(n) * 0.02).astype(np.float32)

        def conv(channels):
            kp = _k_padded(channels)
            w = np.zeros((d, kp), np.float32)
            w[:, :3 * channels] = rng.standard_normal((d, 3 * channels)) * 0.02
            return O.pack_weights(w), vec(d), kp

        self.conv1, self.conv2 = conv(mels), conv(d)
        self.pos = (rng.standard_normal((positions, d)) * 0.02).astype(np.float32)
        self.blocks = [{"qkv": mat(3 * d, d), "qkv_b": vec(3 * d), "out": mat(d, d), "out_b": vec(d),
                        "fc1": mat(f, d), "fc1_b": vec(f), "fc2": mat(d, f), "fc2_b": vec(d),
                        "ln1": (vec(d, True), vec(d)), "ln2": (vec(d, True), vec(d))}
                       for _ in range(self.sample_layers)]
        self.final = (vec(d, True), vec(d))
        self.gelu = gelu_table()
        self.mel = rng.uniform(-1.5, 1.0, (mels, 2 * positions)).astype(np.float32)

    # ------------------------------------------------------------------ pieces
    def _mm(self, blocks, x):
        return O.ref_mul_mat(blocks, np.ascontiguousarray(x, np.float32), "q8_0", threads=self.threads)

    def _gelu(self, x):
        x = np.asarray(x, np.float32)
        y = self.gelu[x.astype(np.float16).view(np.uint16)]
        return np.where(x <= -10.0, np.float32(0.0), np.where(x >= 10.0, x, y)).astype(np.float32)

    def _attention(self, q, k, v):
        import torch
        T, d = q.shape
        H, hd = self.heads, d // self.heads
        P = -(-T // 256) * 256
        kp = np.zeros((P, d), np.float32)
        vp = np.zeros((P, d), np.float32)
        kp[:T], vp[:T] = k, v
        qh = torch.from_numpy(q.astype(np.float16).astype(np.float32)).view(T, H, hd).transpose(0, 1)
        kh = torch.from_numpy(kp).view(P, H, hd).transpose(0, 1)
        vh = torch.from_numpy(vp).view(P, H, hd).transpose(0, 1)
        out = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh, scale=hd ** -0.5)
        return out.transpose(0, 1).reshape(T, d).numpy()

    def stems(self):
        (b1, bias1, k1), (b2, bias2, k2) = self.conv1, self.conv2
        y = self._gelu(self._mm(b1, im2col(self.mel, 1, k1)) + bias1)
        y = self._gelu(self._mm(b2, im2col(np.ascontiguousarray(y.T), 2, k2)) + bias2)
        return (y + self.pos).astype(np.float32)

    def layer(self, x, L):
        d = self.width
        n = layer_norm(x, *L["ln1"])
        a = self._mm(L["qkv"], n) + L["qkv_b"]
        q = a[:, :d].astype(np.float32)
        k = O.fp16_round(a[:, d:2 * d])
        v = O.fp16_round(a[:, 2 * d:])
        x = (x + (self._mm(L["out"], self._attention(q, k, v)) + L["out_b"])).astype(np.float32)
        n = layer_norm(x, *L["ln2"])
        h = self._gelu(self._mm(L["fc1"], n) + L["fc1_b"])
        return (x + (self._mm(L["fc2"], h) + L["fc2_b"])).astype(np.float32)

    def forward_seconds(self) -> float:
        """One sampled forward; returns the extrapolated seconds of a full forward."""
        t0 = time.perf_counter()
        x = self.stems()
        t1 = time.perf_counter()
        for L in self.blocks:
            x = self.layer(x, L)
        t2 = time.perf_counter()
        layer_norm(x, *self.final)
        t3 = time.perf_counter()
        return (t1 - t0) + (t2 - t1) * self.layers / self.sample_layers + (t3 - t2)

    def sample_text(self) -> str:
        return (f"one utterance ({self.positions} positions) of the {self.layers}-layer encoder per step: "
                f"stems + {self.sample_layers} of the {self.layers} identical layers (time scaled by "
                f"{self.layers}/{self.sample_layers}) + final LayerNorm; Q8_0 contractions through the vendored "
                f"ggml x86 quantizer + vec_dot on {self.threads} host threads, LayerNorm / GELU table / "
                f"attention (torch fp32) on the host")
