"""Whisper audio encoder on B200: the stock-Q8 graph of the reference's native
encoder (backends/cpu_ggml/encoder.cpp:400-754) as a chain of tcgen05 GEMMs over
staged Q8_0 operands.

Per utterance (mel [mels, 2 * positions] fp32, channel-major like the
reference's ``audio_features`` input, encoder.cpp:642-643):
  conv1  im2col (kernel 3, pad 1) -> Q8_0 GEMM, K zero-padded to 32
         (convolution_q8, encoder.cpp:45-52, 551), + bias, ggml GELU (tanh table);
  conv2  the same over conv1's time-major output with stride 2, + bias, GELU,
         + embed_positions (encoder.cpp:689) fused as a residual with period
         ``positions``;
  layer  LayerNorm fused into the Q8_0 staging of the fused QKV GEMM
         (encoder.cpp:467-479, 692-696); its epilogue adds the q/k/v biases and
         writes fp16 rows into per-utterance planes padded to 256 positions whose
         tail stays zero (qkv_scatter, encoder.cpp:202-234); attention over the
         padded keys, scale 1/sqrt(head_dim) (fused_attention, encoder.cpp:371-388);
         out_proj + bias + residual in place (encoder_bias_residual,
         encoder.cpp:146-166); LayerNorm-staged fc1 whose epilogue adds the bias,
         applies GELU and Q8_0-quantizes each 32-column block straight into fc2's
         staged operand (encoder_bias_gelu, encoder.cpp:91-112); fc2 + bias +
         residual in place;
  final  LayerNorm to fp32 ``encoder_states`` (encoder.cpp:725).

The GEMMs, staging, LayerNorm and epilogues are this library's kernels. The
attention itself (outside the block-quantized path) is
torch.nn.functional.scaled_dot_product_attention on the fp16 planes, with the
zero keys of the padded planes inside the softmax exactly as in the reference.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import native
from .linear import BlockLinear, layer_norm, stage_conv, stage_rows


@dataclass(frozen=True)
class EncoderConfig:
    mels: int = 80
    width: int = 384
    heads: int = 6
    layers: int = 4
    positions: int = 1500   # max_source_positions; the mel input has 2 * positions frames
    eps: float = 1e-5
    # whisper-tiny; whisper-large-v3 is EncoderConfig(128, 1280, 20, 32)

    @property
    def ffn(self) -> int:
        return 4 * self.width

    @property
    def padded_keys(self) -> int:
        return -(-self.positions // 256) * 256


TINY = EncoderConfig()
LARGE_V3 = EncoderConfig(mels=128, width=1280, heads=20, layers=32)


def weight_shapes(cfg: EncoderConfig) -> dict[str, tuple[int, ...]]:
    """Reference checkpoint names (encoder.cpp:462-479, 670-735) and shapes."""
    d, f = cfg.width, cfg.ffn
    shapes = {"encoder.conv1.weight": (d, cfg.mels, 3), "encoder.conv1.bias": (d,),
              "encoder.conv2.weight": (d, d, 3), "encoder.conv2.bias": (d,),
              "encoder.embed_positions.weight": (cfg.positions, d),
              "encoder.layer_norm.weight": (d,), "encoder.layer_norm.bias": (d,)}
    for i in range(cfg.layers):
        p = f"encoder.layers.{i}."
        for ln in ("self_attn_layer_norm", "final_layer_norm"):
            shapes[p + ln + ".weight"] = (d,)
            shapes[p + ln + ".bias"] = (d,)
        for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
            shapes[p + f"self_attn.{proj}.weight"] = (d, d)
            shapes[p + f"self_attn.{proj}.bias"] = (d,)
        shapes[p + "fc1.weight"] = (f, d)
        shapes[p + "fc1.bias"] = (f,)
        shapes[p + "fc2.weight"] = (d, f)
        shapes[p + "fc2.bias"] = (d,)
    return shapes


def synthetic_weights(cfg: EncoderConfig, seed: int = 1, device="cpu") -> dict[str, torch.Tensor]:
    """Seeded random encoder weights: matrices, convolutions, positions and biases
    N(0, 0.02); LayerNorm weights 1 + N(0, 0.02). The key bias is kept (the
    reference adds whatever k_proj.bias the checkpoint supplies)."""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, shape in weight_shapes(cfg).items():
        t = torch.randn(shape, generator=g) * 0.02
        if "norm" in name and name.endswith(".weight"):
            t = t + 1.0
        out[name] = t.to(device)
    return out


def synthetic_mel(cfg: EncoderConfig, batch: int, seed: int = 2, device="cpu") -> torch.Tensor:
    """log-mel features U(-1.5, 1.0), [batch, mels, 2 * positions]."""
    g = torch.Generator().manual_seed(seed)
    return (torch.rand((batch, cfg.mels, 2 * cfg.positions), generator=g) * 2.5 - 1.5).to(device)


def conv_k_padded(channels: int) -> int:
    return -(-3 * channels // 32) * 32


class WhisperEncoderB200:
    """Prepared encoder for up to ``max_batch`` utterances on the current CUDA device."""

    def __init__(self, weights: dict[str, torch.Tensor], cfg: EncoderConfig = TINY, *, max_batch: int = 1,
                 rounding: str = "arm", device=None):
        if cfg.width % cfg.heads or cfg.width % 32 or (3 * cfg.width) % 32:
            raise ValueError("unsupported encoder geometry")
        self.lib = native.require_capability()
        self.cfg, self.max_batch, self.rounding = cfg, max_batch, rounding
        self.device = torch.device(device or "cuda")
        dev = self.device
        W = {k: v.detach().to(device=dev, dtype=torch.float32).contiguous() for k, v in weights.items()}
        d = cfg.width
        self.k1, self.k2 = conv_k_padded(cfg.mels), conv_k_padded(d)

        def conv(name, channels, kp):
            w = W[name + ".weight"].reshape(d, 3 * channels)
            if kp > 3 * channels:  # only the added K columns are zero (encoder.cpp:620-634)
                w = torch.cat([w, torch.zeros((d, kp - 3 * channels), device=dev)], dim=1)
            lin = BlockLinear(w.contiguous(), bias=W[name + ".bias"])
            lin.prepare_gemm(64)
            return lin

        self.conv1 = conv("encoder.conv1", cfg.mels, self.k1)
        self.conv2 = conv("encoder.conv2", d, self.k2)
        self.positions = W["encoder.embed_positions.weight"]
        self.layers = []
        for i in range(cfg.layers):
            p = f"encoder.layers.{i}."
            qkv_w = torch.cat([W[p + f"self_attn.{n}_proj.weight"] for n in "qkv"], dim=0)
            # a checkpoint without a key bias (public Whisper) adds +0 (encoder.cpp:655-663)
            qkv_b = torch.cat([W.get(p + f"self_attn.{n}_proj.bias", torch.zeros(d, device=dev)) for n in "qkv"], dim=0)
            layer = {
                "ln1": (W[p + "self_attn_layer_norm.weight"], W[p + "self_attn_layer_norm.bias"], cfg.eps),
                "ln2": (W[p + "final_layer_norm.weight"], W[p + "final_layer_norm.bias"], cfg.eps),
                "qkv": BlockLinear(qkv_w, bias=qkv_b),
                "out": BlockLinear(W[p + "self_attn.out_proj.weight"], bias=W[p + "self_attn.out_proj.bias"]),
                "fc1": BlockLinear(W[p + "fc1.weight"], bias=W[p + "fc1.bias"]),
                "fc2": BlockLinear(W[p + "fc2.weight"], bias=W[p + "fc2.bias"]),
            }
            for k in ("qkv", "out", "fc1", "fc2"):
                layer[k].prepare_gemm(64)
            self.layers.append(layer)
        self.final_norm = (W["encoder.layer_norm.weight"], W["encoder.layer_norm.bias"], cfg.eps)
        self._alloc(max_batch)

    def _alloc(self, batch: int) -> None:
        cfg, dev = self.cfg, self.device
        d, T, P = cfg.width, cfg.positions, cfg.padded_keys
        rows1, rows = batch * 2 * T, batch * T
        stage_elems = max(rows1 * self.k1, rows * self.k2, rows * d)
        self.staged = torch.empty(stage_elems, dtype=torch.float16, device=dev)
        self.hidden16 = torch.empty((rows, cfg.ffn), dtype=torch.float16, device=dev)
        self.conv_out = torch.empty((rows1, d), dtype=torch.float32, device=dev)
        self.x = torch.empty((rows, d), dtype=torch.float32, device=dev)
        # fp16 q|k|v rows in per-utterance planes of P rows; rows T..P-1 stay zero
        self.qkv16 = torch.zeros((batch, P, 3 * d), dtype=torch.float16, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)

    def _staged(self, rows: int, k: int) -> torch.Tensor:
        return self.staged[:rows * k].view(rows, k)

    def forward(self, mel: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """mel fp32 [batch, mels, 2 * positions] (device) -> encoder_states fp32 [batch, positions, width]."""
        cfg, r = self.cfg, self.rounding
        B = mel.shape[0]
        if mel.shape[1:] != (cfg.mels, 2 * cfg.positions) or mel.dtype != torch.float32:
            raise ValueError("mel must be fp32 [batch, mels, 2 * positions]")
        if B > self.max_batch:
            raise ValueError("batch exceeds the prepared capacity")
        d, T, P, H = cfg.width, cfg.positions, cfg.padded_keys, cfg.heads
        rows = B * T
        st = self.status
        x = self.x[:rows]
        # convolution stems
        a = stage_conv(mel, time_major=False, stride=1, k_padded=self.k1, rounding=r,
                       out=self._staged(B * 2 * T, self.k1), status=st)
        self.conv1.gemm(a, out=self.conv_out[:B * 2 * T], gelu="tanh", rounding=r, status=st)
        a = stage_conv(self.conv_out[:B * 2 * T].view(B, 2 * T, d), time_major=True, stride=2, k_padded=self.k2,
                       rounding=r, out=self._staged(rows, self.k2), status=st)
        self.conv2.gemm(a, out=x, gelu="tanh", residual=self.positions, residual_period=T, rounding=r, status=st)
        qkv = self.qkv16[:B]
        for L in self.layers:
            a = stage_rows(x, norm=L["ln1"], rounding=r, out=self._staged(rows, d), status=st)
            L["qkv"].gemm(a, out=qkv, out_format="f16", segments=(T, P), rounding=r, status=st)
            q = qkv[:, :T, :d].unflatten(-1, (H, d // H)).transpose(1, 2)
            k = qkv[:, :, d:2 * d].unflatten(-1, (H, d // H)).transpose(1, 2)
            v = qkv[:, :, 2 * d:].unflatten(-1, (H, d // H)).transpose(1, 2)
            att = F.scaled_dot_product_attention(q, k, v, scale=(d // H) ** -0.5)
            att = att.transpose(1, 2).reshape(rows, d)
            a = stage_rows(att, rounding=r, out=self._staged(rows, d), status=st)
            L["out"].gemm(a, out=x, residual=x, rounding=r, status=st)
            a = stage_rows(x, norm=L["ln2"], rounding=r, out=self._staged(rows, d), status=st)
            h = L["fc1"].gemm(a, out=self.hidden16[:rows], out_format="staged", gelu="tanh", rounding=r, status=st)
            L["fc2"].gemm(h, out=x, residual=x, rounding=r, status=st)
        if out is None:
            out = torch.empty((B, T, d), dtype=torch.float32, device=self.device)
        w, b, eps = self.final_norm
        layer_norm(x, w, b, eps, out=out.view(rows, d))
        return out

    __call__ = forward

    def launches_per_forward(self) -> int:
        """This library's kernel launches in one forward: two convolution stagings and GEMMs;
        per layer three stagings (two with the LayerNorm) and four GEMMs; the final LayerNorm.
        The attention between them is torch's."""
        return 4 + 7 * len(self.layers) + 1

    def close(self) -> None:
        for lin in [self.conv1, self.conv2] + [L[k] for L in self.layers for k in ("qkv", "out", "fc1", "fc2")]:
            lin.close()
