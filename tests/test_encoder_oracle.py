"""The encoder oracle's graph wiring against torch's own operators (CPU).

oracle/whisper_encoder_oracle.py restates the reference's stock-Q8 encoder
graph with im2col convolutions, hand-written LayerNorm and attention over the
zero-padded K/V planes. Here the same weights (the fp16-rounded, Q8_0-dequantized
values the oracle multiplies by) go through torch.nn.functional.conv1d,
layer_norm and softmax attention in float64 with unquantized activations, so
the two differ only by Q8_0 activation quantization: within 3e-2 of the
largest |output| (about 1 % per quantized contraction, eight of them per layer).
"""
import numpy as np
import torch
import torch.nn.functional as F

from oracle import oracle as O
from oracle import whisper_encoder_oracle as EO


def test_im2col_is_conv1d():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 11)).astype(np.float32)
    w = rng.standard_normal((4, 5, 3)).astype(np.float32)
    for stride in (1, 2):
        ref = F.conv1d(torch.from_numpy(x)[None].double(), torch.from_numpy(w).double(), stride=stride,
                       padding=1)[0].numpy().T
        got = EO.im2col(x, stride, 32)[:, :15].astype(np.float64) @ w.reshape(4, 15).T.astype(np.float64)
        np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12)
        assert np.all(EO.im2col(x, stride, 32)[:, 15:] == 0)


def test_layer_norm_matches_torch():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((64, 384)) * 3 + 1).astype(np.float32)
    w = (1 + rng.standard_normal(384) * 0.1).astype(np.float32)
    b = (rng.standard_normal(384) * 0.1).astype(np.float32)
    ref = F.layer_norm(torch.from_numpy(x).double(), (384,), torch.from_numpy(w).double(),
                       torch.from_numpy(b).double(), 1e-5).numpy()
    np.testing.assert_allclose(EO.layer_norm(x, w, b), ref, rtol=1e-5, atol=1e-5)


def _dq(w):
    """The weight values the Q8_0 contraction multiplies by (fp16 pre-round, Q8_0)."""
    rows = w.shape[0]
    flat = w.reshape(rows, -1)
    k = flat.shape[1]
    padded = np.zeros((rows, -(-k // 32) * 32), np.float32)  # zero columns, as convolution_q8 pads K
    padded[:, :k] = flat
    return torch.from_numpy(O.dequantize(O.pack_weights(padded), "q8_0")[:, :k]).double()


def _torch_encoder(weights, cfg, mel):
    W = {k: torch.from_numpy(np.asarray(v, np.float64)) for k, v in weights.items()}
    d, H = cfg.width, cfg.heads
    gelu = lambda t: torch.from_numpy(O.gelu_ggml(t.float().numpy())).double()
    x = torch.from_numpy(mel).double()[None]
    c1 = _dq(weights["encoder.conv1.weight"]).reshape(d, cfg.mels, 3)
    c2 = _dq(weights["encoder.conv2.weight"]).reshape(d, d, 3)
    y = gelu(F.conv1d(x, c1, W["encoder.conv1.bias"], padding=1))
    y = gelu(F.conv1d(y, c2, W["encoder.conv2.bias"], stride=2, padding=1))[0].T
    x = y + W["encoder.embed_positions.weight"]
    T = x.shape[0]
    P = -(-T // 256) * 256
    for i in range(cfg.layers):
        p = f"encoder.layers.{i}."
        n = F.layer_norm(x, (d,), W[p + "self_attn_layer_norm.weight"], W[p + "self_attn_layer_norm.bias"], cfg.eps)
        q, k, v = (n @ _dq(weights[p + f"self_attn.{s}_proj.weight"]).T + W[p + f"self_attn.{s}_proj.bias"]
                   for s in "qkv")
        k = torch.cat([k, torch.zeros(P - T, d, dtype=k.dtype)])
        v = torch.cat([v, torch.zeros(P - T, d, dtype=v.dtype)])
        split = lambda t: t.reshape(t.shape[0], H, d // H).transpose(0, 1)
        att = torch.softmax(split(q) @ split(k).transpose(1, 2) / (d // H) ** 0.5, -1) @ split(v)
        att = att.transpose(0, 1).reshape(T, d)
        x = x + att @ _dq(weights[p + "self_attn.out_proj.weight"]).T + W[p + "self_attn.out_proj.bias"]
        n = F.layer_norm(x, (d,), W[p + "final_layer_norm.weight"], W[p + "final_layer_norm.bias"], cfg.eps)
        h = gelu(n @ _dq(weights[p + "fc1.weight"]).T + W[p + "fc1.bias"])
        x = x + h @ _dq(weights[p + "fc2.weight"]).T + W[p + "fc2.bias"]
    return F.layer_norm(x, (d,), W["encoder.layer_norm.weight"], W["encoder.layer_norm.bias"], cfg.eps).numpy()


def test_encoder_oracle_wiring_matches_torch():
    from mstar_accelerators_b200.encoder import EncoderConfig, synthetic_mel, synthetic_weights
    cfg = EncoderConfig(mels=80, width=128, heads=2, layers=2, positions=300)
    w = {k: v.numpy() for k, v in synthetic_weights(cfg, seed=5).items()}
    mel = synthetic_mel(cfg, 1, seed=6).numpy()[0]
    got = EO.WhisperEncoderOracle(w, cfg).forward_one(mel)
    ref = _torch_encoder(w, cfg, mel)
    scale = np.abs(ref).max()
    assert np.abs(got - ref).max() <= 3e-2 * scale
    assert np.abs(got - ref).mean() <= 3e-3 * scale
