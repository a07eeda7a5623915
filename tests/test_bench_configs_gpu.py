"""The timed configurations against the oracle, at their own sizes.

  * Whisper-tiny decoder at the decode bench's configuration: 32 sequences (and
    one), 4 prompt tokens, then 64 greedy decode steps at positions 4..67 over
    shared encoder states [1, 1500, 384], teacher-forced with the oracle's tokens
    so every step of every sequence is compared with the production (ARM)
    rounding of the reference. The B200 logits are bit-identical to the oracle's
    until a sequence's first Q8_0 rounding flip (an activation on a rounding
    boundary, moved by the attention's or a LayerNorm's fp32 order); after it
    the difference is at the quantization-noise level. The reference's own two
    builds differ at that same level at every step (the x86 quantizer,
    arch/x86/quants.c:302-350, against the ARM one, arch/arm/quants.c:41-75:
    1.0-1.4 % of the largest |logit| and 1.2 % of the greedy tokens on this
    workload), so the bars are: per step and sequence, max |logit difference|
    within max(1.5x the x86 build's, 1e-2) and within 2e-2 of the largest
    |logit|; the mean |logit difference| over all steps no larger than 1.5x the
    x86 build's; greedy tokens identical to the oracle's at least as often as the
    x86 build's are, every difference passing the harness's reciprocal top-5
    rule (testing/generation.py:25-57), and identical on every step before the
    sequence's first flip.
  * Free-running greedy generation at the same configuration, the harness's
    sequence policy (testing/generation.py:60-91): identical tokens through the
    first divergence, reciprocal top-5 at it.
  * Whisper-large-v3-shaped encoder (width 1280, 20 heads, mels 128, FFN 5120)
    cut to 2 layers, batch 2 x 1500 positions, against the encoder oracle with
    the same bars as the whisper-tiny encoder test (no farther from the ARM
    oracle than 1.5x the x86 oracle is; 3e-2 max / 3e-3 mean of the largest
    |output|).
  * Each large-v3 GEMM shape (QKV 3840x1280, out_proj 1280x1280, fc1 5120x1280,
    fc2 1280x5120) at the bench's 24,000 rows against the reference's own x86
    ggml mul_mat (quantize_row_q8_0 + vec_dot, oracle/_ref): within 2e-3 of the
    largest |output| (the GEMM bar: one fp16 rounding of each dequantized factor).
  * The thinker MoE layer at the prefill bench size (4096 tokens, 128 experts,
    top-8, I 768, H 2048), bf16 and Q8_0 experts, against the MoE oracle (pinned
    against transformers in tests/test_moe_oracle_pin.py): 2e-2 max / 2e-3 mean
    of the largest |output|.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


# ----------------------------------------------------------------------------- decoder
def _decoder_setup(B):
    from mstar_accelerators_b200.whisper import WhisperConfig, WhisperDecoderB200, synthetic_weights
    from oracle.whisper_oracle import WhisperDecoderOracle
    cfg = WhisperConfig()
    weights = synthetic_weights(cfg, seed=1)
    enc = torch.randn((1, cfg.source, cfg.d_model), generator=torch.Generator().manual_seed(2))
    prompt = np.random.default_rng(3).integers(0, cfg.vocab, (B, 4))
    dec = WhisperDecoderB200(weights, cfg, batch=B)
    arm = WhisperDecoderOracle(weights, cfg, batch=B, rounding="arm")
    x86 = WhisperDecoderOracle(weights, cfg, batch=B, rounding="x86")
    for o in (arm, x86):
        o.set_cross(enc.numpy())
    return cfg, enc, prompt, dec, arm, x86


@pytest.mark.parametrize("B", [32, 1])
def test_decoder_bench_configuration_teacher_forced(B):
    from oracle.whisper_oracle import greedy_agrees
    cfg, enc, prompt, dec, arm, x86 = _decoder_setup(B)
    agree_b200 = agree_x86 = decisions = 0
    mean_b200 = mean_x86 = 0.0
    exact_prefix = [True] * B

    def compare(got_l, got_t, la, ta, lx, tx):
        nonlocal agree_b200, agree_x86, decisions, mean_b200, mean_x86
        for b in range(B):
            finite = np.isfinite(la[b])
            assert np.array_equal(finite, np.isfinite(got_l[b]))
            scale = np.abs(la[b][finite]).max()
            d = np.abs(got_l[b][finite] - la[b][finite])
            spread = np.abs(lx[b][finite] - la[b][finite])
            if exact_prefix[b] and d.max() > 0:
                exact_prefix[b] = False      # this sequence's first rounding flip
            if exact_prefix[b]:
                assert int(got_t[b]) == int(ta[b])
            assert d.max() <= max(1.5 * spread.max(), 1e-2 * scale) and d.max() <= 2e-2 * scale, \
                (b, d.max(), spread.max(), scale)
            mean_b200 += d.mean() / scale
            mean_x86 += spread.mean() / scale
            assert greedy_agrees(int(got_t[b]), la[b], int(ta[b]), got_l[b])
            decisions += 1
            agree_b200 += int(got_t[b]) == int(ta[b])
            agree_x86 += int(tx[b]) == int(ta[b])

    logits, token = dec.prefill(torch.from_numpy(prompt).cuda(), enc.cuda())
    pos0 = np.tile(np.arange(4), (B, 1))
    la, ta = arm.forward(prompt, pos0, "prefill")
    lx, tx = x86.forward(prompt, pos0, "prefill")
    compare(logits.cpu().numpy(), token.cpu().numpy(), la, ta, lx, tx)
    tokens = ta.copy()
    for step in range(64):
        pos = 4 + step
        logits, token = dec.decode(torch.from_numpy(tokens).cuda(), torch.full((B,), pos, dtype=torch.int64))
        la, ta = arm.forward(tokens[:, None], np.full((B, 1), pos), "decode")
        lx, tx = x86.forward(tokens[:, None], np.full((B, 1), pos), "decode")
        compare(logits.cpu().numpy(), token.cpu().numpy(), la, ta, lx, tx)
        tokens = ta.copy()
    assert int(dec.status.cpu()[0]) == 0
    assert agree_b200 >= agree_x86 - 1, (agree_b200, agree_x86, decisions)
    assert mean_b200 <= 1.5 * mean_x86, (mean_b200 / decisions, mean_x86 / decisions)
    dec.close()


def test_decoder_bench_configuration_free_running_greedy():
    from oracle.whisper_oracle import greedy_agrees
    B = 32
    cfg, enc, prompt, dec, arm, _ = _decoder_setup(B)
    logits, token = dec.prefill(torch.from_numpy(prompt).cuda(), enc.cuda())
    la, ta = arm.forward(prompt, np.tile(np.arange(4), (B, 1)), "prefill")
    got_seq, ref_seq, got_l, ref_l = [token.cpu().numpy()], [ta], [logits.cpu().numpy()], [la]
    for step in range(64):
        pos = 4 + step
        logits, token = dec.decode(token, torch.full((B,), pos, dtype=torch.int64))
        la, ta = arm.forward(ta[:, None], np.full((B, 1), pos), "decode")
        got_seq.append(token.cpu().numpy())
        ref_seq.append(ta)
        got_l.append(logits.cpu().numpy())
        ref_l.append(la)
    identical = 0
    for b in range(B):
        for i in range(len(got_seq)):
            if int(got_seq[i][b]) != int(ref_seq[i][b]):
                assert greedy_agrees(int(got_seq[i][b]), ref_l[i][b], int(ref_seq[i][b]), got_l[i][b]), (b, i)
                break
        else:
            identical += 1
    assert identical >= B // 2, identical
    dec.close()


# ----------------------------------------------------------------------------- encoder
def test_large_v3_encoder_two_layers_match_oracle():
    from mstar_accelerators_b200.encoder import EncoderConfig, WhisperEncoderB200, synthetic_mel, synthetic_weights
    from oracle import whisper_encoder_oracle as EO
    cfg = EncoderConfig(mels=128, width=1280, heads=20, layers=2)
    w = synthetic_weights(cfg, seed=1)
    mel = synthetic_mel(cfg, 2, seed=2)
    enc = WhisperEncoderB200({k: v.cuda() for k, v in w.items()}, cfg, max_batch=2)
    got = enc(mel.cuda()).cpu().numpy()
    assert int(enc.status.cpu()[0]) == 0
    enc.close()
    wn = {k: v.numpy() for k, v in w.items()}
    ref = EO.WhisperEncoderOracle(wn, cfg, "arm").forward(mel.numpy())
    x86 = EO.WhisperEncoderOracle(wn, cfg, "x86").forward(mel.numpy())
    scale = np.abs(ref).max()
    diff, spread = np.abs(got - ref), np.abs(x86 - ref)
    assert diff.max() <= max(1.5 * spread.max(), 1e-3 * scale) and diff.max() <= 3e-2 * scale, (diff.max(), spread.max())
    assert diff.mean() <= 1.5 * spread.mean() and diff.mean() <= 3e-3 * scale, (diff.mean(), spread.mean())


@pytest.mark.parametrize("n,k", [(3840, 1280), (1280, 1280), (5120, 1280), (1280, 5120)])
def test_large_v3_gemm_shapes_at_24000_rows_match_ggml(n, k):
    from mstar_accelerators_b200 import linear
    m = 24000
    rng = np.random.default_rng(n + k)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((m, k)).astype(np.float32)
    lin = linear.BlockLinear(torch.from_numpy(w).cuda())
    lin.prepare_gemm(m)
    staged = linear.stage_rows(torch.from_numpy(x).cuda(), rounding="x86")
    got = lin.gemm(staged).cpu().numpy()
    lin.close()
    ref = O.ref_mul_mat(O.pack_weights(w), x, "q8_0")
    assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max()


# ----------------------------------------------------------------------------- MoE
@pytest.mark.parametrize("fmt", ["bf16", "q8_0"])
def test_moe_prefill_4096_matches_oracle(fmt):
    from mstar_accelerators_b200 import linear, moe
    from oracle import moe_oracle as M
    E, I, H, k, T = 128, 768, 2048, 8, 4096
    g = torch.Generator().manual_seed(3)
    w1 = (torch.randn((E, 2 * I, H), generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn((E, H, I), generator=g) * 0.02).to(torch.bfloat16)
    wr = (torch.randn((E, H), generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn((T, H), generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    xb = x.float().numpy()
    rw, rids, _ = M.route(xb, wr.float().numpy(), k)
    if fmt == "bf16":
        backend = moe.ThinkerMoEB200(w1.cuda(), w2.cuda(), fmt="bf16", top_k=k, max_tokens=T)
        ref = M.experts_bf16(xb, w1.float().numpy(), w2.float().numpy(), rw, rids)
    else:
        b1 = linear.pack(w1.float().reshape(-1, H).cuda(), "q8_0", preround=False).reshape(E, 2 * I, -1)
        b2 = linear.pack(w2.float().reshape(-1, I).cuda(), "q8_0", preround=False).reshape(E, H, -1)
        backend = moe.ThinkerMoEB200(b1, b2, fmt="q8_0", top_k=k, max_tokens=T, intermediate=I, hidden=H)
        ref = M.experts_q8(xb, b1.cpu().numpy(), b2.cpu().numpy(), rw, rids, I, H)
    got = backend(x.cuda(), torch.from_numpy(rw).cuda(), torch.from_numpy(rids).cuda()).float().cpu().numpy()
    assert int(backend.status.cpu()[0]) == 0
    backend.close()
    scale = np.abs(ref).max()
    diff = np.abs(got - ref)
    assert diff.max() <= 2e-2 * scale, (diff.max(), scale)
    assert diff.mean() <= 2e-3 * scale, (diff.mean(), scale)
