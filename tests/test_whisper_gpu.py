"""Whisper-tiny decoder on the B200 kernels against the oracle composition of
the reference graph (oracle/whisper_oracle.py).

Fidelity bar: logits within 1e-2 relative to the oracle's largest |logit|
(the stated fidelity bar for logits) and greedy tokens accepted by the
reference harness's policy (testing/generation.py:25-89: the same token, or
reciprocal top-5, compared through the first divergence). Sequences are
teacher-forced with the oracle's tokens so every step is compared.
"""
import numpy as np
import pytest
import torch

from oracle.whisper_oracle import WhisperDecoderOracle, greedy_agrees

pytestmark = pytest.mark.gpu
REL_TOL = 1e-2


@pytest.fixture(scope="module")
def setup():
    from mstar_accelerators_b200.whisper import WhisperConfig, synthetic_weights
    cfg = WhisperConfig()
    weights = synthetic_weights(cfg, seed=1)
    g = torch.Generator().manual_seed(2)
    enc = torch.randn((1, cfg.source, cfg.d_model), generator=g)
    return cfg, weights, enc


def check_logits(got, ref):
    scale = np.abs(ref[np.isfinite(ref)]).max()
    finite = np.isfinite(ref)
    assert np.array_equal(finite, np.isfinite(got))
    assert np.abs(got[finite] - ref[finite]).max() <= REL_TOL * scale


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_decoder_prefill_and_decode_match_oracle(setup, fmt):
    from mstar_accelerators_b200.whisper import WhisperDecoderB200
    cfg, weights, enc = setup
    B = 2
    sup = {"prefill": [50257, 220], "decode": [50257]}
    dec = WhisperDecoderB200(weights, cfg, batch=B, readout_format=fmt, suppressed=sup)
    ref = WhisperDecoderOracle(weights, cfg, batch=B, readout_format=fmt, suppressed=sup)
    ref.set_cross(enc.numpy())
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, cfg.vocab, (B, 4))
    logits, token = dec.prefill(torch.from_numpy(prompt).cuda(), enc.cuda())
    rl, rt = ref.forward(prompt, np.tile(np.arange(4), (B, 1)), "prefill")
    got_l, got_t = logits.cpu().numpy(), token.cpu().numpy()
    assert int(dec.status.cpu()[0]) == 0
    for b in range(B):
        check_logits(got_l[b], rl[b])
        assert greedy_agrees(int(got_t[b]), rl[b], int(rt[b]), got_l[b])
    tokens = rt.copy()
    for step in range(6):
        pos = 4 + step
        logits, token = dec.decode(torch.from_numpy(tokens).cuda(), torch.full((B,), pos, dtype=torch.int64))
        rl, rt = ref.forward(tokens[:, None], np.full((B, 1), pos), "decode")
        got_l, got_t = logits.cpu().numpy(), token.cpu().numpy()
        for b in range(B):
            check_logits(got_l[b], rl[b])
            assert greedy_agrees(int(got_t[b]), rl[b], int(rt[b]), got_l[b])
        tokens = rt.copy()
    assert int(dec.status.cpu()[0]) == 0
    dec.close()


def test_graph_replay_equals_eager_steps(setup):
    from mstar_accelerators_b200.whisper import GraphDecoder, WhisperDecoderB200
    cfg, weights, enc = setup
    B = 4
    rng = np.random.default_rng(4)
    prompt = torch.from_numpy(rng.integers(0, cfg.vocab, (B, 4))).cuda()
    eager = WhisperDecoderB200(weights, cfg, batch=B)
    _, tok = eager.prefill(prompt, enc.cuda())
    seq_eager = []
    t = tok.clone()
    for step in range(5):
        _, t = eager.decode(t, torch.full((B,), 4 + step, dtype=torch.int64))
        seq_eager.append(t.cpu().numpy().copy())
    graphed = WhisperDecoderB200(weights, cfg, batch=B)
    _, tok2 = graphed.prefill(prompt, enc.cuda())
    assert torch.equal(tok, tok2)
    gd = GraphDecoder(graphed)
    gd.tokens.copy_(tok2)
    gd.positions.fill_(4)
    gd.capture()
    seq_graph = []
    for _ in range(5):
        gd.run(1)
        seq_graph.append(gd.tokens.cpu().numpy().copy())
    assert all(np.array_equal(a, b) for a, b in zip(seq_eager, seq_graph))
    eager.close()
    graphed.close()


def test_batch_rows_are_independent(setup):
    """Sequence b of a batch decodes exactly like the same sequence alone."""
    from mstar_accelerators_b200.whisper import WhisperDecoderB200
    cfg, weights, enc = setup
    rng = np.random.default_rng(5)
    prompt = torch.from_numpy(rng.integers(0, cfg.vocab, (3, 4))).cuda()
    many = WhisperDecoderB200(weights, cfg, batch=3)
    one = WhisperDecoderB200(weights, cfg, batch=1)
    l3, t3 = many.prefill(prompt, enc.cuda())
    l1, t1 = one.prefill(prompt[1:2], enc.cuda())
    assert torch.equal(l3[1], l1[0]) and int(t3[1]) == int(t1[0])
    many.close()
    one.close()


@pytest.mark.parametrize("B,fmt,shared", [(32, "q4_0", True), (5, "q8_0", True), (3, "q4_0", False)])
def test_persistent_step_equals_multi_launch_step(setup, B, fmt, shared):
    """The one-kernel decode step (mstar_b200_decode_step_*) produces the same
    logits, bit for bit, and the same tokens as the multi-launch step on the same
    state, over several steps with the tokens fed back; a captured graph of the
    persistent step replays it."""
    from mstar_accelerators_b200.whisper import GraphDecoder, WhisperDecoderB200
    cfg, weights, enc = setup
    rng = np.random.default_rng(B)
    prompt = torch.from_numpy(rng.integers(0, cfg.vocab, (B, 4))).cuda()
    encs = enc.cuda() if shared else enc.cuda().repeat(B, 1, 1)
    ref_dec = WhisperDecoderB200(weights, cfg, batch=B, readout_format=fmt, shared_cross=shared)
    _, tok = ref_dec.prefill(prompt, encs)
    one = WhisperDecoderB200(weights, cfg, batch=B, readout_format=fmt, shared_cross=shared)
    _, tok1 = one.prefill(prompt, encs)
    assert torch.equal(tok, tok1)
    ref = GraphDecoder(ref_dec)
    per = GraphDecoder(one, persistent=True)
    for gd in (ref, per):
        gd.tokens.copy_(tok)
        gd.positions.fill_(4)
    for step in range(3):
        ref._step()
        per._step()
        torch.cuda.synchronize()
        assert torch.equal(ref.logits, per.logits), step
        assert torch.equal(ref.tokens, per.tokens), step
    assert int(one.status.item()) == 0
    per.capture()
    ref.capture()
    for step in range(3):
        ref.run(1)
        per.run(1)
        torch.cuda.synchronize()
        assert torch.equal(ref.logits, per.logits), ("graph", step)
        assert torch.equal(ref.tokens, per.tokens), ("graph", step)
    per.step.close()
    ref_dec.close()
    one.close()
