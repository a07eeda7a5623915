"""The thinker decoder stack on B200 (mstar_accelerators_b200.thinker_stack: Q8_0 fused QKV
and o_proj, the one-launch QK-norm / RoPE / KV write, SDPA over the bf16 cache, the
grouped MoE kernels, the Q8_0 lm_head readout) against the oracle composition
(oracle/thinker_oracle.ThinkerStackOracle) at a reduced geometry (2 layers, hidden
256, 4 query / 2 KV heads of 128, 16 experts top-4, vocabulary 1000): prefill of 3
sequences x 70 tokens (the prefill linears on the tcgen05 GEMM), then 4 decode steps
teacher-forced with the oracle's tokens (the decode linears on the bit-exact GEMV), the
whole decode step replayed as one captured CUDA graph; a second stack stepping eagerly
gives the graph's logits bit for bit.
The bf16 residual stream, bf16 MoE and Q8_0 activations put both sides at the
quantization-noise level of each other after the first layer, so logits are held
within 5e-2 of the largest |logit| (mean 1e-2) and greedy tokens to the harness's
policy (the same token, or reciprocal top-5; testing/generation.py:25-57)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("experts", ["q8_0", "bf16"])
def test_stack_matches_oracle(experts):
    from mstar_accelerators_b200.thinker_stack import ThinkerStackB200, ThinkerStackConfig, head_weights, layer_weights
    from oracle.thinker_oracle import ThinkerStackOracle
    from oracle.whisper_oracle import greedy_agrees
    cfg = ThinkerStackConfig(hidden=256, layers=2, q_heads=4, kv_heads=2, experts=16, top_k=4, moe_intermediate=128,
                             vocab=1000)
    layers = [layer_weights(cfg, i, seed=3) for i in range(cfg.layers)]
    stack = ThinkerStackB200(cfg, max_seqs=3, max_len=80, seed=3, experts=experts, gemm_rows=256,
                             weights=lambda i: layers[i])
    ref = ThinkerStackOracle(cfg, layers, head_weights(cfg, seed=3), experts=experts)
    tokens = np.random.default_rng(4).integers(0, cfg.vocab, (3, 70))

    def check(got, want):
        gl, gt = got[0].cpu().numpy(), got[1].cpu().numpy()
        rl, rt = want
        scale = np.abs(rl).max()
        assert np.abs(gl - rl).max() <= 5e-2 * scale and np.abs(gl - rl).mean() <= 1e-2 * scale, \
            (np.abs(gl - rl).max() / scale, np.abs(gl - rl).mean() / scale)
        for b in range(len(gt)):
            assert greedy_agrees(int(gt[b]), rl[b], int(rt[b]), gl[b])
        return rt

    eager = ThinkerStackB200(cfg, max_seqs=3, max_len=80, seed=3, experts=experts, gemm_rows=256,
                             weights=lambda i: layers[i])
    nxt = check(stack.prefill(torch.from_numpy(tokens).cuda()), ref.prefill(tokens))
    eager.prefill(torch.from_numpy(tokens).cuda())
    for _ in range(4):
        got = stack.decode(torch.from_numpy(nxt).cuda(), graph=True)
        logits = got[0].clone()
        e_logits, _ = eager.decode(torch.from_numpy(nxt).cuda())
        assert torch.equal(logits, e_logits)
        nxt = check(got, ref.decode(nxt))
    assert int(stack.status.item()) == 0 and int(eager.status.item()) == 0
    stack.close()
    eager.close()
