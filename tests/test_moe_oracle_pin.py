"""Pins the MoE oracle (oracle/moe_oracle.py) against the reference's own MoE
oracle: transformers' eager Qwen3OmniMoeThinkerTextSparseMoeBlock (the class the
reference drives in testing/models/qwen3_omni_hf.py:16-53 and
testing/models/qwen_node_reference.py:148-163), run here on the CPU on seeded
bf16 weights. transformers 5.5 is installed; the reference pins 4.57.3
(pyproject.toml:16), whose eager block has the same router and expert steps.

  * router: probabilities within 1e-7, renormalised top-k weights within 1e-7,
    the same expert set wherever the k-th and (k+1)-th probabilities differ
    (bf16 logits tie often; the tie order is torch.topk's);
  * experts, HF rounding points (``experts_bf16_hf``): bit-identical to the
    block's output on >= 99 % of the values; the rest differ by a few bf16 steps
    (float32 vs float64 accumulation of a dot can round g, u or mid to the other
    bf16 neighbour, which moves that pair's whole output row), so max <= 1.5e-2
    and mean <= 2e-5 of the largest |output| (40x tighter on average than the
    distance between the two sets of rounding points below);
  * experts, the reference kernel's rounding points (``experts_bf16``,
    thinker_moe.py:17-101: no bf16 rounding of the down output before the
    routing weight, slot-order fp32 sum instead of a bf16 running sum): within
    2e-2 (max) and 2e-3 (mean) of the largest |output| of the HF block -- the
    tolerance the B200 MoE tests use against this oracle.
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as M


def hf_block(H, E, I, k, seed):
    from transformers.models.qwen3_omni_moe import configuration_qwen3_omni_moe as C
    from transformers.models.qwen3_omni_moe import modeling_qwen3_omni_moe as MM
    cfg = C.Qwen3OmniMoeTextConfig(hidden_size=H, num_experts=E, moe_intermediate_size=I, num_experts_per_tok=k,
                                   norm_topk_prob=True, hidden_act="silu")
    cfg._experts_implementation = "eager"
    blk = MM.Qwen3OmniMoeThinkerTextSparseMoeBlock(cfg)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        blk.experts.gate_up_proj.copy_(torch.randn(E, 2 * I, H, generator=g) * 0.02)
        blk.experts.down_proj.copy_(torch.randn(E, H, I, generator=g) * 0.02)
        blk.gate.weight.copy_(torch.randn(E, H, generator=g) * 0.02)
    return blk.to(torch.bfloat16).eval(), g


def np32(t):
    return t.detach().float().numpy()


@pytest.mark.parametrize("H,E,I,k,T", [(256, 16, 128, 4, 64), (1024, 128, 256, 8, 48)])
def test_moe_oracle_matches_transformers(H, E, I, k, T):
    blk, g = hf_block(H, E, I, k, seed=11 + H)
    x = torch.randn(1, T, H, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        out = np32(blk(x)[0])
        probs, scores, idx = blk.gate(x.view(-1, H))
    xb, wr = np32(x[0]), np32(blk.gate.weight)
    w1, w2 = np32(blk.experts.gate_up_proj), np32(blk.experts.down_proj)

    # router
    rw, rids, p = M.route(xb, wr, k)
    np.testing.assert_allclose(p, np32(probs), rtol=0, atol=1e-7)
    np.testing.assert_allclose(np.sort(rw, 1), np.sort(np32(scores), 1), rtol=0, atol=1e-7)
    ps = -np.sort(-p, axis=-1)
    untied = ps[:, k - 1] > ps[:, k]
    assert untied.mean() > 0.5
    for t in np.nonzero(untied)[0]:
        assert set(rids[t]) == set(idx[t].tolist())

    # experts, driven with the block's own routing
    hw, hids = np32(scores), idx.numpy().astype(np.int32)
    scale = np.abs(out).max()
    hf = M.experts_bf16_hf(xb, w1, w2, hw, hids)
    d = np.abs(hf - out)
    assert (d == 0).mean() >= 0.99 and d.max() <= 1.5e-2 * scale and d.mean() <= 2e-5 * scale, \
        ((d == 0).mean(), d.max() / scale, d.mean() / scale)
    ref = M.experts_bf16(xb, w1, w2, hw, hids)
    d = np.abs(ref - out)
    assert d.max() <= 2e-2 * scale and d.mean() <= 2e-3 * scale, (d.max() / scale, d.mean() / scale)


def test_grouped_oracle_equals_per_pair_order():
    """The oracle contracts each expert's pairs together; a pair-by-pair evaluation in
    token order (the shape of thinker_moe.py's per-slot grid) gives the same bits."""
    rng = np.random.default_rng(0)
    E, I, H, k, T = 8, 64, 128, 4, 19
    w1 = M.bf16(rng.standard_normal((E, 2 * I, H)) * 0.02)
    w2 = M.bf16(rng.standard_normal((E, H, I)) * 0.02)
    x = M.bf16(rng.standard_normal((T, H)))
    rw, rids, _ = M.route(x, M.bf16(rng.standard_normal((E, H)) * 0.02), k)
    out = np.zeros((T, H), np.float32)
    for t in range(T):
        acc = np.zeros(H, np.float32)
        for s in range(k):
            e = int(rids[t, s])
            gg = M.bf16((w1[e, :I].astype(np.float64) @ x[t]).astype(np.float32))
            uu = M.bf16((w1[e, I:].astype(np.float64) @ x[t]).astype(np.float32))
            mid = M._swiglu(gg, uu)
            y = (w2[e].astype(np.float64) @ mid).astype(np.float32)
            acc = (acc + M.bf16((y * rw[t, s]).astype(np.float32))).astype(np.float32)
        out[t] = M.bf16(acc)
    np.testing.assert_array_equal(M.experts_bf16(x, w1, w2, rw, rids), out)
