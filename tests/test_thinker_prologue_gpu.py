"""The thinker attention prologue in one launch (mstar_b200_qknorm_rope: QK RMSNorm,
prepared MRoPE, KV write) against the oracle restatement of the reference's fused op
(oracle/thinker_oracle.py): q / k heads equal the oracle's bit for bit except where the
sum of squares' fp32 order moves a value across a bf16 rounding boundary (at most
1 % of the values, each within a few bf16 steps of the head's largest value); v rows are copied exactly into the
cache rows the slot table names; a slot outside the cache sets status bit 1 and
writes nothing."""
import numpy as np
import pytest
import torch

from oracle import thinker_oracle as TO
from oracle.moe_oracle import bf16

pytestmark = pytest.mark.gpu


def close(got, want):
    d = np.abs(got - want)
    assert (d == 0).mean() >= 0.99, (d == 0).mean()
    # a moved bf16 rounding of n, a or b shifts y by a few bf16 steps of those terms,
    # which are at most the head's largest |y| in size
    assert np.all(d <= 2 ** -6 * np.abs(want).max(axis=-1, keepdims=True)), d.max()


@pytest.mark.parametrize("T,round_products", [(1, True), (8, True), (300, True), (40, False)])
def test_prologue_matches_oracle(T, round_products):
    from mstar_accelerators_b200 import thinker
    rng = np.random.default_rng(T)
    Hq, Hk = 32, 4
    qkv = bf16(rng.standard_normal((T, (Hq + 2 * Hk) * 128)) * 2)       # one fused projection row per token
    qw, kw = bf16(1 + 0.1 * rng.standard_normal(128)), bf16(1 + 0.1 * rng.standard_normal(128))
    ang = rng.uniform(0, 200, (T, 64))
    cos = bf16(np.cos(np.concatenate([ang, ang], -1)))
    sin = bf16(np.sin(np.concatenate([ang, ang], -1)))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda().to(torch.bfloat16)
    x = dev(qkv)
    q = x[:, :Hq * 128].view(T, Hq, 128)
    k = x[:, Hq * 128:(Hq + Hk) * 128].view(T, Hk, 128)
    v = x[:, (Hq + Hk) * 128:].view(T, Hk, 128)
    slots_np = rng.permutation(512)[:T]
    kc = torch.zeros((512, Hk, 128), dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    oq, kc = thinker.qknorm_rope(q, k, dev(qw), dev(kw), dev(cos), dev(sin), eps=1e-6, round_products=round_products,
                                 v=v, k_cache=kc, v_cache=vc, slots=torch.from_numpy(slots_np).cuda(), status=status)
    rq, rk = TO.qknorm_rope(qkv[:, :Hq * 128].reshape(T, Hq, 128), qkv[:, Hq * 128:(Hq + Hk) * 128].reshape(T, Hk, 128),
                            qw, kw, cos, sin, eps=1e-6, round_products=round_products)
    assert int(status.item()) == 0
    close(oq.float().cpu().numpy(), rq)
    close(kc[slots_np].float().cpu().numpy(), rk)
    np.testing.assert_array_equal(vc[slots_np].float().cpu().numpy(), qkv[:, (Hq + Hk) * 128:].reshape(T, Hk, 128))
    untouched = np.setdiff1d(np.arange(512), slots_np)
    assert not kc[untouched].any() and not vc[untouched].any()


def test_out_of_range_slot_sets_status():
    from mstar_accelerators_b200 import thinker
    T, Hq, Hk = 2, 32, 4
    q = torch.randn(T, Hq, 128, device="cuda").to(torch.bfloat16)
    k = torch.randn(T, Hk, 128, device="cuda").to(torch.bfloat16)
    w = torch.ones(128, device="cuda", dtype=torch.bfloat16)
    cs = torch.ones(T, 128, device="cuda", dtype=torch.bfloat16)
    kc = torch.zeros((4, Hk, 128), dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    thinker.qknorm_rope(q, k, w, w, cs, cs, k_cache=kc, slots=torch.tensor([1, 9], device="cuda"), status=status)
    assert int(status.item()) & 1 and kc[1].any() and not kc[[0, 2, 3]].any()


@pytest.mark.parametrize("T", [1, 37, 300])
def test_fp32_rows_equal_their_bf16_rounding(T):
    """mstar_b200_qknorm_rope_f32 on the fp32 projection output gives, bit for bit, what
    mstar_b200_qknorm_rope gives on its .to(bfloat16): q, the k cache rows and the v copies."""
    from mstar_accelerators_b200 import thinker
    g = torch.Generator(device="cuda").manual_seed(T)
    Hq, Hk = 32, 4
    x32 = torch.randn((T, (Hq + 2 * Hk) * 128), device="cuda", generator=g) * 2
    w = (1 + 0.1 * torch.randn((2, 128), device="cuda", generator=g)).to(torch.bfloat16)
    ang = torch.rand((T, 64), device="cuda", generator=g) * 200
    cos = torch.cos(torch.cat([ang, ang], -1)).to(torch.bfloat16)
    sin = torch.sin(torch.cat([ang, ang], -1)).to(torch.bfloat16)
    slots = torch.randperm(512, device="cuda", generator=g)[:T]
    outs = []
    for x in (x32, x32.to(torch.bfloat16)):
        q = x[:, :Hq * 128].view(T, Hq, 128)
        k = x[:, Hq * 128:(Hq + Hk) * 128].view(T, Hk, 128)
        v = x[:, (Hq + Hk) * 128:].view(T, Hk, 128)
        kc = torch.zeros((512, Hk, 128), dtype=torch.bfloat16, device="cuda")
        vc = torch.zeros_like(kc)
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        oq, kc = thinker.qknorm_rope(q, k, w[0], w[1], cos, sin, eps=1e-6, v=v, k_cache=kc, v_cache=vc, slots=slots,
                                     status=status)
        assert int(status.item()) == 0
        outs.append((oq, kc, vc))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_mixed_input_dtypes_are_rejected():
    from mstar_accelerators_b200 import thinker
    q = torch.zeros((2, 4, 128), device="cuda")
    k = torch.zeros((2, 1, 128), device="cuda", dtype=torch.bfloat16)
    w = torch.ones(128, device="cuda", dtype=torch.bfloat16)
    cs = torch.ones(2, 128, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        thinker.qknorm_rope(q, k, w, w, cs, cs)
