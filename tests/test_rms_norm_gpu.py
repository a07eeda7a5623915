"""The thinker layer's RMSNorm in one launch (mstar_b200_rms_norm) against transformers'
Qwen3OmniMoeThinkerTextRMSNorm written in torch (fp32 normalisation, bf16 before the weight,
the reference's input / post-attention norms, implementations/qwen3_omni/amd/
thinker_model.py:106-148). The kernel sums the squares in another order than torch's
reduction, so the mean can move in the last bit: at most 1e-3 of the outputs may sit one
bf16 step away, none further; the fp32 output carries exactly the bf16 output's values.
The layer's bf16 residual add of an fp32 projection (mstar_b200_residual_add_bf16) equals
torch's x + v.to(bf16) bit for bit."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _torch_rms(x, w, eps):
    h = x.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return w * h.to(x.dtype)


@pytest.mark.parametrize("rows,width", [(32, 2048), (37, 2048), (5, 4096), (300, 128), (1, 8)])
def test_rms_norm_matches_torch(rows, width):
    from mstar_accelerators_b200.thinker_stack import rms_norm
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + width)
    x = (torch.randn((rows, width), device="cuda", generator=g) * 3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(width, device="cuda", generator=g)).to(torch.bfloat16)
    ref = _torch_rms(x, w, 1e-6)
    got = rms_norm(x, w, 1e-6)
    got32 = rms_norm(x, w, 1e-6, f32=True)
    assert got.dtype == torch.bfloat16 and got32.dtype == torch.float32
    assert torch.equal(got32, got.float())
    diff = (got.float() - ref.float()).abs()
    step = ref.float().abs().clamp_min(1e-30) * 2.0 ** -7   # one bf16 step at the value
    assert (diff > 0).float().mean().item() <= 1e-3
    assert bool((diff <= step * 1.01).all())


def test_rms_norm_rejects_unaligned_widths():
    from mstar_accelerators_b200.native import NativeError
    from mstar_accelerators_b200.thinker_stack import rms_norm
    x = torch.zeros((4, 12), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(NativeError):
        rms_norm(x, torch.ones(12, dtype=torch.bfloat16, device="cuda"), 1e-6)


@pytest.mark.parametrize("n", [8, 32 * 2048, 1000 * 8])
def test_residual_add_equals_torch(n):
    """mstar_b200_residual_add_bf16 is torch's x + v.to(bf16) bit for bit."""
    from mstar_accelerators_b200.thinker_stack import residual_add
    g = torch.Generator(device="cuda").manual_seed(n)
    x = torch.randn(n, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(n, device="cuda", generator=g) * 0.3
    assert torch.equal(residual_add(x, v), x + v.to(torch.bfloat16))
