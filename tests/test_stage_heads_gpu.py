"""The thinker prefill's attention-output staging in one pass (mstar_b200_stage_heads):
bf16 [seqs, heads, positions, 128] as scaled_dot_product_attention returns it (before the
transpose of implementations/qwen3_omni/amd/thinker_model.py:106-148) -> the o_proj GEMM's
Q8_0-staged operand. It must write the bytes that mstar_b200_stage_rows writes for the
transposed fp32 rows, in every rounding and for strided (already transposed) inputs, and
o_proj through it must equal the linear's own path on those rows bit for bit."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _attention(shape, seed, transposed=False):
    g = torch.Generator(device="cuda").manual_seed(seed)
    S, H, n, D = shape
    if transposed:   # [S, n, H, D] storage viewed as [S, H, n, D]
        return (torch.randn((S, n, H, D), device="cuda", generator=g) * 0.7).to(torch.bfloat16).transpose(1, 2)
    return (torch.randn(shape, device="cuda", generator=g) * 0.7).to(torch.bfloat16)


@pytest.mark.parametrize("shape", [(3, 4, 70, 128), (1, 2, 5, 64), (2, 32, 33, 128), (1, 1, 1, 32)])
@pytest.mark.parametrize("rounding", ["arm", "x86", "ref"])
def test_stage_heads_equals_row_staging(shape, rounding):
    from mstar_accelerators_b200.linear import stage_heads, stage_rows
    att = _attention(shape, seed=sum(shape))
    S, H, n, D = shape
    rows = att.transpose(1, 2).reshape(S * n, H * D).float()
    assert torch.equal(stage_heads(att, rounding=rounding), stage_rows(rows, rounding=rounding))


def test_stage_heads_strided_input():
    from mstar_accelerators_b200.linear import stage_heads, stage_rows
    att = _attention((2, 8, 40, 128), seed=5, transposed=True)
    assert not att.is_contiguous()
    rows = att.transpose(1, 2).reshape(80, 1024).float()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert torch.equal(stage_heads(att, status=status), stage_rows(rows))
    assert int(status.item()) == 0


def test_stage_heads_flags_non_finite_values():
    from mstar_accelerators_b200.linear import stage_heads
    att = _attention((1, 2, 4, 64), seed=9)
    att[0, 1, 2, 7] = float("inf")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stage_heads(att, status=status)
    assert int(status.item()) & 1


def test_stage_heads_rejects_bad_layouts():
    from mstar_accelerators_b200.linear import stage_heads
    from mstar_accelerators_b200.native import NativeError
    with pytest.raises(NativeError):   # head_dim not a multiple of 32
        stage_heads(torch.zeros((1, 2, 4, 48), dtype=torch.bfloat16, device="cuda"))
    base = torch.zeros((1, 2, 4, 66), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(NativeError):   # rows of 66 elements: a stride that is not a multiple of 4
        stage_heads(base[..., :64])


@pytest.mark.parametrize("seqs,positions", [(2, 100), (3, 70)])
def test_o_proj_through_head_staging_is_the_linear(seqs, positions):
    """The thinker's prefill o_proj (stage_heads + the prepared GEMM) gives the linear's own
    result on the transposed fp32 rows (its row staging + the same GEMM) bit for bit."""
    from mstar_accelerators_b200.linear import BlockLinear, stage_heads
    g = torch.Generator(device="cuda").manual_seed(seqs * positions)
    heads, D, hidden = 4, 128, 256
    lin = BlockLinear(torch.randn((hidden, heads * D), device="cuda", generator=g) * 0.02)
    lin.prepare_gemm(256)
    att = _attention((seqs, heads, positions, D), seed=positions)
    rows = att.transpose(1, 2).reshape(seqs * positions, heads * D).float()
    want = lin(rows)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    got = lin.gemm(stage_heads(att, status=status), bias=False, status=status)
    assert torch.equal(got, want)
    assert int(status.item()) == 0
    lin.close()
