"""Thinker attention-prologue linears as Q8_0 B200 contractions.

Q8LinearB200 is ggml_mul_mat(Q8_0 W, x): bit-identical to the oracle for decode
row counts (the GEMV path) and within the fp16-product tolerance of the tcgen05
GEMM for prefill row counts, at the thinker's shapes (q 4096 x 2048, k / v
512 x 2048, o_proj 2048 x 4096). install_thinker_attention_linears on
transformers' Qwen3OmniMoeThinkerTextAttention replaces its four projections
and the layer's output stays within the Q8_0 quantization error of the bf16
layer.
"""
import types

import numpy as np
import pytest
import torch
from torch import nn

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def T():
    from mstar_accelerators_b200 import thinker
    O.build()
    return thinker


@pytest.mark.parametrize("n,k", [(512, 2048), (2048, 4096)])
@pytest.mark.parametrize("rows", [1, 7, 32])
def test_decode_rows_are_bit_exact(T, n, k, rows):
    g = torch.Generator(device="cuda").manual_seed(n + rows)
    lin = nn.Linear(k, n, bias=False).cuda()
    with torch.no_grad():
        lin.weight.copy_(torch.randn((n, k), device="cuda", generator=g) * 0.02)
    q8 = T.Q8LinearB200(lin)
    x = torch.randn((rows, k), device="cuda", generator=g)
    got = q8(x).cpu().numpy()
    ref = O.mul_mat(q8.lin.blocks.cpu().numpy(), x.cpu().numpy(), "q8_0")
    assert np.array_equal(got, ref)
    q8.close()


def test_prefill_rows_on_the_gemm(T):
    g = torch.Generator(device="cuda").manual_seed(3)
    lin = nn.Linear(2048, 4096, bias=False).cuda()
    with torch.no_grad():
        lin.weight.copy_(torch.randn((4096, 2048), device="cuda", generator=g) * 0.02)
    q8 = T.Q8LinearB200(lin, gemm_rows=256)
    x = torch.randn((300, 2048), device="cuda", generator=g)   # a 256-row GEMM chunk, then a 44-row GEMV chunk
    got = q8(x).cpu().numpy()
    ref = O.mul_mat(q8.lin.blocks.cpu().numpy(), x.cpu().numpy(), "q8_0")
    assert np.array_equal(got[256:], ref[256:])
    np.testing.assert_allclose(got[:256], ref[:256], rtol=2e-3, atol=2e-3 * np.abs(ref).max())
    q8.close()


def test_install_on_the_transformers_attention(T):
    mod = pytest.importorskip("transformers.models.qwen3_omni_moe.modeling_qwen3_omni_moe")
    cfg = types.SimpleNamespace(hidden_size=512, num_attention_heads=8, num_key_value_heads=2, head_dim=64,
                                attention_bias=False, attention_dropout=0.0, rms_norm_eps=1e-6,
                                _attn_implementation="eager")
    torch.manual_seed(0)
    attn = mod.Qwen3OmniMoeThinkerTextAttention(cfg, layer_idx=0).cuda().to(torch.bfloat16).eval()
    with torch.no_grad():
        for p in attn.parameters():
            if p.dim() == 2:
                p.copy_(torch.randn_like(p) * 0.02)
    x = torch.randn((2, 40, 512), device="cuda", dtype=torch.bfloat16)
    pos = torch.arange(40, device="cuda", dtype=torch.float32)
    inv = 1.0 / (10000 ** (torch.arange(0, 64, 2, device="cuda", dtype=torch.float32) / 64))
    ang = torch.outer(pos, inv)
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos()[None].to(torch.bfloat16), emb.sin()[None].to(torch.bfloat16)
    with torch.no_grad():
        ref, _ = attn(x, (cos, sin), None)
        assert T.install_thinker_attention_linears(attn) == 4
        assert isinstance(attn.q_proj, T.Q8LinearB200) and isinstance(attn.o_proj, T.Q8LinearB200)
        got, _ = attn(x, (cos, sin), None)
    err = (got.float() - ref.float()).norm() / ref.float().norm()
    assert err.item() < 3e-2
