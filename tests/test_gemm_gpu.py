"""tcgen05 GEMM (prefill / encoder shapes) against the oracle and against the
same fp16-dequantized operands multiplied in fp32.

Tolerance: the GEMM multiplies fp16(q*d) operands, so each product carries one
fp16 rounding of its two factors; outputs must be within 2e-3 of the oracle's
largest |output| (well inside the 1e-2 logits bar), and within 1e-5 relative of
an fp32 matmul of the very same fp16 operands (accumulation order only).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def dequant(blocks, fmt):
    return O.dequantize(blocks, fmt).astype(np.float16).astype(np.float32)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("m,n,k", [(64, 256, 64), (128, 256, 384), (200, 384, 384), (1500, 1152, 384),
                                   (333, 384, 1536), (256, 3072, 384)])
def test_gemm_matches_oracle(fmt, m, n, k):
    from mstar_accelerators_b200 import linear
    rng = np.random.default_rng(m + n + k)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((m, k)).astype(np.float32)
    lin = linear.BlockLinear(dev(w), fmt=fmt)
    lin.prepare_gemm(max(m, 64))
    got = lin(dev(x)).cpu().numpy()
    blocks = O.pack_weights(w, fmt)
    ref = O.mul_mat(blocks, x, fmt)
    assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max()
    # same operands in fp32: only the accumulation order differs
    xq = O.dequantize(O.quantize_q8_0(x, "arm"), "q8_0").astype(np.float16).astype(np.float32)
    exact = torch.from_numpy(xq).double() @ torch.from_numpy(dequant(blocks, fmt)).double().T
    np.testing.assert_allclose(got, exact.numpy(), rtol=1e-4, atol=1e-4 * np.abs(ref).max())
    lin.close()


def test_gemm_epilogues():
    from mstar_accelerators_b200 import linear
    rng = np.random.default_rng(1)
    m, n, k = 300, 1536, 384
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    x = rng.standard_normal((m, k)).astype(np.float32)
    res = rng.standard_normal((m, n)).astype(np.float32)
    lin = linear.BlockLinear(dev(w), bias=dev(b))
    lin.prepare_gemm(m)
    base = O.mul_mat(O.pack_weights(w), x) + b
    tol = 2e-3 * np.abs(base).max()
    assert np.abs(lin(dev(x)).cpu().numpy() - base).max() <= tol
    assert np.abs(lin(dev(x), residual=dev(res)).cpu().numpy() - (res + base)).max() <= tol
    g = lin(dev(x), gelu="tanh").cpu().numpy()
    assert np.abs(g - O.gelu_ggml(base)).max() <= 2 * tol
    lin.close()


def test_gemm_and_gemv_agree_on_prefill_rows():
    """The same handle answers 64+ rows with the GEMM and <=32 rows with the GEMV."""
    from mstar_accelerators_b200 import linear
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((384, 384)) * 0.02).astype(np.float32)
    x = rng.standard_normal((96, 384)).astype(np.float32)
    lin = linear.BlockLinear(dev(w))
    gemv = lin(dev(x)).cpu().numpy()          # not prepared yet: GEMV chunks (bit-exact)
    lin.prepare_gemm(96)
    gemm = lin(dev(x)).cpu().numpy()
    assert np.array_equal(gemv, O.mul_mat(O.pack_weights(w), x))
    assert np.abs(gemm - gemv).max() <= 2e-3 * np.abs(gemv).max()
    lin.close()
