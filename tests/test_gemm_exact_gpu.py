"""The exact Q8_0 GEMM (mstar_b200_gemm_q8_exact: one tcgen05 kind::i8 MMA per 32-element
block, the blocks rescaled and summed in ggml's generic order on the CUDA cores) is
bit-identical to the oracle's generic-order mul_mat (ggml-cpu/quants.c:451-480) and to
the decode GEMV at every row count -- including ragged rows, ragged columns, a block
count that leaves a partial 4-block stage, and the Whisper-large-v3 fc1 shape at the
bench's 24,000 rows."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("m,n,k", [(1, 384, 384), (7, 200, 64), (200, 1536, 384), (333, 384, 1536), (130, 256, 416),
                                   (1000, 1152, 384)])
@pytest.mark.parametrize("mode", ["arm", "x86"])
def test_exact_gemm_is_bit_identical_to_oracle(m, n, k, mode):
    from mstar_accelerators_b200 import linear
    rng = np.random.default_rng(m * 7 + n + k)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    x = (rng.standard_normal((m, k)) * 2).astype(np.float32)
    lin = linear.BlockLinear(dev(w), bias=dev(b))
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    got = lin.exact(dev(x), rounding=mode, status=st).cpu().numpy()
    assert int(st.item()) == 0
    ref = (O.mul_mat(O.pack_weights(w), x, "q8_0", mode=mode) + b).astype(np.float32)
    np.testing.assert_array_equal(got, ref)
    if m <= 32:   # the decode GEMV gives the same bits
        np.testing.assert_array_equal(lin(dev(x), rounding=mode).cpu().numpy(), got)
    lin.close()


def test_exact_gemm_fc1_shape_at_24000_rows():
    from mstar_accelerators_b200 import linear
    rng = np.random.default_rng(24)
    w = (rng.standard_normal((5120, 1280)) * 0.02).astype(np.float32)
    x = rng.standard_normal((24000, 1280)).astype(np.float32)
    lin = linear.BlockLinear(dev(w))
    got = lin.exact(dev(x)).cpu().numpy()
    np.testing.assert_array_equal(got, O.mul_mat(O.pack_weights(w), x, "q8_0"))
    lin.close()
