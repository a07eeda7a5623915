"""GGUF-imported Q8_0 / Q4_0 weights run on the B200 linears unchanged: a
BlockLinear made from the file's block bytes gives the oracle's generic-order
ggml mul_mat of those same bytes bit for bit (decode GEMV, <= 32 rows), and the
F32 tensor of the same weights, packed on the device, gives the same blocks
with the fp16 pre-round switched off."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_gguf_linear_matches_oracle(tmp_path, fmt):
    import gguf
    from gguf import quants
    from mstar_accelerators_b200.gguf_import import GGUFFile, load_linear
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((384, 384)) * 0.02).astype(np.float32)
    x = rng.standard_normal((5, 384)).astype(np.float32)
    T = gguf.GGMLQuantizationType
    q = (quants.Q8_0 if fmt == "q8_0" else quants.Q4_0).quantize(w)
    path = tmp_path / "w.gguf"
    wr = gguf.GGUFWriter(str(path), "test")
    wr.add_tensor("w", q, raw_dtype=T.Q8_0 if fmt == "q8_0" else T.Q4_0)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    with GGUFFile(path) as gf:
        lin = load_linear(gf, "w")
        blocks = gf.raw("w")
    got = lin(torch.from_numpy(x).cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, O.mul_mat(blocks, x, fmt))
    np.testing.assert_array_equal(lin.blocks.cpu().numpy(), blocks)
    lin.close()
