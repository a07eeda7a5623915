"""GGUF Q8_0 / Q4_0 import (mstar_accelerators_b200/gguf_import.py) on the CPU.

Files are written with the gguf package (the GGUF writer of the ggml project)
from seeded weights quantized by its own Q8_0 / Q4_0 quantizers. The importer
must return each tensor's logical shape and exactly its block bytes, and those
bytes must equal the packers' bytes for the same weights (the oracle's
restatement of quantize_row_q8_0_ref / quantize_row_q4_0_ref, without the fp16
pre-round a ggml checkpoint does not carry), so a ggml-quantized checkpoint
feeds the B200 linears unchanged. Malformed files are refused the way ggml's
reader refuses them.
"""
import numpy as np
import pytest

from oracle import oracle as O


def write(path, tensors, align=None):
    import gguf
    w = gguf.GGUFWriter(str(path), "test")
    if align:
        w.add_custom_alignment(align)
    w.add_string("general.name", "blocks")
    for name, (arr, qtype, shape) in tensors.items():
        w.add_tensor(name, arr, raw_dtype=qtype)   # quantized arrays carry their byte shape
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def weights(rows, k, seed):
    return (np.random.default_rng(seed).standard_normal((rows, k)) * 0.02).astype(np.float32)


@pytest.mark.parametrize("align", [None, 64])
def test_gguf_blocks_equal_packer_bytes(tmp_path, align):
    import gguf
    from gguf import quants
    from mstar_accelerators_b200.gguf_import import GGUFFile
    T = gguf.GGMLQuantizationType
    w8, w4, wf = weights(48, 96, 1), weights(40, 64, 2), weights(8, 32, 3)
    tensors = {"blk.0.q8": (quants.Q8_0.quantize(w8), T.Q8_0, (48, 96)),
               "blk.0.q4": (quants.Q4_0.quantize(w4), T.Q4_0, (40, 64)),
               "blk.0.f32": (wf, T.F32, (8, 32)),
               "blk.0.f16": (wf.astype(np.float16), T.F16, (8, 32))}
    path = tmp_path / "w.gguf"
    write(path, tensors, align)
    with GGUFFile(path) as gf:
        assert gf.metadata["general.name"] == "blocks"
        assert {k: (t.shape, t.format) for k, t in gf.tensors.items()} == {
            "blk.0.q8": ((48, 96), "q8_0"), "blk.0.q4": ((40, 64), "q4_0"),
            "blk.0.f32": ((8, 32), "f32"), "blk.0.f16": ((8, 32), "f16")}
        q8, q4 = gf.raw("blk.0.q8"), gf.raw("blk.0.q4")
        np.testing.assert_array_equal(q8, O.pack_weights(w8, "q8_0", preround=False))
        np.testing.assert_array_equal(q4, O.pack_weights(w4, "q4_0", preround=False))
        np.testing.assert_array_equal(gf.raw("blk.0.f32").view(np.float32).reshape(8, 32), wf)
        np.testing.assert_array_equal(gf.raw("blk.0.f16").view(np.float16).reshape(8, 32), wf.astype(np.float16))


def test_gguf_rejects_malformed_files(tmp_path):
    import gguf
    from gguf import quants
    from mstar_accelerators_b200.gguf_import import GGUFError, GGUFFile
    T = gguf.GGMLQuantizationType
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + bytes(60))
    with pytest.raises(GGUFError):
        GGUFFile(bad)
    good = tmp_path / "good.gguf"
    write(good, {"w": (quants.Q8_0.quantize(weights(4, 64, 4)), T.Q8_0, (4, 64))})
    data = good.read_bytes()
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(data[:-40])                     # data section shorter than the tensor
    with pytest.raises(GGUFError):
        GGUFFile(cut)
    q41 = tmp_path / "q41.gguf"
    write(q41, {"w": (quants.Q4_1.quantize(weights(4, 64, 5)), T.Q4_1, (4, 64))})
    with pytest.raises(GGUFError):                  # not a format of this path
        GGUFFile(q41)
