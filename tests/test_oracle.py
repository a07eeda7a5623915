"""The oracle is pinned before it is trusted: reference known-answer tests,
the reference's own Python packer output, and the vendored ggml arithmetic
compiled from the reference sources (oracle/_ref)."""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module", autouse=True)
def built():
    O.build()


def test_q8_known_answers_from_reference_tests():
    # tests/whisper/test_q8_readout.py:13-36: roundf ties, fp32 scale, fp16 underflow
    z = np.load(GOLDEN / "q8_kat.npz")
    for i in range(3):
        got = O.pack_weights(z[f"w{i}"], "q8_0", preround=False)
        assert bytes(got.reshape(-1)) == bytes(z[f"bytes{i}"])


def test_q8_matches_reference_python_packer():
    z = np.load(GOLDEN / "q8_pack.npz")
    assert np.array_equal(O.pack_weights(z["w"], "q8_0", preround=False), z["packed"])


@pytest.mark.parametrize("bad", [np.nan, np.inf, -np.inf])
def test_packers_reject_nonfinite(bad):
    w = np.zeros((2, 32), np.float32)
    w[1, 3] = bad
    for fmt in ("q8_0", "q4_0"):
        with pytest.raises(ValueError, match="nonfinite"):
            O.pack_weights(w, fmt)


def test_q4_packer_rejects_fp16_overflow():
    # decoder.cpp:829-833: a finite fp32 weight that overflows F16 is refused
    w = np.zeros((1, 32), np.float32)
    w[0, 0] = 1e10
    with pytest.raises(ValueError, match="overflows"):
        O.pack_weights(w, "q4_0")


def test_q4_reference_fixture_both_rounding_contracts():
    # tests/test_cpu_ggml_q4_readout.py:79-91 fixture; the compiled ggml uses FMA
    z = np.load(GOLDEN / "q4_pack.npz")
    assert np.array_equal(O.pack_weights(z["x"], "q4_0", fused=True), z["fma"])
    assert np.array_equal(O.pack_weights(z["x"], "q4_0", fused=False), z["separate"])
    assert np.array_equal(z["fma"], z["ggml"])
    assert not np.array_equal(z["fma"], z["separate"])  # the fixture separates the contracts


def test_q4_all_zero_block_is_negative_zero_scale():
    # d = max / -8 with max == +0 stores -0.0 (0x8000); every nibble is 8
    b = O.pack_weights(np.zeros((1, 32), np.float32), "q4_0")[0]
    assert bytes(b[:2]) == b"\x00\x80" and set(b[2:].tolist()) == {0x88}


def test_generic_mul_mat_matches_reference_golden():
    z = np.load(GOLDEN / "mul_mat.npz")
    for tag in ("q8_0_40x384x5", "q4_0_40x384x3", "q8_0_16x1536x2"):
        fmt = tag[:4]
        got = O.mul_mat(z[tag + "_blocks"], z[tag + "_x"], fmt, mode="x86")
        assert np.array_equal(got, z[tag + "_out"]), tag


def test_argmax_rules():
    # decoder.cpp:686-696 / readout.c:47-53
    nan = np.nan
    assert O.argmax([1, 3, 3, 2])[1] == 1                    # first index of the maximum
    assert O.argmax([1, nan, 5, nan])[1] == 1                # first NaN wins over any value
    assert O.argmax([-0.0, 0.0])[1] == 0                     # signed zeros tie
    assert O.argmax([-np.inf, -np.inf])[1] == 0              # all -inf
    logits, tok = O.argmax([1, 9, 3], suppressed=[1])
    assert tok == 2 and logits[1] == -np.inf


ref_missing = pytest.mark.skipif(O.ref_lib() is None, reason="oracle/_ref not built")


@ref_missing
@pytest.mark.parametrize("mode,which", [("ref", "q8_ref"), ("x86", "q8_x86")])
def test_activation_quantizer_matches_compiled_reference(mode, which):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((64, 1536)) * rng.uniform(1e-3, 30, (64, 1))).astype(np.float32)
    x[0, :64] = 0
    x[1, :32] = np.arange(32) - 15.5        # many exact halves after scaling
    assert np.array_equal(O.quantize_q8_0(x, mode), O.ref_quantize(x, which))


def test_arm_rounding_differs_from_ref_only_on_ties():
    x = np.zeros((1, 32), np.float32)
    x[0, 0] = 127.0
    x[0, 1] = 0.5      # id == 1: 0.5 rounds to 0 (half-even) vs 1 (half away)
    x[0, 2] = 2.5
    arm, ref = O.quantize_q8_0(x, "arm")[0], O.quantize_q8_0(x, "ref")[0]
    assert arm[2 + 1] == 0 and ref[2 + 1] == 1
    assert arm[2 + 2] == 2 and ref[2 + 2] == 3


@ref_missing
def test_q4_quantizer_matches_compiled_reference():
    rng = np.random.default_rng(4)
    x = O.fp16_round(rng.standard_normal((128, 384)).astype(np.float32))
    assert np.array_equal(O.quantize_q4_0(x, fused=True), O.ref_quantize(x, "q4_ref"))


@ref_missing
@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_simd_reference_mul_mat_is_a_reordering(fmt):
    rng = np.random.default_rng(6)
    blocks = O.pack_weights((rng.standard_normal((64, 768)) * 0.02).astype(np.float32), fmt)
    x = rng.standard_normal((3, 768)).astype(np.float32)
    generic = O.mul_mat(blocks, x, fmt, mode="x86")
    simd = O.ref_mul_mat(blocks, x, fmt, threads=2)
    np.testing.assert_allclose(simd, generic, rtol=1e-5, atol=1e-5)


def test_block_sums_are_exact_integers():
    rng = np.random.default_rng(7)
    blocks = O.pack_weights((rng.standard_normal((1, 96)) * 0.02).astype(np.float32), "q8_0")
    xq = O.quantize_q8_0(rng.standard_normal((1, 96)).astype(np.float32))
    sums = O.block_sums(blocks[0], xq[0])
    w = blocks[0].reshape(3, 34)[:, 2:].view(np.int8).astype(np.int64)
    a = xq[0].reshape(3, 34)[:, 2:].view(np.int8).astype(np.int64)
    assert np.array_equal(sums, (w * a).sum(1))


def test_gelu_table_form():
    x = np.array([-11, -1, 0, 0.5, 3, 11], np.float32)
    y = O.gelu_ggml(x)
    assert y[0] == 0 and y[-1] == 11 and y[2] == 0
    assert np.allclose(y[1:5], 0.5 * x[1:5] * (1 + np.tanh(0.7978845608 * (x[1:5] + 0.044715 * x[1:5] ** 3))),
                       rtol=2e-3, atol=1e-3)
