"""The categorical sampler's oracle (oracle/q8_oracle.c, philox4x32-10-gumbel23-v1)
pinned on the CPU: the Random123 Philox4x32-10 known-answer vectors listed in the
reference's backends/pi/docs/categorical.md, and the draws of the reference's own
scalar oracle (backends/pi/torch/tests/categorical_reference.py, imported by
tests/golden/make_golden.py into tests/golden/categorical.npz): ordinary rows at
several temperatures with 64-bit seeds and offsets, tied maxima, -inf masks, +inf
entries, a NaN row, an all -inf row, invalid temperatures, and 2000 draws of one
row."""
from pathlib import Path

import numpy as np

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden" / "categorical.npz"
M = 0xFFFFFFFF


def test_philox_known_answers():
    assert O.philox4x32_10((0, 0, 0, 0), (0, 0)) == (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)
    assert O.philox4x32_10((M, M, M, M), (M, M)) == (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)
    assert O.philox4x32_10((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0)) == (
        0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)


def test_oracle_draws_equal_reference_golden():
    g = np.load(GOLDEN)
    got = O.categorical(g["logits"], g["seeds"], g["offsets"], g["temperatures"])
    np.testing.assert_array_equal(got, g["tokens"])
    assert list(got[-4:]) == [-1, -1, -1, -1]         # NaN row, all -inf row, T = 0, T < 0
    assert got[4] in (3, 100, 200) and got[6] in (7, 150)
    n = len(g["many_offsets"])
    many = O.categorical(np.tile(g["many_logits"], (n, 1)), np.full(n, 12345), g["many_offsets"],
                         np.full(n, 0.9, np.float32))
    np.testing.assert_array_equal(many, g["many_tokens"])
