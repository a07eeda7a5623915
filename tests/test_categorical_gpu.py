"""Categorical sampling on B200 (mstar_b200_categorical) against the oracle, which is
pinned to the reference's scalar oracle (tests/test_categorical.py).

Tokens must equal the oracle's exactly: the Philox words are integer arithmetic and
the kernel evaluates the two logarithms in double and rounds them, as the oracle
does. Cases: the golden rows (ties, masks, +inf, NaN, invalid temperatures), readout-
sized rows (51865 entries, 32 rows, several temperatures, 64-bit seeds and offsets),
independence from the row's position in the batch, and the draw frequencies of one
row against softmax(logits / T) over 4000 offsets."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "categorical.npz"


def draw(logits, seeds, offsets, temps):
    from mstar_accelerators_b200 import linear
    t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a, dt)).cuda()
    return linear.categorical(t(logits, np.float32), t(seeds, np.int64), t(offsets, np.int64),
                              t(temps, np.float32)).cpu().numpy()


def test_golden_rows():
    g = np.load(GOLDEN)
    np.testing.assert_array_equal(draw(g["logits"], g["seeds"], g["offsets"], g["temperatures"]), g["tokens"])


def test_readout_sized_rows_match_oracle():
    rng = np.random.default_rng(5)
    rows, vocab = 32, 51865
    logits = (rng.standard_normal((rows, vocab)) * rng.uniform(0.2, 6.0, (rows, 1))).astype(np.float32)
    logits[3, ::7] = -np.inf
    seeds = rng.integers(-(1 << 63), (1 << 63) - 1, rows, dtype=np.int64)
    offsets = rng.integers(0, 1 << 40, rows, dtype=np.int64)
    temps = rng.uniform(0.05, 2.0, rows).astype(np.float32)
    got = draw(logits, seeds, offsets, temps)
    np.testing.assert_array_equal(got, O.categorical(logits, seeds, offsets, temps))
    # a row's draw depends on its logits, seed, offset and temperature only
    perm = rng.permutation(rows)
    np.testing.assert_array_equal(draw(logits[perm], seeds[perm], offsets[perm], temps[perm]), got[perm])


def test_draw_frequencies_follow_softmax():
    rng = np.random.default_rng(6)
    logits = (rng.standard_normal(12) * 1.2).astype(np.float32)
    n, T = 4000, np.float32(0.8)
    toks = draw(np.tile(logits, (n, 1)), np.full(n, 99), np.arange(n), np.full(n, T))
    np.testing.assert_array_equal(toks, O.categorical(np.tile(logits, (n, 1)), np.full(n, 99), np.arange(n),
                                                      np.full(n, T)))
    p = np.exp((logits - logits.max()) / T)
    p /= p.sum()
    counts = np.bincount(toks, minlength=12)
    chi2 = float(((counts - n * p) ** 2 / (n * p)).sum())
    assert chi2 < 40.0, (chi2, counts, n * p)     # 11 degrees of freedom: p ~ 1e-4 at 40


def test_rejects_bad_operands():
    from mstar_accelerators_b200 import linear, native
    x = torch.zeros(2, 8, device="cuda")
    s = torch.zeros(2, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError):
        linear.categorical(x, s[:1], s, torch.ones(2, device="cuda"))
    lib = native.require_capability()
    e = native.error_buffer()
    assert lib.mstar_b200_categorical(x.data_ptr(), 2, 8, 4, s.data_ptr(), s.data_ptr(), x.data_ptr(),
                                      s.data_ptr(), s.data_ptr(), 32, None, e, len(e)) == -1   # ld < vocab
