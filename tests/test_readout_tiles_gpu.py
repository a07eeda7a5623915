"""The vocab readout on the 16-row tile layout (prepare_readout) against the oracle.

The tile kernel computes the same per-block int32 dots and folds them in
ggml's generic order, so logits must be bit-identical to the oracle's
mul_mat and to the decode-GEMV readout of the same handle; tokens follow the
first-index / NaN-first rule after suppression (decoder.cpp:686-696).
Covered: every n-tile count (1, 2, 4 queries per 8), ragged row counts (rows
not a multiple of 16), one and several chunks per tile, suppression of the
first / last rows and of every row, NaN logits, and repeated calls (the
cross-CTA state must reset itself).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    from mstar_accelerators_b200 import linear
    O.build()
    return linear


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def _check(lin, blocks, fmt, x, sup):
    logits, token, status = lin.readout(dev(x), dev(sup) if sup.size else None)
    ref = O.mul_mat(blocks, x, fmt)
    got, toks = host(logits), host(token)
    for i in range(x.shape[0]):
        masked, tok = O.argmax(ref[i], sup)
        assert np.array_equal(got[i], masked), f"logits of query {i}"
        assert toks[i] == tok, f"token of query {i}"
    assert host(status)[0] == 0
    return got, toks


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("n,k,m", [(51865, 384, 32), (51865, 384, 1), (4099, 384, 17), (3001, 96, 9),
                                   (1000, 1280, 16), (777, 4096, 8), (40, 64, 5)])
def test_tile_readout_matches_oracle(L, fmt, n, k, m):
    rng = np.random.default_rng(n + k + m)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    w[n - 1] = w[min(123, n - 2)]                  # duplicate rows: a tie candidate
    x = rng.standard_normal((m, k)).astype(np.float32)
    blocks = O.pack_weights(w, fmt)
    lin = L.BlockLinear(blocks=dev(blocks), fmt=fmt, rows=n, width=k)
    sup = np.array(sorted({0, 5, n // 2, n - 1}), np.int64)
    plain = lin.readout(dev(x), dev(sup))          # decode-GEMV readout of the same handle
    lin.prepare_readout()
    got, toks = _check(lin, blocks, fmt, x, sup)
    assert np.array_equal(got, host(plain[0])) and np.array_equal(toks, host(plain[1]))
    # again: the argmax state of the previous call must have been reset
    _check(lin, blocks, fmt, x[::-1].copy(), np.array([], np.int64))
    lin.close()


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_tile_readout_ties_nan_and_full_suppression(L, fmt):
    rng = np.random.default_rng(9)
    n, k = 5000, 384
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    w[4777] = w[1234]
    blocks = O.pack_weights(w, fmt)
    lin = L.BlockLinear(blocks=dev(blocks), fmt=fmt, rows=n, width=k)
    lin.prepare_readout()
    x = rng.standard_normal((3, k)).astype(np.float32)
    x[0] = w[1234] * 400.0                          # the duplicated rows are the maximum: the first wins
    _, toks = _check(lin, blocks, fmt, x, np.array([], np.int64))
    assert toks[0] == 1234
    # every row suppressed: all logits -inf, the first index wins
    everything = np.arange(n, dtype=np.int64)
    _, toks = _check(lin, blocks, fmt, x, everything)
    assert toks.tolist() == [0, 0, 0]
    # NaN scales make NaN logits: the first NaN row wins over every number
    bad = blocks.copy()
    bs = O.Q4_BLOCK if fmt == "q4_0" else O.Q8_BLOCK
    for r in (3000, 2500):
        bad[r, 0:2] = np.frombuffer(np.float16(np.nan).tobytes(), np.uint8)
    lin2 = L.BlockLinear(blocks=dev(bad), fmt=fmt, rows=n, width=k)
    lin2.prepare_readout()
    logits, token, status = lin2.readout(dev(x))
    assert host(token).tolist() == [2500, 2500, 2500] and host(status)[0] == 0
    assert np.isnan(host(logits)[:, 2500]).all()
    assert bs in (18, 34)
    lin.close()
    lin2.close()


def test_tile_readout_in_a_cuda_graph(L):
    rng = np.random.default_rng(3)
    n, k, m = 51865, 384, 32
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    blocks = O.pack_weights(w, "q4_0")
    lin = L.BlockLinear(blocks=dev(blocks), fmt="q4_0", rows=n, width=k)
    lin.prepare_readout()
    x = torch.zeros((m, k), device="cuda")
    lg = torch.empty((m, n), device="cuda")
    tk = torch.empty(m, dtype=torch.int64, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        lin.readout(x, logits=lg, token=tk, status=st)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        lin.readout(x, logits=lg, token=tk, status=st)
    for seed in (1, 2):
        xs = np.random.default_rng(seed).standard_normal((m, k)).astype(np.float32)
        x.copy_(dev(xs))
        graph.replay()
        ref = O.mul_mat(blocks, xs, "q4_0")
        assert np.array_equal(host(lg), ref)
        assert host(tk).tolist() == [O.argmax(ref[i])[1] for i in range(m)]
    graph = None
    lin.close()


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_tile_readout_status_and_fused_layernorm(L, fmt):
    rng = np.random.default_rng(21)
    n, k, m = 3000, 384, 7
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    blocks = O.pack_weights(w, fmt)
    tiles = L.BlockLinear(blocks=dev(blocks), fmt=fmt, rows=n, width=k)
    tiles.prepare_readout()
    plain = L.BlockLinear(blocks=dev(blocks), fmt=fmt, rows=n, width=k)
    x = (rng.standard_normal((m, k)) * 3 + 1).astype(np.float32)
    lw = rng.uniform(0.5, 1.5, k).astype(np.float32)
    lb = (rng.standard_normal(k) * 0.1).astype(np.float32)
    norm = (dev(lw), dev(lb), 1e-5)
    # the fused LayerNorm + quantization prologue matches the stand-alone quantize kernel bit for bit
    for rounding in ("ref", "arm", "x86"):
        got = tiles.readout(dev(x), norm=norm, rounding=rounding)
        ref = plain.readout(dev(x), norm=norm, rounding=rounding)
        assert np.array_equal(host(got[0]), host(ref[0])) and np.array_equal(host(got[1]), host(ref[1]))
        assert host(got[2])[0] == 0
    # a non-finite query value sets bit 0 of this call's status only
    bad = x.copy()
    bad[3, 100] = np.inf
    assert host(tiles.readout(dev(bad))[2])[0] == 1
    assert host(tiles.readout(dev(x))[2])[0] == 0
    tiles.close()
    plain.close()


@pytest.mark.parametrize("m", [1, 17, 32, 40])
def test_tile_gemv_equals_the_split_gemv(L, m):
    """linear_run on a handle with the tile layout (the logits-only tile kernel) gives the bytes of
    the fragment-layout GEMV: bias, residual and the fused LayerNorm included."""
    rng = np.random.default_rng(40 + m)
    n, k = 1000, 2048
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    blocks = O.pack_weights(w, "q8_0")
    plain = L.BlockLinear(blocks=dev(blocks), fmt="q8_0", rows=n, width=k, bias=dev(bias))
    tiles = L.BlockLinear(blocks=dev(blocks), fmt="q8_0", rows=n, width=k, bias=dev(bias))
    tiles.prepare_readout()
    x = (rng.standard_normal((m, k)) * 2).astype(np.float32)
    res = rng.standard_normal((m, n)).astype(np.float32)
    lw = rng.uniform(0.5, 1.5, k).astype(np.float32)
    lb = (rng.standard_normal(k) * 0.1).astype(np.float32)
    for kw in ({}, {"norm": (dev(lw), dev(lb), 1e-5)}):
        a = host(plain(dev(x), **kw))
        b = host(tiles(dev(x), **kw))
        assert np.array_equal(a, b)
        ra = dev(res.copy())
        rb = dev(res.copy())
        plain(dev(x), out=ra, residual=ra, **kw)
        tiles(dev(x), out=rb, residual=rb, **kw)
        assert np.array_equal(host(ra), host(rb))
    assert np.array_equal(host(tiles(dev(x), bias=False)), O.mul_mat(blocks, x, "q8_0"))
    plain.close()
    tiles.close()
