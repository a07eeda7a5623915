"""Thinker MoE on B200 against the oracle (oracle/moe_oracle.py).

Router: ids equal the oracle's wherever the k-th probability is not tied with
the next one (the reference's own router test is tie-tolerant,
tests/qwen3_omni/test_predictor_fusions.py:47-72); weights within 1e-5.
Experts: driven with the oracle's top-k so both sides use the same routing;
outputs within 2e-2 of the largest |output| elementwise (one bf16 rounding of
g, u, act or mid may land on the other side of a boundary, as the reference's
fp32 accumulation order is unspecified) and within 2e-3 on average.
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as M
from oracle import oracle as O

pytestmark = pytest.mark.gpu

GEOMS = {"small": (16, 128, 256, 4), "thinker": (128, 768, 2048, 8)}


def make(geom, seed=0):
    E, I, H, k = GEOMS[geom]
    g = torch.Generator().manual_seed(seed)
    w1 = (torch.randn((E, 2 * I, H), generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn((E, H, I), generator=g) * 0.02).to(torch.bfloat16)
    wr = (torch.randn((E, H), generator=g) * 0.02).to(torch.bfloat16)
    return E, I, H, k, w1, w2, wr


def bf(t):
    return t.float().numpy()


@pytest.mark.parametrize("geom,T", [("small", 1), ("small", 37), ("thinker", 1), ("thinker", 32), ("thinker", 300)])
def test_router_matches_oracle(geom, T):
    from mstar_accelerators_b200 import moe
    E, I, H, k, w1, w2, wr = make(geom, 1)
    x = torch.randn((T, H), generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    w, ids = moe.route(x.cuda(), wr.cuda(), top_k=k)
    rw, rids, p = M.route(bf(x), bf(wr), k)
    got_w, got_ids = w.cpu().numpy(), ids.cpu().numpy()
    ps = -np.sort(-p, axis=-1)
    for t in range(T):
        if ps[t, k - 1] - ps[t, k] > 1e-6:  # no tie at the boundary
            assert set(got_ids[t]) == set(rids[t])
            order = np.argsort(rids[t])
            np.testing.assert_allclose(got_w[t][np.argsort(got_ids[t])], rw[t][order], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("fmt", ["bf16", "q8_0"])
@pytest.mark.parametrize("geom,T", [("small", 1), ("small", 37), ("thinker", 1), ("thinker", 32), ("thinker", 200)])
def test_experts_match_oracle(fmt, geom, T):
    from mstar_accelerators_b200 import linear, moe
    E, I, H, k, w1, w2, wr = make(geom, 3)
    x = torch.randn((T, H), generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    rw, rids, _ = M.route(bf(x), bf(wr), k)
    if fmt == "bf16":
        backend = moe.ThinkerMoEB200(w1.cuda(), w2.cuda(), fmt="bf16", top_k=k, max_tokens=max(T, 64))
        ref = M.experts_bf16(bf(x), bf(w1), bf(w2), rw, rids)
    else:
        b1 = linear.pack(w1.float().reshape(-1, H).cuda(), "q8_0", preround=False).reshape(E, 2 * I, -1)
        b2 = linear.pack(w2.float().reshape(-1, I).cuda(), "q8_0", preround=False).reshape(E, H, -1)
        backend = moe.ThinkerMoEB200(b1, b2, fmt="q8_0", top_k=k, max_tokens=max(T, 64), intermediate=I, hidden=H)
        ref = M.experts_q8(bf(x), b1.cpu().numpy(), b2.cpu().numpy(), rw, rids, I, H)
    out = backend(x.cuda(), torch.from_numpy(rw).cuda(), torch.from_numpy(rids).cuda())
    got = out.float().cpu().numpy()
    assert int(backend.status.cpu()[0]) == 0
    scale = np.abs(ref).max()
    diff = np.abs(got - ref)
    assert diff.max() <= 2e-2 * scale, (diff.max(), scale)
    assert diff.mean() <= 2e-3 * scale
    backend.close()


def test_experts_skip_out_of_range_ids():
    """An id outside [0, E) sets status bit value 4 and its slot adds nothing."""
    from mstar_accelerators_b200 import moe
    E, I, H, k, w1, w2, wr = make("small", 5)
    backend = moe.ThinkerMoEB200(w1.cuda(), w2.cuda(), fmt="bf16", top_k=k, max_tokens=8)
    x = torch.randn((2, H), generator=torch.Generator().manual_seed(6)).to(torch.bfloat16)
    ids = np.array([[0, 1, 2, 3], [4, 5, 6, E]], np.int32)
    w = np.full((2, k), 0.25, np.float32)
    out = backend(x.cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(ids).cuda()).float().cpu().numpy()
    assert int(backend.status.cpu()[0]) & 4
    w_skip = w.copy()
    w_skip[1, 3] = 0.0  # the invalid slot contributes +0 (bf16(0 * y) = 0)
    ids_skip = ids.copy()
    ids_skip[1, 3] = 0
    ref = M.experts_bf16(bf(x), bf(w1), bf(w2), w_skip, ids_skip)
    scale = np.abs(ref).max()
    assert np.abs(out - ref).max() <= 2e-2 * scale
    backend.close()


def test_thinker_experts_backend_installs_and_chunks():
    """install_thinker_experts swaps the experts_backend of thinker-shaped MoE
    layers; the backend keeps the reference call signature and splits calls
    larger than max_tokens into row chunks with identical results."""
    from mstar_accelerators_b200 import moe
    E, I, H, k, w1, w2, wr = make("thinker", 7)

    class Bank(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_up_proj = torch.nn.Parameter(w1.cuda(), requires_grad=False)
            self.down_proj = torch.nn.Parameter(w2.cuda(), requires_grad=False)

    class Layer(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.experts = Bank()
            self.experts_backend = None

    root = torch.nn.Sequential(Layer(), torch.nn.Linear(4, 4))
    assert moe.install_thinker_experts(root, max_tokens=64) == 1
    layer = root[0]
    T = 150
    x = torch.randn((T, H), generator=torch.Generator().manual_seed(8)).to(torch.bfloat16)
    rw, rids, _ = M.route(bf(x), bf(wr), k)
    args = (x.cuda(), layer.experts.gate_up_proj, layer.experts.down_proj, torch.from_numpy(rw).cuda(),
            torch.from_numpy(rids).cuda())
    chunked = layer.experts_backend(*args).float().cpu().numpy()
    whole = moe.ThinkerMoEB200(w1.cuda(), w2.cuda(), top_k=k, max_tokens=T)
    ref = whole(args[0], args[3], args[4]).float().cpu().numpy()
    np.testing.assert_array_equal(chunked, ref)
    with pytest.raises(ValueError):
        layer.experts_backend(args[0], args[2], args[1], args[3], args[4])
    whole.close()
    layer.experts_backend.close()
