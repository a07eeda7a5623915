"""The expert-parallel send-side plan on one B200 (mstar_b200_moe_dispatch)
against the torch restatement, and the caller-rows combine against an fp32
slot-ordered sum.

The plan is integer and copy work, so meta, rows, (local id, weight bits)
pairs and inverse positions must be identical: every rank count from 1 to 8,
token counts that are not multiples of the 1024-pair rounds, ranks that get no
pairs, ids outside [0, E) (flagged in meta), int64 ids, and zero tokens.
"""
import pytest
import torch

from mstar_accelerators_b200.moe_ep import torch_dispatch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    from mstar_accelerators_b200 import native
    return native.require_capability()


def _inputs(T, k, E, H, seed, *, skew=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16).cuda()
    w = torch.rand((T, k), generator=g).cuda()
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]) if T else torch.zeros((0, k))
    ids = ids.to(torch.int32)
    if skew:  # every pair on the first quarter of the experts: later ranks receive nothing
        ids = ids % max(1, E // 4)
    return x, w, ids.cuda()


@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
@pytest.mark.parametrize("T,k,H", [(1, 8, 2048), (37, 8, 2048), (4096, 8, 2048), (300, 3, 72), (129, 1, 512),
                                   (50, 2, 36)])
def test_dispatch_equals_the_torch_plan(lib, ranks, T, k, H):
    from mstar_accelerators_b200.moe_ep import b200_dispatch
    E = 128
    x, w, ids = _inputs(T, k, E, H, seed=T * 31 + ranks)
    got = b200_dispatch(lib)(x, w, ids, k, E, ranks)
    ref = torch_dispatch(x, w, ids, k, E, ranks)
    for a, b, name in zip(got, ref, ("meta", "rows", "pairs", "inverse")):
        assert a.dtype == b.dtype and torch.equal(a, b), name


def test_dispatch_skew_invalid_ids_int64_and_zero_tokens(lib):
    from mstar_accelerators_b200.moe_ep import b200_dispatch
    run = b200_dispatch(lib)
    E, k, H = 64, 4, 256
    x, w, ids = _inputs(2500, k, E, H, seed=4, skew=True)
    for a, b in zip(run(x, w, ids, k, E, 8), torch_dispatch(x, w, ids, k, E, 8)):
        assert torch.equal(a, b)
    meta = run(x, w, ids, k, E, 8)[0].view(8, 2)
    assert meta[2:, 0].sum().item() == 0 and meta[:, 1].sum().item() == 0
    bad = ids.clone().long()
    bad[7, 2] = E + 5
    bad[2400, 0] = -3
    bad[11, 1] = 1 << 40                      # outside int32 as well
    got = run(x, w, bad, k, E, 4)
    ref = torch_dispatch(x, w, bad.clamp(-1, E), k, E, 4)
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    assert got[0].view(4, 2)[:, 1].tolist() == [1, 1, 1, 1]
    empty = run(x[:0], w[:0], ids[:0], k, E, 4)
    assert empty[0].tolist() == [0] * 8 and empty[1].shape == (0, H)


@pytest.mark.parametrize("H", [2048, 36])
def test_combine_rows_is_the_slot_ordered_sum(lib, H):
    from mstar_accelerators_b200.moe_ep import b200_combine
    T, k = 333, 8
    g = torch.Generator().manual_seed(H)
    y = torch.randn((T * k + 5, H), generator=g).to(torch.bfloat16).cuda()
    rows = torch.randperm(T * k + 5, generator=g)[:T * k].to(torch.int32)
    rows[17] = -1                              # outside [0, y_rows): adds nothing
    rows[40] = T * k + 5
    rows = rows.cuda()
    got = b200_combine(lib)(y, rows, k)
    ref = torch.zeros((T, H), dtype=torch.float32, device="cuda")
    yf = y.float()
    r = rows.view(T, k).long()
    for s in range(k):
        ok = (r[:, s] >= 0) & (r[:, s] < y.shape[0])
        ref += torch.where(ok[:, None], yf[r[:, s].clamp(0, y.shape[0] - 1)], torch.zeros_like(ref))
    assert torch.equal(got, ref.to(torch.bfloat16))
