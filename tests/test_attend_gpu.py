"""Split-key decode attention (mstar_b200_attend) against a float64 reference.

The kernel walks key tiles of 64 on the tensor cores (fp16 K and V, Q and P as
fp16 hi + lo pairs, fp32 accumulation) with an online softmax and, over shared
planes, splits the keys across CTAs and merges the partial sums. Results must
match exact attention over the fp16 K/V planes within 5e-5 (absolute and
relative; outputs are O(1)). Covers shared
planes (all batch*queries rows against one K/V tile, as the decoder's cross
attention), causal per-sequence planes with the new K/V rows appended at
positions that straddle a 64-key chunk boundary, per-sequence lengths that are
not multiples of 64, and invalid positions (status bit value 8, rows zeroed).
"""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

H, D = 6, 64


def attend(lib, q, kp, vp, capacity, batch, nq, causal, shared, begin=None, kv_len=None, k_new=None, v_new=None):
    from mstar_accelerators_b200 import native
    out = torch.full((batch * nq, H * D), 123.0, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    n = int(lib.mstar_b200_attend_workspace(H, batch, nq, capacity, int(shared)))
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    e = native.error_buffer()
    native.check(lib.mstar_b200_attend(
        q.data_ptr(), q.stride(0), k_new.data_ptr() if k_new is not None else None,
        v_new.data_ptr() if v_new is not None else None, k_new.stride(0) if k_new is not None else 0,
        kp.data_ptr(), vp.data_ptr(), capacity, H, D, batch, nq,
        begin.data_ptr() if begin is not None else None, kv_len.data_ptr() if kv_len is not None else None,
        int(causal), int(shared), out.data_ptr(), out.stride(0), 1.0 / math.sqrt(D), status.data_ptr(),
        ws.data_ptr(), n, torch.cuda.current_stream().cuda_stream, e, len(e)), e, "attention")
    torch.cuda.synchronize()
    return out.cpu().numpy(), int(status.item())


def reference(q, kpl, vpl, limits, seqs):
    """q [rows, H*D]; kpl/vpl [seq, cap, H*D] (float64); limits/seqs per row."""
    out = np.zeros_like(q, dtype=np.float64)
    for r in range(q.shape[0]):
        L, s = limits[r], seqs[r]
        if L == 0:
            continue
        for h in range(H):
            qh = q[r, h * D:(h + 1) * D].astype(np.float64)
            k = kpl[s, :L, h * D:(h + 1) * D]
            v = vpl[s, :L, h * D:(h + 1) * D]
            sc = k @ qh / math.sqrt(D)
            p = np.exp(sc - sc.max())
            out[r, h * D:(h + 1) * D] = (p / p.sum()) @ v
    return out


@pytest.mark.parametrize("nq", [1, 4])
def test_shared_planes(nq):
    from mstar_accelerators_b200 import native
    lib = native.require_capability()
    g = torch.Generator().manual_seed(nq)
    B, cap = 32, 1500
    kp = torch.randn((1, cap, H * D), generator=g).half().cuda()
    vp = torch.randn((1, cap, H * D), generator=g).half().cuda()
    q = torch.randn((B * nq, H * D), generator=g).cuda()
    kv_len = torch.full((B,), cap, dtype=torch.int64, device="cuda")
    kv_len[3] = 700  # rows of one sequence see fewer keys of the shared plane
    got, st = attend(lib, q, kp, vp, cap, B, nq, False, True, kv_len=kv_len)
    assert st == 0
    lens = kv_len.cpu().numpy()
    ref = reference(q.cpu().numpy(), kp.double().cpu().numpy(), vp.double().cpu().numpy(),
                    [lens[r // nq] for r in range(B * nq)], [0] * (B * nq))
    np.testing.assert_allclose(got, ref, rtol=5e-5, atol=5e-5)


@pytest.mark.parametrize("nq,begins", [(1, [0, 63, 100]), (4, [0, 62, 300])])
def test_causal_append(nq, begins):
    from mstar_accelerators_b200 import native
    lib = native.require_capability()
    g = torch.Generator().manual_seed(10 + nq)
    B, cap = len(begins), 448
    kp = torch.randn((B, cap, H * D), generator=g).half().cuda()
    vp = torch.randn((B, cap, H * D), generator=g).half().cuda()
    qkv = torch.randn((B * nq, 3 * H * D), generator=g).cuda()
    q, kn, vn = qkv[:, :H * D], qkv[:, H * D:2 * H * D], qkv[:, 2 * H * D:]
    begin = torch.tensor(begins, dtype=torch.int64, device="cuda")
    kref, vref = kp.double().cpu().numpy(), vp.double().cpu().numpy()
    for b, b0 in enumerate(begins):
        kref[b, b0:b0 + nq] = kn[b * nq:(b + 1) * nq].half().double().cpu().numpy()
        vref[b, b0:b0 + nq] = vn[b * nq:(b + 1) * nq].half().double().cpu().numpy()
    got, st = attend(lib, q, kp, vp, cap, B, nq, True, False, begin=begin, k_new=kn, v_new=vn)
    assert st == 0
    limits = [begins[r // nq] + r % nq + 1 for r in range(B * nq)]
    ref = reference(q.cpu().numpy(), kref, vref, limits, [r // nq for r in range(B * nq)])
    np.testing.assert_allclose(got, ref, rtol=5e-5, atol=5e-5)
    # the new rows were written to the planes in fp16
    np.testing.assert_array_equal(kp.double().cpu().numpy(), kref)
    np.testing.assert_array_equal(vp.double().cpu().numpy(), vref)


def test_per_sequence_lengths_and_invalid_rows():
    from mstar_accelerators_b200 import native
    lib = native.require_capability()
    g = torch.Generator().manual_seed(20)
    lens = [1, 65, 1500, 0]  # the last one is invalid
    B, cap, nq = len(lens), 1500, 1
    kp = torch.randn((B, cap, H * D), generator=g).half().cuda()
    vp = torch.randn((B, cap, H * D), generator=g).half().cuda()
    q = torch.randn((B, H * D), generator=g).cuda()
    kv_len = torch.tensor(lens, dtype=torch.int64, device="cuda")
    got, st = attend(lib, q, kp, vp, cap, B, nq, False, False, kv_len=kv_len)
    assert st & 8
    ref = reference(q.cpu().numpy(), kp.double().cpu().numpy(), vp.double().cpu().numpy(), lens, list(range(B)))
    np.testing.assert_allclose(got, ref, rtol=5e-5, atol=5e-5)
    assert np.all(got[3] == 0.0)


def _attend_q8(lib, frags, q, kp, vp, capacity, batch, nq, causal, shared, begin=None, kv_len=None):
    import ctypes as C
    from mstar_accelerators_b200 import native
    out = torch.empty((batch * nq, H * D), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    n = int(lib.mstar_b200_attend_workspace(H, batch, nq, capacity, int(shared)))
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    e = native.error_buffer()
    native.check(lib.mstar_b200_attend_q8(
        q.data_ptr(), q.stride(0), None, None, 0, kp.data_ptr(), vp.data_ptr(), capacity, H, D, batch, nq,
        begin.data_ptr() if begin is not None else None, kv_len.data_ptr() if kv_len is not None else None,
        int(causal), int(shared), out.data_ptr(), out.stride(0), 1.0 / math.sqrt(D), status.data_ptr(),
        ws.data_ptr(), n, C.byref(frags), torch.cuda.current_stream().cuda_stream, e, len(e)), e, "attention")
    return out, status


@pytest.mark.parametrize("shared,batch", [(True, 32), (False, 32), (False, 5), (True, 12)])
@pytest.mark.parametrize("rounding", ["arm", "x86", "ref"])
def test_attention_output_fragments_equal_the_linear_quantizer(shared, batch, rounding):
    """attend_q8 + run_frags on a Q8_0 out-projection gives the bytes of attend + linear_run."""
    from mstar_accelerators_b200 import native
    from mstar_accelerators_b200.linear import BlockLinear
    lib = native.load()
    g = torch.Generator(device="cuda").manual_seed(batch + int(shared))
    cap = 1500 if shared else 448
    nseq = 1 if shared else batch
    kp = (torch.randn((nseq, cap, H * D), device="cuda", generator=g)).half()
    vp = (torch.randn((nseq, cap, H * D), device="cuda", generator=g)).half()
    q = torch.randn((batch, H * D), device="cuda", generator=g)
    lin = BlockLinear(torch.randn((H * D, H * D), device="cuda", generator=g) * 0.02,
                      bias=torch.randn(H * D, device="cuda", generator=g) * 0.1)
    x = torch.randn((batch, H * D), device="cuda", generator=g)
    if shared:
        kv_len = torch.full((batch,), cap, dtype=torch.int64, device="cuda")
        kv_len[0] = 77
        args = dict(causal=False, shared=True, kv_len=kv_len)
    else:
        begin = torch.randint(0, 200, (batch,), device="cuda", generator=g)
        args = dict(causal=True, shared=False, begin=begin)
    att, st = _attend_q8(lib, lin.frags(batch, rounding), q, kp, vp, cap, batch, 1, **args)
    got = lin.run_frags(batch, out=x.clone(), residual=None)
    got_res = x.clone()
    att2, _ = _attend_q8(lib, lin.frags(batch, rounding), q, kp, vp, cap, batch, 1, **args)
    lin.run_frags(batch, out=got_res, residual=got_res)
    ref = lin(att, rounding=rounding)
    ref_res = lin(att, out=x.clone(), residual=x.clone(), rounding=rounding)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert torch.equal(att, att2)
    assert torch.equal(got, ref) and torch.equal(got_res, ref_res)
    lin.close()


@pytest.mark.parametrize("m", [1, 9, 16, 32])
@pytest.mark.parametrize("rounding", ["arm", "ref", "x86"])
def test_fc1_fragment_output_equals_the_fc2_quantizer(m, rounding):
    """fc1 (LayerNorm, bias, GELU) with next_frags + fc2.run_frags gives the bytes of fc1 then fc2."""
    from mstar_accelerators_b200.linear import BlockLinear
    g = torch.Generator(device="cuda").manual_seed(m)
    d, f = 384, 1536
    fc1 = BlockLinear(torch.randn((f, d), device="cuda", generator=g) * 0.05,
                      bias=torch.randn(f, device="cuda", generator=g) * 0.1)
    fc2 = BlockLinear(torch.randn((d, f), device="cuda", generator=g) * 0.05,
                      bias=torch.randn(d, device="cuda", generator=g) * 0.1)
    x = torch.randn((m, d), device="cuda", generator=g) * 2
    lw = torch.rand(d, device="cuda", generator=g) + 0.5
    lb = torch.randn(d, device="cuda", generator=g) * 0.1
    norm = (lw, lb, 1e-5)
    h_ref = fc1(x, norm=norm, gelu="tanh", rounding=rounding)
    xr = x.clone()
    fc2(h_ref, out=xr, residual=xr, rounding=rounding)
    h = torch.empty_like(h_ref)
    fc1(x, out=h, norm=norm, gelu="tanh", rounding=rounding, next_frags=fc2.frags(m, rounding))
    xg = x.clone()
    fc2.run_frags(m, out=xg, residual=xg)
    torch.cuda.synchronize()
    assert torch.equal(h, h_ref)
    assert torch.equal(xg, xr)
    fc1.close()
    fc2.close()
