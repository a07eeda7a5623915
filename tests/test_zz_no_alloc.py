"""The Q8_0 readout that allocates nothing (mstar_b200_q8_readout_noalloc).

It exists for callers that cannot allocate device memory at call time: a
runtime that owns every device buffer and hands kernels only buffers it
planned, or a latency-bound caller that must not pay for cudaMalloc. It reads
the caller's canonical Q8_0 bytes and keeps its scratch in a fixed device
array, so its results must equal the handle-based entry point
(mstar_b200_q8_readout) exactly — the same bit-identical bar the other readout
tests use — call after call, since every call reuses that array.

This file is named to be collected last.
"""
import errno

import pytest
import torch

pytestmark = pytest.mark.gpu


def _call_both(lib, handle, blocks, rows, k, x, suppressed, stream):
    sup_ptr = suppressed.data_ptr() if suppressed is not None else None
    count = suppressed.numel() if suppressed is not None else 0
    ref = torch.empty(rows, device="cuda")
    ref_tok = torch.empty(1, dtype=torch.int64, device="cuda")
    ref_st = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.mstar_b200_q8_readout(handle, x.data_ptr(), ref.data_ptr(), ref_tok.data_ptr(), ref_st.data_ptr(),
                                     sup_ptr, count, stream) == 0
    out = torch.empty(rows, device="cuda")
    tok = torch.empty(1, dtype=torch.int64, device="cuda")
    st = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    assert lib.mstar_b200_q8_readout_noalloc(blocks.data_ptr(), blocks.numel(), rows, k, x.data_ptr(),
                                             out.data_ptr(), tok.data_ptr(), st.data_ptr(), sup_ptr, count,
                                             stream) == 0
    torch.cuda.synchronize()
    return (ref, ref_tok, ref_st), (out, tok, st)


@pytest.mark.parametrize("rows,k", [(51865, 384), (1000, 416), (5, 4096)])
def test_noalloc_readout_equals_handle_readout_on_consecutive_calls(rows, k):
    """Vocabulary width with an even block count (384: 12 blocks), an odd block count
    (416: 13, so the quantizer writes a padding block into the shared array), and the
    widest activation the array holds (4096), with and without suppression."""
    from mstar_accelerators_b200 import linear, native
    lib = native.load()
    native.require_capability(lib)
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(7 + k)
    blocks = linear.pack(torch.randn(rows, k, device="cuda", generator=g) * 0.02, "q8_0")
    head = linear.BlockLinear(blocks=blocks, fmt="q8_0", rows=rows, width=k)
    stream = torch.cuda.current_stream().cuda_stream
    suppression = [None, torch.tensor(sorted({3 % rows, 77 % rows, rows - 1}), dtype=torch.int64, device="cuda")]
    for call, sup in enumerate(suppression):
        x = torch.randn(k, device="cuda", generator=g)
        (ref, ref_tok, ref_st), (out, tok, st) = _call_both(lib, head.handle, blocks, rows, k, x, sup, stream)
        assert torch.equal(out, ref), f"call {call}: logits differ"
        assert int(tok) == int(ref_tok), f"call {call}: token differs"
        assert int(st) == 0 and int(ref_st) == 0
        if sup is not None:
            assert torch.isinf(out[sup]).all()
    # free device memory is read right around a lone no-allocation call whose every
    # operand exists beforehand: the call itself must not change it
    x = torch.randn(k, device="cuda", generator=g)
    out = torch.empty(rows, device="cuda")
    tok = torch.empty(1, dtype=torch.int64, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    before = torch.cuda.mem_get_info()[0]
    assert lib.mstar_b200_q8_readout_noalloc(blocks.data_ptr(), blocks.numel(), rows, k, x.data_ptr(),
                                             out.data_ptr(), tok.data_ptr(), st.data_ptr(), None, 0, stream) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == before, "the call changed free device memory"
    head.close()


def test_noalloc_readout_rejects_widths_beyond_its_scratch():
    from mstar_accelerators_b200 import native
    lib = native.load()
    native.require_capability(lib)
    rows, k = 8, 4128
    blocks = torch.zeros(rows * (k // 32) * 34, dtype=torch.uint8, device="cuda")
    x = torch.zeros(k, device="cuda")
    out = torch.empty(rows, device="cuda")
    tok = torch.empty(1, dtype=torch.int64, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.mstar_b200_q8_readout_noalloc(blocks.data_ptr(), blocks.numel(), rows, k, x.data_ptr(),
                                             out.data_ptr(), tok.data_ptr(), st.data_ptr(), None, 0,
                                             stream) == errno.E2BIG
