"""Every device wait in the library is bounded and reports a timeout in the
call's status word instead of hanging the GPU. Each test makes one wait run
out on purpose with a limit of about a millisecond, on one GPU, with nothing
faulted or trapped:

  * an mbarrier that nothing arrives at (the wait of every TMA / tcgen05
    pipeline, mbar_wait_bounded): status bit value 2;
  * the persistent decode step's grid barrier with a CTA that never arrives:
    status bit value 32;
  * the tensor-parallel peer barrier (mstar_b200_tp_barrier) with world = 2
    where the "peer" is a second local buffer whose flag nothing ever sets:
    status bit value 16, after the limit set by mstar_b200_set_wait_limits.

After each, the same stream runs an ordinary kernel to show the context is
still usable.
"""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def lib():
    from mstar_accelerators_b200 import native
    return native.require_capability()


def run(fn, *args):
    from mstar_accelerators_b200.native import check, error_buffer
    e = error_buffer()
    check(fn(*args, e, len(e)), e, "wait test")


def still_usable():
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float((x * 2).sum().item()) == 1023 * 1024


@pytest.mark.parametrize("kind,bit", [(0, 2), (1, 32)])
def test_selftest_wait_gives_up(kind, bit):
    L = lib()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    words = torch.zeros(2, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    run(L.mstar_b200_wait_selftest, kind, 20000, words.data_ptr(), status.data_ptr(), stream)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 30.0
    assert int(status.item()) & bit
    still_usable()


def test_tp_barrier_gives_up_when_a_peer_never_arrives():
    L = lib()
    mine = torch.zeros(2, dtype=torch.int32, device="cuda")
    peer = torch.zeros(2, dtype=torch.int32, device="cuda")   # stands in for rank 1's flags; nothing answers
    ptrs = torch.tensor([mine.data_ptr(), peer.data_ptr()], dtype=torch.int64, device="cuda")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    run(L.mstar_b200_set_wait_limits, 10000, 0)      # ~1 ms of 100 ns polls
    try:
        t0 = time.perf_counter()
        run(L.mstar_b200_tp_barrier, ptrs.data_ptr(), mine.data_ptr(), 0, 2, counter.data_ptr(), status.data_ptr(),
            stream)
        torch.cuda.synchronize()
        assert time.perf_counter() - t0 < 30.0
    finally:
        run(L.mstar_b200_set_wait_limits, 0, 0)      # back to the defaults
    assert int(status.item()) & 16
    assert int(counter.item()) == 1 and int(mine[0].item()) == 1 and int(peer[0].item()) == 1
    still_usable()


def test_wait_limits_reject_negative_values():
    from mstar_accelerators_b200 import native
    L = lib()
    with pytest.raises(native.NativeError):
        run(L.mstar_b200_set_wait_limits, -1, 0)
