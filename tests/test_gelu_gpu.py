"""The epilogue GELU equals ggml's fp16 GELU table for every input.

ggml's stock GELU (ggml-cpu/vec.h:963-969, 1000-1013) is a lookup in a 65536-entry
fp16 table built with the host's tanhf (ggml-cpu.c:3889); the oracle
(orc_gelu_ggml) restates it. The kernels look up the same table, which the
library builds on the host in ggml's operation order, so the results must be
bit-identical to the oracle on all 65536 fp16 inputs (NaN where the oracle gives
NaN) and on arbitrary fp32 inputs, through both the tcgen05 GEMM epilogue (table
in shared memory) and the decode GEMV epilogue (table in global memory). The
inputs enter as the bias of an all-zero weight matrix, so the epilogue sees
exactly bias + 0.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def inputs():
    every = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32)
    rng = np.random.default_rng(3)
    extra = rng.uniform(-12, 12, 65536).astype(np.float32)
    near = (np.float32(10.0) + rng.uniform(-0.02, 0.02, 4096)).astype(np.float32)
    return np.concatenate([every, extra, near, -near])


def expect(v):
    return O.gelu_ggml((v + np.float32(0.0)).astype(np.float32))


def same(got, ref):
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_gelu_gemm_epilogue_matches_table():
    from mstar_accelerators_b200 import linear
    v = inputs()
    n = v.size
    lin = linear.BlockLinear(torch.zeros(n, 64, device="cuda"), bias=torch.from_numpy(v).cuda())
    lin.prepare_gemm(64)
    a = linear.stage_rows(torch.zeros(128, 64, device="cuda"))
    got = lin.gemm(a, gelu="tanh")[0].cpu().numpy()
    same(got, expect(v))
    lin.close()


def test_gelu_gemv_epilogue_matches_table():
    from mstar_accelerators_b200 import linear
    v = inputs()
    n = v.size
    lin = linear.BlockLinear(torch.zeros(n, 64, device="cuda"), bias=torch.from_numpy(v).cuda())
    got = lin(torch.zeros(1, 64, device="cuda"), gelu="tanh")[0].cpu().numpy()
    same(got, expect(v))
    lin.close()
