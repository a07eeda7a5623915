"""Host-side argument validation of the C-ABI: a malformed call returns -1 with the
reason in the error buffer before anything reaches the device (the reference's
native ABIs validate the same way, backends/cpu_ggml/decoder.cpp:29-49, 414-446).
These run on any host: every case is refused by a check that precedes the first
CUDA call of its entry point."""
import ctypes as C

import pytest

from mstar_accelerators_b200 import build, native

FAKE = 0x10000   # a 64 KB-aligned address that is never dereferenced: validation stops first


@pytest.fixture(scope="module")
def lib():
    build.build()
    return native.load()


def _call(fn, *args):
    e = C.create_string_buffer(256)
    rc = fn(*args, e, len(e))
    return rc, e.value.decode()


def _stage_heads(lib, seqs=2, heads=4, positions=8, head_dim=128, strides=None, attention=FAKE, staged=FAKE,
                 rounding=1):
    s0, s1, s2 = strides or (heads * positions * head_dim, positions * head_dim, head_dim)
    return _call(lib.mstar_b200_stage_heads, attention, seqs, heads, positions, head_dim, s0, s1, s2, staged,
                 1 << 30, rounding, FAKE, None)


def test_stage_heads_refusals(lib):
    assert _stage_heads(lib, head_dim=48) == (-1, "invalid attention layout (head_dim a multiple of 32)")
    assert _stage_heads(lib, strides=(4096, 1028, 128))[1] == \
        "attention strides must be non-negative multiples of 8 elements"
    assert _stage_heads(lib, attention=FAKE + 8) == (-1, "attention output must be 16-byte aligned")
    assert _stage_heads(lib, attention=None)[1] == "missing staging operand"
    assert _stage_heads(lib, rounding=3)[1] == "unknown Q8_0 activation rounding"


def _qknorm(fn, head_dim=128, q=FAKE, q_s0=5120, eps=1e-6):
    return _call(fn, q, q_s0, 128, FAKE, q_s0, 128, None, 0, 0, FAKE, FAKE, FAKE, 128, FAKE, 128, 4, 32, 4, head_dim,
                 C.c_float(eps), 1, FAKE, FAKE, None, 512, None, 64, FAKE, None)


@pytest.mark.parametrize("name", ["mstar_b200_qknorm_rope", "mstar_b200_qknorm_rope_f32"])
def test_qknorm_rope_refusals(lib, name):
    fn = getattr(lib, name)
    assert _qknorm(fn, head_dim=64) == (-1, "head_dim must be 128")
    assert _qknorm(fn, eps=float("nan"))[1] == "invalid RMSNorm epsilon"
    assert _qknorm(fn, q_s0=5122)[1] == "strides must keep 8-byte alignment"
    assert _qknorm(fn, q=None)[1] == "missing prologue operand"


def test_qknorm_rope_f32_wants_16_byte_rows(lib):
    assert _qknorm(lib.mstar_b200_qknorm_rope_f32, q=FAKE + 8)[1] == "fp32 q / k / v rows must be 16-byte aligned"
    # the bf16 form accepts the same 8-byte aligned rows and fails only later, at the device check
    assert _qknorm(lib.mstar_b200_qknorm_rope, q=FAKE + 8)[1] != "fp32 q / k / v rows must be 16-byte aligned"


def test_stage_rows_refusals(lib):
    def stage(fmt=0, width=1280, stride=1280, x=FAKE):
        return _call(lib.mstar_b200_stage_rows, x, fmt, stride, 16, width, None, None, C.c_float(0.0), FAKE,
                     1 << 30, 1, FAKE, None)
    assert stage(fmt=7) == (-1, "staged rows are fp32 or fp16")
    assert stage(width=48)[1] == "invalid staging shape"
    assert stage(stride=1282)[1] == "row stride must be a multiple of 4 elements"
    assert stage(x=FAKE + 4)[1] == "activation rows must be aligned"


def test_rms_norm_and_residual_refusals(lib):
    def rms(width=2048, eps=1e-6, x=FAKE):
        return _call(lib.mstar_b200_rms_norm, x, width, 4, width, FAKE, C.c_float(eps), FAKE, width, None, 0, None)
    assert rms(width=12)[0] == -1
    assert rms(x=None)[1] == "missing RMSNorm operand"
    assert rms(eps=-1.0)[1] == "invalid epsilon"
    rc, msg = _call(lib.mstar_b200_residual_add_bf16, FAKE, FAKE, 12, FAKE, None)
    assert (rc, msg) == (-1, "element count must be a multiple of 8")


def test_pack_refusals(lib):
    def pack(fmt=8, rows=4, width=64, inp=FAKE, out=FAKE + 4096, out_bytes=4 * 2 * 34):
        return _call(lib.mstar_b200_pack, fmt, inp, rows * width * 4, out, out_bytes, rows, width, 1, 1, None)
    assert pack(fmt=3) == (-1, "unsupported block format")
    assert pack(width=48)[0] == -1 and pack(width=48)[1] != "unsupported block format"
    # borrowed extents must be exactly the bytes the shape implies
    assert pack(out_bytes=4 * 2 * 34 + 2)[1] == "invalid borrowed storage extent/alignment: packing output"
    assert pack(out=FAKE + 512)[1] == "packing input/output overlap"


def test_categorical_refusals(lib):
    def cat(rows=2, vocab=100, ld=100, workspace_bytes=1 << 16, seeds=FAKE):
        return _call(lib.mstar_b200_categorical, FAKE, rows, vocab, ld, seeds, FAKE + 256, FAKE + 512, FAKE + 768,
                     FAKE + 1024, workspace_bytes, None)
    assert cat(rows=0) == (-1, "rows must be 1..65535")
    assert cat(ld=50)[1] == "invalid vocabulary extent"
    assert cat(seeds=None)[1] == "missing sampling operand"
    assert cat(workspace_bytes=1)[1] == "sampling workspace too small"


def test_router_refusals(lib):
    def route(experts=128, top_k=8, x=FAKE):
        return _call(lib.mstar_b200_moe_route, x, 4, 2048, FAKE, experts, top_k, 1, FAKE, FAKE, FAKE, None)
    assert route(x=None) == (-1, "missing router operand")
    assert route(experts=300)[1] == "router geometry: 1..256 experts"
    assert route(top_k=9)[1] == "top_k outside 1..8"
