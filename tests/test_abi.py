"""The C-ABI library loads on any host and exports exactly what the public
header declares; capability is refused without an sm_100 device."""
import ctypes as C
import hashlib

import pytest

from mstar_accelerators_b200 import build, native


@pytest.fixture(scope="module")
def lib():
    build.build()
    return native.load()


def test_every_declared_symbol_is_exported(lib):
    declared = native.declared_symbols()
    assert len(declared) >= 10
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing
    assert set(declared) == set(native.SIGNATURES)


def test_abi_and_capability(lib):
    import torch
    assert lib.mstar_b200_abi() == 1
    expect = torch.cuda.is_available() and torch.cuda.get_device_capability() == (10, 0)
    assert lib.mstar_b200_capability() == int(expect)


def test_sha256_pin_is_enforced(lib):
    digest = hashlib.sha256(native.LIBRARY.read_bytes()).hexdigest()
    assert native.load(sha256=digest) is not None
    with pytest.raises(native.NativeError, match="SHA256"):
        native.load(sha256="0" * 64)


def test_create_without_capability_reports_an_error(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("device present")
    e = native.error_buffer()
    assert not lib.mstar_b200_linear_create(native.Q8_0, None, 0, 8, 32, None, e, len(e))
    assert b"capability" in e.value


def test_errno_mirrors_refuse_without_device(lib):
    import errno
    import torch
    if torch.cuda.is_available():
        pytest.skip("device present")
    assert lib.mstar_b200_q8_quantize(None, None, 0, 1, 32, 1, None) == errno.ENOTSUP


def test_close_of_null_handle_is_a_no_op(lib):
    e = native.error_buffer()
    assert lib.mstar_b200_linear_close(None, e, len(e)) == 0
