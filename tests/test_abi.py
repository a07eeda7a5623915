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


def _ctype_of(decl: str):
    """The ctypes type a C parameter or return declaration of the header maps to."""
    d = " ".join(decl.replace("const ", "").split())
    if "*" in d:
        return "char*" if d.startswith("char") else "ptr"
    base = d.rsplit(" ", 1)[0] if " " in d else d
    return {"int": C.c_int, "int32_t": C.c_int32, "int64_t": C.c_int64, "uint64_t": C.c_uint64,
            "uint32_t": C.c_uint32, "size_t": C.c_size_t, "float": C.c_float, "double": C.c_double,
            "void": None}[base]


def test_signatures_match_the_header():
    """Every ctypes signature in native.SIGNATURES has the header's parameter count and, per
    parameter, the same kind of type (pointer, char pointer, or the same scalar width)."""
    import re
    text = re.sub(r"/\*.*?\*/", "", native.HEADER.read_text(), flags=re.S)
    decls = re.findall(r"MSTAR_B200_API\s+([\w\s\*]+?)\b(mstar_b200_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.S)
    assert len(decls) == len(native.SIGNATURES)
    for ret, name, params in decls:
        restype, argtypes = native.SIGNATURES[name]
        plist = [p.strip() for p in params.split(",")] if params.strip() not in ("", "void") else []
        assert len(plist) == len(argtypes), name
        for i, (p, t) in enumerate(zip(plist, argtypes)):
            want = _ctype_of(p)
            if want == "ptr":
                assert t is C.c_void_p or (isinstance(t, type) and issubclass(t, C._Pointer)), (name, i, p)
            elif want == "char*":
                assert t is C.c_char_p, (name, i, p)
            else:
                assert C.sizeof(t) == C.sizeof(want) and (t in (C.c_float, C.c_double)) == (want in (C.c_float, C.c_double)), \
                    (name, i, p, t)
        r = _ctype_of(ret.strip() + " x") if "*" not in ret else "ptr"
        if r == "ptr":
            assert restype is C.c_void_p, name
        elif r is None:
            assert restype is None, name
        else:
            assert C.sizeof(restype) == C.sizeof(r), name
