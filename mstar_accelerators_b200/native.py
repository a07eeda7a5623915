"""ctypes binding of libmstar_b200 (declared in include/mstar_b200.h).

Loading follows the reference's artifact discipline
(implementations/whisper/cpu_ggml.py:78-96, backends/torch/q8.py:42-77): an
optional SHA256 pin, an ABI check (``mstar_b200_abi() == 1``) and a separate
capability query (``mstar_b200_capability() == 1`` only on an sm_100 device).
There is no fallback: a missing library or capability raises.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import re
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
LIBRARY = PACKAGE / "libmstar_b200.so"
HEADER = PACKAGE.parent / "include" / "mstar_b200.h"

Q8_REF, Q8_ARM, Q8_X86 = 0, 1, 2
ROUNDING = {"ref": Q8_REF, "arm": Q8_ARM, "x86": Q8_X86}
Q8_0, Q4_0, BF16 = 8, 4, 16
FORMATS = {"q8_0": Q8_0, "q4_0": Q4_0, "bf16": BF16}
BIAS, GELU, RESIDUAL, GELU_ERF = 1, 2, 4, 8
ACT_F32, ACT_F16 = 0, 1
OUT_F32, OUT_F16, OUT_STAGED = 0, 1, 2


class Q8Frags(C.Structure):
    """mstar_b200_q8_frags: a handle's Q8_0 activation-fragment buffers."""
    _fields_ = [("fragments", C.c_void_p), ("scales", C.c_void_p), ("sums", C.c_void_p), ("blocks", C.c_int64),
                ("rows", C.c_int64), ("rounding", C.c_int32)]

_vp, _i64, _u64, _sz, _int = C.c_void_p, C.c_int64, C.c_uint64, C.c_size_t, C.c_int
_err = [C.c_char_p, _sz]

# name -> (restype, argtypes)
SIGNATURES = {
    "mstar_b200_abi": (_int, []),
    "mstar_b200_capability": (_int, []),
    "mstar_b200_pack": (_int, [_int, _vp, _u64, _vp, _u64, _i64, _i64, _int, _int, _vp, *_err]),
    "mstar_b200_q8_quantize": (_int, [_vp, _vp, _sz, _i64, _i64, _int, _vp]),
    "mstar_b200_linear_create": (_vp, [_int, _vp, _u64, _i64, _i64, _vp, *_err]),
    "mstar_b200_linear_run": (_int, [_vp, _vp, _i64, _i64, _vp, _i64, _vp, _int, _vp, _vp, C.c_float, _int, _vp,
                                     *_err]),
    "mstar_b200_linear_block_sums": (_int, [_vp, _vp, _i64, _vp, _u64, _int, _vp, *_err]),
    "mstar_b200_linear_readout": (_int, [_vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _u64, _vp, _vp, C.c_float, _int,
                                         _vp, *_err]),
    "mstar_b200_linear_close": (_int, [_vp, *_err]),
    "mstar_b200_linear_set_split": (_int, [_vp, _int, *_err]),
    "mstar_b200_linear_prepare_gemm": (_int, [_vp, _vp, _u64, _i64, *_err]),
    "mstar_b200_linear_prepare_readout": (_int, [_vp, _vp, _u64, *_err]),
    "mstar_b200_linear_frags": (_int, [_vp, _i64, C.c_int32, _vp, *_err]),
    "mstar_b200_linear_run_frags": (_int, [_vp, _i64, _vp, _i64, _vp, _int, _vp, *_err]),
    "mstar_b200_linear_run_q8out": (_int, [_vp, _vp, _i64, _i64, _vp, _i64, _vp, _int, _vp, _vp, C.c_float, _int,
                                           _vp, _vp, *_err]),
    "mstar_b200_linear_gemm": (_int, [_vp, _vp, _u64, _i64, _vp, _u64, _i64, C.c_int32, _vp, _u64, _i64, _i64, _i64,
                                      _i64, C.c_int32, C.c_int32, _vp, _vp, *_err]),
    "mstar_b200_residual_add_bf16": (_int, [_vp, _vp, _i64, _vp, _vp, *_err]),
    "mstar_b200_stage_heads": (_int, [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _u64, C.c_int32, _vp,
                                      _vp, *_err]),
    "mstar_b200_rms_norm": (_int, [_vp, _i64, _i64, _i64, _vp, C.c_float, _vp, _i64, _vp, _i64, _vp, *_err]),
    "mstar_b200_tp_barrier": (_int, [_vp, _vp, C.c_int32, C.c_int32, _vp, _vp, _vp, *_err]),
    "mstar_b200_linear_gemm_push": (_int, [_vp, _vp, _u64, _i64, _vp, _vp, C.c_int32, C.c_int32, _i64, _vp, _vp,
                                           *_err]),
    "mstar_b200_tp_reduce_recv": (_int, [_vp, _vp, C.c_int32, _i64, _i64, _i64, _vp, _vp, _vp, _vp, C.c_float, _vp,
                                         _vp, _i64, C.c_int32, _vp, _vp, *_err]),
    "mstar_b200_tp_reduce_multicast": (_int, [_vp, C.c_int32, _i64, _i64, _vp, _vp, _vp, _vp, C.c_float, _vp, _i64,
                                              C.c_int32, _vp, _vp, *_err]),
    "mstar_b200_set_wait_limits": (_int, [_i64, _i64, *_err]),
    "mstar_b200_categorical_workspace": (_u64, [_i64]),
    "mstar_b200_q8_exact_pad": (_i64, [_i64]),
    "mstar_b200_q8_exact_weights": (_int, [_vp, _u64, _i64, _i64, _vp, _vp, _vp, *_err]),
    "mstar_b200_q8_exact_activations": (_int, [_vp, _i64, _i64, _i64, C.c_int32, _vp, _vp, _vp, _vp, *_err]),
    "mstar_b200_gemm_q8_exact": (_int, [_vp, _vp, _i64, _vp, _vp, _i64, _i64, _vp, _vp, _i64, _vp, _vp, *_err]),
    "mstar_b200_qknorm_rope": (_int, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _vp, _i64,
                                      _i64, C.c_int32, C.c_int32, C.c_int32, C.c_float, C.c_int32, _vp, _vp, _vp, _i64,
                                      _vp, _i64, _vp, _vp, *_err]),
    "mstar_b200_qknorm_rope_f32": (_int, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _vp,
                                          _i64, _i64, C.c_int32, C.c_int32, C.c_int32, C.c_float, C.c_int32, _vp, _vp,
                                          _vp, _i64, _vp, _i64, _vp, _vp, *_err]),
    "mstar_b200_categorical": (_int, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _u64, _vp, *_err]),
    "mstar_b200_wait_selftest": (_int, [C.c_int32, _i64, _vp, _vp, _vp, *_err]),
    "mstar_b200_tp_reduce": (_int, [_vp, C.c_int32, _i64, _i64, _vp, _vp, _vp, _vp, C.c_float, _vp, _i64,
                                    C.c_int32, _vp, _vp, *_err]),
    "mstar_b200_stage_rows": (_int, [_vp, C.c_int32, _i64, _i64, _i64, _vp, _vp, C.c_float, _vp, _u64, C.c_int32, _vp,
                                     _vp, *_err]),
    "mstar_b200_stage_conv": (_int, [_vp, C.c_int32, _i64, _i64, _i64, C.c_int32, _i64, _vp, _u64, C.c_int32, _vp, _vp,
                                     *_err]),
    "mstar_b200_layer_norm": (_int, [_vp, _i64, _i64, _i64, _vp, _vp, C.c_float, _vp, _i64, _vp, *_err]),
    "mstar_b200_q8_readout": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "mstar_b200_embed": (_int, [_vp, _i64, _vp, _i64, _i64, _vp, _vp, _i64, C.c_float, _vp, _vp, _vp, *_err]),
    "mstar_b200_attend_workspace": (_u64, [C.c_int32, C.c_int32, C.c_int32, _i64, C.c_int32]),
    "mstar_b200_attend": (_int, [_vp, _i64, _vp, _vp, _i64, _vp, _vp, _i64, C.c_int32, C.c_int32, C.c_int32,
                                 C.c_int32, _vp, _vp, C.c_int32, C.c_int32, _vp, _i64, C.c_float, _vp, _vp, _u64,
                                 _vp, *_err]),
    "mstar_b200_attend_q8": (_int, [_vp, _i64, _vp, _vp, _i64, _vp, _vp, _i64, C.c_int32, C.c_int32, C.c_int32,
                                 C.c_int32, _vp, _vp, C.c_int32, C.c_int32, _vp, _i64, C.c_float, _vp, _vp, _u64,
                                 _vp, _vp, *_err]),
    "mstar_b200_fill_kv": (_int, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _vp, *_err]),
    "mstar_b200_moe_route": (_int, [_vp, _i64, _i64, _vp, C.c_int32, C.c_int32, C.c_int32, _vp, _vp, _vp, _vp,
                                    *_err]),
    "mstar_b200_moe_create": (_vp, [C.c_int32, _vp, _u64, _vp, _u64, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                    C.c_int32, *_err]),
    "mstar_b200_moe_run": (_int, [_vp, _vp, _i64, _vp, _vp, _vp, _vp, C.c_int32, _vp, *_err]),
    "mstar_b200_moe_close": (_int, [_vp, *_err]),
    "mstar_b200_moe_combine": (_int, [_vp, _i64, _vp, _i64, C.c_int32, _i64, _vp, _vp, *_err]),
    "mstar_b200_moe_run_experts": (_int, [_vp, _vp, _i64, _vp, _vp, C.c_int32, C.c_int32, _vp, _i64, _i64, _vp,
                                          _vp, C.c_int32, _vp, *_err]),
    "mstar_b200_thinker_reduce": (_int, [_vp, _vp, C.c_int32, C.c_int32, _i64, _i64, _i64, _vp, *_err]),
    "mstar_b200_thinker_combine": (_int, [_vp, _vp, _i64, _vp, C.c_int32, C.c_int32, C.c_int32, _vp,
                                          C.c_int32, C.c_int32, _i64, _i64, _i64, _vp, _vp, *_err]),
    "mstar_b200_moe_dispatch": (_int, [_vp, _i64, _i64, _vp, _vp, C.c_int32, C.c_int32, C.c_int32, _vp, _vp, _vp,
                                       _vp, _vp, *_err]),
    "mstar_b200_decode_step_create": (_vp, [_vp, *_err]),
    "mstar_b200_decode_step_run": (_int, [_vp, _vp, *_err]),
    "mstar_b200_decode_step_close": (_int, [_vp, *_err]),
    "mstar_b200_q8_readout_noalloc": (_int, [_vp, _sz, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
}


class NativeError(RuntimeError):
    pass


def declared_symbols(header: Path = HEADER) -> list[str]:
    """Every entry point the public header declares."""
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    return re.findall(r"MSTAR_B200_API\s+[\w\s\*]+?\b(mstar_b200_\w+)\s*\(", text)


_cache: dict[tuple, C.CDLL] = {}


def load(path: str | Path | None = None, sha256: str | None = None) -> C.CDLL:
    """Load (once) and type the library; verify its digest when one is pinned."""
    path = Path(path or LIBRARY).resolve()
    key = (str(path), sha256)
    if key in _cache:
        return _cache[key]
    if not path.is_file():
        raise NativeError(f"libmstar_b200 is not built: {path} (run mstar_accelerators_b200.build)")
    if sha256 is not None:
        with path.open("rb") as stream:
            if hashlib.file_digest(stream, "sha256").hexdigest() != sha256:
                raise NativeError("libmstar_b200 artifact SHA256 differs")
    lib = C.CDLL(str(path))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if lib.mstar_b200_abi() != 1:
        raise NativeError("libmstar_b200 ABI differs")
    _cache[key] = lib
    return lib


def capability(lib: C.CDLL | None = None) -> bool:
    return (lib or load()).mstar_b200_capability() == 1


def require_capability(lib: C.CDLL | None = None) -> C.CDLL:
    lib = lib or load()
    if lib.mstar_b200_capability() != 1:
        raise NativeError("sm_100a capability is unavailable on the current CUDA device")
    return lib


def error_buffer():
    return C.create_string_buffer(1024)


def check(status: int, error, what: str) -> None:
    if status:
        raise NativeError(f"{what}: {error.value.decode(errors='replace')}")
