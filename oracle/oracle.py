"""ORACLE — test infrastructure only.

numpy/ctypes front end of the CPU restatement in ``q8_oracle.c`` and of the
reference's own vendored ggml quantizers compiled into ``_ref/`` (see the
Makefile). Only tests, ``__graft_entry__.smoke`` and bench.py's CPU-baseline
leg import this module, and only to compare against. The product package never
imports it.

Byte formats follow ggml-common.h:194-199 (Q4_0, 18-byte blocks) and
ggml-common.h:251-256 (Q8_0, 34-byte blocks), row-major [rows][K/32] blocks.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libggml_quant_ref.so"
REF_LIB_512 = HERE / "_ref" / "libggml_quant_ref_avx512.so"   # AVX-512 VNNI build of the same sources

Q8_REF, Q8_ARM, Q8_X86 = 0, 1, 2
MODES = {"ref": Q8_REF, "arm": Q8_ARM, "x86": Q8_X86}
Q8_BLOCK, Q4_BLOCK = 34, 18

_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")


def build() -> None:
    """Compile liboracle.so (and _ref when the reference checkout exists)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "CC=gcc"], check=True)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not ORACLE_LIB.exists():
            build()
        L = C.CDLL(str(ORACLE_LIB))
        L.orc_fp32_to_fp16.argtypes = [C.c_float]
        L.orc_fp32_to_fp16.restype = C.c_uint16
        L.orc_fp16_to_fp32.argtypes = [C.c_uint16]
        L.orc_fp16_to_fp32.restype = C.c_float
        L.orc_quantize_row_q8_0.argtypes = [_f32p, _u8p, C.c_int64, C.c_int]
        L.orc_quantize_row_q4_0.argtypes = [_f32p, _u8p, C.c_int64, C.c_int]
        L.orc_pack_weights.argtypes = [_f32p, _u8p, C.c_int64, C.c_int64, C.c_int, C.c_int, C.c_int]
        L.orc_pack_weights.restype = C.c_int
        L.orc_block_sums_q8_0.argtypes = [_u8p, _u8p, C.c_int64, _i32p]
        L.orc_block_sums_q4_0.argtypes = [_u8p, _u8p, C.c_int64, _i32p]
        L.orc_mul_mat.argtypes = [_u8p, C.c_int, _f32p, _f32p, C.c_int64, C.c_int64, C.c_int64, C.c_int, _u8p]
        L.orc_argmax.argtypes = [_f32p, C.c_int64, _i64p, C.c_int64]
        L.orc_argmax.restype = C.c_int64
        L.orc_gelu_ggml.argtypes = [C.c_float]
        L.orc_gelu_ggml_rows.argtypes = [_f32p, _f32p, C.c_int64]
        L.orc_gelu_ggml_rows.restype = None
        L.orc_gelu_ggml.restype = C.c_float
        _u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
        L.orc_philox4x32_10.argtypes = [_u32p, _u32p, _u32p]
        L.orc_philox4x32_10.restype = None
        L.orc_categorical.argtypes = [_f32p, C.c_int64, C.c_int64, _i64p, _i64p, _f32p, _i64p]
        L.orc_categorical.restype = None
        _lib = L
    return _lib


def _host_has_avx512_vnni() -> bool:
    try:
        flags = Path("/proc/cpuinfo").read_text()
    except OSError:
        return False
    return all(f in flags for f in ("avx512f", "avx512bw", "avx512vl", "avx512dq", "avx512_vnni", "avx_vnni"))


def ref_lib():
    """The reference's ggml quantizers/dots (the AVX-512 VNNI build where the host has
    it, as ggml built with -march=native would be; else AVX2); None when not built."""
    global _ref
    path = REF_LIB_512 if REF_LIB_512.exists() and _host_has_avx512_vnni() else REF_LIB
    if _ref is None and path.exists():
        L = C.CDLL(str(path))
        for name in ("ref_quantize_q8_0_ref", "ref_quantize_q8_0_x86", "ref_quantize_q4_0_ref"):
            getattr(L, name).argtypes = [_f32p, _u8p, C.c_int64]
        L.ref_vec_dot.argtypes = [C.c_int, C.c_int, C.c_int, _u8p, _u8p]
        L.ref_vec_dot.restype = C.c_float
        L.ref_mul_mat.argtypes = [_u8p, C.c_int, _f32p, _f32p, C.c_int64, C.c_int64, C.c_int64, _u8p, C.c_int]
        _ref = L
    return _ref


def _f32(x):
    return np.ascontiguousarray(x, dtype=np.float32)


def quantize_q8_0(x, mode="arm") -> np.ndarray:
    """Activation/weight rows [..., K] fp32 -> Q8_0 bytes [..., K/32*34]."""
    x = _f32(x)
    k = x.shape[-1]
    out = np.zeros(x.shape[:-1] + (k // 32 * Q8_BLOCK,), np.uint8)
    lib().orc_quantize_row_q8_0(x.reshape(-1), out.reshape(-1), x.size, MODES[mode])
    return out


def quantize_q4_0(x, fused=True) -> np.ndarray:
    x = _f32(x)
    k = x.shape[-1]
    out = np.zeros(x.shape[:-1] + (k // 32 * Q4_BLOCK,), np.uint8)
    lib().orc_quantize_row_q4_0(x.reshape(-1), out.reshape(-1), x.size, int(fused))
    return out


def pack_weights(w, fmt="q8_0", preround=True, fused=True) -> np.ndarray:
    """Logical fp32 [rows, K] -> ggml blocks (decoder.cpp:307-316 / :816-842)."""
    w = _f32(w)
    rows, k = w.shape
    q4 = fmt == "q4_0"
    out = np.zeros((rows, k // 32 * (Q4_BLOCK if q4 else Q8_BLOCK)), np.uint8)
    status = lib().orc_pack_weights(w.reshape(-1), out.reshape(-1), rows, k, int(q4), int(preround), int(fused))
    if status == -1:
        raise ValueError("nonfinite weight")
    if status == -2:
        raise ValueError("weight overflows F16")
    if status:
        raise ValueError("invalid packing shape")
    return out


def block_sums(w_row: np.ndarray, x_row: np.ndarray, fmt="q8_0") -> np.ndarray:
    """Exact per-block int32 dots of one weight row and one Q8_0 activation row."""
    nb = x_row.size // Q8_BLOCK
    out = np.zeros(nb, np.int32)
    fn = lib().orc_block_sums_q4_0 if fmt == "q4_0" else lib().orc_block_sums_q8_0
    fn(np.ascontiguousarray(w_row, np.uint8), np.ascontiguousarray(x_row, np.uint8), nb, out)
    return out


def mul_mat(w_blocks: np.ndarray, x, fmt="q8_0", mode="arm") -> np.ndarray:
    """out[M, N] = generic-order ggml mul_mat of blocks W[N] with fp32 x[M, K]."""
    x = _f32(x)
    m, k = x.shape
    n = w_blocks.shape[0]
    out = np.zeros((m, n), np.float32)
    scratch = np.zeros(m * (k // 32) * Q8_BLOCK, np.uint8)
    lib().orc_mul_mat(np.ascontiguousarray(w_blocks, np.uint8).reshape(-1), int(fmt == "q4_0"),
                      x.reshape(-1), out.reshape(-1), m, n, k, MODES[mode], scratch)
    return out


def argmax(logits, suppressed=()) -> tuple[np.ndarray, int]:
    """Suppression + first-index / NaN-first argmax; returns (masked logits, token)."""
    l = _f32(logits).copy()
    s = np.ascontiguousarray(np.asarray(suppressed, np.int64).reshape(-1))
    tok = lib().orc_argmax(l, l.size, s, s.size)
    return l, int(tok)


def philox4x32_10(counter, key) -> tuple[int, ...]:
    """Random123 Philox4x32-10 of four counter and two key words."""
    out = np.zeros(4, np.uint32)
    lib().orc_philox4x32_10(np.asarray(counter, np.uint32), np.asarray(key, np.uint32), out)
    return tuple(int(v) for v in out)


def categorical(logits, seeds, offsets, temperatures) -> np.ndarray:
    """philox4x32-10-gumbel23-v1 draws of each row of fp32 logits [rows, vocab] (-1: invalid row)."""
    x = _f32(logits)
    rows, vocab = x.shape
    out = np.zeros(rows, np.int64)
    lib().orc_categorical(x.reshape(-1), rows, vocab, np.ascontiguousarray(seeds, np.int64).reshape(-1),
                          np.ascontiguousarray(offsets, np.int64).reshape(-1),
                          _f32(temperatures).reshape(-1), out)
    return out


def fp16_round(x) -> np.ndarray:
    return _f32(x).astype(np.float16).astype(np.float32)


def dequantize(blocks: np.ndarray, fmt="q8_0") -> np.ndarray:
    """Block bytes [rows, nb*B] -> fp32 values [rows, K] (value = q * d)."""
    rows = blocks.shape[0]
    bsz = Q4_BLOCK if fmt == "q4_0" else Q8_BLOCK
    b = blocks.reshape(rows, -1, bsz)
    d = b[..., :2].copy().view(np.float16).astype(np.float32)
    if fmt == "q4_0":
        qs = b[..., 2:]
        lo = (qs & 0x0F).astype(np.int32) - 8
        hi = (qs >> 4).astype(np.int32) - 8
        q = np.concatenate([lo, hi], axis=-1)
    else:
        q = b[..., 2:].view(np.int8).astype(np.int32)
    return (q * d).reshape(rows, -1).astype(np.float32)


def gelu_ggml(x) -> np.ndarray:
    x = _f32(x)
    y = np.empty_like(x)
    lib().orc_gelu_ggml_rows(x.reshape(-1), y.reshape(-1), x.size)
    return y


def ref_quantize(x, which: str) -> np.ndarray:
    """The reference's compiled quantizer: 'q8_ref', 'q8_x86' or 'q4_ref'."""
    L = ref_lib()
    x = _f32(x)
    k = x.shape[-1]
    bsz = Q4_BLOCK if which == "q4_ref" else Q8_BLOCK
    out = np.zeros(x.shape[:-1] + (k // 32 * bsz,), np.uint8)
    fn = {"q8_ref": L.ref_quantize_q8_0_ref, "q8_x86": L.ref_quantize_q8_0_x86,
          "q4_ref": L.ref_quantize_q4_0_ref}[which]
    rows = x.reshape(-1, k)
    o = out.reshape(rows.shape[0], -1)
    for i in range(rows.shape[0]):
        fn(np.ascontiguousarray(rows[i]), o[i], k)
    return out


def ref_mul_mat(w_blocks, x, fmt="q8_0", threads=0) -> np.ndarray:
    """The reference's x86 ggml mul_mat arithmetic (AVX2 quantizer + vec_dot)."""
    L = ref_lib()
    x = _f32(x)
    m, k = x.shape
    n = w_blocks.shape[0]
    out = np.zeros((m, n), np.float32)
    scratch = np.zeros(m * (k // 32) * Q8_BLOCK, np.uint8)
    L.ref_mul_mat(np.ascontiguousarray(w_blocks, np.uint8).reshape(-1), int(fmt == "q4_0"),
                  x.reshape(-1), out.reshape(-1), m, n, k, scratch, int(threads))
    return out


def cpu_cores() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
