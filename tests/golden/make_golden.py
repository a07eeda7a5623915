"""Generate the committed golden vectors under tests/golden/ (run in a
container where the reference checkout exists; the GPU machine only reads the
.npz files).

Sources of truth, all from the reference itself:
  * q8_kat.npz     — the explicit known-answer bytes of the reference's
                     tests/whisper/test_q8_readout.py:13-36 (roundf ties, fp32
                     scale vs fp16 storage, fp16 underflow), restated here.
  * q8_pack.npz    — the reference's Python packer pack_q8_0
                     (src/mstar_accelerators/implementations/whisper/pi_v3d/q8.py:16-45)
                     imported from the checkout (its unrelated M* imports are
                     stubbed) and run on seeded weights with planted ties.
  * q4_pack.npz    — the reference's own Q4 fixture input
                     (tests/test_cpu_ggml_q4_readout.py:79: linspace(-1.71, 1.83, 7*384))
                     packed by the vendored ggml quantize_row_q4_0_ref compiled
                     into oracle/_ref, after the fp16 pre-round of
                     backends/cpu_ggml/decoder.cpp:816-842, plus the test's two
                     scalar rounding models (fma / separate).
  * mul_mat.npz    — generic-order ggml vec_dot results (oracle/_ref) for seeded
                     Q8_0 and Q4_0 weights and activations at small shapes.
"""
from __future__ import annotations

import importlib.util
import os
import struct
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
# the reference checkout: MSTAR_REFERENCE in the environment, else its usual place here
REFERENCE = Path(os.environ.get("MSTAR_REFERENCE", "/root/reference"))
sys.path.insert(0, str(REPO))

from oracle import oracle as O  # noqa: E402


def reference_pack_q8_0():
    """Import pack_q8_0 from the reference checkout with its M* imports stubbed."""
    import torch  # noqa: F401  (the packer is torch code)
    stub = types.ModuleType("mstar_accelerators.backends.graph")
    stub.NativeGraphProvider = object
    for name in ("mstar_accelerators", "mstar_accelerators.backends"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["mstar_accelerators.backends.graph"] = stub
    path = REFERENCE / "src/mstar_accelerators/implementations/whisper/pi_v3d/q8.py"
    spec = importlib.util.spec_from_file_location("_reference_q8", path)
    module = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = module
    spec.loader.exec_module(module)
    return module.pack_q8_0


def q8_kat():
    cases = []
    values = [127, -127, .5, -.5, 1.5, -1.5, 2.5, -2.5, 126.5, -126.5] + [0] * 22
    w = np.array([values, [0] * 32], np.float32)
    exp = struct.pack('<e32b', 1, 127, -127, 1, -1, 2, -2, 3, -3, 127, -127, *([0] * 22)) + bytes(34)
    cases.append((w, exp))
    w = np.zeros((2, 32), np.float32)
    w[:, :4] = [63.5, -63.5, .25, -.25]
    cases.append((w.copy(), struct.pack('<e32b', .5, 127, -127, 1, -1, *([0] * 28)) * 2))
    w = np.zeros((2, 32), np.float32)
    w[:, 0] = 1e-12
    cases.append((w.copy(), struct.pack('<e32b', 0, 127, *([0] * 31)) * 2))
    out = {}
    for i, (w, e) in enumerate(cases):
        out[f"w{i}"] = w
        out[f"bytes{i}"] = np.frombuffer(e, np.uint8)
    np.savez(HERE / "q8_kat.npz", **out)


def q8_pack():
    import torch
    pack = reference_pack_q8_0()
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((24, 384)) * 0.02).astype(np.float32)
    w[0, :32] = 0.0
    w[1, :32] = np.linspace(-127, 127, 32) / 127 * 0.5   # exact-ish ties region
    w[2, :4] = [63.5, -63.5, 0.25, -0.25]
    w[2, 4:32] = 0
    w[3, :32] = 1e-12
    packed = pack(torch.from_numpy(w)).view(torch.uint8).numpy().reshape(24, -1)
    np.savez(HERE / "q8_pack.npz", w=w, packed=packed)


def q4_pack():
    x = np.linspace(-1.71, 1.83, 7 * 384, dtype=np.float32).reshape(7, 384)
    xh = O.fp16_round(x)
    ref = O.ref_quantize(xh, "q4_ref")
    # The reference test's scalar model (tests/test_cpu_ggml_q4_readout.py:79-91).
    b = xh.reshape(-1, 32)
    idx = np.abs(b).argmax(1)
    mx = b[np.arange(b.shape[0]), idx]
    d = (mx / np.float32(-8)).astype(np.float32)
    inv = np.where(d != 0, (np.float32(1) / np.where(d != 0, d, 1)).astype(np.float32), np.float32(0))
    models = {}
    for mode in ("fma", "separate"):
        if mode == "fma":
            t = (b.astype(np.float64) * inv[:, None].astype(np.float64) + 8.5).astype(np.float32)
        else:
            t = ((b * inv[:, None]).astype(np.float32) + np.float32(8.5)).astype(np.float32)
        q = np.minimum(t.astype(np.int32), 15).astype(np.uint8)
        blk = np.concatenate([d.astype(np.float16).view(np.uint8).reshape(-1, 2), q[:, :16] | (q[:, 16:] << 4)], 1)
        models[mode] = blk.reshape(7, -1)
    np.savez(HERE / "q4_pack.npz", x=x, ggml=ref.reshape(7, -1), fma=models["fma"], separate=models["separate"])


def mul_mat():
    L = O.ref_lib()
    rng = np.random.default_rng(5)
    out = {}
    for fmt, n, k, m in (("q8_0", 40, 384, 5), ("q4_0", 40, 384, 3), ("q8_0", 16, 1536, 2)):
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        blocks = O.pack_weights(w, fmt)
        x = rng.standard_normal((m, k)).astype(np.float32)
        xq = O.ref_quantize(x, "q8_x86")
        res = np.array([[L.ref_vec_dot(int(fmt == "q4_0"), 1, k, np.ascontiguousarray(blocks[r]),
                                       np.ascontiguousarray(xq[i])) for r in range(n)] for i in range(m)],
                       np.float32)
        tag = f"{fmt}_{n}x{k}x{m}"
        out[tag + "_blocks"], out[tag + "_x"], out[tag + "_out"] = blocks, x, res
    np.savez(HERE / "mul_mat.npz", **out)


def reference_categorical():
    """The reference's own scalar categorical oracle, imported from the checkout
    (backends/pi/torch/tests/categorical_reference.py; it imports only the standard library)."""
    path = REFERENCE / "backends/pi/torch/tests/categorical_reference.py"
    spec = importlib.util.spec_from_file_location("_reference_categorical", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def categorical():
    """Draws of the reference's scalar oracle on seeded rows: ordinary finite rows at
    several temperatures, 64-bit seeds and offsets, exact ties, -inf masks, +inf
    entries, a NaN row, an all -inf row and invalid temperatures."""
    ref = reference_categorical()
    ref.known_answers()
    rng = np.random.default_rng(31)
    V = 257
    rows = [rng.standard_normal(V).astype(np.float32) * s for s in (0.5, 2.0, 8.0, 0.1)]
    r = np.zeros(V, np.float32); r[[3, 100, 200]] = 5.0; rows.append(r)                    # tied maxima
    r = rng.standard_normal(V).astype(np.float32); r[::2] = -np.inf; rows.append(r)         # masked entries
    r = rng.standard_normal(V).astype(np.float32); r[[7, 150]] = np.inf; rows.append(r)    # +inf entries
    r = rng.standard_normal(V).astype(np.float32); r[42] = np.nan; rows.append(r)          # NaN
    rows.append(np.full(V, -np.inf, np.float32))                                          # nothing to draw
    rows.append(rng.standard_normal(V).astype(np.float32))                                # invalid temperature
    rows.append(rng.standard_normal(V).astype(np.float32))                                # invalid temperature
    logits = np.stack(rows)
    n = len(rows)
    seeds = rng.integers(-(1 << 63), (1 << 63) - 1, n, dtype=np.int64)
    offsets = rng.integers(-(1 << 63), (1 << 63) - 1, n, dtype=np.int64)
    temps = np.array([1.0, 0.8, 2.5, 1e-5, 1.0, 0.7, 1.0, 1.0, 1.0, 0.0, -1.0], np.float32)
    tokens = np.array([ref.categorical_row(logits[i].tolist(), int(seeds[i]) & ((1 << 64) - 1),
                                           int(offsets[i]) & ((1 << 64) - 1), float(temps[i]))
                       for i in range(n)], np.int64)
    # many draws of one row, for the statistics of the sampler
    many_logits = (rng.standard_normal(16) * 1.5).astype(np.float32)
    many_offsets = np.arange(2000, dtype=np.int64)
    many_tokens = np.array([ref.categorical_row(many_logits.tolist(), 12345, int(o), 0.9) for o in many_offsets],
                           np.int64)
    np.savez(HERE / "categorical.npz", logits=logits, seeds=seeds, offsets=offsets, temperatures=temps,
             tokens=tokens, many_logits=many_logits, many_offsets=many_offsets, many_tokens=many_tokens)


if __name__ == "__main__":
    O.build()
    q8_kat()
    q8_pack()
    q4_pack()
    mul_mat()
    categorical()
    print("golden vectors written to", HERE)
