"""The sm_100a device Condition for B200 registry entries.

Mirrors the reference's capability gates (CPUQ8EncoderAvailable,
implementations/whisper/cpu_ggml_q8.py:31-41; ArmQ8Available,
backends/torch/q8.py:42-77): UNKNOWN without a binding, otherwise YES only when
the binding's device is CUDA, the device is compute capability 10.0, the
configured library's SHA256 matches, and mstar_b200_abi() == 1 and
mstar_b200_capability() == 1 on that device. Absence is NO, never a fallback.

Deployment setting (runtime_extension.b200 in the deployment YAML, same shape
as runtime_extension.cpu_ggml, implementations/whisper/cpu_ggml.py:17-27):
    b200: {library: /abs/path/libmstar_b200.so, sha256: <lowercase hex>}
Without the setting the in-tree library is used unpinned.
"""
from __future__ import annotations

import enum
from collections.abc import Mapping
from dataclasses import dataclass
from pathlib import Path

try:  # the M* runtime supplies the tri-state used by every reference Condition
    from mstar.engine.execution import Support
except ImportError:  # M* absent (tests, bench): an equivalent stand-in
    class Support(enum.Enum):
        YES = "yes"
        NO = "no"
        UNKNOWN = "unknown"

try:
    from mstar_accelerators.conditions import Constant
except ImportError:
    @dataclass(frozen=True)
    class Constant:
        value: Support

        def evaluate(self, facts):
            return self.value

        def specialize(self, facts):
            return self


def setting(binding):
    """Validated runtime_extension.b200 setting, or None."""
    config = getattr(binding, "model_config", None) or {}
    value = config.get("runtime_extension", {}).get("b200")
    if value is None:
        return None
    if (not isinstance(value, Mapping) or set(value) != {"library", "sha256"}
            or not isinstance(value["library"], str) or not Path(value["library"]).is_absolute()
            or not isinstance(value["sha256"], str) or len(value["sha256"]) != 64
            or any(c not in "0123456789abcdef" for c in value["sha256"])):
        raise ValueError("b200 requires an absolute library and lowercase SHA256")
    return dict(value)


def library(binding):
    """The loaded, capability-checked library for this binding, or None."""
    from . import native
    device = getattr(binding, "device", None)
    if device is None or getattr(device, "type", None) != "cuda":
        return None
    value = setting(binding)
    key = ("mstar_b200_library", tuple(sorted(value.items())) if value else None)
    prepared = getattr(binding, "prepared", None)
    if prepared is not None and key in prepared:
        return prepared[key]
    try:
        import torch
        if not torch.cuda.is_available():
            return None
        index = device.index if device.index is not None else torch.cuda.current_device()
        if torch.cuda.get_device_capability(index) != (10, 0):
            return None
        lib = native.load(value["library"] if value else None, value["sha256"] if value else None)
        with torch.cuda.device(index):
            if lib.mstar_b200_abi() != 1 or lib.mstar_b200_capability() != 1:
                return None
    except native.NativeError:
        return None
    if prepared is not None:
        prepared[key] = lib
    return lib


@dataclass(frozen=True)
class SM100aAvailable:
    """YES only on a CUDA binding whose device runs libmstar_b200's sm_100a kernels."""

    def evaluate(self, facts):
        binding = facts.get("binding")
        if binding is None:
            return Support.UNKNOWN
        return Support.YES if library(binding) is not None else Support.NO

    def specialize(self, facts):
        value = self.evaluate(facts)
        return self if value is Support.UNKNOWN else Constant(value)
