"""Build libmstar_b200.so in-tree: every CUDA source for sm_100a only.

``python -m mstar_accelerators_b200.build`` (or ``build()``) compiles
csrc/*.cu with nvcc into mstar_accelerators_b200/libmstar_b200.so. The
shared object is git-ignored and travels with the source tree.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
LIBRARY = PACKAGE / "libmstar_b200.so"
INCLUDE = PACKAGE.parent / "include"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-Xcompiler", "-ffp-contract=off",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > built for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIBRARY
    nvcc = os.environ.get("NVCC", "nvcc")
    objdir = PACKAGE / "_build"
    objdir.mkdir(exist_ok=True)
    env = dict(os.environ)
    env.pop("CC", None)   # nvcc's host compiler is the system gcc on PATH
    env.pop("CXX", None)
    objects = []
    procs = []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        procs.append((subprocess.Popen(cmd, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT), src))
        objects.append(obj)
    failed = []
    for p, src in procs:
        out, _ = p.communicate()
        text = out.decode(errors="replace")
        if p.returncode:
            failed.append(f"{src.name}:\n{text}")
        elif verbose and text.strip():
            print(text)
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *map(str, objects), "-o", str(tmp)]
    subprocess.run(cmd, env=env, check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIBRARY)
