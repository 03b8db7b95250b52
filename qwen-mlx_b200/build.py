"""Build recipe of the product library libgdn_b200.so (in-tree, sm_100a).

    python qwen-mlx_b200/build.py [--force] [--verbose]

Compiles every CUDA source (and the host-only C++ sources) under csrc/ with nvcc for sm_100a
(-gencode arch=compute_100a,code=sm_100a) into qwen-mlx_b200/libgdn_b200.so,
which exports the C ABI declared in include/gdn.h and include/gdn_host.h.  The CUDA runtime is linked
statically; cuBLASLt (the projection GEMMs) dynamically, with an rpath to the
toolkit.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libgdn_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "-shared", "--expt-relaxed-constexpr"]


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not (force or _stale()):
        return LIB
    cmd = [NVCC, *ARCH, *FLAGS, "-I", str(INCLUDE), "-I", str(CSRC)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [str(s) for s in sources()] + ["-o", str(LIB)]
    # cuBLASLt (projection GEMMs); rpath so the library loads without LD_LIBRARY_PATH
    cmd += ["-L/usr/local/cuda/lib64", "-lcublasLt", "-Xlinker", "-rpath,/usr/local/cuda/lib64"]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build("--force" in sys.argv, "--verbose" in sys.argv))
