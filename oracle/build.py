"""Build recipe for the oracle (TEST INFRASTRUCTURE ONLY).

  oracle/_build/libgdn_oracle.so   C restatement of the reference layer (gdn_oracle.c)
  oracle/_ref/libgdn_metal_ref.so  the reference's own Metal kernel body
                                   (src/models/metal_gdn.rs:10-67), compiled for
                                   the CPU through metal_ref_shim.hpp

The second library is only built where the reference tree is present; its
source is read from the reference and piped to g++ on stdin, so no copy of it
is written anywhere.  Both outputs are git-ignored build products.
"""
from __future__ import annotations

import os
import re
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF_OUT = HERE / "_ref"
# The reference tree: $GDN_REFERENCE_TREE, else a directory named "reference" beside this repository.
REF_TREE = Path(os.environ.get("GDN_REFERENCE_TREE", str(HERE.parent.parent / "reference")))
METAL_RS = "src/models/metal_gdn.rs"

ORACLE_SO = BUILD / "libgdn_oracle.so"
REF_SO = REF_OUT / "libgdn_metal_ref.so"

CFLAGS = ["-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-std=c11"]


def _stale(out: Path, deps) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build_oracle(force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    src = HERE / "gdn_oracle.c"
    if force or _stale(ORACLE_SO, [src, __file__]):
        cmd = ["gcc", *CFLAGS, str(src), "-o", str(ORACLE_SO), "-lm"]
        subprocess.run(cmd, check=True)
    return ORACLE_SO


def extract_metal_body(rs_text: str) -> str:
    """Return the raw-string body of GDN_KERNEL_SOURCE (metal_gdn.rs:10-67)."""
    m = re.search(r'const\s+GDN_KERNEL_SOURCE\s*:\s*&str\s*=\s*r#"(.*?)"#;', rs_text, re.S)
    if not m:
        raise RuntimeError("GDN_KERNEL_SOURCE not found in " + METAL_RS)
    return m.group(1)


def build_ref(force: bool = False) -> Path | None:
    """Compile the reference Metal kernel body for the CPU; None when the reference is absent."""
    rs = REF_TREE / METAL_RS
    if not rs.exists():
        return REF_SO if REF_SO.exists() else None
    REF_OUT.mkdir(exist_ok=True)
    deps = [rs, HERE / "metal_ref_shim.hpp", HERE / "metal_ref_tail.hpp", __file__]
    if not (force or _stale(REF_SO, deps)):
        return REF_SO
    body = extract_metal_body(rs.read_text())
    tu = "\n".join([
        '#include "metal_ref_shim.hpp"',
        "GDN_SIMDGROUP_SIGNATURE {",
        "GDN_PRELUDE",
        "#define float LF",
        f'#line 11 "{METAL_RS}"',
        body,
        "#undef float",
        "}",
        '#include "metal_ref_tail.hpp"',
        "",
    ])
    cmd = ["g++", "-O2", "-fPIC", "-shared", "-std=c++17", "-ffp-contract=off", "-fno-fast-math",
           "-I", str(HERE), "-x", "c++", "-", "-o", str(REF_SO)]
    subprocess.run(cmd, input=tu.encode(), check=True)
    return REF_SO


if __name__ == "__main__":
    force = "--force" in sys.argv
    print(build_oracle(force))
    print(build_ref(force))
