"""Build libxencb.so (the C ABI of include/xencb.h) in-tree for sm_100a.

    python -m kv_skill_v2_b200.csrc.build          # or __graft_entry__.build()

One nvcc invocation over xencb.cu (which includes the kernel headers); the result is written next to the
package (kv_skill_v2_b200/libxencb.so) so it travels with the source tree. cudart is linked statically, so
the library only needs the NVIDIA driver at run time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
ROOT = PKG.parent
OUT = PKG / "libxencb.so"
SOURCES = [HERE / "xencb.cu"]
DEPS = sorted(HERE.glob("*.cuh")) + [ROOT / "include" / "xencb.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-shared", "-cudart", "static",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in SOURCES + DEPS + [Path(__file__)])


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(ROOT / "include"), *map(str, SOURCES), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
