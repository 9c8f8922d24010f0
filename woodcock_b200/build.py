"""Builds the native library woodcock_b200/lib/libwoodcock_b200.so for sm_100a.

    python -m woodcock_b200.build [--verbose]

One nvcc invocation over woodcock_b200/csrc/runtime.cu (which includes the kernel
headers). The CUDA runtime is linked statically; the library exports only the
C ABI of include/woodcock_b200.h.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libwoodcock_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + \
        [REPO / "include" / "woodcock_b200.h"]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(s.stat().st_mtime <= t for s in sources())


def build(verbose: bool = False, force: bool = False, ptxas_info: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "--use_fast_math=false",
           "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared", "-cudart", "static",
           "-I", str(REPO / "include"), str(CSRC / "runtime.cu"), "-o", str(tmp)]
    cmd = [c for c in cmd if c != "--use_fast_math=false"]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libwoodcock_b200.so")
    if verbose or ptxas_info:
        sys.stderr.write(r.stderr)
    tmp.replace(LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose, a.force, a.ptxas_info))


if __name__ == "__main__":
    main()
