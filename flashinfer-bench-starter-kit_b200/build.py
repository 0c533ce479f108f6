"""Builds libdsa_b200.so (the C-ABI library) in-tree for sm_100a with nvcc.

    python flashinfer-bench-starter-kit_b200/build.py [--verbose]

The library lands next to the Python package (dsa_b200/libdsa_b200.so) so a
snapshot of the source tree carries it; nothing is installed elsewhere.
"""

from __future__ import annotations

import os
import pathlib
import shutil
import subprocess
import sys

ROOT = pathlib.Path(__file__).resolve().parent
REPO = ROOT.parent
CSRC = ROOT / "csrc"
OUT = ROOT / "dsa_b200" / "libdsa_b200.so"
SOURCES = ["capi.cu", "indexer.cu", "attention.cu", "noalloc.cu", "cache_write.cu", "prefill.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def build(verbose: bool = False, force: bool = False) -> pathlib.Path:
    srcs = [CSRC / s for s in SOURCES]
    deps = srcs + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [REPO / "include" / "dsa_b200.h"]
    if OUT.exists() and not force:
        newest = max(p.stat().st_mtime for p in deps)
        if OUT.stat().st_mtime >= newest:
            return OUT
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-std=c++17", "-lineinfo", "--shared",
           "-Xcompiler", "-fPIC,-fvisibility=hidden", "-Xcompiler", "-Wall",
           "-I", str(REPO / "include"), "-I", str(CSRC),
           "-o", str(OUT), *map(str, srcs)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stdout.write(res.stdout)
        sys.stderr.write(res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed with exit code {res.returncode}")
    return OUT


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force=True)
