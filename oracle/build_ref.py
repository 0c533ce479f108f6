"""Builds the reference's own DSA solutions into oracle/_ref/ (TEST INFRASTRUCTURE ONLY).

    python oracle/build_ref.py [--force]

The reference's two operators are CUDA C++ held in Python strings and compiled
at first use with ``torch.utils.cpp_extension.load_inline``:

* dsa_indexer/solution/triton/kernel.py:47-319 (``_cpp_src`` / ``_cuda_src``),
  built at :324-336 as module ``dsa_topk_s11`` exporting ``dsa_topk_run_ms``;
* dsa_attention/solution/triton/kernel.py:17-218, built at :225-236 as module
  ``dsa_sparse_v8`` exporting ``dsa_sparse_attention``.

This recipe reads those strings where they lie under /root/reference (it
imports the two files, which define the strings at module level and compile
nothing on import) and compiles them with the same ``load_inline`` call, the
same module names, functions and flags, for compute capability 10.0 -- the
target the reference's JIT picks on a B200, since it passes no architecture
flag.  Only the two extension libraries are kept (``oracle/_ref/*.so``,
git-ignored, travelling with a copy of the source tree); the generated build
folders, which hold the sources, are deleted.  Nothing under /root/reference
is written.

The libraries are used by ``oracle.ref_gpu`` for a second parity check (against
the reference itself, run on the GPU) and as the same-box GPU baseline.
"""

from __future__ import annotations

import importlib.util
import os
import pathlib
import shutil
import sys

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_ref"
REF_ROOT = pathlib.Path("/root/reference")

# module name -> (reference file, functions, extra_cflags, extra_cuda_cflags), as the
# reference's own load_inline calls give them.
TARGETS = {
    "dsa_topk_s11": ("dsa_indexer/solution/triton/kernel.py", ["dsa_topk_run_ms"],
                     ["-O3", "-std=c++17"], ["-O3", "-std=c++17"]),
    "dsa_sparse_v8": ("dsa_attention/solution/triton/kernel.py", ["dsa_sparse_attention"],
                      ["-O3"], ["-O3", "--use_fast_math"]),
}


def _load_sources(path: pathlib.Path):
    spec = importlib.util.spec_from_file_location(f"_ref_src_{path.parent.parent.parent.name}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod._cpp_src, mod._cuda_src


def stale(name: str) -> bool:
    so = OUT / f"{name}.so"
    src = REF_ROOT / TARGETS[name][0]
    if not so.exists():
        return True
    return so.stat().st_mtime < max(src.stat().st_mtime, pathlib.Path(__file__).stat().st_mtime)


def build(force: bool = False, verbose: bool = False) -> list:
    """Builds every target that is missing or older than its source; returns
    the library paths.  Where /root/reference is absent it only reports what
    is already built."""
    if not REF_ROOT.exists():
        return sorted(OUT.glob("*.so"))
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0"
    from torch.utils.cpp_extension import load_inline

    OUT.mkdir(exist_ok=True)
    built = []
    for name, (rel, functions, cflags, cuda_cflags) in TARGETS.items():
        so = OUT / f"{name}.so"
        if force or stale(name):
            cpp_src, cuda_src = _load_sources(REF_ROOT / rel)
            bdir = OUT / f"_build_{name}"
            if bdir.exists():
                shutil.rmtree(bdir)
            bdir.mkdir()
            load_inline(name=name, cpp_sources=cpp_src, cuda_sources=cuda_src,
                        functions=functions, extra_cflags=cflags,
                        extra_cuda_cflags=cuda_cflags, build_directory=str(bdir),
                        verbose=verbose)
            shutil.copy2(bdir / f"{name}.so", so)
            shutil.rmtree(bdir)
        built.append(so)
    return built


if __name__ == "__main__":
    for p in build(force="--force" in sys.argv, verbose="--verbose" in sys.argv):
        print(p)
