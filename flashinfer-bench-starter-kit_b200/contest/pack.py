"""Packs the B200 DSA kernels as contest solutions.

    python flashinfer-bench-starter-kit_b200/contest/pack.py [-o OUT_DIR] [--variant V]

For each operator directory (dsa_indexer/, dsa_attention/) the config.toml
names the definition and the entry point; this writes
OUT_DIR/<operator>/packed_solution.json in the Solution shape the starter
kit's README documents (name, definition, author, spec with language,
target hardware, entry point, dependencies, destination-passing style and
binding, then the sources as path/content pairs), which the
evaluation pipeline uses directly when it finds it (FAQ.md:53-55).  The
sources are the library's own files, flattened into one directory: the
entry points, the C ABI and the kernels.  Three variants:

  cuda     (default, the operators' config.toml) language "cuda", binding
           "torch": contest/kernel.cu::dsa_indexer / ::dsa_attention.
  tvm-ffi  language "cuda", binding "tvm-ffi" (the harness's default
           binding): contest/kernel_tvm.cu::dsa_indexer / ::dsa_attention.
  python   language "python": kernel.py::run, the entry point name the
           reference's config.toml files use (dsa_indexer/config.toml:8,
           dsa_attention/config.toml:7).  Each operator's packed kernel.py is
           contest/kernel.py plus a `run` with that operator's arguments,
           calling run_indexer / run_attention, which compile the packed CUDA
           sources for sm_100a themselves through tvm_ffi.cpp.load.  The harness's CUDA builders
           set no SM target and take no flags (FAQ.md:144-154), so this is the
           variant that builds the sm_100a kernels under a stock harness.
"""

from __future__ import annotations

import argparse
import json
import pathlib
import tomllib

HERE = pathlib.Path(__file__).resolve().parent
PKG = HERE.parent
REPO = PKG.parent
LIBRARY = [
    PKG / "csrc" / "capi.cu",
    PKG / "csrc" / "indexer.cu",
    PKG / "csrc" / "attention.cu",
    PKG / "csrc" / "ptx.cuh",
    PKG / "csrc" / "host.h",
    REPO / "include" / "dsa_b200.h",
]
OPERATORS = ("dsa_indexer", "dsa_attention")
# variant -> (language, binding, entry file, sources in front of the library,
#             entry function per operator; None: the config.toml's)
VARIANTS = {
    "cuda": ("cuda", "torch", "kernel.cu", [HERE / "kernel.cu"], None),
    "tvm-ffi": ("cuda", "tvm-ffi", "kernel_tvm.cu", [HERE / "kernel_tvm.cu"], None),
    "python": ("python", None, "kernel.py", [HERE / "kernel.py", HERE / "kernel_tvm.cu"],
               {"dsa_indexer": "run", "dsa_attention": "run"}),
}
# The python variant's per-operator entry point, appended to its kernel.py.
PY_RUN = {
    "dsa_indexer": '''

def run(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices):
    """The operator's entry point, kernel.py::run (dsa_indexer/config.toml:8)."""
    run_indexer(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices)
''',
    "dsa_attention": '''

def run(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, output, lse):
    """The operator's entry point, kernel.py::run (dsa_attention/config.toml:7)."""
    run_attention(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, output, lse)
''',
}


def solution(op: str, variant: str = "cuda") -> dict:
    cfg = tomllib.loads((HERE / op / "config.toml").read_text())
    sol, build = cfg["solution"], cfg["build"]
    language, binding, entry_file, front, fns = VARIANTS[variant]
    fn = fns[op] if fns else build["entry_point"].split("::")[1]
    spec = {
        "language": language,
        "target_hardware": ["cuda"],
        "entry_point": f"{entry_file}::{fn}",
        "dependencies": [],
        "destination_passing_style": bool(build.get("destination_passing_style", True)),
    }
    if binding is not None:
        spec["binding"] = binding
    return {
        "name": sol["name"] if variant == "cuda" else f"{sol['name']}-{variant}",
        "definition": sol["definition"],
        "author": sol["author"],
        "spec": spec,
        "sources": [{"path": p.name,
                     "content": p.read_text() + (PY_RUN[op] if variant == "python" and p.name == "kernel.py" else "")}
                    for p in front + LIBRARY],
    }


def pack(out_dir: pathlib.Path, variant: str = "cuda") -> list:
    written = []
    for op in OPERATORS:
        d = out_dir / op
        d.mkdir(parents=True, exist_ok=True)
        path = d / "packed_solution.json"
        path.write_text(json.dumps(solution(op, variant), indent=2))
        written.append(path)
    return written


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("-o", "--out", type=pathlib.Path, default=HERE / "packed")
    ap.add_argument("--variant", choices=sorted(VARIANTS), default="cuda")
    args = ap.parse_args()
    for p in pack(args.out, args.variant):
        print(p)


if __name__ == "__main__":
    main()
