"""Packs the B200 DSA kernels as contest CUDA solutions.

    python flashinfer-bench-starter-kit_b200/contest/pack.py [-o OUT_DIR]

For each operator directory (dsa_indexer/, dsa_attention/) the config.toml
names the definition and the entry point; this writes
OUT_DIR/<operator>/packed_solution.json in the Solution shape the starter
kit's README documents (name, definition, author, spec with language
"cuda", target hardware, entry point, dependencies, destination-passing
style and binding, then the sources as path/content pairs), which the
evaluation pipeline uses directly when it finds it (FAQ.md:53-55).  The
sources are the library's own files, flattened into one directory: the
torch-binding entry points (contest/kernel.cu), the C ABI and the kernels.
"""

from __future__ import annotations

import argparse
import json
import pathlib
import tomllib

HERE = pathlib.Path(__file__).resolve().parent
PKG = HERE.parent
REPO = PKG.parent
SOURCES = [
    HERE / "kernel.cu",
    PKG / "csrc" / "capi.cu",
    PKG / "csrc" / "indexer.cu",
    PKG / "csrc" / "attention.cu",
    PKG / "csrc" / "ptx.cuh",
    PKG / "csrc" / "host.h",
    REPO / "include" / "dsa_b200.h",
]
OPERATORS = ("dsa_indexer", "dsa_attention")


def solution(op: str) -> dict:
    cfg = tomllib.loads((HERE / op / "config.toml").read_text())
    sol, build = cfg["solution"], cfg["build"]
    return {
        "name": sol["name"],
        "definition": sol["definition"],
        "author": sol["author"],
        "spec": {
            "language": build["language"],
            "target_hardware": ["cuda"],
            "entry_point": build["entry_point"],
            "dependencies": [],
            "destination_passing_style": bool(build.get("destination_passing_style", True)),
            "binding": build.get("binding", "tvm-ffi"),
        },
        "sources": [{"path": p.name, "content": p.read_text()} for p in SOURCES],
    }


def pack(out_dir: pathlib.Path) -> list:
    written = []
    for op in OPERATORS:
        d = out_dir / op
        d.mkdir(parents=True, exist_ok=True)
        path = d / "packed_solution.json"
        path.write_text(json.dumps(solution(op), indent=2))
        written.append(path)
    return written


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("-o", "--out", type=pathlib.Path, default=HERE / "packed")
    args = ap.parse_args()
    for p in pack(args.out):
        print(p)


if __name__ == "__main__":
    main()
