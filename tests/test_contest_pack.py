"""Contest packaging: the packed CUDA solutions are complete and well-formed
(CPU), and on the GPU their sources build as a torch extension whose entry
points return exactly what dsa_b200 returns."""

import importlib.util
import json
import pathlib
import re

import pytest
import torch

REPO = pathlib.Path(__file__).resolve().parent.parent
_spec = importlib.util.spec_from_file_location(
    "dsa_contest_pack", REPO / "flashinfer-bench-starter-kit_b200" / "contest" / "pack.py")
pack = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(pack)


def test_packed_solutions_are_complete(tmp_path):
    paths = pack.pack(tmp_path)
    assert [p.parent.name for p in paths] == ["dsa_indexer", "dsa_attention"]
    defs = {"dsa_indexer": "dsa_topk_indexer_fp8_h64_d128_topk2048_ps64",
            "dsa_attention": "dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64"}
    for p in paths:
        sol = json.loads(p.read_text())
        assert sol["definition"] == defs[p.parent.name]
        spec = sol["spec"]
        assert spec["language"] == "cuda" and spec["target_hardware"] == ["cuda"]
        assert spec["destination_passing_style"] is True and spec["binding"] == "torch"
        fname, fn = spec["entry_point"].split("::")
        files = {s["path"]: s["content"] for s in sol["sources"]}
        assert fname in files and re.search(r"\bvoid %s\(" % fn, files[fname])
        assert f'm.def("{fn}"' in files[fname]
        # every quoted include resolves inside the packed directory
        for name, text in files.items():
            for inc in re.findall(r'#include "([^"]+)"', text):
                assert inc in files, (name, inc)


@pytest.mark.gpu
def test_packed_sources_build_and_match_the_library(cuda_device, tmp_path):
    from torch.utils import cpp_extension

    from dsa_b200 import attention, indexer, workloads

    sol = json.loads(pack.pack(tmp_path)[0].read_text())
    src = tmp_path / "src"
    src.mkdir()
    for s in sol["sources"]:
        (src / s["path"]).write_text(s["content"])
    build = tmp_path / "build"
    build.mkdir()
    mod = cpp_extension.load(
        name="dsa_b200_contest_solution",
        sources=[str(src / f) for f in ("kernel.cu", "capi.cu", "indexer.cu", "attention.cu")],
        extra_include_paths=[str(src)],
        extra_cuda_cflags=["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17"],
        extra_ldflags=["-lcuda"], build_directory=str(build), verbose=False)

    lens = [3000, 70000, 129, 0, 2049]
    dec = workloads.make_decode_inputs(lens, seed=31, device=cuda_device)
    ix = dec.indexer
    want = torch.full((5, 2048), 7, dtype=torch.int32, device=cuda_device)
    got = torch.full_like(want, 7)
    indexer.run(ix.q_index_fp8, ix.k_index_cache_fp8, ix.weights, ix.seq_lens, ix.block_table, want)
    mod.dsa_indexer(ix.q_index_fp8, ix.k_index_cache_fp8, ix.weights, ix.seq_lens, ix.block_table, got)
    torch.cuda.synchronize()
    assert torch.equal(got, want)

    o1 = torch.empty(5, 16, 512, dtype=torch.bfloat16, device=cuda_device)
    l1 = torch.empty(5, 16, dtype=torch.float32, device=cuda_device)
    o2, l2 = torch.empty_like(o1), torch.empty_like(l1)
    attention.run(dec.q_nope, dec.q_pe, dec.ckv_cache, dec.kpe_cache, want, dec.sm_scale, o1, l1)
    mod.dsa_attention(dec.q_nope, dec.q_pe, dec.ckv_cache, dec.kpe_cache, want, dec.sm_scale, o2, l2)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(l1.nan_to_num(), l2.nan_to_num())
