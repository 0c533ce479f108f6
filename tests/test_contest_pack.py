"""Contest packaging: the packed solutions (CUDA with the torch or TVM-FFI
binding, and the Python solution that compiles the CUDA sources itself) are
complete and well-formed, the TVM-FFI module builds for sm_100a and checks its
arguments (CPU); on the GPU the packed sources build and their entry points
return exactly what dsa_b200 returns."""

import ast
import importlib.util
import json
import pathlib
import re
import shutil

import pytest
import torch

REPO = pathlib.Path(__file__).resolve().parent.parent
_spec = importlib.util.spec_from_file_location(
    "dsa_contest_pack", REPO / "flashinfer-bench-starter-kit_b200" / "contest" / "pack.py")
pack = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(pack)


DEFS = {"dsa_indexer": "dsa_topk_indexer_fp8_h64_d128_topk2048_ps64",
        "dsa_attention": "dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64"}
# The reference operators' argument lists (dsa_indexer/solution/triton/kernel.py:364,
# dsa_attention/solution/triton/kernel.py:241): the harness binds by these names.
ARGS = {"dsa_indexer": ["q_index_fp8", "k_index_cache_fp8", "weights", "seq_lens", "block_table",
                        "topk_indices"],
        "dsa_attention": ["q_nope", "q_pe", "ckv_cache", "kpe_cache", "sparse_indices", "sm_scale",
                          "output", "lse"]}


@pytest.mark.parametrize("variant,language,binding", [
    ("cuda", "cuda", "torch"), ("tvm-ffi", "cuda", "tvm-ffi"), ("python", "python", None)])
def test_packed_solutions_are_complete(tmp_path, variant, language, binding):
    paths = pack.pack(tmp_path, variant)
    assert [p.parent.name for p in paths] == ["dsa_indexer", "dsa_attention"]
    names = set()
    for p in paths:
        op = p.parent.name
        sol = json.loads(p.read_text())
        names.add(sol["name"])
        assert sol["definition"] == DEFS[op]
        spec = sol["spec"]
        assert spec["language"] == language and spec["target_hardware"] == ["cuda"]
        assert spec["destination_passing_style"] is True and spec.get("binding") == binding
        fname, fn = spec["entry_point"].split("::")
        files = {s["path"]: s["content"] for s in sol["sources"]}
        assert fname in files
        if language == "cuda":
            assert re.search(r"\bvoid %s\(" % fn, files[fname])
            if binding == "torch":
                assert f'm.def("{fn}"' in files[fname]
            else:
                assert f"TVM_FFI_DLL_EXPORT_TYPED_FUNC({fn}, {fn});" in files[fname]
        else:
            tree = ast.parse(files[fname])
            funcs = {f.name: [a.arg for a in f.args.args] for f in tree.body if isinstance(f, ast.FunctionDef)}
            assert funcs[fn] == ARGS[op]
            # the CUDA sources the Python solution compiles are all packed
            srcs = next(n.value for n in tree.body if isinstance(n, ast.Assign)
                        and n.targets[0].id == "SOURCES")
            assert all(ast.literal_eval(e) in files for e in srcs.elts)
        # every quoted include resolves inside the packed directory
        for name, text in files.items():
            for inc in re.findall(r'#include "([^"]+)"', text):
                assert inc in files, (name, inc)
    assert len(names) == 2


def unpack(tmp_path, variant, op="dsa_indexer"):
    sol = json.loads(pack.pack(tmp_path / "packed", variant)[0 if op == "dsa_indexer" else 1].read_text())
    src = tmp_path / "src"
    src.mkdir(exist_ok=True)
    for s in sol["sources"]:
        (src / s["path"]).write_text(s["content"])
    return src


def load_python_solution(tmp_path, monkeypatch):
    """Imports the packed Python solution from its unpacked directory and
    builds its TVM-FFI module (cached under tmp_path)."""
    src = unpack(tmp_path, "python")
    monkeypatch.setenv("TVM_FFI_CACHE_DIR", str(tmp_path / "tvm-ffi-cache"))
    spec = importlib.util.spec_from_file_location("dsa_packed_python_solution", src / "kernel.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.module()
    return mod


needs_tvm_build = pytest.mark.skipif(
    shutil.which("nvcc") is None or importlib.util.find_spec("tvm_ffi") is None,
    reason="needs nvcc and tvm_ffi")


@needs_tvm_build
def test_python_solution_builds_for_sm100a_and_checks_arguments(tmp_path, monkeypatch):
    import os

    before = os.environ.get("TVM_FFI_CUDA_ARCH_LIST")
    sol = load_python_solution(tmp_path, monkeypatch)
    assert os.environ.get("TVM_FFI_CUDA_ARCH_LIST") == before  # restored after the build
    ninja = next((tmp_path / "tvm-ffi-cache").glob("*/build.ninja")).read_text()
    assert set(re.findall(r"-gencode=?\s*arch=[^ ]+", ninja)) == {"-gencode=arch=compute_100a,code=sm_100a"}
    # Argument checks run before any CUDA call: bad dtypes and host tensors raise.
    B = 2
    q = torch.zeros(B, 64, 128, dtype=torch.float8_e4m3fn)
    kc = torch.zeros(4, 8448, dtype=torch.uint8)
    w = torch.zeros(B, 64)
    sl = torch.zeros(B, dtype=torch.int32)
    bt = torch.zeros(B, 4, dtype=torch.int32)
    out = torch.zeros(B, 2048, dtype=torch.int32)
    with pytest.raises(ValueError, match="topk_indices"):
        sol.run_indexer(q, kc, w, sl, bt, out.long())
    with pytest.raises(ValueError, match="seq_lens"):
        sol.run_indexer(q, kc, w, sl.long(), bt, out)
    with pytest.raises(ValueError, match="CUDA device"):
        sol.run_indexer(q, kc, w, sl, bt, out)
    qn = torch.zeros(B, 16, 512, dtype=torch.bfloat16)
    qp = torch.zeros(B, 16, 64, dtype=torch.bfloat16)
    ckv = torch.zeros(64, 512, dtype=torch.bfloat16)
    kpe = torch.zeros(64, 64, dtype=torch.bfloat16)
    lse = torch.zeros(B, 16)
    with pytest.raises(ValueError, match="kpe_cache"):
        sol.run_attention(qn, qp, ckv, kpe[:32], out, 0.1, qn, lse)
    with pytest.raises(ValueError, match="lse"):
        sol.run_attention(qn, qp, ckv, kpe, out, 0.1, qn, lse.double())
    with pytest.raises(ValueError, match="CUDA device"):
        sol.run_attention(qn, qp, ckv, kpe, out, 0.1, qn, lse)


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


@pytest.mark.gpu
@needs_tvm_build
def test_python_solution_matches_the_library_and_captures(cuda_device, tmp_path, monkeypatch):
    # The Python solution (TVM-FFI entry points compiled by itself for sm_100a)
    # returns exactly what dsa_b200 returns, and launches on torch's current
    # stream: its calls capture into a CUDA graph on a side stream (a launch
    # on any other stream would invalidate the capture).
    from dsa_b200 import attention, indexer, workloads

    sol = load_python_solution(tmp_path, monkeypatch)
    lens = [3000, 70000, 129, 0, 2049]
    dec = workloads.make_decode_inputs(lens, seed=37, device=cuda_device)
    ix = dec.indexer
    want = torch.full((5, 2048), 7, dtype=torch.int32, device=cuda_device)
    indexer.run(ix.q_index_fp8, ix.k_index_cache_fp8, ix.weights, ix.seq_lens, ix.block_table, want)
    o1 = torch.empty(5, 16, 512, dtype=torch.bfloat16, device=cuda_device)
    l1 = torch.empty(5, 16, dtype=torch.float32, device=cuda_device)
    attention.run(dec.q_nope, dec.q_pe, dec.ckv_cache, dec.kpe_cache, want, dec.sm_scale, o1, l1)

    got = torch.full_like(want, 7)
    o2, l2 = torch.empty_like(o1), torch.empty_like(l1)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # first calls on the capture stream size its workspaces
        # kernel.py::run, the packed indexer's entry point (as the reference names it)
        sol.run(ix.q_index_fp8, ix.k_index_cache_fp8, ix.weights, ix.seq_lens, ix.block_table, got)
        sol.run_attention(dec.q_nope, dec.q_pe, dec.ckv_cache, dec.kpe_cache, got, dec.sm_scale, o2, l2)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(o1, o2) and torch.equal(l1.nan_to_num(), l2.nan_to_num())

    got.fill_(7)
    o2.zero_()
    l2.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        sol.run_indexer(ix.q_index_fp8, ix.k_index_cache_fp8, ix.weights, ix.seq_lens, ix.block_table, got)
        sol.run_attention(dec.q_nope, dec.q_pe, dec.ckv_cache, dec.kpe_cache, got, dec.sm_scale, o2, l2)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(o1, o2) and torch.equal(l1.nan_to_num(), l2.nan_to_num())
    del g
