"""Python entry points of the B200 DSA kernels for the contest harness.

The harness's CUDA builders pass no custom compile flags and set no SM target
(FAQ.md:144-154 of the starter kit), while these kernels use sm_100a-only
instructions (tcgen05, TMA).  The FAQ's remedy is a Python solution that
compiles its CUDA sources itself: on first use this module builds the packed
sources that sit beside it (the TVM-FFI entry points in kernel_tvm.cu, the C
ABI and the kernels) with ``tvm_ffi.cpp.load`` for ``sm_100a`` and keeps the
module; the build is cached by TVM-FFI across processes
(``TVM_FFI_CACHE_DIR``, default ``~/.cache/tvm-ffi``).

``run_indexer`` and ``run_attention`` keep the reference operators' argument
names and destination-passing style (dsa_indexer/solution/triton/kernel.py:364,
dsa_attention/solution/triton/kernel.py:241): the outputs are written in place
on the current torch stream; the calls raise on bad arguments and on a failed
launch, as the reference's do.
"""

from __future__ import annotations

import os
import pathlib
import threading

HERE = pathlib.Path(__file__).resolve().parent
SOURCES = ("kernel_tvm.cu", "capi.cu", "indexer.cu", "attention.cu")
ARCH = "10.0a"  # -gencode=arch=compute_100a,code=sm_100a

_lock = threading.Lock()
_module = None


def module():
    """The compiled TVM-FFI module (built on the first call)."""
    global _module
    with _lock:
        if _module is None:
            import tvm_ffi.cpp

            prev = os.environ.get("TVM_FFI_CUDA_ARCH_LIST")
            os.environ["TVM_FFI_CUDA_ARCH_LIST"] = ARCH
            try:
                _module = tvm_ffi.cpp.load(
                    "dsa_b200_tvm_ffi",
                    cuda_files=[str(HERE / f) for f in SOURCES],
                    extra_cuda_cflags=["-O3", "-lineinfo"],
                    extra_include_paths=[str(HERE)],
                )
            finally:
                if prev is None:
                    os.environ.pop("TVM_FFI_CUDA_ARCH_LIST", None)
                else:
                    os.environ["TVM_FFI_CUDA_ARCH_LIST"] = prev
        return _module


def run_indexer(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices):
    """Top-2048 global slot ids per request into ``topk_indices`` ([B, 2048] int32, -1 padded)."""
    module().dsa_indexer(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices)


def run_attention(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, output, lse):
    """Sparse MLA attention into ``output`` ([T, 16, 512] bf16) and ``lse`` ([T, 16] fp32, base 2)."""
    module().dsa_attention(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, float(sm_scale), output, lse)
