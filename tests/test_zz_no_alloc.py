"""GPU test of dsa_indexer_run_noalloc, the indexer entry point for callers
that cannot allocate device memory when they call (C / JNI / FFI hosts whose
device memory belongs to another allocator, serving loops that forbid
cudaMalloc after warm-up).  It must return exactly what the workspace entry
point returns, on back-to-back calls that reuse the library's one scratch
array, and refuse problems larger than that array.

The file name makes pytest collect it last; it also passes on its own in a
fresh process."""

import ctypes

import pytest
import torch

from dsa_b200 import _native, indexer, workloads

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _noalloc(ix, out):
    lib = _native.lib()
    B, max_pages = ix.block_table.shape
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.dsa_indexer_run_noalloc(_p(ix.q_index_fp8), _p(ix.k_index_cache_fp8),
                                       ix.num_pages, _p(ix.weights), _p(ix.seq_lens),
                                       _p(ix.block_table), B, max_pages, _p(out), stream)


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(cuda_device):
    # Two calls in a row through the shared scratch: the second has a larger
    # batch, so its histogram rows sit where the first call's scores were.
    cases = (([3000, 70000, 129, 0, 2049], 1200, 41), ([65536, 8192, 4097, 65, 30000, 1, 2048, 9000], 1100, 42))
    for lens, pool, seed in cases:
        ix = workloads.make_indexer_inputs(lens, pool_pages=pool, seed=seed, device=cuda_device)
        ref = torch.full((len(lens), 2048), 7, dtype=torch.int32, device=cuda_device)
        indexer.run(ix.q_index_fp8, ix.k_index_cache_fp8, ix.weights, ix.seq_lens,
                    ix.block_table, ref)
        got = torch.full_like(ref, 7)
        assert _noalloc(ix, got) == _native.DSA_OK
        torch.cuda.synchronize()
        # Index outputs are compared exactly, as in the other indexer tests.
        assert torch.equal(got, ref), lens


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_device):
    lib = _native.lib()
    limit = lib.dsa_indexer_workspace_bytes(64, 256)
    assert limit <= (256 + 32768 + 64 * 2048 * 4 + 1048576 * 4)
    assert lib.dsa_indexer_workspace_bytes(64, 300) > (256 + 32768 + 64 * 2048 * 4 + 1048576 * 4)
    ix = workloads.make_indexer_inputs([64] * 64, pool_pages=300, seed=43, device=cuda_device,
                                       max_pages=300)
    out = torch.full((64, 2048), 7, dtype=torch.int32, device=cuda_device)
    assert _noalloc(ix, out) == 3  # DSA_ERR_WORKSPACE_TOO_SMALL
    torch.cuda.synchronize()
    assert (out == 7).all()  # nothing was launched
