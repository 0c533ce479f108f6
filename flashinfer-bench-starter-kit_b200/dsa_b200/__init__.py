"""dsa_b200 -- B200-native (sm_100a) DSA decode: FP8 lightning indexer with
top-2048 select, and sparse MLA attention over the selected slots.

Operators (destination-passing, same signatures as the reference solutions):

* ``dsa_b200.indexer.run(q_index_fp8, k_index_cache_fp8, weights, seq_lens,
  block_table, topk_indices)``
* ``dsa_b200.attention.run(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices,
  sm_scale, output, lse)``

The kernels live in libdsa_b200.so (C ABI: include/dsa_b200.h); there is no
CPU or library fallback.
"""

from . import attention, indexer, workloads  # noqa: F401
from ._native import DsaError, LIB_PATH  # noqa: F401

__all__ = ["attention", "indexer", "workloads", "DsaError", "LIB_PATH"]
