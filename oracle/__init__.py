"""CPU oracle for the two-stage DSA decode path (TEST INFRASTRUCTURE ONLY).

This package restates, on the CPU, what the reference computes for the DSA
lightning indexer and the DSA sparse MLA attention:

* ``oracle.indexer``   -- dsa_indexer/solution/triton/kernel.py (scoring, top-k,
                          page-table translation, -1 padding).
* ``oracle.attention`` -- the ``dsa_paged`` definition reference that
                          dsa_attention/solution/triton/kernel.py is graded
                          against (flashinfer 0.6.11.post2,
                          flashinfer/trace/templates/attention.py:644-684).
* ``oracle.compare``   -- set / tolerance comparators with boundary-swap
                          counting for the indexer and the harness tolerance
                          rule (fail only if abs > atol AND rel > rtol) for
                          attention.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package, and only to check results against it or as the
timed CPU baseline.  The product path (``dsa_b200``) never imports it and has no CPU
fallback.

Parity pinning: the attention restatement and the top-k/page-table step are
pinned against fixtures produced by importing the published flashinfer
references; the indexer scoring is pinned against fixtures produced by the
DeepGEMM paged-MQA-logits torch reference shipped in vllm 0.22
(``fp8_paged_mqa_logits_torch``).  The generating script is
``tests/golden/make_golden.py``.  No golden workload of the contest dataset
itself is available, so the indexer's exact reference arithmetic (cuBLAS
SGEMM order) is not pinned bit-for-bit: near-boundary swaps are counted, not
forbidden.
"""
