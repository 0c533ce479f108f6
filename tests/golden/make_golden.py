"""Generates the golden fixtures in this directory from published references.

Run in a container where the third-party references import (no GPU needed):

    python tests/golden/make_golden.py

* attention_small.npz -- outputs of ``_dsa_paged_reference`` from
  flashinfer 0.6.11.post2 (flashinfer/trace/templates/attention.py:644-684),
  the definition reference of dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64.
* indexer_small.npz -- index scores from ``fp8_paged_mqa_logits_torch``
  (vllm 0.22, vllm/v1/attention/ops/rocm_aiter_mla_sparse.py; the DeepGEMM
  paged MQA-logits test reference, same 8448-byte page layout), and the
  top-k + page-table translation from ``_top_k_page_table_transform_reference``
  (flashinfer/trace/templates/sampling.py:721-749).

Inputs are stored in the fixtures, so tests never need these packages.
"""

from __future__ import annotations

import math
import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "flashinfer-bench-starter-kit_b200"))

from dsa_b200 import workloads  # noqa: E402


def attention_fixture() -> None:
    from flashinfer.trace.templates.attention import _dsa_paged_reference

    g = torch.Generator().manual_seed(20260101)
    T, pages = 3, 4
    qn = torch.randn(T, 16, 512, generator=g).to(torch.bfloat16)
    qp = torch.randn(T, 16, 64, generator=g).to(torch.bfloat16)
    ckv = torch.randn(pages, 64, 512, generator=g).to(torch.bfloat16)
    kpe = torch.randn(pages, 64, 64, generator=g).to(torch.bfloat16)
    idx = torch.randint(0, pages * 64, (T, 2048), generator=g, dtype=torch.int32)
    pad = torch.randperm(2048, generator=g)[:1048]
    idx[1, pad] = -1          # token 1: 1000 valid entries scattered among -1
    idx[2, :] = -1            # token 2: no valid entry -> output 0, lse -inf
    sm_scale = 1.0 / math.sqrt(192.0)
    out, lse = _dsa_paged_reference(qn, qp, ckv, kpe, idx, sm_scale)
    np.savez_compressed(
        HERE / "attention_small.npz",
        q_nope=qn.view(torch.int16).numpy(), q_pe=qp.view(torch.int16).numpy(),
        ckv=ckv.view(torch.int16).numpy(), kpe=kpe.view(torch.int16).numpy(),
        indices=idx.numpy(), sm_scale=np.float32(sm_scale),
        output=out.view(torch.int16).numpy(), lse=lse.numpy())


def indexer_fixture() -> None:
    from flashinfer.trace.templates.sampling import _top_k_page_table_transform_reference
    from vllm.v1.attention.ops.rocm_aiter_mla_sparse import fp8_paged_mqa_logits_torch

    seq_lens = [2500, 130, 0, 71]
    ix = workloads.make_indexer_inputs(seq_lens, pool_pages=64, seed=4242, device="cpu")
    max_pages = ix.block_table.shape[1]
    logits = fp8_paged_mqa_logits_torch(
        ix.q_index_fp8[:, None], ix.k_index_cache_fp8, ix.weights, ix.seq_lens,
        ix.block_table, max_pages * 64)
    # The transform maps token positions through a token-level table, so
    # expand the 64-token page table to slot ids: page*64 + token % 64.
    tok = torch.arange(max_pages * 64)
    slot_table = (ix.block_table.long()[:, tok // 64] * 64 + tok % 64).to(torch.int32)
    topk = _top_k_page_table_transform_reference(logits, slot_table, ix.seq_lens, 2048)
    np.savez_compressed(
        HERE / "indexer_small.npz",
        q=ix.q_index_fp8.view(torch.uint8).numpy(), k_cache=ix.k_index_cache_fp8.numpy(),
        weights=ix.weights.numpy(), seq_lens=ix.seq_lens.numpy(),
        block_table=ix.block_table.numpy(), logits=logits.numpy(), topk=topk.numpy())


if __name__ == "__main__":
    attention_fixture()
    indexer_fixture()
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))
