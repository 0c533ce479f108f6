"""CPU restatement of DSA sparse MLA attention (TEST INFRASTRUCTURE ONLY).

The reference solution (dsa_attention/solution/triton/kernel.py:240-252) is
graded against the ``dsa_paged`` definition reference; the installed
flashinfer 0.6.11.post2 ships that definition as ``_dsa_paged_reference``
(flashinfer/trace/templates/attention.py:644-684).  Restated here:

* caches flattened to global slots: ckv ``[-1, 512]``, kpe ``[-1, 64]``
  (attention.py:657-658; reference kernel.py:245-246);
* per query token, the entries of ``sparse_indices`` equal to -1 are dropped
  (attention.py:667-669; the reference masks them to -inf, kernel.py:130);
* ``logits = q_nope @ Kc^T + q_pe @ Kp^T`` in fp32, times ``sm_scale``
  (attention.py:676-678; kernel.py:198-201, 129);
* ``lse = logsumexp(logits) / ln 2`` -- base 2 (attention.py:679;
  kernel.py:166-168);
* ``output = softmax(logits) @ Kc`` cast to bf16 (attention.py:680-681;
  kernel.py:216-217);
* a token with no valid index gets output 0 and lse -inf
  (attention.py:660-671).
"""

from __future__ import annotations

import math

import torch

NUM_HEADS = 16
DIM_CKV = 512
DIM_KPE = 64
TOPK = 2048


@torch.no_grad()
def attention_reference(q_nope: torch.Tensor, q_pe: torch.Tensor,
                        ckv_cache: torch.Tensor, kpe_cache: torch.Tensor,
                        sparse_indices: torch.Tensor, sm_scale: float):
    qn_all = q_nope.cpu().to(torch.float32)
    qp_all = q_pe.cpu().to(torch.float32)
    kc_all = ckv_cache.cpu().reshape(-1, DIM_CKV)
    kp_all = kpe_cache.cpu().reshape(-1, DIM_KPE)
    idx_all = sparse_indices.cpu().to(torch.int64)
    T, H, _ = qn_all.shape
    out = torch.zeros((T, H, DIM_CKV), dtype=torch.bfloat16)
    lse = torch.full((T, H), -math.inf, dtype=torch.float32)
    for t in range(T):
        idx = idx_all[t]
        idx = idx[idx != -1]
        if idx.numel() == 0:
            continue
        kc = kc_all[idx].to(torch.float32)
        kp = kp_all[idx].to(torch.float32)
        logits = qn_all[t] @ kc.T + qp_all[t] @ kp.T
        logits = logits * float(sm_scale)
        lse[t] = torch.logsumexp(logits, dim=-1) / math.log(2.0)
        out[t] = (torch.softmax(logits, dim=-1) @ kc).to(torch.bfloat16)
    return out, lse
