"""CPU restatement of the DSA top-k indexer (TEST INFRASTRUCTURE ONLY).

Follows dsa_indexer/solution/triton/kernel.py of the reference:

* page layout (``PAGE_BYTES = 8448``, kernel.py:76-80, 120-124): each page holds
  64 tokens x 128 FP8-E4M3FN bytes, followed by 64 little-endian fp32 scales
  (one per token) at byte offset ``64*128 + tok*4``;
* dequantisation ``K = fp8(k).float() * scale`` (kernel.py:108-135);
* ``scores = q.float() @ K.T`` over the request's pages (kernel.py:208, 293);
* ``v <= 0 ? 0 : v`` then ``* w[h]`` (kernel.py:141-151, NaN passes through);
* ``final = scores.sum(0)`` over the 64 heads (kernel.py:300);
* ``topk(final, min(L, 2048))`` sorted descending (kernel.py:284, 301);
* global slot id ``block_table[b, tok // 64] * 64 + tok % 64`` (kernel.py:156-169);
* untouched entries stay ``-1`` (kernel.py:206); ``L == 0`` rows are skipped
  (kernel.py:280).

The reference leaves the order of equal scores to ``at::topk``.  This oracle
fixes it: descending score, ties broken by the lowest token index, with NaN
ranked above every number (torch's topk convention) and -0.0 equal to +0.0.
"""

from __future__ import annotations

import math

import numpy as np
import torch

PAGE_SIZE = 64
NUM_HEADS = 64
HEAD_DIM = 128
TOPK = 2048
PAGE_BYTES = PAGE_SIZE * HEAD_DIM + PAGE_SIZE * 4  # 8448


def decode_e4m3fn(byte: int) -> float:
    """Value of one FP8 E4M3FN byte, from the format's bit layout.

    1 sign bit, 4 exponent bits (bias 7), 3 mantissa bits; exponent field 0 is
    subnormal (m/8 * 2^-6); S.1111.111 is NaN; there are no infinities.  This
    is the format the reference decodes in software (kernel.py:86-103) and is
    used to pin torch's ``float8_e4m3fn`` conversion table.
    """
    sign = -1.0 if (byte & 0x80) else 1.0
    exp = (byte >> 3) & 0xF
    man = byte & 0x7
    if exp == 0xF and man == 0x7:
        return math.nan
    if exp == 0:
        return sign * (man / 8.0) * 2.0 ** -6
    return sign * (1.0 + man / 8.0) * 2.0 ** (exp - 7)


def e4m3_table() -> np.ndarray:
    """fp32 value of every FP8 byte, via torch's float8_e4m3fn conversion."""
    b = torch.arange(256, dtype=torch.uint8)
    return b.view(torch.float8_e4m3fn).to(torch.float32).numpy()


def request_pages(block_table_row: torch.Tensor, seq_len: int) -> torch.Tensor:
    n_pages = (seq_len + PAGE_SIZE - 1) // PAGE_SIZE
    return block_table_row[:n_pages].to(torch.long)


def dequant_request(k_cache_u8: torch.Tensor, pages: torch.Tensor):
    """fp32 K [n_pages*64, 128], per-token scales [n_pages*64] (kernel.py:108-135)."""
    pg = k_cache_u8.reshape(-1, PAGE_BYTES)[pages]  # [P, 8448]
    kf = pg[:, : PAGE_SIZE * HEAD_DIM].contiguous().view(torch.float8_e4m3fn)
    kf = kf.to(torch.float32).reshape(-1, HEAD_DIM)
    sc = pg[:, PAGE_SIZE * HEAD_DIM :].contiguous().view(torch.float32).reshape(-1)
    return kf, sc


def score_request(q_b: torch.Tensor, k_cache_u8: torch.Tensor, w_b: torch.Tensor,
                  seq_len: int, block_table_row: torch.Tensor) -> torch.Tensor:
    """fp32 index scores [seq_len] of one request (kernel.py:288-300)."""
    if seq_len <= 0:
        return torch.zeros(0, dtype=torch.float32)
    pages = request_pages(block_table_row, seq_len)
    kf, sc = dequant_request(k_cache_u8, pages)
    K = kf * sc[:, None]                                   # fp8 * scale in fp32
    s = q_b.to(torch.float32) @ K.T                        # [64, P*64]
    s = torch.where(s <= 0, torch.zeros_like(s), s)        # NaN passes through
    s = s * w_b.to(torch.float32)[:, None]
    return s.sum(0)[:seq_len].contiguous()


def score_error_bound(q_b: torch.Tensor, k_cache_u8: torch.Tensor, w_b: torch.Tensor,
                      seq_len: int, block_table_row: torch.Tensor) -> torch.Tensor:
    """Per-token bound on fp32 reordering error of the score.

    Any fp32 evaluation order of sum_h w_h * relu(s * sum_d q_hd k_d) differs
    from another by at most about (n_terms) * 2^-24 * sum of |terms|; with
    128 + 64 + a few terms, 256 * 2^-24 * sum_h |w_h| |s| sum_d |q_hd k_d| is a
    safe bound.
    """
    if seq_len <= 0:
        return torch.zeros(0, dtype=torch.float32)
    pages = request_pages(block_table_row, seq_len)
    kf, sc = dequant_request(k_cache_u8, pages)
    absdot = q_b.to(torch.float32).abs() @ kf.abs().T      # [64, P*64]
    mag = (w_b.to(torch.float32).abs()[:, None] * absdot).sum(0) * sc.abs()
    return (256.0 * 2.0 ** -24 * mag)[:seq_len].contiguous()


def order_keys(scores: np.ndarray) -> np.ndarray:
    """Order-preserving uint32 keys: larger key == larger score.

    NaN maps to the largest key; -0.0 maps to the key of +0.0.
    """
    s = np.ascontiguousarray(scores, dtype=np.float32)
    u = s.view(np.uint32).copy()
    u[(u & np.uint32(0x7FFFFFFF)) == 0] = 0                 # -0.0 -> +0.0
    neg = (u & np.uint32(0x80000000)) != 0
    key = np.where(neg, ~u, u | np.uint32(0x80000000)).astype(np.uint32)
    key[np.isnan(s)] = np.uint32(0xFFFFFFFF)
    return key


def topk_order(scores: np.ndarray, k: int = TOPK) -> np.ndarray:
    """Token indices of the top-min(L, k) scores: score desc, then index asc."""
    n = scores.shape[0]
    kk = min(n, k)
    if kk == 0:
        return np.zeros(0, dtype=np.int64)
    key = order_keys(scores).astype(np.int64)
    idx = np.arange(n, dtype=np.int64)
    order = np.lexsort((idx, -key))   # primary: key desc, secondary: index asc
    return order[:kk]


def indexer_reference(q_index_fp8: torch.Tensor, k_index_cache_fp8: torch.Tensor,
                      weights: torch.Tensor, seq_lens: torch.Tensor,
                      block_table: torch.Tensor, topk: int = TOPK):
    """Returns (topk_indices [B, topk] int32, per-request fp32 scores list)."""
    q = q_index_fp8.cpu()
    k_u8 = k_index_cache_fp8.cpu().contiguous().view(torch.uint8).reshape(-1)
    w = weights.cpu().to(torch.float32)
    sl = seq_lens.cpu().to(torch.int64)
    bt = block_table.cpu().to(torch.int64)
    B = q.shape[0]
    out = np.full((B, topk), -1, dtype=np.int32)
    all_scores = []
    for b in range(B):
        L = int(sl[b])
        sc = score_request(q[b], k_u8, w[b], L, bt[b])
        all_scores.append(sc)
        if L <= 0:
            continue
        order = topk_order(sc.numpy(), topk)
        phys = bt[b].numpy()[order // PAGE_SIZE]
        out[b, : order.shape[0]] = (phys * PAGE_SIZE + order % PAGE_SIZE).astype(np.int32)
    return torch.from_numpy(out), all_scores


def rows_block_table(block_table: torch.Tensor, cu_seqlens_q: torch.Tensor, rows) -> torch.Tensor:
    """Block-table row of each query row in `rows`: request r owns rows
    cu_seqlens_q[r] .. cu_seqlens_q[r+1]-1."""
    cu = cu_seqlens_q.cpu().to(torch.int64)
    bt = block_table.cpu()
    req = torch.searchsorted(cu, torch.as_tensor(list(rows), dtype=torch.int64), right=True) - 1
    return bt[req]


def prefill_reference(q_index_fp8: torch.Tensor, k_index_cache_fp8: torch.Tensor,
                      weights: torch.Tensor, seq_lens: torch.Tensor, block_table: torch.Tensor,
                      cu_seqlens_q: torch.Tensor, rows=None, topk: int = TOPK):
    """Many query rows per request: row t of request r is the decode problem
    (q[t], weights[t], seq_lens[t], block_table[r]), so this is
    ``indexer_reference`` on the selected rows with each row's request's
    block-table row.  The reference's indexer definition is decode-only
    (one query per request, kernel.py:364); this is that computation applied
    row by row.  Returns (topk_indices [len(rows), topk], scores list)."""
    rows = list(range(q_index_fp8.shape[0])) if rows is None else list(rows)
    return indexer_reference(q_index_fp8[rows], k_index_cache_fp8, weights[rows], seq_lens[rows],
                             rows_block_table(block_table, cu_seqlens_q, rows), topk)
