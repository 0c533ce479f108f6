"""Seeded synthetic inputs with the shapes and value distributions of the DSA
decode workloads, plus the algorithmic byte model used for rooflines.

The contest's own workloads (HF dataset flashinfer-ai/mlsys26-contest) are
not available offline; these generators stand in for them:

* indexer q: N(0,1) bf16 quantised to FP8 E4M3 with one per-tensor scale
  (absmax / 448); the run() API takes no q scale, so that positive constant
  is folded into the head weights (it does not change the selected set);
* paged K cache: N(0,1) rows, per-token scale absmax / 448, stored as
  64 x 128 FP8 bytes then 64 fp32 scales per 8448-byte page;
* head weights N(0,1) / 8;
* attention q_nope / q_pe / ckv / kpe: N(0,1) bf16; sparse indices: 2048
  distinct random positions below the row's length, mapped through a random
  page table to global slot ids; sm_scale = 1/sqrt(192).

Shape-like random choices (lengths, page tables, positions) come from a CPU
generator so they do not depend on the device; bulk values come from a
generator on the target device.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

PAGE = 64
IX_HEADS, IX_DIM = 64, 128
PAGE_BYTES = PAGE * IX_DIM + PAGE * 4
A_HEADS, CKV, KPE = 16, 512, 64
TOPK = 2048
FP8_MAX = 448.0


@dataclass
class IndexerInputs:
    q_index_fp8: torch.Tensor        # [B, 64, 128] float8_e4m3fn
    k_index_cache_fp8: torch.Tensor  # [pages, 64, 1, 132] uint8
    weights: torch.Tensor            # [B, 64] float32
    seq_lens: torch.Tensor           # [B] int32
    block_table: torch.Tensor        # [B, max_pages] int32

    @property
    def num_pages(self) -> int:
        return self.k_index_cache_fp8.shape[0]


@dataclass
class AttentionInputs:
    q_nope: torch.Tensor          # [T, 16, 512] bf16
    q_pe: torch.Tensor            # [T, 16, 64] bf16
    ckv_cache: torch.Tensor       # [pages, 64, 512] bf16
    kpe_cache: torch.Tensor       # [pages, 64, 64] bf16
    sparse_indices: torch.Tensor  # [T, 2048] int32
    sm_scale: float


def _gens(seed: int, device) -> tuple:
    cpu = torch.Generator().manual_seed(seed)
    dev = torch.Generator(device=device).manual_seed(seed + 1)
    return cpu, dev


def quantize_pages(rows: torch.Tensor) -> torch.Tensor:
    """[pages*64, 128] float rows -> [pages, 64, 1, 132] uint8 paged FP8 cache."""
    n = rows.shape[0]
    assert n % PAGE == 0
    pages = n // PAGE
    r = rows.to(torch.float32)
    scale = r.abs().amax(dim=1).clamp_min(1e-30) / FP8_MAX
    q = (r / scale[:, None]).to(torch.float8_e4m3fn).view(torch.uint8)
    data = q.reshape(pages, PAGE * IX_DIM)
    sc = scale.contiguous().view(torch.uint8).reshape(pages, PAGE * 4)
    return torch.cat([data, sc], dim=1).reshape(pages, PAGE, 1, IX_DIM + 4).contiguous()


def quantize_q(q: torch.Tensor) -> tuple:
    """Per-tensor FP8 quantisation; returns (fp8 tensor, scale)."""
    qf = q.to(torch.float32)
    scale = float(qf.abs().max().clamp_min(1e-30)) / FP8_MAX
    return (qf / scale).to(torch.float8_e4m3fn), scale


def uniform_lengths(batch: int, lo: int, hi: int, gen: torch.Generator) -> list:
    return torch.randint(lo, hi + 1, (batch,), generator=gen).tolist()


def log_uniform_lengths(batch: int, lo: int, hi: int, gen: torch.Generator) -> list:
    u = torch.rand(batch, generator=gen, dtype=torch.float64)
    return [int(round(math.exp(math.log(lo) + x * (math.log(hi) - math.log(lo))))) for x in u.tolist()]


def pages_needed(seq_lens: list) -> list:
    return [(max(0, int(l)) + PAGE - 1) // PAGE for l in seq_lens]


def page_tables(seq_lens: list, pool_pages: int, gen: torch.Generator, disjoint: bool,
                max_pages: int | None = None) -> torch.Tensor:
    """[B, max_pages] int32 page tables.

    disjoint: request b gets its own ceil(L_b/64) pages of a random
    permutation of the pool and the rest of its row is -1 (never read);
    otherwise every row is an independent random permutation of the pool
    truncated to the table width (requests may share pages).
    """
    need = pages_needed(seq_lens)
    width = max(1, max(need) if need else 1, max_pages or 0)
    B = len(seq_lens)
    if disjoint:
        assert pool_pages >= sum(need), "pool too small for disjoint page tables"
        perm = torch.randperm(pool_pages, generator=gen)
        bt = torch.full((B, width), -1, dtype=torch.int32)
        off = 0
        for b, n in enumerate(need):
            bt[b, :n] = perm[off:off + n].to(torch.int32)
            off += n
        return bt
    assert pool_pages >= width, "pool smaller than one request's pages"
    rows = [torch.randperm(pool_pages, generator=gen)[:width] for _ in range(B)]
    return torch.stack(rows).to(torch.int32).contiguous() if rows else torch.zeros(0, width, dtype=torch.int32)


def make_indexer_inputs(seq_lens: list, pool_pages: int, seed: int = 0, device="cuda",
                        disjoint: bool = False, max_pages: int | None = None) -> IndexerInputs:
    cpu, dev = _gens(seed, device)
    B = len(seq_lens)
    bt = page_tables(seq_lens, pool_pages, cpu, disjoint, max_pages)
    q = torch.randn(B, IX_HEADS, IX_DIM, generator=dev, device=device, dtype=torch.float32)
    q8, q_scale = quantize_q(q.to(torch.bfloat16))
    rows = torch.randn(pool_pages * PAGE, IX_DIM, generator=dev, device=device,
                       dtype=torch.float32).to(torch.bfloat16)
    kc = quantize_pages(rows)
    del rows
    w = torch.randn(B, IX_HEADS, generator=dev, device=device, dtype=torch.float32) / 8.0 * q_scale
    return IndexerInputs(q8, kc, w, torch.tensor(seq_lens, dtype=torch.int32, device=device),
                         bt.to(device))


def sparse_indices_for(lengths: list, pool_pages: int, gen: torch.Generator,
                       valid_counts: list | None = None) -> torch.Tensor:
    """[T, 2048] int32 slot ids: distinct positions < L_t through a random page table."""
    out = torch.full((len(lengths), TOPK), -1, dtype=torch.int32)
    for t, L in enumerate(lengths):
        n_pages = (L + PAGE - 1) // PAGE
        pt = torch.randperm(pool_pages, generator=gen)[:n_pages]
        k = min(L, TOPK) if valid_counts is None else min(valid_counts[t], L, TOPK)
        pos = torch.randperm(L, generator=gen)[:k]
        out[t, :k] = (pt[pos // PAGE] * PAGE + pos % PAGE).to(torch.int32)
    return out


def make_attention_inputs(num_tokens: int, pool_pages: int, seed: int = 0, device="cuda",
                          len_range: tuple = (4096, 16384),
                          valid_counts: list | None = None) -> AttentionInputs:
    cpu, dev = _gens(seed, device)
    lengths = uniform_lengths(num_tokens, len_range[0], min(len_range[1], pool_pages * PAGE), cpu)
    idx = sparse_indices_for(lengths, pool_pages, cpu, valid_counts)
    qn = torch.randn(num_tokens, A_HEADS, CKV, generator=dev, device=device).to(torch.bfloat16)
    qp = torch.randn(num_tokens, A_HEADS, KPE, generator=dev, device=device).to(torch.bfloat16)
    ckv = torch.randn(pool_pages, PAGE, CKV, generator=dev, device=device).to(torch.bfloat16)
    kpe = torch.randn(pool_pages, PAGE, KPE, generator=dev, device=device).to(torch.bfloat16)
    return AttentionInputs(qn, qp, ckv, kpe, idx.to(device), 1.0 / math.sqrt(192.0))


@dataclass
class DecodeInputs:
    """One decode step: indexer inputs plus attention queries over the same pages."""
    indexer: IndexerInputs
    q_nope: torch.Tensor
    q_pe: torch.Tensor
    ckv_cache: torch.Tensor
    kpe_cache: torch.Tensor
    sm_scale: float


def make_decode_inputs(seq_lens: list, seed: int = 0, device="cuda",
                       pool_pages: int | None = None) -> DecodeInputs:
    """Each request owns disjoint pages of one pool shared by the FP8 index
    cache and the ckv / kpe caches (slot ids mean the same row in all three)."""
    B = len(seq_lens)
    pool = pool_pages or max(1, sum(pages_needed(seq_lens)))
    ix = make_indexer_inputs(seq_lens, pool, seed, device, disjoint=True)
    _, dev = _gens(seed + 7, device)
    qn = torch.randn(B, A_HEADS, CKV, generator=dev, device=device).to(torch.bfloat16)
    qp = torch.randn(B, A_HEADS, KPE, generator=dev, device=device).to(torch.bfloat16)
    ckv = torch.randn(pool, PAGE, CKV, generator=dev, device=device).to(torch.bfloat16)
    kpe = torch.randn(pool, PAGE, KPE, generator=dev, device=device).to(torch.bfloat16)
    return DecodeInputs(ix, qn, qp, ckv, kpe, 1.0 / math.sqrt(192.0))


@dataclass
class PrefillInputs:
    """Query rows of several requests over paged FP8 K caches (prefill)."""
    q_index_fp8: torch.Tensor        # [T, 64, 128] float8_e4m3fn
    k_index_cache_fp8: torch.Tensor  # [pages, 64, 1, 132] uint8
    weights: torch.Tensor            # [T, 64] float32
    seq_lens: torch.Tensor           # [T] int32, causal lengths
    block_table: torch.Tensor        # [R, max_pages] int32
    cu_seqlens_q: torch.Tensor       # [R + 1] int32

    @property
    def num_pages(self) -> int:
        return self.k_index_cache_fp8.shape[0]


def make_prefill_inputs(prefixes: list, chunks: list, seed: int = 0, device="cuda",
                        extra_pages: int = 0) -> PrefillInputs:
    """Request r has `prefixes[r]` cached tokens and appends `chunks[r]` query
    tokens; query t of the chunk sees positions <= prefix + t (causal), so its
    row's length is prefix + t + 1.  Requests own disjoint pages of one pool."""
    cpu, dev = _gens(seed, device)
    totals = [p + c for p, c in zip(prefixes, chunks)]
    need = pages_needed(totals)
    pool = sum(need) + extra_pages
    bt = page_tables(totals, pool, cpu, disjoint=True)
    lens = [p + t + 1 for p, c in zip(prefixes, chunks) for t in range(c)]
    T = len(lens)
    cu = [0]
    for c in chunks:
        cu.append(cu[-1] + c)
    q = torch.randn(T, IX_HEADS, IX_DIM, generator=dev, device=device, dtype=torch.float32)
    q8, q_scale = quantize_q(q.to(torch.bfloat16))
    del q
    rows = torch.randn(pool * PAGE, IX_DIM, generator=dev, device=device,
                       dtype=torch.float32).to(torch.bfloat16)
    kc = quantize_pages(rows)
    del rows
    w = torch.randn(T, IX_HEADS, generator=dev, device=device, dtype=torch.float32) / 8.0 * q_scale
    return PrefillInputs(q8, kc, w, torch.tensor(lens, dtype=torch.int32, device=device),
                         bt.to(device), torch.tensor(cu, dtype=torch.int32, device=device))


def prefill_flops(seq_lens: list) -> int:
    """FP8 MACs x 2 of the per-row scores actually needed (each row's own length)."""
    return sum(2 * IX_HEADS * IX_DIM * max(0, int(L)) for L in seq_lens)


# ------------------------------------------------------------ byte model
def indexer_bytes(seq_lens: list) -> int:
    """Algorithmic HBM bytes of one indexer call: 132 B per context token
    (128 FP8 + 4 scale), q (8 KiB), weights (256 B), the request's page-table
    entries, seq_len and the 8 KiB output row, per request."""
    total = 0
    for L in seq_lens:
        L = max(0, int(L))
        total += 132 * L + IX_HEADS * IX_DIM + IX_HEADS * 4 + 4 * ((L + PAGE - 1) // PAGE) + 4 + TOPK * 4
    return total


def attention_bytes(num_tokens: int, valid_rows: int | None = None) -> int:
    """Algorithmic HBM bytes of one attention call: 1152 B per selected row
    (512 + 64 bf16), q (18 KiB), indices (8 KiB), output (16 KiB), lse."""
    rows = TOPK * num_tokens if valid_rows is None else valid_rows
    per_tok = A_HEADS * (CKV + KPE) * 2 + TOPK * 4 + A_HEADS * CKV * 2 + A_HEADS * 4
    return rows * (CKV + KPE) * 2 + num_tokens * per_tok


def indexer_flops(seq_lens: list) -> int:
    return sum(2 * IX_HEADS * IX_DIM * max(0, int(L)) for L in seq_lens)


def attention_flops(num_tokens: int) -> int:
    return num_tokens * A_HEADS * TOPK * 2 * (CKV + KPE + CKV)
