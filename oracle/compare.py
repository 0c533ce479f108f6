"""Comparators for parity tests (TEST INFRASTRUCTURE ONLY).

Indexer: outputs are compared as sets of global slot ids per request, plus the
-1 padding layout.  A slot that only one side selected is a *boundary swap*;
a swap is accepted only when the two tokens' oracle scores are within the
fp32 reordering bound of each other (``oracle.indexer.score_error_bound``),
i.e. when a different fp32 accumulation order could flip them.  Swaps are
counted and returned so tests and the bench can report them.  The order is
checked too (the reference returns torch.topk's sorted order): in a row that
is not identical to the oracle's, every output must score at least the next
one's oracle score minus the two tokens' rounding bounds.

Attention: the contest harness rule -- an element fails only if
``abs_err > atol`` AND ``rel_err > rtol`` -- with atol = rtol = 1e-2 for the
bf16 output and 1e-3 for the base-2 lse; -inf lse entries must match exactly.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import indexer as _ix


@dataclass
class TopkReport:
    ok: bool = True
    rows: int = 0
    exact_rows: int = 0            # identical row, order included
    swaps: int = 0                 # slots selected by only one side
    max_swap_gap: float = 0.0      # largest |score gap| of an accepted swap
    order_violations: int = 0      # adjacent outputs out of score order
    problems: list = field(default_factory=list)


def _slot_to_token(bt_row: np.ndarray, seq_len: int, num_pages: int) -> np.ndarray:
    n_pages = (seq_len + _ix.PAGE_SIZE - 1) // _ix.PAGE_SIZE
    inv = np.full(num_pages, -1, dtype=np.int64)
    inv[bt_row[:n_pages]] = np.arange(n_pages)
    return inv


def compare_topk(got: torch.Tensor, ref: torch.Tensor, scores: list, bounds: list,
                 seq_lens: torch.Tensor, block_table: torch.Tensor, num_pages: int,
                 topk: int = _ix.TOPK) -> TopkReport:
    got = got.cpu().numpy().astype(np.int64)
    ref = ref.cpu().numpy().astype(np.int64)
    sl = seq_lens.cpu().numpy().astype(np.int64)
    bt = block_table.cpu().numpy().astype(np.int64)
    rep = TopkReport(rows=got.shape[0])
    for b in range(got.shape[0]):
        L = int(sl[b])
        kk = min(max(L, 0), topk)
        g, r = got[b], ref[b]
        if np.array_equal(g, r):
            rep.exact_rows += 1
            continue
        if not (np.all(g[kk:] == -1) and np.all(g[:kk] >= 0)):
            rep.ok = False
            rep.problems.append(f"row {b}: padding layout wrong (k={kk})")
            continue
        gs, rs = set(g[:kk].tolist()), set(r[:kk].tolist())
        if len(gs) != kk:
            rep.ok = False
            rep.problems.append(f"row {b}: duplicate slots")
            continue
        only_g, only_r = gs - rs, rs - gs
        inv = _slot_to_token(bt[b], L, num_pages)
        sc = scores[b].numpy().astype(np.float64)
        eb = bounds[b].numpy().astype(np.float64)

        def tok(slot):
            t = inv[slot // _ix.PAGE_SIZE]
            return -1 if t < 0 else int(t * _ix.PAGE_SIZE + slot % _ix.PAGE_SIZE)

        tall = np.array([tok(s) for s in g[:kk]], dtype=np.int64)
        if kk and (tall.min() < 0 or tall.max() >= L):
            rep.ok = False
            rep.problems.append(f"row {b}: slot outside the request's pages")
            continue
        s_all, e_all = sc[tall], eb[tall]
        bad = np.nonzero(s_all[1:] - s_all[:-1] > e_all[1:] + e_all[:-1])[0]
        if bad.size:
            rep.ok = False
            rep.order_violations += int(bad.size)
            i = int(bad[0])
            rep.problems.append(f"row {b}: output {i + 1} (score {s_all[i + 1]:.7g}) ranks below "
                                f"output {i} (score {s_all[i]:.7g})")
            continue
        if not only_g:
            continue  # same set, different order of (near-)equal scores
        tg = [tok(s) for s in only_g]
        tr = [tok(s) for s in only_r]
        # every GPU-only token must be within rounding of every ref-only token
        worst_ref = min(tr, key=lambda t: sc[t])
        best_got = max(tg, key=lambda t: sc[t])
        lo_ref = sc[worst_ref]
        for t in tg:
            gap = lo_ref - sc[t]
            if gap > eb[t] + eb[worst_ref]:
                rep.ok = False
                rep.problems.append(
                    f"row {b}: token {t} (score {sc[t]:.7g}) selected over {worst_ref} "
                    f"(score {lo_ref:.7g}); gap {gap:.3g} exceeds rounding bound")
                break
            rep.max_swap_gap = max(rep.max_swap_gap, float(abs(gap)))
        del best_got
        rep.swaps += len(only_g)
    return rep


@dataclass
class CloseReport:
    ok: bool
    max_abs: float
    max_rel: float
    n_bad: int


def harness_close(got: torch.Tensor, ref: torch.Tensor, atol: float, rtol: float) -> CloseReport:
    """Element fails only if abs_err > atol AND rel_err > rtol (FAQ.md:110-116)."""
    g = got.detach().cpu().to(torch.float64)
    r = ref.detach().cpu().to(torch.float64)
    both_inf = torch.isinf(g) & torch.isinf(r) & (torch.sign(g) == torch.sign(r))
    diff = (g - r).abs()
    diff = torch.where(both_inf, torch.zeros_like(diff), diff)
    rel = diff / r.abs().clamp_min(1e-30)
    rel = torch.where(both_inf, torch.zeros_like(rel), rel)
    bad = (diff > atol) & (rel > rtol)
    bad = bad | (torch.isnan(g) != torch.isnan(r))
    bad = bad | ((torch.isinf(g) | torch.isinf(r)) & ~both_inf)
    finite = torch.isfinite(diff)
    return CloseReport(ok=not bool(bad.any()),
                       max_abs=float(diff[finite].max()) if finite.any() else 0.0,
                       max_rel=float(rel[finite].max()) if finite.any() else 0.0,
                       n_bad=int(bad.sum()))
