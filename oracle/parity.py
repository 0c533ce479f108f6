"""Oracle check of sampled decode rows, possibly from other ranks (TEST INFRASTRUCTURE ONLY).

A rank packs, for a few of its requests, everything the CPU oracle needs to
redo them -- the request's query, weights, length and FP8 K pages, the query
token's attention inputs and the ckv / kpe rows at the slots the indexer
selected -- into a bundle of CPU tensors (``pack_rows``).  The bundles travel
to rank 0 next to the NCCL-gathered outputs, and ``check_bundles`` compares
the gathered outputs with the oracle there:

* indexer: set equality with boundary swaps judged by the fp32 reordering
  bound (``oracle.compare.compare_topk``), after mapping the rank's global
  slot ids to request-local ones through the packed block-table row;
* attention over the indexer's own selections: output within atol = rtol =
  1e-2, lse within 1e-3 (the harness rule: an element fails only if both
  limits are exceeded).
"""

from __future__ import annotations

import numpy as np
import torch

from . import attention as oatt
from . import compare
from . import indexer as oix

OUT_TOL = 1e-2
LSE_TOL = 1e-3


def pack_rows(dec, topk: torch.Tensor, rows: list, rank: int = 0) -> list:
    """CPU bundle per sampled request of a decode step (`dec`: the step's
    DecodeInputs, `topk`: its indexer output on the device)."""
    ix = dec.indexer
    out = []
    for b in rows:
        L = int(ix.seq_lens[b])
        n_pages = (max(L, 0) + 63) // 64
        bt_row = ix.block_table[b, :n_pages].long()
        idx = topk[b].long()
        valid = idx >= 0
        rows_ = torch.where(valid, idx, torch.zeros_like(idx))
        out.append({
            "rank": rank, "row": b, "L": L,
            "q": ix.q_index_fp8[b].view(torch.uint8).cpu(),
            "w": ix.weights[b].cpu(),
            "bt": bt_row.cpu(),
            "kpages": ix.k_index_cache_fp8[bt_row].cpu(),
            "topk": topk[b].cpu(),
            "q_nope": dec.q_nope[b].cpu(), "q_pe": dec.q_pe[b].cpu(),
            "ckv_rows": dec.ckv_cache.reshape(-1, 512)[rows_].cpu(),
            "kpe_rows": dec.kpe_cache.reshape(-1, 64)[rows_].cpu(),
            "sm_scale": float(dec.sm_scale),
        })
    return out


def _local_slots(slots: np.ndarray, bt_row: np.ndarray) -> np.ndarray:
    """Global slot ids of one request -> ids in its pages renumbered 0..n-1
    (-1 stays -1; a slot outside the request's pages becomes -2)."""
    inv = {int(p): j for j, p in enumerate(bt_row.tolist())}
    res = np.full(slots.shape, -1, dtype=np.int64)
    for i, s in enumerate(slots.tolist()):
        if s >= 0:
            j = inv.get(s // 64)
            res[i] = -2 if j is None else j * 64 + s % 64
    return res


def check_bundles(bundles: list, gathered: list | None = None) -> dict:
    """Oracle check of every bundle.  `gathered` (rank 0 of a multi-GPU run):
    per rank (topk, output, lse) as received by the output gather; the
    indices checked are then the gathered ones (and must equal the bundle's)."""
    rep = {"rows": 0, "exact_rows": 0, "swaps": 0, "max_swap_gap": 0.0, "tokens": 0,
           "out_max_abs": 0.0, "out_max_rel": 0.0, "lse_max_abs": 0.0, "lse_max_rel": 0.0,
           "ok": True, "problems": []}
    for bd in bundles:
        r, b, L = bd["rank"], bd["row"], bd["L"]
        got_topk, got_out, got_lse = bd["topk"], None, None
        if gathered is not None:
            g_topk, g_out, g_lse = gathered[r]
            got_topk = g_topk[b].cpu()
            got_out, got_lse = g_out[b].cpu(), g_lse[b].cpu()
            if not torch.equal(got_topk, bd["topk"]):
                rep["ok"] = False
                rep["problems"].append(f"rank {r} row {b}: gathered indices differ from the rank's")
        n_pages = bd["bt"].numel()
        local_bt = torch.arange(max(n_pages, 1), dtype=torch.int32)[None]
        kc = bd["kpages"]
        q8 = bd["q"].view(torch.float8_e4m3fn)[None]
        w = bd["w"][None]
        sl = torch.tensor([L], dtype=torch.int32)
        ref, scores = oix.indexer_reference(q8, kc, w, sl, local_bt)
        ku = kc.view(torch.uint8).reshape(-1)
        bound = oix.score_error_bound(q8[0], ku, w[0], L, local_bt[0].long())
        mine = torch.from_numpy(_local_slots(got_topk.numpy().astype(np.int64), bd["bt"].numpy()))
        if (mine == -2).any():
            rep["ok"] = False
            rep["problems"].append(f"rank {r} row {b}: a slot outside the request's pages")
            continue
        tr = compare.compare_topk(mine.to(torch.int32)[None], ref, scores, [bound], sl, local_bt,
                                  max(n_pages, 1))
        rep["rows"] += 1
        rep["exact_rows"] += tr.exact_rows
        rep["swaps"] += tr.swaps
        rep["max_swap_gap"] = max(rep["max_swap_gap"], tr.max_swap_gap)
        if not tr.ok:
            rep["ok"] = False
            rep["problems"].extend(f"rank {r} row {b}: {p}" for p in tr.problems[:3])
        if got_out is None:
            continue
        # attention over this row's own selections, rows compacted
        valid = got_topk >= 0
        local = torch.where(valid, torch.arange(valid.numel()), torch.full_like(got_topk, -1).long())
        ro, rl = oatt.attention_reference(bd["q_nope"][None], bd["q_pe"][None],
                                          bd["ckv_rows"], bd["kpe_rows"], local[None], bd["sm_scale"])
        co = compare.harness_close(got_out[None], ro, OUT_TOL, OUT_TOL)
        cl = compare.harness_close(got_lse[None], rl, LSE_TOL, LSE_TOL)
        rep["tokens"] += 1
        rep["out_max_abs"] = max(rep["out_max_abs"], co.max_abs)
        rep["out_max_rel"] = max(rep["out_max_rel"], co.max_rel)
        rep["lse_max_abs"] = max(rep["lse_max_abs"], cl.max_abs)
        rep["lse_max_rel"] = max(rep["lse_max_rel"], cl.max_rel)
        if not (co.ok and cl.ok):
            rep["ok"] = False
            rep["problems"].append(f"rank {r} token {b}: output {co} lse {cl}")
    return rep
