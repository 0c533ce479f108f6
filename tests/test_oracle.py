"""CPU tests that pin the oracle to the published references (via the
committed golden fixtures) and check the comparators."""

import math
import pathlib

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import compare
from oracle import indexer as oix

GOLD = pathlib.Path(__file__).resolve().parent / "golden"


def test_e4m3_table_matches_bit_layout():
    table = oix.e4m3_table()
    for b in range(256):
        want = oix.decode_e4m3fn(b)
        got = float(table[b])
        if math.isnan(want):
            assert math.isnan(got), b
        else:
            assert got == want, (b, got, want)
    assert oix.decode_e4m3fn(0x7E) == 448.0
    assert oix.decode_e4m3fn(0x01) == 2.0 ** -9


def test_order_keys_total_order():
    vals = np.array([-np.inf, -3.5, -1e-30, -0.0, 0.0, 1e-30, 2.0, np.inf, np.nan], np.float32)
    keys = oix.order_keys(vals)
    assert keys[3] == keys[4]                      # -0 == +0
    assert np.all(np.diff(keys[[0, 1, 2, 4, 5, 6, 7]].astype(np.int64)) > 0)
    assert keys[8] == 0xFFFFFFFF                   # NaN ranks first


def test_topk_tie_break_lowest_index():
    s = np.zeros(5000, np.float32)
    s[4000] = 1.0
    order = oix.topk_order(s, 2048)
    assert order[0] == 4000
    assert np.array_equal(order[1:], np.arange(2047))


def test_topk_short_rows():
    s = np.array([0.5, 2.0, -1.0], np.float32)
    assert list(oix.topk_order(s, 2048)) == [1, 0, 2]
    assert oix.topk_order(np.zeros(0, np.float32), 2048).shape == (0,)


def _load_indexer_fixture():
    z = np.load(GOLD / "indexer_small.npz")
    q = torch.from_numpy(z["q"]).view(torch.float8_e4m3fn)
    return (q, torch.from_numpy(z["k_cache"]), torch.from_numpy(z["weights"]),
            torch.from_numpy(z["seq_lens"]), torch.from_numpy(z["block_table"]),
            torch.from_numpy(z["logits"]), torch.from_numpy(z["topk"]))


def test_indexer_scores_match_deepgemm_reference():
    q, kc, w, sl, bt, logits, _ = _load_indexer_fixture()
    _, scores = oix.indexer_reference(q, kc, w, sl, bt)
    kc_u8 = kc.view(torch.uint8).reshape(-1)
    for b in range(q.shape[0]):
        L = int(sl[b])
        ref = logits[b, :L]
        # DeepGEMM applies the token scale after the head sum, the reference
        # solution before the ReLU: equal for positive scales up to fp32
        # reordering, which the bound covers.
        bound = oix.score_error_bound(q[b], kc_u8, w[b], L, bt[b].long())
        assert ((scores[b] - ref).abs() <= bound).all(), b
        assert torch.isinf(logits[b, L:]).all()


def test_indexer_topk_matches_flashinfer_transform():
    q, kc, w, sl, bt, _, gold = _load_indexer_fixture()
    got, scores = oix.indexer_reference(q, kc, w, sl, bt)
    kc_u8 = kc.view(torch.uint8).reshape(-1)
    bounds = [oix.score_error_bound(q[b], kc_u8, w[b], int(sl[b]), bt[b].long())
              for b in range(q.shape[0])]
    # flashinfer's transform leaves 0 (not -1) past min(L, k); the reference
    # solution pads with -1 (kernel.py:206).
    ref = gold.clone()
    for b in range(q.shape[0]):
        ref[b, min(int(sl[b]), 2048):] = -1
    rep = compare.compare_topk(got, ref, scores, bounds, sl, bt, kc.shape[0])
    assert rep.ok, rep.problems
    assert rep.exact_rows + (rep.swaps > 0) >= q.shape[0] - 1


def test_attention_oracle_matches_flashinfer_reference():
    z = np.load(GOLD / "attention_small.npz")
    qn = torch.from_numpy(z["q_nope"]).view(torch.bfloat16)
    qp = torch.from_numpy(z["q_pe"]).view(torch.bfloat16)
    ckv = torch.from_numpy(z["ckv"]).view(torch.bfloat16)
    kpe = torch.from_numpy(z["kpe"]).view(torch.bfloat16)
    idx = torch.from_numpy(z["indices"])
    out, lse = oatt.attention_reference(qn, qp, ckv, kpe, idx, float(z["sm_scale"]))
    gold_out = torch.from_numpy(z["output"]).view(torch.bfloat16)
    gold_lse = torch.from_numpy(z["lse"])
    assert compare.harness_close(out, gold_out, 1e-6, 1e-6).ok
    assert compare.harness_close(lse, gold_lse, 1e-6, 1e-6).ok
    assert torch.isinf(lse[2]).all() and (out[2] == 0).all()


def test_compare_topk_rejects_a_planted_wrong_index():
    q, kc, w, sl, bt, _, _ = _load_indexer_fixture()
    ref, scores = oix.indexer_reference(q, kc, w, sl, bt)
    kc_u8 = kc.view(torch.uint8).reshape(-1)
    bounds = [oix.score_error_bound(q[b], kc_u8, w[b], int(sl[b]), bt[b].long())
              for b in range(q.shape[0])]
    bad = ref.clone()
    # Plant a mistake: replace the best token of row 0 by an unselected one.
    L = int(sl[0])
    order = oix.topk_order(scores[0].numpy(), 2048)
    loser = int(oix.topk_order(scores[0].numpy(), L)[-1])
    bad[0, 0] = int(bt[0, loser // 64]) * 64 + loser % 64
    assert order[0] != loser
    rep = compare.compare_topk(bad, ref, scores, bounds, sl, bt, kc.shape[0])
    assert not rep.ok


def test_compare_topk_rejects_a_planted_wrong_order():
    q, kc, w, sl, bt, _, _ = _load_indexer_fixture()
    ref, scores = oix.indexer_reference(q, kc, w, sl, bt)
    kc_u8 = kc.view(torch.uint8).reshape(-1)
    bounds = [oix.score_error_bound(q[b], kc_u8, w[b], int(sl[b]), bt[b].long())
              for b in range(q.shape[0])]
    # Same set, but the best and the 100th outputs of row 0 trade places.
    bad = ref.clone()
    bad[0, 0], bad[0, 99] = ref[0, 99].item(), ref[0, 0].item()
    rep = compare.compare_topk(bad, ref, scores, bounds, sl, bt, kc.shape[0])
    assert not rep.ok and rep.order_violations > 0
    # Exactly equal scores may come in either order only when bounds allow:
    # the oracle's own output passes untouched.
    assert compare.compare_topk(ref, ref, scores, bounds, sl, bt, kc.shape[0]).ok


def test_harness_close_rule():
    ref = torch.tensor([1.0, 100.0, -math.inf])
    assert compare.harness_close(torch.tensor([1.005, 100.5, -math.inf]), ref, 0.01, 0.01).ok
    assert not compare.harness_close(torch.tensor([1.05, 100.0, -math.inf]), ref, 0.01, 0.01).ok
    assert not compare.harness_close(torch.tensor([1.0, 100.0, 0.0]), ref, 0.01, 0.01).ok


@pytest.mark.parametrize("L", [1, 63, 64, 65, 129])
def test_indexer_oracle_small_lengths_pad_with_minus_one(L):
    from dsa_b200 import workloads
    ix = workloads.make_indexer_inputs([L], pool_pages=8, seed=L, device="cpu")
    out, _ = oix.indexer_reference(ix.q_index_fp8, ix.k_index_cache_fp8, ix.weights,
                                   ix.seq_lens, ix.block_table)
    assert (out[0, L:] == -1).all() and (out[0, :L] >= 0).all()
    assert len(set(out[0, :L].tolist())) == L
