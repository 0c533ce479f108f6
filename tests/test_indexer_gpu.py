"""GPU parity of the indexer (dsa_b200.indexer.run -> C ABI -> sm_100a
kernels) against the CPU oracle and the golden fixture."""

import pathlib

import numpy as np
import pytest
import torch

from dsa_b200 import DsaError, indexer, workloads
from dsa_b200 import workspace as ws_mod
from oracle import compare
from oracle import indexer as oix

pytestmark = pytest.mark.gpu
GOLD = pathlib.Path(__file__).resolve().parent / "golden"


def run_gpu(ix, out=None):
    B = ix.q_index_fp8.shape[0]
    if out is None:
        out = torch.full((B, 2048), 7, dtype=torch.int32, device=ix.q_index_fp8.device)
    indexer.run(ix.q_index_fp8, ix.k_index_cache_fp8, ix.weights, ix.seq_lens, ix.block_table, out)
    torch.cuda.synchronize()
    return out


def oracle_check(ix, got, rows=None):
    """Compares `got` with the oracle on `rows` (all by default)."""
    rows = list(range(ix.q_index_fp8.shape[0])) if rows is None else rows
    q = ix.q_index_fp8[rows].cpu()
    kc = ix.k_index_cache_fp8.cpu()
    w = ix.weights[rows].cpu()
    sl = ix.seq_lens[rows].cpu()
    bt = ix.block_table[rows].cpu()
    ref, scores = oix.indexer_reference(q, kc, w, sl, bt)
    ku = kc.view(torch.uint8).reshape(-1)
    bounds = [oix.score_error_bound(q[i], ku, w[i], int(sl[i]), bt[i].long())
              for i in range(len(rows))]
    rep = compare.compare_topk(got[rows].cpu(), ref, scores, bounds, sl, bt, kc.shape[0])
    assert rep.ok, rep.problems[:5]
    return rep


@pytest.mark.parametrize("seq_lens", [
    [100], [2048], [2049], [1, 63, 64, 65, 127, 128, 129], [2500, 130, 0, 71], [0, 0, 0],
])
def test_small_lengths(cuda_device, seq_lens):
    ix = workloads.make_indexer_inputs(seq_lens, pool_pages=64, seed=sum(seq_lens) + 1,
                                       device=cuda_device)
    got = run_gpu(ix)
    rep = oracle_check(ix, got)
    assert rep.swaps == 0


def test_eight_requests_2k_to_8k(cuda_device):
    g = torch.Generator().manual_seed(0)
    lens = workloads.uniform_lengths(8, 2048, 8192, g)
    ix = workloads.make_indexer_inputs(lens, pool_pages=1024, seed=0, device=cuda_device)
    got = run_gpu(ix)
    rep = oracle_check(ix, got)
    print(f"8 requests of 2048-8192 tokens: exact rows {rep.exact_rows}/8, boundary swaps {rep.swaps}")


def test_golden_fixture(cuda_device):
    z = np.load(GOLD / "indexer_small.npz")
    ix = workloads.IndexerInputs(
        torch.from_numpy(z["q"]).view(torch.float8_e4m3fn).to(cuda_device),
        torch.from_numpy(z["k_cache"]).to(cuda_device),
        torch.from_numpy(z["weights"]).to(cuda_device),
        torch.from_numpy(z["seq_lens"]).to(cuda_device),
        torch.from_numpy(z["block_table"]).to(cuda_device))
    got = run_gpu(ix).cpu()
    gold = torch.from_numpy(z["topk"])
    for b in range(gold.shape[0]):
        L = int(z["seq_lens"][b])
        k = min(L, 2048)
        assert set(got[b, :k].tolist()) == set(gold[b, :k].tolist()), b
        assert (got[b, k:] == -1).all()
    oracle_check(ix, got.to(cuda_device))


def test_all_equal_scores_break_ties_by_index(cuda_device):
    # q == 0 makes every score 0: the top-2048 are the first 2048 tokens, in
    # token order.  L > the shared-memory candidate capacity exercises the
    # global fallback of the select.
    for L in (5000, 100000):
        ix = workloads.make_indexer_inputs([L], pool_pages=L // 64 + 2, seed=3, device=cuda_device)
        ix.q_index_fp8.zero_()
        got = run_gpu(ix).cpu()[0]
        bt = ix.block_table.cpu()[0].long()
        tok = torch.arange(2048)
        want = (bt[tok // 64] * 64 + tok % 64).to(torch.int32)
        assert torch.equal(got, want), L


def test_outlier_scores_keep_sorted_order(cuda_device):
    # Scales 10^4 times larger on one page give a few scores far above the
    # rest: the select's bucket sort then sees the other keys crowd into a few
    # buckets and sorts with its merge-sort path instead.
    ix = workloads.make_indexer_inputs([8192, 8192], pool_pages=300, seed=41, device=cuda_device)
    kc = ix.k_index_cache_fp8.view(torch.uint8).reshape(ix.num_pages, -1)
    page = int(ix.block_table[0, 0])
    kc[page, 64 * 128:].view(torch.float32).mul_(1e4)
    got = run_gpu(ix)
    rep = oracle_check(ix, got)
    assert rep.order_violations == 0


def test_repeated_page_ties(cuda_device):
    # Every page of the request is the same physical page: 64 distinct
    # scores, each repeated L/64 times -> ties resolved by token index.
    L = 8192
    ix = workloads.make_indexer_inputs([L], pool_pages=160, seed=5, device=cuda_device)
    ix.block_table.fill_(3)
    got = run_gpu(ix)
    rep = oracle_check(ix, got)
    assert rep.exact_rows == 1


def test_longer_block_table_and_minus_one_tail(cuda_device):
    lens = [3000, 700]
    ix = workloads.make_indexer_inputs(lens, pool_pages=128, seed=9, device=cuda_device,
                                       max_pages=100)
    bt = ix.block_table.clone()
    bt[0, 47:] = -1   # beyond ceil(3000/64) = 47 pages: never read
    bt[1, 11:] = -1
    ix.block_table = bt
    got = run_gpu(ix)
    oracle_check(ix, got)


def test_bad_page_id_is_reported(cuda_device):
    ix = workloads.make_indexer_inputs([300], pool_pages=16, seed=11, device=cuda_device)
    ix.block_table[0, 2] = 10_000
    with pytest.raises(DsaError, match="block_table"):
        run_gpu(ix)


def test_bad_seq_len_is_reported(cuda_device):
    ix = workloads.make_indexer_inputs([300], pool_pages=16, seed=12, device=cuda_device)
    ix.seq_lens[0] = ix.block_table.shape[1] * 64 + 1
    with pytest.raises(DsaError, match="seq_len"):
        run_gpu(ix)


def test_graph_capture_reads_seq_lens_on_device(cuda_device):
    lens = [4000, 2500, 9000]
    ix = workloads.make_indexer_inputs(lens, pool_pages=512, seed=21, device=cuda_device,
                                       max_pages=160)
    out = torch.empty(3, 2048, dtype=torch.int32, device=cuda_device)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up on the capture stream sizes its workspace
        run_gpu(ix, out)
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        indexer.run(ix.q_index_fp8, ix.k_index_cache_fp8, ix.weights, ix.seq_lens,
                    ix.block_table, out)
    torch.cuda.current_stream().wait_stream(s)
    for new in ([4000, 2500, 9000], [10000, 64, 2049], [0, 5000, 1]):
        ix.seq_lens.copy_(torch.tensor(new, dtype=torch.int32))
        g.replay()
        torch.cuda.synchronize()
        oracle_check(ix, out.clone())


def test_score_precision_vs_oracle(cuda_device):
    # The fp32 scores live in the workspace after a call; their deviation from
    # the oracle must stay inside the reordering bound the comparator uses.
    lens = [6000, 3000]
    ix = workloads.make_indexer_inputs(lens, pool_pages=256, seed=31, device=cuda_device)
    run_gpu(ix)
    stream_id = torch.cuda.current_stream(cuda_device).cuda_stream
    buf = ws_mod.all_buffers()[(cuda_device.index, "indexer", stream_id)]
    stride = ix.block_table.shape[1] * 64
    off = 256 + 32768 + 2 * 2048 * 4   # header, ready counters, then the radix histograms
    scores = buf[off:off + 4 * 2 * stride].view(torch.float32).reshape(2, stride).cpu()
    q, kc, w = ix.q_index_fp8.cpu(), ix.k_index_cache_fp8.cpu(), ix.weights.cpu()
    bt = ix.block_table.cpu()
    ku = kc.view(torch.uint8).reshape(-1)
    worst = 0.0
    for b, L in enumerate(lens):
        ref = oix.score_request(q[b], ku, w[b], L, bt[b].long())
        bound = oix.score_error_bound(q[b], ku, w[b], L, bt[b].long())
        ratio = float(((scores[b, :L] - ref).abs() / bound).max())
        worst = max(worst, ratio)
    print(f"max |gpu - oracle| / bound = {worst:.3g}")
    assert worst <= 1.0


def test_64_requests_32k_to_128k(cuda_device):
    g = torch.Generator().manual_seed(2)
    lens = workloads.uniform_lengths(64, 32768, 131072, g)
    ix = workloads.make_indexer_inputs(lens, pool_pages=150_000, seed=2, device=cuda_device)
    got = run_gpu(ix)
    rep = oracle_check(ix, got, rows=[0, 17, 63])
    # Size-independent properties on every row: 2048 distinct slots, each in
    # one of the request's pages.
    bt = ix.block_table.cpu()
    for b in range(64):
        row = got[b].cpu()
        assert (row >= 0).all() and row.unique().numel() == 2048, b
        pages = set(bt[b, : (lens[b] + 63) // 64].tolist())
        assert set((row // 64).tolist()) <= pages, b
    print(f"64 requests of 32768-131072 tokens, sampled: exact {rep.exact_rows}/3, swaps {rep.swaps}")


def test_workspace_reuse_across_sizes(cuda_device):
    # One stream, one workspace; growing the batch at a fixed workspace size
    # moves the histogram region onto bytes that held scores before (the 6-row
    # call after the 2-row one): every call clears its histogram rows before
    # the score kernel adds to them.  Largest first, so later calls reuse
    # (never regrow) the workspace.
    for lens, mp in (([5000] * 9, 80), ([9000] * 2, 160), ([6000] * 6, 100), ([2100] * 4, 160)):
        ix = workloads.make_indexer_inputs(lens, pool_pages=512, seed=len(lens), device=cuda_device,
                                           max_pages=mp)
        oracle_check(ix, run_gpu(ix))
    # Histograms left over from a previous call never leak into the next one:
    # the same call twice gives the same result.
    ix = workloads.make_indexer_inputs([6000] * 6, pool_pages=512, seed=6, device=cuda_device,
                                       max_pages=100)
    first = run_gpu(ix)
    assert torch.equal(first, run_gpu(ix))


def test_select_wide_and_narrow_ctas_agree(cuda_device):
    """More rows than SMs run the select as 512-thread CTAs (two per SM); at most
    one row per SM as 1024-thread CTAs.  A row's result does not depend on which
    variant ran it: degenerate rows (all scores equal, so the staging areas
    overflow and the winners crowd one bucket) and rows of <= 2048 tokens
    included."""
    n_sm = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    B = n_sm + 20
    g = torch.Generator().manual_seed(95)
    lens = workloads.uniform_lengths(B, 2049, 40000, g)
    lens[1], lens[7], lens[n_sm + 2] = 2048, 300, 0
    ix = workloads.make_indexer_inputs(lens, pool_pages=1024, seed=96, device=cuda_device)
    for r in (3, n_sm + 5):
        ix.q_index_fp8[r].zero_()  # every score of the row is 0
    wide = run_gpu(ix)  # B > SMs: 512-thread CTAs
    for lo, hi in ((0, n_sm), (n_sm - 10, B)):
        narrow = torch.full((hi - lo, 2048), 7, dtype=torch.int32, device=cuda_device)
        indexer.run(ix.q_index_fp8[lo:hi], ix.k_index_cache_fp8, ix.weights[lo:hi], ix.seq_lens[lo:hi],
                    ix.block_table[lo:hi], narrow)
        torch.cuda.synchronize()
        assert torch.equal(narrow, wide[lo:hi]), (lo, hi)
    oracle_check(ix, wide, rows=[0, 1, 3, 7, n_sm + 2, n_sm + 5, B - 1])


def test_ready_wait_timeout_is_reported_and_the_next_call_is_exact(cuda_device):
    """Each request's select waits, bounded, until the score kernel has published
    the request's ready count.  The failure path, made to happen without
    faulting anything: a test hook makes the score kernel publish nothing for
    request 0 and shortens the select's wait to 1 ms.  Request 0's select gives
    up, reports DSA_DEV_WAIT_TIMEOUT and writes its row as all -1; the other
    rows are exact.  The select then takes request 0's scored count as consumed,
    so the next call on the same workspace is exact again."""
    from dsa_b200 import _native
    ix = workloads.make_indexer_inputs([70000, 3000, 65536, 129], pool_pages=1200, seed=97,
                                       device=cuda_device)
    good = run_gpu(ix).clone()
    lib = _native.lib()
    assert lib.dsa_b200_test_inject(_native.TEST_SKIP_READY, 1_000_000) == 0
    out = torch.full_like(good, 7)
    try:
        with pytest.raises(DsaError, match="timed out"):
            run_gpu(ix, out)
    finally:
        lib.dsa_b200_test_inject(_native.TEST_NONE, 0)
    assert (out[0] == -1).all()
    assert torch.equal(out[1:], good[1:])
    for _ in range(2):
        assert torch.equal(run_gpu(ix), good)
