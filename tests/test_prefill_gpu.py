"""GPU parity of the many-rows-per-request indexer (dsa_b200.indexer.run_prefill
-> C ABI -> sm_100a kernels): every row must match the decode oracle for its
(q, weights, seq_len, request block-table row), and the decode kernel run on
the same rows one request per row."""

import pytest
import torch

from dsa_b200 import DsaError, indexer, workloads
from oracle import compare
from oracle import indexer as oix

pytestmark = pytest.mark.gpu


def run_prefill(pf, out=None):
    T = pf.q_index_fp8.shape[0]
    if out is None:
        out = torch.full((T, 2048), 7, dtype=torch.int32, device=pf.q_index_fp8.device)
    indexer.run_prefill(pf.q_index_fp8, pf.k_index_cache_fp8, pf.weights, pf.seq_lens,
                        pf.block_table, pf.cu_seqlens_q, out)
    torch.cuda.synchronize()
    return out


def oracle_check(pf, got, rows):
    ref, scores = oix.prefill_reference(pf.q_index_fp8.cpu(), pf.k_index_cache_fp8.cpu(),
                                        pf.weights.cpu(), pf.seq_lens.cpu(), pf.block_table.cpu(),
                                        pf.cu_seqlens_q.cpu(), rows)
    ku = pf.k_index_cache_fp8.cpu().view(torch.uint8).reshape(-1)
    bt = oix.rows_block_table(pf.block_table, pf.cu_seqlens_q, rows)
    q = pf.q_index_fp8[rows].cpu()
    w = pf.weights[rows].cpu()
    sl = pf.seq_lens[rows].cpu()
    bounds = [oix.score_error_bound(q[i], ku, w[i], int(sl[i]), bt[i].long()) for i in range(len(rows))]
    rep = compare.compare_topk(got[rows].cpu(), ref, scores, bounds, sl, bt, pf.num_pages)
    assert rep.ok, rep.problems[:5]
    return rep


def decode_equivalent(pf):
    """The same rows as decode requests: block-table row of each row's request."""
    T = pf.q_index_fp8.shape[0]
    bt = oix.rows_block_table(pf.block_table, pf.cu_seqlens_q, range(T)).to(pf.block_table.device)
    out = torch.full((T, 2048), 7, dtype=torch.int32, device=pf.q_index_fp8.device)
    indexer.run(pf.q_index_fp8, pf.k_index_cache_fp8, pf.weights, pf.seq_lens, bt.contiguous(), out)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("prefixes,chunks", [
    ([0], [5]),                 # rows of length 1..5, one partial group
    ([100], [7]),               # short rows, a full and a partial group
    ([2000, 30], [6, 3]),       # two requests, rows across the 2048 boundary
    ([3000, 0, 500], [9, 1, 4]),
])
def test_prefill_small_matches_oracle(cuda_device, prefixes, chunks):
    pf = workloads.make_prefill_inputs(prefixes, chunks, seed=sum(prefixes) + len(chunks),
                                       device=cuda_device, extra_pages=3)
    got = run_prefill(pf)
    T = pf.q_index_fp8.shape[0]
    rep = oracle_check(pf, got, list(range(T)))
    assert rep.order_violations == 0


def test_prefill_empty_requests_and_zero_length_rows(cuda_device):
    # Requests with no rows (equal consecutive cu_seqlens_q entries), rows of
    # length 0 inside a group, and a request whose rows span three groups.
    pf = workloads.make_prefill_inputs([300, 2600, 0], [3, 9, 2], seed=31, device=cuda_device,
                                       extra_pages=2)
    R = pf.block_table.shape[0]
    bt = torch.cat([pf.block_table[:1], pf.block_table[:1], pf.block_table[1:], pf.block_table[2:]])
    cu = torch.tensor([0, 3, 3, 12, 12, 14], dtype=torch.int32, device=cuda_device)  # requests 1, 4 empty
    assert bt.shape[0] == R + 2
    pf.block_table, pf.cu_seqlens_q = bt.contiguous(), cu
    pf.seq_lens[1] = 0      # a zero-length row in the first group
    pf.seq_lens[7] = 0      # and one in the middle of the long request
    got = run_prefill(pf)
    T = pf.q_index_fp8.shape[0]
    oracle_check(pf, got, list(range(T)))
    assert (got[1] == -1).all() and (got[7] == -1).all()


def test_prefill_equals_decode_kernel(cuda_device):
    # 3 requests, 4k-16k contexts, 37 rows: the GEMM-shaped path and the
    # decode path score with the same per-token arithmetic.
    pf = workloads.make_prefill_inputs([4000, 9000, 15000], [13, 11, 13], seed=5, device=cuda_device)
    got = run_prefill(pf)
    dec = decode_equivalent(pf)
    same = (got == dec).all(dim=1)
    if not bool(same.all()):
        rows = [int(i) for i in torch.nonzero(~same).flatten().tolist()]
        oracle_check(pf, got, rows)  # differing rows must still be within rounding
    assert float(same.float().mean()) >= 0.9


def test_prefill_4096_rows_sampled(cuda_device):
    # One request, 4096 query rows appended to a 61440-token prefix (rows of
    # length 61441 .. 65536): sampled rows against the oracle.
    pf = workloads.make_prefill_inputs([61440], [4096], seed=3, device=cuda_device)
    got = run_prefill(pf)
    rows = [0, 1, 2, 3, 1000, 2047, 4094, 4095]
    rep = oracle_check(pf, got, rows)
    print(f"prefill, 4096 rows, sampled: exact {rep.exact_rows}/{len(rows)}, swaps {rep.swaps}")


def test_prefill_repeated_calls_and_graph(cuda_device):
    pf = workloads.make_prefill_inputs([5000], [33], seed=9, device=cuda_device)
    first = run_prefill(pf)
    out = torch.empty_like(first)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        indexer.run_prefill(pf.q_index_fp8, pf.k_index_cache_fp8, pf.weights, pf.seq_lens,
                            pf.block_table, pf.cu_seqlens_q, out)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        indexer.run_prefill(pf.q_index_fp8, pf.k_index_cache_fp8, pf.weights, pf.seq_lens,
                            pf.block_table, pf.cu_seqlens_q, out)
    torch.cuda.current_stream().wait_stream(s)
    out.fill_(7)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(first, out)


def test_prefill_bad_cu_seqlens_is_reported(cuda_device):
    pf = workloads.make_prefill_inputs([300, 300], [4, 4], seed=11, device=cuda_device)
    pf.cu_seqlens_q = torch.tensor([0, 4, 7], dtype=torch.int32, device=cuda_device)  # last != rows
    with pytest.raises(DsaError, match="seq_len"):
        run_prefill(pf)
