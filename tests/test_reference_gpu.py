"""Parity against the reference itself: the reference's own DSA solutions,
compiled unmodified from their sources (oracle/build_ref.py) and driven the
way their run() wrappers drive them (oracle/ref_gpu.py), on the same seeded
inputs as this library.

Indexer: rows are compared as sets of global slot ids.  A row whose set
differs from the reference's is judged with the CPU oracle's fp32 scores: a
token only one side selected must lie within the fp32 reordering bound of the
other side's boundary token (a different accumulation order may flip them);
such boundary swaps are counted.  The reference is checked against the oracle
the same way, which pins the oracle to the reference's own output.

Attention: output within atol = rtol = 1e-2 (bf16, the harness rule: an
element fails only if both are exceeded), lse within atol = rtol = 1e-3.
Rows whose indices are all -1 are left out: the reference's softmax gives NaN
there, the definition reference 0 / -inf."""

import pytest
import torch

from dsa_b200 import attention, indexer, pipeline, workloads
from oracle import compare, ref_gpu
from oracle import indexer as oix

pytestmark = pytest.mark.gpu
OUT_TOL = 1e-2
LSE_TOL = 1e-3


@pytest.fixture(scope="module")
def ref_indexer(cuda_device):
    if not ref_gpu.available():
        pytest.skip("reference solutions not built (oracle/build_ref.py needs the reference sources)")
    return ref_gpu.RefIndexer()


def ours_indexer(ix):
    out = torch.full((ix.q_index_fp8.shape[0], 2048), 7, dtype=torch.int32, device=ix.seq_lens.device)
    indexer.run(ix.q_index_fp8, ix.k_index_cache_fp8, ix.weights, ix.seq_lens, ix.block_table, out)
    torch.cuda.synchronize()
    return out.cpu()


def reference_indexer(ref, ix, calls=5):
    """Runs the reference's run() `calls` times (3 eager warm-ups, the
    capture, then replays) and checks every call gives the same output."""
    outs = []
    for _ in range(calls):
        out = torch.full((ix.q_index_fp8.shape[0], 2048), 7, dtype=torch.int32, device=ix.seq_lens.device)
        ref.run(ix.q_index_fp8, ix.k_index_cache_fp8, ix.weights, ix.seq_lens, ix.block_table, out)
        torch.cuda.synchronize()
        outs.append(out.cpu())
    for o in outs[1:]:
        assert torch.equal(o, outs[0]), "reference output changed between its eager and graph calls"
    return outs[0]


def compare_with_reference(ix, ours, theirs):
    """(rows with identical sets, boundary swaps) of `ours` against the
    reference; differing rows must pass the oracle's swap rule, and so must
    the reference's own rows against the oracle."""
    sl = ix.seq_lens.cpu()
    same, diff = 0, []
    for b in range(ours.shape[0]):
        k = min(max(int(sl[b]), 0), 2048)
        if (set(ours[b, :k].tolist()) == set(theirs[b, :k].tolist())
                and bool((ours[b, k:] == -1).all()) and bool((theirs[b, k:] == -1).all())):
            same += 1
        else:
            diff.append(b)
    swaps = 0
    if diff:
        q = ix.q_index_fp8[diff].cpu()
        kc = ix.k_index_cache_fp8.cpu()
        w, sld, bt = ix.weights[diff].cpu(), sl[diff], ix.block_table[diff].cpu()
        oref, scores = oix.indexer_reference(q, kc, w, sld, bt)
        ku = kc.view(torch.uint8).reshape(-1)
        bounds = [oix.score_error_bound(q[i], ku, w[i], int(sld[i]), bt[i].long()) for i in range(len(diff))]
        rep = compare.compare_topk(ours[diff], theirs[diff], scores, bounds, sld, bt, kc.shape[0])
        assert rep.ok, rep.problems[:5]
        swaps = rep.swaps
        rep_ref = compare.compare_topk(theirs[diff], oref, scores, bounds, sld, bt, kc.shape[0])
        assert rep_ref.ok, ("reference vs oracle", rep_ref.problems[:5])
    return same, swaps


def test_indexer_8_requests_2k_to_8k_vs_reference(cuda_device, ref_indexer):
    g = torch.Generator().manual_seed(0)
    lens = workloads.uniform_lengths(8, 2048, 8192, g)
    ix = workloads.make_indexer_inputs(lens, pool_pages=1024, seed=0, device=cuda_device)
    same, swaps = compare_with_reference(ix, ours_indexer(ix), reference_indexer(ref_indexer, ix))
    print(f"8 requests of 2048-8192 tokens vs reference: {same}/8 rows identical as sets, {swaps} boundary swaps")


def test_indexer_short_rows_vs_reference(cuda_device, ref_indexer):
    # L < 2048 (-1 padding), L == 0 (row skipped by the reference), page tails.
    lens = [100, 2048, 2049, 0, 65, 1, 4097, 63]
    ix = workloads.make_indexer_inputs(lens, pool_pages=256, seed=11, device=cuda_device)
    ours, theirs = ours_indexer(ix), reference_indexer(ref_indexer, ix)
    same, swaps = compare_with_reference(ix, ours, theirs)
    assert same == len(lens) and swaps == 0
    assert (ours[3] == -1).all() and (theirs[3] == -1).all()


def test_indexer_64_requests_32k_to_128k_vs_reference(cuda_device, ref_indexer):
    g = torch.Generator().manual_seed(2)
    lens = workloads.uniform_lengths(64, 32768, 131072, g)
    ix = workloads.make_indexer_inputs(lens, pool_pages=150000, seed=2, device=cuda_device)
    same, swaps = compare_with_reference(ix, ours_indexer(ix), reference_indexer(ref_indexer, ix, calls=4))
    print(f"64 requests of 32768-131072 tokens vs reference: {same}/64 rows identical as sets, {swaps} boundary swaps")


def _attention_pair(a):
    T = a.q_nope.shape[0]
    dev = a.q_nope.device
    out = torch.full((T, 16, 512), float("nan"), dtype=torch.bfloat16, device=dev)
    lse = torch.full((T, 16), float("nan"), dtype=torch.float32, device=dev)
    attention.run(a.q_nope, a.q_pe, a.ckv_cache, a.kpe_cache, a.sparse_indices, a.sm_scale, out, lse)
    rout, rlse = torch.empty_like(out), torch.empty_like(lse)
    ref_gpu.ref_attention_run(a.q_nope, a.q_pe, a.ckv_cache, a.kpe_cache, a.sparse_indices,
                              a.sm_scale, rout, rlse)
    torch.cuda.synchronize()
    return out.cpu(), lse.cpu(), rout.cpu(), rlse.cpu()


def test_attention_eleven_tokens_vs_reference(cuda_device, ref_indexer):
    # Eight tokens of 2048 valid indices plus tokens with 1, 100 and 2047 (the rest -1).
    a = workloads.make_attention_inputs(11, pool_pages=2048, seed=1, device=cuda_device,
                                        valid_counts=[2048] * 8 + [1, 100, 2047])
    out, lse, rout, rlse = _attention_pair(a)
    ro = compare.harness_close(out, rout, OUT_TOL, OUT_TOL)
    rl = compare.harness_close(lse, rlse, LSE_TOL, LSE_TOL)
    assert ro.ok, f"output: {ro}"
    assert rl.ok, f"lse: {rl}"
    print(f"11 tokens vs reference: output max_abs {ro.max_abs:.3g} max_rel {ro.max_rel:.3g}; "
          f"lse max_abs {rl.max_abs:.3g}")


def test_decode_step_64x65536_vs_reference(cuda_device, ref_indexer):
    """The decode step of 64 requests x 65536 tokens: the whole indexer
    output against the reference's, and attention over this library's
    selections against the reference's attention over the same selections."""
    dec = workloads.make_decode_inputs([65536] * 64, seed=1000, device=cuda_device)
    step = pipeline.DecodeStep(dec, use_graph=True)
    step()
    torch.cuda.synchronize()
    ix = dec.indexer
    ours = step.topk.cpu()
    same, swaps = compare_with_reference(ix, ours, reference_indexer(ref_indexer, ix, calls=4))
    rout = torch.empty_like(step.out)
    rlse = torch.empty_like(step.lse)
    ref_gpu.ref_attention_run(dec.q_nope, dec.q_pe, dec.ckv_cache, dec.kpe_cache, step.topk,
                              dec.sm_scale, rout, rlse)
    torch.cuda.synchronize()
    ro = compare.harness_close(step.out.cpu(), rout.cpu(), OUT_TOL, OUT_TOL)
    rl = compare.harness_close(step.lse.cpu(), rlse.cpu(), LSE_TOL, LSE_TOL)
    assert ro.ok, f"output: {ro}"
    assert rl.ok, f"lse: {rl}"
    print(f"64 x 65536 decode step vs reference: {same}/64 indexer rows identical as sets, {swaps} boundary "
          f"swaps; attention output max_abs {ro.max_abs:.3g} max_rel {ro.max_rel:.3g}, "
          f"lse max_abs {rl.max_abs:.3g}")
