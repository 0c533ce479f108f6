"""The captured decode step (dsa_b200.pipeline.DecodeStep): one stream against
two streams inside one CUDA graph (the batch split in halves, indexer ->
attention of one half on a side stream, joined by events), the way the
reference forks its indexer over pooled streams inside its captured graph
(dsa_indexer/solution/triton/kernel.py:233-241, 270-273, 315-318).

The indexer's result does not depend on how the batch is split.  Attention
splits each call's tiles over the SMs, so a half-batch call merges partial
softmax sums at other points than the whole-batch call: the two-stream step
must equal, bit for bit, eager calls on the same halves, and the one-stream
step within the output tolerance (atol = rtol = 1e-2, lse 1e-3)."""

import pytest
import torch

from dsa_b200 import attention, indexer, pipeline, workloads
from oracle import compare

pytestmark = pytest.mark.gpu


def test_two_stream_graph_matches_one_stream(cuda_device):
    lens = [5000, 70000, 2049, 129, 40000, 3000, 0, 65536]
    dec = workloads.make_decode_inputs(lens, seed=71, device=cuda_device)
    one = pipeline.DecodeStep(dec, use_graph=True, streams=1)
    two = pipeline.DecodeStep(dec, use_graph=True, streams=2)
    for _ in range(2):  # replays of the same graphs give the same results
        one()
        two()
        torch.cuda.synchronize()
        assert torch.equal(one.topk, two.topk)
        ro = compare.harness_close(two.out, one.out, 1e-2, 1e-2)
        rl = compare.harness_close(two.lse, one.lse, 1e-3, 1e-3)
        assert ro.ok and rl.ok, (ro, rl)

    ix = dec.indexer
    for lo, hi in two.parts:
        topk = torch.full((hi - lo, 2048), 7, dtype=torch.int32, device=cuda_device)
        indexer.run(ix.q_index_fp8[lo:hi], ix.k_index_cache_fp8, ix.weights[lo:hi], ix.seq_lens[lo:hi],
                    ix.block_table[lo:hi], topk)
        out = torch.empty(hi - lo, 16, 512, dtype=torch.bfloat16, device=cuda_device)
        lse = torch.empty(hi - lo, 16, dtype=torch.float32, device=cuda_device)
        attention.run(dec.q_nope[lo:hi], dec.q_pe[lo:hi], dec.ckv_cache, dec.kpe_cache, topk, dec.sm_scale,
                      out, lse)
        torch.cuda.synchronize()
        assert torch.equal(topk, two.topk[lo:hi])
        assert torch.equal(out, two.out[lo:hi]) and torch.equal(lse, two.lse[lo:hi])


def test_host_io_graph_matches_the_device_step(cuda_device):
    """DecodeStep(host_io=True): one graph copies the pinned inputs in, runs the
    step and copies the outputs back; results equal the device-resident step's
    bit for bit, and inputs rewritten on the host reach the next replay."""
    lens = [5000, 70000, 2049, 129, 0, 3000]
    dec = workloads.make_decode_inputs(lens, seed=72, device=cuda_device)
    ref = pipeline.DecodeStep(dec, use_graph=True)
    io = pipeline.DecodeStep(dec, use_graph=True, host_io=True)
    for new_len in (None, 4000):
        if new_len is not None:
            io.host_in[2][0] = new_len          # seq_lens, written on the host
            dec.indexer.seq_lens[0] = new_len   # the same change for the device step
        ref()
        io.replay_io()
        torch.cuda.synchronize()
        topk, out, lse = io.host_out
        assert torch.equal(topk, ref.topk.cpu())
        assert torch.equal(out, ref.out.cpu()) and torch.equal(lse, ref.lse.cpu())
    assert int((io.host_out[0][0] >= 0).sum()) == 2048
