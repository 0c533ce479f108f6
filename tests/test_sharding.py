"""Host-side logic of the multi-GPU path, on CPU: request sharding, and the
step statistics and per-rank results gathered across ranks, run as two gloo
processes (the GPU runs use NCCL with the same calls).  Decode requests are
independent, so a sharded run must give each request exactly the result of a
single-process run."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsa_b200 import sharding, workloads
from oracle import attention as oatt
from oracle import indexer as oix
from oracle import parity


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_every_request_on_exactly_one_rank(world):
    g = torch.Generator().manual_seed(world)
    lens = [0, 7] + workloads.log_uniform_lengths(61, 64, 131072, g)
    shards = sharding.shard_requests(lens, world)
    assert len(shards) == world
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(len(lens)))
    for s in shards:
        assert s == sorted(s)  # original order kept inside a rank


def test_lpt_balance_and_imbalance_metric():
    g = torch.Generator().manual_seed(5)
    lens = workloads.log_uniform_lengths(512, 4096, 131072, g)
    for world in (2, 4, 8):
        shards = sharding.shard_requests(lens, world)
        loads = [sum(lens[i] for i in s) for s in shards]
        # Longest-first greedy: no rank exceeds another by more than one request.
        assert max(loads) - min(loads) <= max(lens)
        assert 1.0 <= sharding.shard_imbalance(lens, shards) < 1.05
    assert sharding.shard_requests([], 4) == [[], [], [], []]
    with pytest.raises(ValueError):
        sharding.shard_requests([1], 0)


def test_single_rank_stats_pass_through():
    assert sharding.reduce_step_stats(2.5, 10.0, 3.0, 1) == (2.5, 10.0, 3.0)


LENS = [100, 3000, 2049, 64, 5000, 0, 129]


def _problem():
    return workloads.make_indexer_inputs(LENS, pool_pages=260, seed=77, device=torch.device("cpu"))


def _decode_problem(rank):
    # shards of different sizes: rank r holds 2 + r requests
    lens = [300 + 500 * i for i in range(2 + rank)]
    return workloads.make_decode_inputs(lens, seed=50 + rank, device=torch.device("cpu"))


def _rank_main(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ix = _problem()
        mine = sharding.shard_requests(LENS, world)[rank]
        idx = torch.tensor(mine, dtype=torch.long)
        topk, _ = oix.indexer_reference(ix.q_index_fp8[idx], ix.k_index_cache_fp8, ix.weights[idx],
                                        ix.seq_lens[idx], ix.block_table[idx])
        # Step statistics: time is the max over ranks, bytes and requests sum.
        ms, nbytes, nreq = sharding.reduce_step_stats(1.0 + rank, 100.0 * (rank + 1), float(len(mine)), world)
        gathered = [None] * world
        dist.all_gather_object(gathered, (mine, topk.tolist()))
        # The verification flag every rank contributes (bench.py's verify()).
        flag = torch.tensor([1], dtype=torch.int32)
        flags = [torch.zeros_like(flag) for _ in range(world)]
        dist.all_gather(flags, flag)
        # bench.py's verify(): every rank's (indices, output, lse) gathered to
        # rank 0 (shards of different sizes), plus the sampled rows' oracle
        # bundles; rank 0 checks the gathered outputs against the oracle.
        # Here the "outputs" are the oracle's own, computed per rank.
        dec = _decode_problem(rank)
        d_topk, _ = oix.indexer_reference(dec.indexer.q_index_fp8, dec.indexer.k_index_cache_fp8,
                                          dec.indexer.weights, dec.indexer.seq_lens,
                                          dec.indexer.block_table)
        d_out, d_lse = oatt.attention_reference(dec.q_nope, dec.q_pe, dec.ckv_cache, dec.kpe_cache,
                                                d_topk, dec.sm_scale)
        outs = sharding.gather_outputs([d_topk, d_out, d_lse], world)
        B = d_topk.shape[0]
        bundles = [None] * world
        dist.all_gather_object(bundles, parity.pack_rows(dec, d_topk, [0, B - 1], rank))
        if rank == 0:
            rep = parity.check_bundles([b for bs in bundles for b in bs], outs)
            torch.save({"stats": (ms, nbytes, nreq), "gathered": gathered,
                        "flags": [int(f.item()) for f in flags],
                        "out_rows": [o[0].shape[0] for o in outs], "parity": rep},
                       os.path.join(out_dir, "r0.pt"))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_match_a_single_process(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    r = torch.load(tmp_path / "r0.pt")
    assert r["stats"] == (2.0, 300.0, float(len(LENS)))
    assert r["flags"] == [1, 1]
    assert r["out_rows"] == [2, 3]
    rep = r["parity"]
    assert rep["ok"], rep["problems"]
    assert rep["rows"] == 4 and rep["exact_rows"] == 4 and rep["tokens"] == 4
    ix = _problem()
    full, _ = oix.indexer_reference(ix.q_index_fp8, ix.k_index_cache_fp8, ix.weights,
                                    ix.seq_lens, ix.block_table)
    seen = set()
    for mine, rows in r["gathered"]:
        for i, row in zip(mine, rows):
            assert row == full[i].tolist(), i
            seen.add(i)
    assert seen == set(range(len(LENS)))
