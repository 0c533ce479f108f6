"""GPU parity of sparse MLA attention (dsa_b200.attention.run -> C ABI ->
sm_100a kernels) against the CPU oracle and the golden fixture.

Tolerances: output within atol = rtol = 1e-2 (bf16, harness rule: an element
fails only if both are exceeded); lse within atol = rtol = 1e-3."""

import pathlib

import numpy as np
import pytest
import torch

from dsa_b200 import DsaError, attention, workloads
from dsa_b200 import workspace as ws_mod
from oracle import attention as oatt
from oracle import compare

pytestmark = pytest.mark.gpu
GOLD = pathlib.Path(__file__).resolve().parent / "golden"
OUT_TOL = 1e-2
LSE_TOL = 1e-3


def run_gpu(a):
    T = a.q_nope.shape[0]
    dev = a.q_nope.device
    out = torch.full((T, 16, 512), float("nan"), dtype=torch.bfloat16, device=dev)
    lse = torch.full((T, 16), float("nan"), dtype=torch.float32, device=dev)
    attention.run(a.q_nope, a.q_pe, a.ckv_cache, a.kpe_cache, a.sparse_indices, a.sm_scale, out, lse)
    torch.cuda.synchronize()
    return out, lse


def check(a, out, lse, tokens=None):
    tokens = list(range(a.q_nope.shape[0])) if tokens is None else tokens
    ref_out, ref_lse = oatt.attention_reference(
        a.q_nope[tokens].cpu(), a.q_pe[tokens].cpu(), a.ckv_cache.cpu(), a.kpe_cache.cpu(),
        a.sparse_indices[tokens].cpu(), a.sm_scale)
    ro = compare.harness_close(out[tokens].cpu(), ref_out, OUT_TOL, OUT_TOL)
    rl = compare.harness_close(lse[tokens].cpu(), ref_lse, LSE_TOL, LSE_TOL)
    assert ro.ok, f"output: {ro}"
    assert rl.ok, f"lse: {rl}"
    return ro, rl


@pytest.mark.parametrize("T", [1, 2, 3, 8])
def test_small_batches(cuda_device, T):
    a = workloads.make_attention_inputs(T, pool_pages=max(256, 32 * T), seed=T,
                                        device=cuda_device)
    out, lse = run_gpu(a)
    ro, rl = check(a, out, lse)
    print(f"T={T}: out max_abs {ro.max_abs:.3g}, lse max_abs {rl.max_abs:.3g}")


def test_eight_tokens(cuda_device):
    a = workloads.make_attention_inputs(8, pool_pages=2048, seed=1, device=cuda_device)
    out, lse = run_gpu(a)
    check(a, out, lse)


def test_golden_fixture(cuda_device):
    z = np.load(GOLD / "attention_small.npz")
    d = cuda_device
    a = workloads.AttentionInputs(
        torch.from_numpy(z["q_nope"]).view(torch.bfloat16).to(d),
        torch.from_numpy(z["q_pe"]).view(torch.bfloat16).to(d),
        torch.from_numpy(z["ckv"]).view(torch.bfloat16).to(d),
        torch.from_numpy(z["kpe"]).view(torch.bfloat16).to(d),
        torch.from_numpy(z["indices"]).to(d), float(z["sm_scale"]))
    out, lse = run_gpu(a)
    gold_out = torch.from_numpy(z["output"]).view(torch.bfloat16)
    gold_lse = torch.from_numpy(z["lse"])
    assert compare.harness_close(out.cpu(), gold_out, OUT_TOL, OUT_TOL).ok
    assert compare.harness_close(lse.cpu(), gold_lse, LSE_TOL, LSE_TOL).ok
    assert torch.isinf(lse[2]).all() and (out[2] == 0).all()


def test_padding_patterns(cuda_device):
    T = 6
    a = workloads.make_attention_inputs(T, pool_pages=512, seed=7, device=cuda_device)
    idx = a.sparse_indices.clone()
    idx[0, :] = -1                 # nothing valid
    idx[1, 1024:] = -1             # valid prefix
    idx[2, :1024] = -1             # valid suffix
    idx[3, ::2] = -1               # every other entry
    idx[4, :2047] = -1             # a single valid entry
    a.sparse_indices = idx
    out, lse = run_gpu(a)
    check(a, out, lse)
    assert torch.isinf(lse[0]).all() and (out[0] == 0).all()


def test_duplicate_indices(cuda_device):
    a = workloads.make_attention_inputs(2, pool_pages=4, seed=13, device=cuda_device,
                                        len_range=(256, 256))
    a.sparse_indices = torch.randint(0, 256, (2, 2048), dtype=torch.int32, device=cuda_device)
    out, lse = run_gpu(a)
    check(a, out, lse)


@pytest.mark.parametrize("T", [64, 300])
def test_many_tokens(cuda_device, T):
    # T=64 splits every token across CTAs; T=300 also has tokens that one CTA
    # covers entirely (written without the combine pass).
    a = workloads.make_attention_inputs(T, pool_pages=4096, seed=100 + T, device=cuda_device)
    out, lse = run_gpu(a)
    check(a, out, lse, tokens=list(range(0, T, max(1, T // 24))) + [T - 1])


@pytest.mark.parametrize("T", [512, 1500])
def test_many_segments_per_cta(cuda_device, T):
    # 148 CTAs over T*32 tiles give every CTA 4+ token segments, so both
    # Q slots are refilled at least twice; the teardown drains only the last
    # load of each slot (an older one's phase parity would read as pending
    # and the drain would run out, raising the wait-timeout status bit).
    import time
    a = workloads.make_attention_inputs(T, pool_pages=4096, seed=200 + T, device=cuda_device)
    run_gpu(a)
    t0 = time.perf_counter()
    out, lse = run_gpu(a)
    dt = time.perf_counter() - t0
    check(a, out, lse, tokens=list(range(0, T, max(1, T // 24))) + [T - 1])
    assert dt < 0.05, f"{T} tokens took {dt * 1e3:.1f} ms"


def test_merge_counters_are_left_zero_and_stale_ones_reported(cuda_device):
    # 64 tokens over the SM count: every token is split and merged.  Each
    # call leaves its merge counters (arrival tickets and publications, at
    # the end of the workspace) at zero; an arrival counter planted non-zero
    # is reported, by this call and the next, instead of silently pairing
    # parts of different calls.
    T = 64
    a = workloads.make_attention_inputs(T, pool_pages=2048, seed=43, device=cuda_device)
    out, lse = run_gpu(a)
    check(a, out, lse, tokens=[0, 31, 63])
    dev = torch.device(cuda_device)
    buf = ws_mod.get(dev, "attention", 0, torch.cuda.current_stream(dev).cuda_stream)
    W = buf.numel()
    off = (W - 8 * T) & ~3
    assert int(buf[off:off + 8 * T].view(torch.int32).abs().sum()) == 0
    arrive0 = off + 4 * T
    buf[arrive0:arrive0 + 4].view(torch.int32).fill_(1000)
    try:
        for _ in range(2):
            with pytest.raises(DsaError, match="merge counter"):
                run_gpu(a)
    finally:
        buf.zero_()
    out, lse = run_gpu(a)
    check(a, out, lse, tokens=[0, 31, 63])


@pytest.mark.parametrize("T", [64, 5])
def test_wait_timeout_is_reported_and_the_next_call_is_exact(cuda_device, T):
    # The failure path, made to happen without faulting anything: a test hook
    # makes every CTA's producers skip their second tile (no copy is issued,
    # no barrier arrival made) and shortens every bounded wait to 1 ms.  The
    # MMA issuers' wait for that tile runs out, the CTA aborts, drains and
    # frees its tensor memory, and settles the merge counters of the tokens
    # it still owed.  The call must return with DSA_DEV_WAIT_TIMEOUT set, and
    # the next call on the same workspace must be exact.  T = 5 gives tokens
    # of many parts (merged from records at the end of a CTA); T = 64 tokens
    # of 3-4 parts (merged by the last one as its segment ends).
    from dsa_b200 import _native
    a = workloads.make_attention_inputs(T, pool_pages=2048, seed=600 + T, device=cuda_device)
    good_out, good_lse = run_gpu(a)
    check(a, good_out, good_lse, tokens=[0, T // 2, T - 1])
    dev = torch.device(cuda_device)
    buf = ws_mod.get(dev, "attention", 0, torch.cuda.current_stream(dev).cuda_stream)
    lib = _native.lib()
    assert lib.dsa_b200_test_inject(_native.TEST_SKIP_ARRIVAL, 1_000_000) == 0
    try:
        with pytest.raises(DsaError, match="timed out"):
            run_gpu(a)
    finally:
        lib.dsa_b200_test_inject(_native.TEST_NONE, 0)
    W = buf.numel()
    off = (W - 8 * T) & ~3
    assert int(buf[off:off + 8 * T].view(torch.int32).abs().sum()) == 0, "merge counters left set"
    out, lse = run_gpu(a)
    assert torch.equal(out, good_out) and torch.equal(lse, good_lse)


def test_large_logits_rescale(cuda_device):
    # Scaled logits spanning many units of log2 force the lazy rescale path.
    a = workloads.make_attention_inputs(4, pool_pages=512, seed=17, device=cuda_device)
    a.q_nope.mul_(8.0)
    a.ckv_cache[::3].mul_(4.0)
    out, lse = run_gpu(a)
    check(a, out, lse)


def test_bad_index_is_reported(cuda_device):
    a = workloads.make_attention_inputs(2, pool_pages=64, seed=19, device=cuda_device)
    a.sparse_indices[1, 5] = 64 * 64 + 3
    with pytest.raises(DsaError, match="sparse index"):
        run_gpu(a)


def test_graph_capture(cuda_device):
    a = workloads.make_attention_inputs(8, pool_pages=512, seed=23, device=cuda_device)
    out, lse = run_gpu(a)
    out2 = torch.empty_like(out)
    lse2 = torch.empty_like(lse)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up on the capture stream sizes its workspace
        attention.run(a.q_nope, a.q_pe, a.ckv_cache, a.kpe_cache, a.sparse_indices, a.sm_scale,
                      out2, lse2)
    torch.cuda.synchronize()
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        attention.run(a.q_nope, a.q_pe, a.ckv_cache, a.kpe_cache, a.sparse_indices, a.sm_scale,
                      out2, lse2)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, out2) and torch.equal(lse, lse2)


def test_workspace_reuse_across_sizes(cuda_device):
    # One stream, one workspace, token counts that move the merge counters
    # onto bytes a previous call used for partial records.
    for T, seed in ((64, 31), (3, 32), (20, 33), (1, 34), (64, 35)):
        a = workloads.make_attention_inputs(T, pool_pages=2048, seed=seed, device=cuda_device)
        out, lse = run_gpu(a)
        check(a, out, lse, tokens=list(range(0, T, max(1, T // 6))) + [T - 1])
