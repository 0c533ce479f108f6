"""Indexer K-cache writer (quantise new keys into the 8448-byte FP8 pages):
the CPU oracle's arithmetic, the C ABI's argument checks, and on the GPU
bit-exact parity with the oracle, parity with vLLM's own writer when it can
be loaded, and a round trip through the indexer."""

import ctypes

import pytest
import torch

from dsa_b200 import _native, workloads
from oracle import cache_write as ocw
from oracle import compare
from oracle import indexer as oix


def _keys(n, seed):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(n, 128, generator=g)
    k = k * torch.exp2(torch.randint(-12, 12, (n, 1), generator=g).float())  # wide per-token range
    k[0] = 0.0  # amax 0 -> scale 1e-4 / 448
    return k.to(torch.bfloat16)


def test_oracle_scales_and_rounding():
    k = _keys(64, 1)
    q, s = ocw.quantize(k)
    amax = k.float().abs().amax(-1)
    assert torch.equal(s, torch.clamp(amax, min=1e-4) / 448.0)
    assert (q.view(torch.float8_e4m3fn).float().abs().amax(-1) <= 448).all()
    # ue8m0 scales are powers of two, the smallest not below the plain scale
    _, s2 = ocw.quantize(k, ue8m0=True)
    m, e = torch.frexp(s2)
    assert (m == 0.5).all() and (s2 >= s).all() and (s2 < 2 * s).all()
    # dequantised keys are within half an e4m3 step (3 mantissa bits) of the input
    err = (q.view(torch.float8_e4m3fn).float() * s[:, None] - k.float()).abs()
    assert (err <= s[:, None] * 448 * 2.0 ** -4 + 1e-30).all()


def test_oracle_write_skips_padding():
    k = _keys(5, 2)
    cache = torch.full((3 * ocw.PAGE_BYTES,), 0x5A, dtype=torch.uint8)
    slots = torch.tensor([0, -1, 130, 65, -7])
    out = ocw.write_cache(k, slots, cache)
    for i, sl in enumerate(slots.tolist()):
        if sl >= 0:
            assert torch.allclose(ocw.dequantize_slot(out, sl), ocw.dequantize_slot(
                ocw.write_cache(k[i:i + 1], torch.tensor([sl]), cache), sl))
    touched = torch.zeros_like(cache, dtype=torch.bool)
    for sl in (0, 130, 65):
        p, t = divmod(sl, 64)
        touched[p * 8448 + t * 128: p * 8448 + t * 128 + 128] = True
        touched[p * 8448 + 8192 + 4 * t: p * 8448 + 8192 + 4 * t + 4] = True
    assert (out[~touched] == 0x5A).all()


def test_c_abi_rejects_bad_arguments():
    lib = _native.lib()
    P = ctypes.c_void_p
    assert lib.dsa_index_cache_write(P(16), P(16), -1, P(16), 1, 0, None, None) == 1
    assert lib.dsa_index_cache_write(P(16), P(16), 0, P(16), 1, 0, None, None) == 0
    assert lib.dsa_index_cache_write(None, P(16), 4, P(16), 1, 0, None, None) == 1
    assert lib.dsa_index_cache_write(P(16), P(16), 4, P(8), 1, 0, None, None) == 2  # cache not 16-B aligned


def _gpu_case(device, n, pages, seed, pad_every=7):
    k = _keys(n, seed)
    g = torch.Generator().manual_seed(seed + 100)
    slots = torch.randperm(pages * 64, generator=g)[:n].to(torch.int64)
    slots[::pad_every] = -1
    cache = torch.randint(0, 256, (pages * ocw.PAGE_BYTES,), generator=g, dtype=torch.uint8)
    return k, slots, cache


@pytest.mark.gpu
@pytest.mark.parametrize("ue8m0", [False, True])
def test_gpu_matches_oracle_bit_exact(cuda_device, ue8m0):
    from dsa_b200 import cache as kc

    for n, pages, seed in ((1, 2, 3), (300, 16, 4), (4096, 100, 5)):
        k, slots, cache = _gpu_case(cuda_device, n, pages, seed)
        want = ocw.write_cache(k, slots, cache, ue8m0)
        got = cache.to(cuda_device)
        kc.write_index_k(k.to(cuda_device), slots.to(cuda_device), got, ue8m0=ue8m0)
        torch.cuda.synchronize()
        assert torch.equal(got.cpu(), want), (n, ue8m0)


@pytest.mark.gpu
@pytest.mark.parametrize("ue8m0", [False, True])
def test_gpu_quotients_match_ieee_division(cuda_device, ue8m0):
    """The kernel forms k / scale with a reciprocal and an FMA correction;
    every byte must equal IEEE division followed by the e4m3 conversion (the
    oracle's quantize on the CPU: on the GPU torch divides by a Python scalar
    as a multiplication by its reciprocal, which is not IEEE division), over
    half a million tokens whose rows span 40 decades and whose values span 6
    decades in a row."""
    from dsa_b200 import cache as kc

    n = 1 << 19
    g = torch.Generator(device=cuda_device).manual_seed(11)
    rows = torch.pow(10.0, torch.empty(n, 1, device=cuda_device).uniform_(-20, 20, generator=g))
    spread = torch.pow(10.0, torch.empty(n, 128, device=cuda_device).uniform_(-6, 0, generator=g))
    k = (torch.randn(n, 128, generator=g, device=cuda_device) * rows * spread).to(torch.bfloat16)
    cache = torch.zeros(n // 64 * ocw.PAGE_BYTES, dtype=torch.uint8, device=cuda_device)
    kc.write_index_k(k, torch.arange(n, device=cuda_device), cache, ue8m0=ue8m0)
    q, scale = ocw.quantize(k.cpu(), ue8m0)
    want = torch.cat([q.reshape(n // 64, 64 * 128),
                      scale.contiguous().view(torch.uint8).reshape(n // 64, 64 * 4)], dim=1).reshape(-1)
    bad = (cache.cpu() != want).nonzero()
    assert bad.numel() == 0, f"{bad.numel()} bytes differ, first at {bad[:4].flatten().tolist()}"


@pytest.mark.gpu
def test_gpu_out_of_range_slot_is_reported_not_written(cuda_device):
    lib = _native.lib()
    k = _keys(3, 6).to(cuda_device)
    cache = torch.zeros(2 * ocw.PAGE_BYTES, dtype=torch.uint8, device=cuda_device)
    slots = torch.tensor([5, 128, 200], dtype=torch.int64, device=cuda_device)  # 2 pages = 128 slots
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    st = lib.dsa_index_cache_write(P(k), P(slots), 3, P(cache), 2, 0, P(status),
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    assert int(status.item()) & _native.DEV_BAD_INDEX
    want = ocw.write_cache(k[:1].cpu(), slots[:1].cpu(), torch.zeros(2 * ocw.PAGE_BYTES, dtype=torch.uint8))
    assert torch.equal(cache.cpu(), want)


def _vllm_writer():
    try:
        import vllm._custom_ops as ops  # noqa: F401  (loads vLLM's compiled ops)
        return torch.ops._C_cache_ops.indexer_k_quant_and_cache
    except Exception:
        return None


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["", "ue8m0"])
def test_gpu_matches_vllm_writer(cuda_device, fmt):
    op = _vllm_writer()
    if op is None:
        pytest.skip("vLLM's compiled cache ops cannot be loaded here")
    from dsa_b200 import cache as kc

    k, slots, cache = _gpu_case(cuda_device, 2000, 64, 7, pad_every=11)
    theirs = cache.to(cuda_device).view(64, 64, 132)
    try:
        op(k.to(cuda_device), theirs, slots.to(cuda_device), 128, fmt)
    except Exception as ex:  # signature differs in this vLLM build
        pytest.skip(f"vLLM writer call failed: {ex}")
    ours = cache.to(cuda_device)
    kc.write_index_k(k.to(cuda_device), slots.to(cuda_device), ours, ue8m0=(fmt == "ue8m0"))
    torch.cuda.synchronize()
    assert torch.equal(ours.cpu(), theirs.reshape(-1).cpu())


@pytest.mark.gpu
def test_gpu_written_cache_feeds_the_indexer(cuda_device):
    from dsa_b200 import cache as kc
    from dsa_b200 import indexer

    lens = [3000, 700, 2100]
    ix = workloads.make_indexer_inputs(lens, pool_pages=120, seed=8, device=cuda_device)
    g = torch.Generator().manual_seed(9)
    n = sum(lens)
    k = (torch.randn(n, 128, generator=g) * 0.5).to(torch.bfloat16)
    # Disjoint pages per request, so every slot is written exactly once.
    perm = torch.randperm(120, generator=g)
    bt = torch.full_like(ix.block_table.cpu().long(), -1)
    used = 0
    for b, L in enumerate(lens):
        npg = (L + 63) // 64
        bt[b, :npg] = perm[used:used + npg]
        used += npg
    ix.block_table = bt.to(torch.int32).to(cuda_device)
    slots = torch.cat([bt[b, torch.arange(L) // 64] * 64 + torch.arange(L) % 64 for b, L in enumerate(lens)])
    cache = ix.k_index_cache_fp8.view(torch.uint8).reshape(-1)
    before = cache.cpu().clone()
    kc.write_index_k(k.to(cuda_device), slots.to(cuda_device), cache)
    out = torch.full((3, 2048), 7, dtype=torch.int32, device=cuda_device)
    indexer.run(ix.q_index_fp8, ix.k_index_cache_fp8, ix.weights, ix.seq_lens, ix.block_table, out)
    torch.cuda.synchronize()
    ref, scores = oix.indexer_reference(ix.q_index_fp8.cpu(), ix.k_index_cache_fp8.cpu(), ix.weights.cpu(),
                                        ix.seq_lens.cpu(), ix.block_table.cpu())
    ku = ix.k_index_cache_fp8.cpu().view(torch.uint8).reshape(-1)
    bounds = [oix.score_error_bound(ix.q_index_fp8[b].cpu(), ku, ix.weights[b].cpu(), lens[b], bt[b])
              for b in range(3)]
    rep = compare.compare_topk(out.cpu(), ref, scores, bounds, ix.seq_lens.cpu(), ix.block_table.cpu(),
                               ix.k_index_cache_fp8.shape[0])
    assert rep.ok, rep.problems[:5]
    # and the cache holds exactly what the oracle writes
    want = ocw.write_cache(k, slots, before)
    assert torch.equal(cache.cpu(), want)
