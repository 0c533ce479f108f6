"""CPU restatement of the indexer K-cache writer (TEST INFRASTRUCTURE ONLY).

Quantises new indexer keys into the paged FP8 cache the indexer reads.  The
page layout is the reference's (dsa_indexer/solution/triton/kernel.py:76-80,
120-124: a page holds 64 tokens x 128 float8_e4m3fn bytes, then 64 fp32
per-token scales at byte offset 64*128 + tok*4).  The reference does not
write this cache; the quantisation is the published algorithm of the vLLM
indexer cache writer, ``indexer_k_quant_and_cache`` (vllm 0.22,
vllm/v1/attention/ops/rocm_aiter_mla_sparse.py:27-87, one scale per 128-dim
key, a third-party dependency outside the reference), restated here:

* ``amax = max_d |k_d|`` over the token's 128 values (in fp32);
* ``scale = max(1e-4, amax) / 448`` in fp32;
* scale format "ue8m0": ``scale = 2^ceil(log2(scale))``, computed exactly on
  the float's bits (a mantissa of zero keeps the value, anything else goes
  to the next power of two);
* ``fp8 = e4m3fn(k / scale)``, round to nearest even;
* a negative slot is padding and writes nothing.
"""

from __future__ import annotations

import torch

PAGE_SIZE = 64
DIM = 128
PAGE_BYTES = PAGE_SIZE * DIM + PAGE_SIZE * 4  # 8448


def pow2_ceil(scale: torch.Tensor) -> torch.Tensor:
    """2^ceil(log2(s)) for positive normal fp32 values, exactly."""
    u = scale.view(torch.int32)
    up = (u & 0x7F800000) + 0x00800000
    return torch.where((u & 0x007FFFFF) == 0, u, up).view(torch.float32)


def quantize(k: torch.Tensor, ue8m0: bool = False) -> tuple:
    """k [N, 128] (any float dtype) -> (fp8 bytes uint8 [N, 128], scales fp32 [N])."""
    kf = k.float()
    amax = kf.abs().amax(dim=-1)
    scale = torch.clamp(amax, min=1e-4) / 448.0
    if ue8m0:
        scale = pow2_ceil(scale)
    q = (kf / scale[:, None]).to(torch.float8_e4m3fn)
    return q.view(torch.uint8), scale


def write_cache(k: torch.Tensor, slot_mapping: torch.Tensor, cache: torch.Tensor,
                ue8m0: bool = False) -> torch.Tensor:
    """Returns a copy of the byte cache (uint8, num_pages * 8448) with the
    tokens' quantised keys and scales written at their slots."""
    out = cache.clone().reshape(-1)
    q, scale = quantize(k, ue8m0)
    sb = scale.contiguous().view(torch.uint8).reshape(-1, 4)
    for i, slot in enumerate(slot_mapping.tolist()):
        if slot < 0:
            continue
        page, tok = divmod(int(slot), PAGE_SIZE)
        base = page * PAGE_BYTES
        out[base + tok * DIM: base + (tok + 1) * DIM] = q[i]
        out[base + PAGE_SIZE * DIM + 4 * tok: base + PAGE_SIZE * DIM + 4 * tok + 4] = sb[i]
    return out


def dequantize_slot(cache: torch.Tensor, slot: int) -> torch.Tensor:
    """fp32 [128] key stored at `slot` (fp8 * scale)."""
    page, tok = divmod(int(slot), PAGE_SIZE)
    base = page * PAGE_BYTES
    flat = cache.reshape(-1)
    q = flat[base + tok * DIM: base + (tok + 1) * DIM].view(torch.float8_e4m3fn).float()
    s = flat[base + PAGE_SIZE * DIM + 4 * tok: base + PAGE_SIZE * DIM + 4 * tok + 4].view(torch.float32)
    return q * s
