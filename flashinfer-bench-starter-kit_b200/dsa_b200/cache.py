"""Writer of the indexer's paged FP8 K cache (destination-passing style).

    write_index_k(k, slot_mapping, k_index_cache_fp8, ue8m0=False) -> None

The step before the indexer in a serving loop: each new token's 128-dim
indexer key is quantised to float8_e4m3fn with one fp32 scale per token
(scale = max(1e-4, max|k|)/448, or its power-of-two ceiling with
``ue8m0=True``) and stored at its slot of the 8448-byte pages that
``dsa_b200.indexer.run`` reads.  Negative slots are padding and skipped; a
slot beyond the cache is reported (``DSA_B200_CHECK=1``) and not written.
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _native

DIM = 128
PAGE_SIZE = 64
PAGE_BYTES = PAGE_SIZE * DIM + PAGE_SIZE * 4

_CHECK = os.environ.get("DSA_B200_CHECK", "0") not in ("", "0")


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(f"dsa_index_cache_write: {msg}")


@torch.no_grad()
def write_index_k(k: torch.Tensor, slot_mapping: torch.Tensor, k_index_cache_fp8: torch.Tensor,
                  ue8m0: bool = False) -> None:
    dev = k.device
    _require(dev.type == "cuda", "tensors must be on a CUDA device")
    _require(slot_mapping.device == dev and k_index_cache_fp8.device == dev,
             "k, slot_mapping and the cache must share a device")
    _require(k.dtype == torch.bfloat16 and k.dim() == 2 and k.shape[1] == DIM,
             f"k must be bf16 [N, {DIM}], got {k.dtype} {tuple(k.shape)}")
    _require(slot_mapping.dim() == 1 and slot_mapping.shape[0] == k.shape[0],
             "slot_mapping must be [N]")
    _require(k_index_cache_fp8.element_size() == 1 and k_index_cache_fp8.is_contiguous(),
             "the cache must be a contiguous 1-byte tensor (written in place)")
    nbytes = k_index_cache_fp8.numel()
    _require(nbytes % PAGE_BYTES == 0, f"the cache holds {nbytes} bytes, not pages of {PAGE_BYTES}")
    n = k.shape[0]
    if n == 0:
        return
    kk = k.contiguous()
    sm = slot_mapping.to(torch.int64).contiguous()
    status = torch.zeros(1, dtype=torch.int32, device=dev) if _CHECK else None
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    with torch.cuda.device(dev):
        st = _native.lib().dsa_index_cache_write(
            _ptr(kk), _ptr(sm), n, _ptr(k_index_cache_fp8), nbytes // PAGE_BYTES, int(bool(ue8m0)),
            _ptr(status) if status is not None else None, stream)
    _native.check(st, "dsa_index_cache_write")
    if status is not None and not torch.cuda.is_current_stream_capturing():
        bits = int(status.item())
        if bits:
            raise _native.DsaError(f"dsa_index_cache_write: {_native.describe_device_status(bits)}")
