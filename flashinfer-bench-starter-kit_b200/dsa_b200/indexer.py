"""DSA top-k indexer operator (destination-passing style).

``run`` keeps the reference entry point's signature, argument meaning and
in-place output (dsa_indexer/solution/triton/kernel.py:364-436):

    run(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table,
        topk_indices) -> None

Differences that are deliberate:

* ``seq_lens`` is never copied to the host (the reference calls
  ``seq_lens.cpu()`` every call, kernel.py:375, which blocks and keys a graph
  cache on the values); every launch here is asynchronous on the current
  stream and can be captured into a caller's CUDA graph.
* The order of equal scores is defined: lower token index first.
* Bad page ids / lengths do not read out of bounds; they set a sticky status
  bit (``device_status``) -- with ``DSA_B200_CHECK=1`` each call synchronises
  and raises on such bits.
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _native, workspace

PAGE_SIZE = 64
NUM_HEADS = 64
HEAD_DIM = 128
TOPK = 2048
PAGE_BYTES = PAGE_SIZE * HEAD_DIM + PAGE_SIZE * 4  # 8448

_CHECK = os.environ.get("DSA_B200_CHECK", "0") not in ("", "0")
_ws_bytes: dict = {}  # (batch, max_pages) -> dsa_indexer_workspace_bytes


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(f"dsa_indexer.run: {msg}")


def num_pages_of(k_index_cache_fp8: torch.Tensor) -> int:
    nbytes = k_index_cache_fp8.numel() * k_index_cache_fp8.element_size()
    if k_index_cache_fp8.element_size() != 1:
        _fail(f"k_index_cache_fp8 must have a 1-byte dtype, got {k_index_cache_fp8.dtype}")
    if nbytes % PAGE_BYTES != 0 or nbytes <= 0:
        _fail(f"k_index_cache_fp8 holds {nbytes} bytes, not a positive multiple of {PAGE_BYTES}")
    return nbytes // PAGE_BYTES


def _fail(msg: str) -> None:
    raise ValueError(f"dsa_indexer.run: {msg}")


# No torch.no_grad() wrapper on the entry points: they write through raw
# pointers and build no autograd graph, and the decorator alone costs ~3 us
# of host time per call.
def run(q_index_fp8: torch.Tensor, k_index_cache_fp8: torch.Tensor, weights: torch.Tensor,
        seq_lens: torch.Tensor, block_table: torch.Tensor, topk_indices: torch.Tensor) -> None:
    # Every message is formatted only on failure: this runs once per decode step.
    dev = q_index_fp8.device
    if dev.type != "cuda":
        _fail("tensors must be on a CUDA device")
    for name, t in (("k_index_cache_fp8", k_index_cache_fp8), ("weights", weights),
                    ("seq_lens", seq_lens), ("block_table", block_table),
                    ("topk_indices", topk_indices)):
        if t.device != dev:
            _fail(f"{name} is on {t.device}, expected {dev}")
    if q_index_fp8.dtype != torch.float8_e4m3fn:
        _fail(f"q_index_fp8 must be float8_e4m3fn, got {q_index_fp8.dtype}")
    if q_index_fp8.dim() != 3 or q_index_fp8.shape[1:] != (NUM_HEADS, HEAD_DIM):
        _fail(f"q_index_fp8 must be [B, {NUM_HEADS}, {HEAD_DIM}], got {tuple(q_index_fp8.shape)}")
    B = q_index_fp8.shape[0]
    if weights.dtype != torch.float32 or weights.shape != (B, NUM_HEADS):
        _fail(f"weights must be float32 [{B}, {NUM_HEADS}]")
    if seq_lens.dtype != torch.int32 or seq_lens.shape != (B,):
        _fail(f"seq_lens must be int32 [{B}]")
    if block_table.dim() != 2 or block_table.shape[0] != B or block_table.shape[1] < 1:
        _fail(f"block_table must be [{B}, max_pages]")
    if block_table.dtype != torch.int32 and block_table.dtype != torch.int64:
        _fail("block_table must be int32 or int64")
    if topk_indices.dtype != torch.int32 or topk_indices.shape != (B, TOPK):
        _fail(f"topk_indices must be int32 [{B}, {TOPK}]")
    if not topk_indices.is_contiguous():
        _fail("topk_indices must be contiguous (written in place)")
    num_pages = num_pages_of(k_index_cache_fp8)
    if B == 0:
        return
    q = q_index_fp8.contiguous()
    k = k_index_cache_fp8.contiguous()
    w = weights.contiguous()
    sl = seq_lens.contiguous()
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    bt = bt.contiguous()
    max_pages = bt.shape[1]

    L = _native.lib()
    nbytes = _ws_bytes.get((B, max_pages))
    if nbytes is None:
        nbytes = _ws_bytes[(B, max_pages)] = L.dsa_indexer_workspace_bytes(B, max_pages)
    cur = _native.current_stream(dev)
    ws = workspace.get(dev, "indexer", nbytes, cur)
    st = _native.call_on(dev, L.dsa_indexer_run, q.data_ptr(), k.data_ptr(), num_pages, w.data_ptr(),
                         sl.data_ptr(), bt.data_ptr(), B, max_pages, topk_indices.data_ptr(),
                         ws.data_ptr(), ws.numel(), cur)
    _native.check(st, "dsa_indexer_run")
    if _CHECK and not torch.cuda.is_current_stream_capturing():
        raise_on_device_status(dev)


def run_prefill(q_index_fp8: torch.Tensor, k_index_cache_fp8: torch.Tensor, weights: torch.Tensor,
                seq_lens: torch.Tensor, block_table: torch.Tensor, cu_seqlens_q: torch.Tensor,
                topk_indices: torch.Tensor) -> None:
    """Indexer for many query rows per request (prefill / chunked prefill).

    Row t of request r (rows ``cu_seqlens_q[r] .. cu_seqlens_q[r+1]-1``) is
    the decode problem ``run`` solves for ``(q[t], weights[t], seq_lens[t],
    block_table[r])``; causal rows of a chunk pass growing ``seq_lens``.  The
    rows of a request are scored four at a time as one FP8 GEMM, so each K
    tile is read once per four rows instead of once per row.
    """
    dev = q_index_fp8.device
    _require(dev.type == "cuda", "tensors must be on a CUDA device")
    for name, t in (("k_index_cache_fp8", k_index_cache_fp8), ("weights", weights),
                    ("seq_lens", seq_lens), ("block_table", block_table),
                    ("cu_seqlens_q", cu_seqlens_q), ("topk_indices", topk_indices)):
        _require(t.device == dev, f"{name} is on {t.device}, expected {dev}")
    _require(q_index_fp8.dtype == torch.float8_e4m3fn,
             f"q_index_fp8 must be float8_e4m3fn, got {q_index_fp8.dtype}")
    _require(q_index_fp8.dim() == 3 and tuple(q_index_fp8.shape[1:]) == (NUM_HEADS, HEAD_DIM),
             f"q_index_fp8 must be [T, {NUM_HEADS}, {HEAD_DIM}], got {tuple(q_index_fp8.shape)}")
    T = q_index_fp8.shape[0]
    _require(weights.dtype == torch.float32 and tuple(weights.shape) == (T, NUM_HEADS),
             f"weights must be float32 [{T}, {NUM_HEADS}]")
    _require(seq_lens.dtype == torch.int32 and tuple(seq_lens.shape) == (T,),
             f"seq_lens must be int32 [{T}]")
    _require(block_table.dim() == 2 and block_table.shape[1] >= 1, "block_table must be [R, max_pages]")
    _require(block_table.dtype in (torch.int32, torch.int64), "block_table must be int32 or int64")
    R = block_table.shape[0]
    _require(cu_seqlens_q.dtype in (torch.int32, torch.int64) and tuple(cu_seqlens_q.shape) == (R + 1,),
             f"cu_seqlens_q must be int32 [{R + 1}] (one more than block_table rows)")
    _require(topk_indices.dtype == torch.int32 and tuple(topk_indices.shape) == (T, TOPK),
             f"topk_indices must be int32 [{T}, {TOPK}]")
    _require(topk_indices.is_contiguous(), "topk_indices must be contiguous (written in place)")
    num_pages = num_pages_of(k_index_cache_fp8)
    if T == 0:
        return
    _require(1 <= R <= T, f"need 1 <= requests <= rows, got {R} requests for {T} rows")
    q = q_index_fp8.contiguous()
    k = k_index_cache_fp8.contiguous()
    w = weights.contiguous()
    sl = seq_lens.contiguous()
    bt = block_table.to(torch.int32).contiguous()
    cu = cu_seqlens_q.to(torch.int32).contiguous()
    max_pages = bt.shape[1]

    L = _native.lib()
    nbytes = L.dsa_indexer_prefill_workspace_bytes(T, R, max_pages)
    cur = torch.cuda.current_stream(dev).cuda_stream
    ws = workspace.get(dev, "indexer_prefill", nbytes, cur)
    stream = ctypes.c_void_p(cur)
    with torch.cuda.device(dev):
        st = L.dsa_indexer_prefill_run(_ptr(q), _ptr(k), num_pages, _ptr(w), _ptr(sl), _ptr(bt),
                                       _ptr(cu), T, R, max_pages, _ptr(topk_indices), _ptr(ws),
                                       ws.numel(), stream)
    _native.check(st, "dsa_indexer_prefill_run")
    if _CHECK and not torch.cuda.is_current_stream_capturing():
        raise_on_device_status(dev)


def device_status(device: torch.device, clear: bool = True) -> int:
    """OR of the sticky device status bits of every indexer workspace on
    `device` (synchronises)."""
    bits = 0
    stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    for ws in workspace.buffers_of(device, "indexer") + workspace.buffers_of(device, "indexer_prefill"):
        out = ctypes.c_uint32(0)
        with torch.cuda.device(device):
            st = _native.lib().dsa_read_device_status(_ptr(ws), ctypes.byref(out), int(clear),
                                                      stream)
        _native.check(st, "dsa_read_device_status")
        bits |= int(out.value)
    return bits


def raise_on_device_status(device: torch.device) -> None:
    bits = device_status(device, clear=True)
    if bits:
        raise _native.DsaError(f"dsa_indexer: {_native.describe_device_status(bits)} "
                               f"(status bits {bits:#x})")
