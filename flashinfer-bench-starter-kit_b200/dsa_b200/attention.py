"""DSA sparse MLA attention operator (destination-passing style).

``run`` keeps the reference entry point's signature, argument meaning and
in-place outputs (dsa_attention/solution/triton/kernel.py:240-252):

    run(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale,
        output, lse) -> None

``lse`` is the base-2 log-sum-exp of the scaled logits; a row whose indices
are all -1 yields output 0 and lse -inf (the definition reference's
behaviour; the reference solution's softmax kernel would give NaN there).
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _native, workspace

NUM_HEADS = 16
DIM_CKV = 512
DIM_KPE = 64
TOPK = 2048

_CHECK = os.environ.get("DSA_B200_CHECK", "0") not in ("", "0")


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(f"dsa_attention.run: {msg}")


@torch.no_grad()
def run(q_nope: torch.Tensor, q_pe: torch.Tensor, ckv_cache: torch.Tensor,
        kpe_cache: torch.Tensor, sparse_indices: torch.Tensor, sm_scale,
        output: torch.Tensor, lse: torch.Tensor) -> None:
    dev = q_nope.device
    _require(dev.type == "cuda", "tensors must be on a CUDA device")
    for name, t in (("q_pe", q_pe), ("ckv_cache", ckv_cache), ("kpe_cache", kpe_cache),
                    ("sparse_indices", sparse_indices), ("output", output), ("lse", lse)):
        _require(t.device == dev, f"{name} is on {t.device}, expected {dev}")
    for name, t in (("q_nope", q_nope), ("q_pe", q_pe), ("ckv_cache", ckv_cache),
                    ("kpe_cache", kpe_cache), ("output", output)):
        _require(t.dtype == torch.bfloat16, f"{name} must be bfloat16, got {t.dtype}")
    _require(q_nope.dim() == 3 and tuple(q_nope.shape[1:]) == (NUM_HEADS, DIM_CKV),
             f"q_nope must be [T, {NUM_HEADS}, {DIM_CKV}], got {tuple(q_nope.shape)}")
    T = q_nope.shape[0]
    _require(tuple(q_pe.shape) == (T, NUM_HEADS, DIM_KPE), f"q_pe must be [{T}, 16, 64]")
    _require(ckv_cache.shape[-1] == DIM_CKV, "ckv_cache last dim must be 512")
    _require(kpe_cache.shape[-1] == DIM_KPE, "kpe_cache last dim must be 64")
    num_slots = ckv_cache.numel() // DIM_CKV
    _require(kpe_cache.numel() // DIM_KPE == num_slots,
             "ckv_cache and kpe_cache must hold the same number of slots")
    _require(tuple(sparse_indices.shape) == (T, TOPK), f"sparse_indices must be [{T}, {TOPK}]")
    _require(sparse_indices.dtype in (torch.int32, torch.int64),
             "sparse_indices must be int32 or int64")
    _require(tuple(output.shape) == (T, NUM_HEADS, DIM_CKV) and output.is_contiguous(),
             f"output must be contiguous bfloat16 [{T}, 16, 512]")
    _require(lse.dtype == torch.float32 and tuple(lse.shape) == (T, NUM_HEADS)
             and lse.is_contiguous(), f"lse must be contiguous float32 [{T}, 16]")
    if isinstance(sm_scale, torch.Tensor):
        sm_scale = float(sm_scale.item())
    if T == 0:
        return
    # Flatten the caches to slots (kernel.py:245-246) and take int32 indices
    # (kernel.py:248).
    qn = q_nope.contiguous()
    qp = q_pe.contiguous()
    ckv = ckv_cache.contiguous()
    kpe = kpe_cache.contiguous()
    idx = sparse_indices.to(torch.int32).contiguous()

    L = _native.lib()
    with torch.cuda.device(dev):
        nbytes = L.dsa_attention_workspace_bytes(T)
    cur = torch.cuda.current_stream(dev).cuda_stream
    ws = workspace.get(dev, "attention", nbytes, cur)
    stream = ctypes.c_void_p(cur)
    with torch.cuda.device(dev):
        st = L.dsa_attention_run(_ptr(qn), _ptr(qp), _ptr(ckv), _ptr(kpe), num_slots, _ptr(idx), T,
                                 float(sm_scale), _ptr(output), _ptr(lse), _ptr(ws), ws.numel(),
                                 stream)
    _native.check(st, "dsa_attention_run")
    if _CHECK and not torch.cuda.is_current_stream_capturing():
        raise_on_device_status(dev)


def device_status(device: torch.device, clear: bool = True) -> int:
    """OR of the sticky device status bits of every attention workspace on
    `device` (synchronises)."""
    bits = 0
    stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    for ws in workspace.buffers_of(device, "attention"):
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
        raise _native.DsaError(f"dsa_attention: {_native.describe_device_status(bits)} "
                               f"(status bits {bits:#x})")
