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


def _fail(msg: str) -> None:
    raise ValueError(f"dsa_attention.run: {msg}")


_ws_bytes: dict = {}  # (device index, tokens) -> dsa_attention_workspace_bytes


def _workspace_bytes(dev: torch.device, T: int) -> int:
    key = (dev.index, T)
    n = _ws_bytes.get(key)
    if n is None:
        n = _native.call_on(dev, _native.lib().dsa_attention_workspace_bytes, T)
        _ws_bytes[key] = n
    return n


def run(q_nope: torch.Tensor, q_pe: torch.Tensor, ckv_cache: torch.Tensor,
        kpe_cache: torch.Tensor, sparse_indices: torch.Tensor, sm_scale,
        output: torch.Tensor, lse: torch.Tensor) -> None:
    # Every message is formatted only on failure: this runs once per decode step.
    dev = q_nope.device
    if dev.type != "cuda":
        _fail("tensors must be on a CUDA device")
    for name, t in (("q_pe", q_pe), ("ckv_cache", ckv_cache), ("kpe_cache", kpe_cache),
                    ("sparse_indices", sparse_indices), ("output", output), ("lse", lse)):
        if t.device != dev:
            _fail(f"{name} is on {t.device}, expected {dev}")
    for name, t in (("q_nope", q_nope), ("q_pe", q_pe), ("ckv_cache", ckv_cache),
                    ("kpe_cache", kpe_cache), ("output", output)):
        if t.dtype != torch.bfloat16:
            _fail(f"{name} must be bfloat16, got {t.dtype}")
    if q_nope.dim() != 3 or q_nope.shape[1:] != (NUM_HEADS, DIM_CKV):
        _fail(f"q_nope must be [T, {NUM_HEADS}, {DIM_CKV}], got {tuple(q_nope.shape)}")
    T = q_nope.shape[0]
    if q_pe.shape != (T, NUM_HEADS, DIM_KPE):
        _fail(f"q_pe must be [{T}, 16, 64]")
    if ckv_cache.shape[-1] != DIM_CKV:
        _fail("ckv_cache last dim must be 512")
    if kpe_cache.shape[-1] != DIM_KPE:
        _fail("kpe_cache last dim must be 64")
    num_slots = ckv_cache.numel() // DIM_CKV
    if kpe_cache.numel() // DIM_KPE != num_slots:
        _fail("ckv_cache and kpe_cache must hold the same number of slots")
    if sparse_indices.shape != (T, TOPK):
        _fail(f"sparse_indices must be [{T}, {TOPK}]")
    if sparse_indices.dtype != torch.int32 and sparse_indices.dtype != torch.int64:
        _fail("sparse_indices must be int32 or int64")
    if output.shape != (T, NUM_HEADS, DIM_CKV) or not output.is_contiguous():
        _fail(f"output must be contiguous bfloat16 [{T}, 16, 512]")
    if lse.dtype != torch.float32 or lse.shape != (T, NUM_HEADS) or not lse.is_contiguous():
        _fail(f"lse must be contiguous float32 [{T}, 16]")
    if isinstance(sm_scale, torch.Tensor):
        sm_scale = float(sm_scale.item())
    if T == 0:
        return
    qn = q_nope.contiguous()
    qp = q_pe.contiguous()
    ckv = ckv_cache.contiguous()
    kpe = kpe_cache.contiguous()
    idx = sparse_indices if sparse_indices.dtype == torch.int32 else sparse_indices.to(torch.int32)
    idx = idx.contiguous()
    cur = _native.current_stream(dev)
    ws = workspace.get(dev, "attention", _workspace_bytes(dev, T), cur)
    st = _native.call_on(dev, _native.lib().dsa_attention_run, qn.data_ptr(), qp.data_ptr(),
                         ckv.data_ptr(), kpe.data_ptr(), num_slots, idx.data_ptr(), T,
                         float(sm_scale), output.data_ptr(), lse.data_ptr(), ws.data_ptr(),
                         ws.numel(), cur)
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
