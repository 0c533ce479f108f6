"""Persistent device workspaces for the two operators.

The reference keeps per-device static scratch alive across calls
(dsa_indexer/solution/triton/kernel.py:220-251); the contest rules allow
persistent workspace as long as its contents are recomputed on every call
(FAQ.md:180-182).  Here each (device, operator, stream) owns one uint8 buffer
-- calls on different streams may run concurrently, so they must not share
scratch --
zero-filled when created (its first 4 bytes are the sticky device status
word) and grown only when a larger problem arrives.  Code that captures CUDA
graphs must call ``reserve`` first so no buffer moves after capture.
"""

from __future__ import annotations

import threading

import torch

_buffers: dict = {}
_lock = threading.Lock()


def get(device: torch.device, name: str, nbytes: int, stream: int = 0) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(), name, stream)
    with _lock:
        buf = _buffers.get(key)
        if buf is None or buf.numel() < nbytes:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(
                    f"dsa_b200 workspace '{name}' must grow to {nbytes} bytes during CUDA graph "
                    "capture; call dsa_b200.workspace.reserve() before capturing")
            new = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
            if buf is not None:
                new[:4].copy_(buf[:4])  # keep pending status bits
            buf = new
            _buffers[key] = buf
        return buf


def reserve(device: torch.device, name: str, nbytes: int, stream: int = 0) -> torch.Tensor:
    return get(device, name, nbytes, stream)


def all_buffers():
    with _lock:
        return dict(_buffers)


def buffers_of(device: torch.device, name: str) -> list:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _lock:
        return [b for (d, n, _), b in _buffers.items() if d == idx and n == name]
