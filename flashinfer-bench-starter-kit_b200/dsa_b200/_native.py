"""ctypes binding of libdsa_b200.so (the C ABI declared in include/dsa_b200.h).

The library is built in-tree by ``build.py``; there is deliberately no
fallback: if it is missing or the GPU is not an sm_100 part, calls raise.
"""

from __future__ import annotations

import ctypes
import pathlib
import threading

import torch

LIB_PATH = pathlib.Path(__file__).resolve().with_name("libdsa_b200.so")

DSA_OK = 0
DEV_BAD_SEQ_LEN = 0x1
DEV_BAD_PAGE = 0x2
DEV_BAD_INDEX = 0x4
DEV_WAIT_TIMEOUT = 0x8
DEV_STALE_WORKSPACE = 0x10

# name -> (restype, argtypes); every symbol include/dsa_b200.h declares.
_P = ctypes.c_void_p
SIGNATURES = {
    "dsa_b200_abi_version": (ctypes.c_int, []),
    "dsa_b200_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "dsa_indexer_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32]),
    "dsa_indexer_run": (ctypes.c_int, [_P, _P, ctypes.c_int64, _P, _P, _P, ctypes.c_int32,
                                       ctypes.c_int32, _P, _P, ctypes.c_size_t, _P]),
    "dsa_attention_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int32]),
    "dsa_attention_run": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_int64, _P, ctypes.c_int32,
                                         ctypes.c_float, _P, _P, _P, ctypes.c_size_t, _P]),
    "dsa_read_device_status": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_uint32), ctypes.c_int,
                                              _P]),
    "dsa_indexer_run_noalloc": (ctypes.c_int, [_P, _P, ctypes.c_int64, _P, _P, _P, ctypes.c_int32,
                                               ctypes.c_int32, _P, _P]),
    "dsa_index_cache_write": (ctypes.c_int, [_P, _P, ctypes.c_int32, _P, ctypes.c_int64,
                                             ctypes.c_int32, _P, _P]),
    "dsa_indexer_prefill_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32,
                                                              ctypes.c_int32]),
    "dsa_indexer_prefill_run": (ctypes.c_int, [_P, _P, ctypes.c_int64, _P, _P, _P, _P, ctypes.c_int32,
                                               ctypes.c_int32, ctypes.c_int32, _P, _P, ctypes.c_size_t,
                                               _P]),
    "dsa_b200_test_inject": (ctypes.c_int, [ctypes.c_int, ctypes.c_uint64]),
}

# dsa_b200_test_inject kinds (failure-path tests only)
TEST_NONE = 0
TEST_SKIP_ARRIVAL = 1
TEST_SKIP_READY = 2

_lib = None
_lock = threading.Lock()


class DsaError(RuntimeError):
    """A dsa_b200 entry point returned a non-zero status."""


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise DsaError(f"{LIB_PATH.name} is not built; run "
                                   "flashinfer-bench-starter-kit_b200/build.py (or "
                                   "__graft_entry__.build())")
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def current_stream(device: torch.device) -> int:
    """Raw handle of torch's current stream on a CUDA `device` (no Stream
    object is built: this sits on every call's host path)."""
    return torch._C._cuda_getCurrentRawStream(device.index)


def call_on(device: torch.device, fn, *args):
    """fn(*args) with `device` current; the device is switched (and restored)
    only when another one is current."""
    if torch._C._cuda_getDevice() == device.index:
        return fn(*args)
    with torch.cuda.device(device):
        return fn(*args)


def check(status: int, what: str) -> None:
    if status != DSA_OK:
        msg = lib().dsa_b200_status_string(status).decode()
        raise DsaError(f"{what} failed: {msg} (status {status})")


def describe_device_status(bits: int) -> str:
    names = []
    if bits & DEV_BAD_SEQ_LEN:
        names.append("seq_len outside [0, max_pages*64]")
    if bits & DEV_BAD_PAGE:
        names.append("block_table entry outside the page pool")
    if bits & DEV_BAD_INDEX:
        names.append("sparse index outside [-1, num_slots)")
    if bits & DEV_WAIT_TIMEOUT:
        names.append("a kernel pipeline wait timed out")
    if bits & DEV_STALE_WORKSPACE:
        names.append("workspace contents inconsistent: a merge counter not zero on entry or a "
                     "histogram not matching its scores (zero-fill the workspace)")
    return ", ".join(names) if names else "ok"
