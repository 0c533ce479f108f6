"""CPU tests of the C ABI: the library loads, exports every symbol the header
declares, and rejects bad arguments on the host before touching a GPU."""

import ctypes
import pathlib
import re

import pytest

from dsa_b200 import _native

HEADER = pathlib.Path(__file__).resolve().parent.parent / "include" / "dsa_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:DSA_API\s+)?(?:const\s+char\s*\*|int|size_t)\s+(dsa_\w+)\s*\(",
                                 text, re.M)))


def test_header_declares_the_abi():
    names = declared_functions()
    assert "dsa_indexer_run" in names and "dsa_attention_run" in names
    assert set(names) == set(_native.SIGNATURES), names


def test_every_return_code_has_its_own_message():
    codes = dict(re.findall(r"^#define\s+(DSA_(?:OK|ERR_\w+))\s+(\d+)", HEADER.read_text(), re.M))
    assert int(codes.pop("DSA_OK")) == _native.DSA_OK == 0
    lib = _native.lib()
    msgs = {lib.dsa_b200_status_string(int(v)) for v in codes.values()}
    assert len(msgs) == len(codes) and b"unknown status" not in msgs, msgs


def test_device_status_bits_match_the_header():
    bits = dict(re.findall(r"^#define\s+DSA_DEV_(\w+)\s+(0x[0-9a-fA-F]+)u", HEADER.read_text(), re.M))
    assert {k: int(v, 16) for k, v in bits.items()} == {
        "BAD_SEQ_LEN": _native.DEV_BAD_SEQ_LEN, "BAD_PAGE": _native.DEV_BAD_PAGE,
        "BAD_INDEX": _native.DEV_BAD_INDEX, "WAIT_TIMEOUT": _native.DEV_WAIT_TIMEOUT,
        "STALE_WORKSPACE": _native.DEV_STALE_WORKSPACE}
    # Every bit has its own message.
    for b in bits.values():
        assert _native.describe_device_status(int(b, 16)), b


def test_test_hook_kinds_match_the_header():
    kinds = dict(re.findall(r"^#define\s+DSA_TEST_(\w+)\s+(\d+)", HEADER.read_text(), re.M))
    assert {k: int(v) for k, v in kinds.items()} == {
        "NONE": _native.TEST_NONE, "SKIP_ARRIVAL": _native.TEST_SKIP_ARRIVAL,
        "SKIP_READY": _native.TEST_SKIP_READY}


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_version_and_status_strings():
    lib = _native.lib()
    assert lib.dsa_b200_abi_version() == 1
    assert lib.dsa_b200_status_string(0) == b"ok"
    assert b"workspace" in lib.dsa_b200_status_string(3)
    assert lib.dsa_b200_status_string(999) == b"unknown status"


def test_workspace_sizes():
    lib = _native.lib()
    assert lib.dsa_indexer_workspace_bytes(64, 1024) == 256 + 32768 + 4 * 64 * 2048 + 4 * 64 * 1024 * 64
    assert lib.dsa_indexer_workspace_bytes(0, 10) == 256 + 32768
    assert lib.dsa_attention_workspace_bytes(0) == 256
    assert lib.dsa_attention_workspace_bytes(8) > lib.dsa_attention_workspace_bytes(1)


NULL = ctypes.c_void_p(0)
FAKE = ctypes.c_void_p(4096)  # never dereferenced: every case fails validation first


@pytest.mark.parametrize("batch,max_pages,num_pages,ptr,expect", [
    (-1, 1, 1, FAKE, 1),        # negative batch
    (0, 1, 1, NULL, 0),         # empty batch: nothing to do
    (4, 1, 1, NULL, 1),         # null pointers
    (4, 0, 1, FAKE, 1),         # max_pages < 1
    (4, 1, 0, FAKE, 1),         # empty pool
    (5000, 1, 1, FAKE, 1),      # batch above the per-call limit
])
def test_indexer_host_validation(batch, max_pages, num_pages, ptr, expect):
    lib = _native.lib()
    st = lib.dsa_indexer_run(ptr, ptr, num_pages, ptr, ptr, ptr, batch, max_pages, ptr, ptr,
                             1 << 30, NULL)
    assert st == expect


def test_indexer_misaligned_and_small_workspace():
    lib = _native.lib()
    odd = ctypes.c_void_p(4097)
    assert lib.dsa_indexer_run(odd, FAKE, 1, FAKE, FAKE, FAKE, 1, 1, FAKE, FAKE, 1 << 30, NULL) == 2
    assert lib.dsa_indexer_run(FAKE, FAKE, 1, FAKE, FAKE, FAKE, 1, 1, FAKE, FAKE, 16, NULL) == 3


@pytest.mark.parametrize("tokens,slots,ptr,expect", [
    (-1, 1, FAKE, 1), (0, 1, NULL, 0), (2, 1, NULL, 1), (2, 0, FAKE, 1),
])
def test_attention_host_validation(tokens, slots, ptr, expect):
    lib = _native.lib()
    st = lib.dsa_attention_run(ptr, ptr, ptr, ptr, slots, ptr, tokens, 0.07, ptr, ptr, ptr,
                               1 << 30, NULL)
    assert st == expect


def test_attention_misaligned():
    lib = _native.lib()
    odd = ctypes.c_void_p(4098)
    assert lib.dsa_attention_run(FAKE, odd, FAKE, FAKE, 10, FAKE, 1, 0.07, FAKE, FAKE, FAKE,
                                 1 << 30, NULL) == 2


def test_test_hook_validation():
    lib = _native.lib()
    assert lib.dsa_b200_test_inject(7, 1000) == 1           # unknown kind
    assert lib.dsa_b200_test_inject(_native.TEST_SKIP_ARRIVAL, 0) == 1
    assert lib.dsa_b200_test_inject(_native.TEST_SKIP_ARRIVAL, 1000) == 0
    assert lib.dsa_b200_test_inject(_native.TEST_SKIP_READY, 0) == 1
    assert lib.dsa_b200_test_inject(_native.TEST_SKIP_READY, 1 << 56) == 1
    assert lib.dsa_b200_test_inject(_native.TEST_SKIP_READY, 1000) == 0
    assert lib.dsa_b200_test_inject(_native.TEST_NONE, 0) == 0  # disarms both again


def test_read_status_rejects_null():
    lib = _native.lib()
    out = ctypes.c_uint32(0)
    assert lib.dsa_read_device_status(NULL, ctypes.byref(out), 0, NULL) == 1
