"""The reference's specification tests for the host layer (BlockTable,
KVBlockLayout, CacheView structure, MemoryAllocator, SwapBackend
bookkeeping, KVCacheManager, Scheduler and its watermark policy),
re-expressed in tests/native/reference_cases.cpp. They run on bookkeeping-only
pools, so the whole suite runs on the CPU."""
import ctypes as C
import os

import pytest

LIB = os.path.join(os.path.dirname(__file__), "native", "libqvp_refcases.so")


def _lib():
    return C.CDLL(LIB)


def _names():
    if not os.path.exists(LIB):
        return []
    buf = C.create_string_buffer(1 << 16)
    _lib().qvp_refcases_list(buf, len(buf))
    return [n for n in buf.value.decode().splitlines() if n]


@pytest.mark.parametrize("name", _names())
def test_reference_case(name):
    msg = C.create_string_buffer(4096)
    rc = _lib().qvp_refcases_run(name.encode(), msg, len(msg))
    assert rc == 0, msg.value.decode()


def test_reference_case_suite_is_built():
    assert len(_names()) >= 40
