"""The reference's specification tests for the host layer (BlockTable,
KVBlockLayout, CacheView structure, MemoryAllocator, SwapBackend
bookkeeping, KVCacheManager, Scheduler and its watermark policy),
re-expressed in tests/native/reference_cases.cpp. They run on bookkeeping-only
pools, so the whole suite runs on the CPU."""
import os

import pytest

from helpers import NativeCases

CASES = NativeCases(os.path.join(os.path.dirname(__file__), "native", "libqvp_refcases.so"), "qvp_refcases")

@pytest.mark.parametrize("name", CASES.names())
def test_reference_case(name):
    rc, msg = CASES.run(name)
    assert rc == 0, msg


def test_reference_case_suite_is_built():
    assert len(CASES.names()) >= 40
