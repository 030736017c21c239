"""GPU tests of the C++ host layer (tests/native/native_tests.cpp): device
pool, batched copy-on-write, host and device swap backends, the
paged_attention_decode<T> shim, PagedDecodeBatch and a scheduler-driven end
to end run, re-expressed from the reference suite."""
import os

import pytest

from helpers import NativeCases

CASES = NativeCases(os.path.join(os.path.dirname(__file__), "native", "libqvp_native_tests.so"), "qvp_native")

@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES.names())
def test_native(name):
    rc, msg = CASES.run(name)
    assert rc == 0, msg


def test_native_suite_is_built_and_lists_its_cases():
    assert len(CASES.names()) >= 12
