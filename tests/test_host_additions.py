"""Host checks of this library's additions to the reference interface
(tests/native/table_cases.cpp): the resident block tables (every packet the
planner emits, applied to a host mirror of the device table, must reproduce a
full per-step flatten, and steady decode uploads a row only when a sequence
gains a block), host-visible pools, the refusal rules of PagedPrefillBatch
and KVAppendBatch, and LruEvictionPolicy."""
import os

import pytest

from helpers import NativeCases

CASES = NativeCases(os.path.join(os.path.dirname(__file__), "native", "libqvp_tablecases.so"), "qvp_tablecases")

@pytest.mark.parametrize("name", CASES.names())
def test_table_case(name):
    rc, msg = CASES.run(name)
    assert rc == 0, msg


def test_table_case_suite_is_built():
    assert len(CASES.names()) >= 6
