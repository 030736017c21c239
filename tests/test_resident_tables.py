"""Host checks of the device-resident block tables (tests/native/table_cases.cpp):
every packet the planner emits, applied to a host mirror of the device table,
must reproduce a full per-step flatten of every sequence's table, and steady
decode must upload a row only when a sequence gains a block."""
import ctypes as C
import os

import pytest

LIB = os.path.join(os.path.dirname(__file__), "native", "libqvp_tablecases.so")


def _names():
    if not os.path.exists(LIB):
        return []
    buf = C.create_string_buffer(1 << 16)
    C.CDLL(LIB).qvp_tablecases_list(buf, len(buf))
    return [n for n in buf.value.decode().splitlines() if n]


@pytest.mark.parametrize("name", _names())
def test_table_case(name):
    msg = C.create_string_buffer(4096)
    rc = C.CDLL(LIB).qvp_tablecases_run(name.encode(), msg, len(msg))
    assert rc == 0, msg.value.decode()


def test_table_case_suite_is_built():
    assert len(_names()) >= 6
