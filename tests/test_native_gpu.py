"""GPU tests of the C++ host layer (tests/native/native_tests.cpp): device
pool, batched copy-on-write, host and device swap backends, the
paged_attention_decode<T> shim, PagedDecodeBatch and a scheduler-driven end
to end run, re-expressed from the reference suite."""
import ctypes as C
import os

import pytest

LIB = os.path.join(os.path.dirname(__file__), "native", "libqvp_native_tests.so")


def _names():
    if not os.path.exists(LIB):
        return []
    lib = C.CDLL(LIB)
    buf = C.create_string_buffer(1 << 16)
    lib.qvp_native_list(buf, len(buf))
    return [n for n in buf.value.decode().splitlines() if n]


@pytest.mark.gpu
@pytest.mark.parametrize("name", _names())
def test_native(name):
    lib = C.CDLL(LIB)
    msg = C.create_string_buffer(4096)
    rc = lib.qvp_native_run(name.encode(), msg, len(msg))
    assert rc == 0, msg.value.decode()


def test_native_suite_is_built_and_lists_its_cases():
    assert len(_names()) >= 12
