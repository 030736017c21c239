"""GPU checks of PagedDecodeBatch with device-resident block tables
(tests/native/resident_gpu_checks.cpp): bit-identical outputs to the per-step
flatten across block growth, copy on write, reordering and a refused
swapped-out sequence, with no table rows uploaded on steady steps.

Not collected yet (no test_ prefix): run it on a GPU with
`python -m pytest tests/resident_tables_gpu_checks.py -q`, then rename it to
test_resident_tables_gpu.py."""
import ctypes as C
import os

import pytest

LIB = os.path.join(os.path.dirname(__file__), "native", "libqvp_residentchecks.so")


def _names():
    if not os.path.exists(LIB):
        return []
    buf = C.create_string_buffer(1 << 16)
    C.CDLL(LIB).qvp_residentchecks_list(buf, len(buf))
    return [n for n in buf.value.decode().splitlines() if n]


@pytest.mark.gpu
@pytest.mark.parametrize("name", _names())
def test_resident_check(name):
    msg = C.create_string_buffer(4096)
    rc = C.CDLL(LIB).qvp_residentchecks_run(name.encode(), msg, len(msg))
    assert rc == 0, msg.value.decode()
