"""GPU checks of the host layer's additions (tests/native/host_layer_gpu_checks.cpp):
PagedDecodeBatch with device-resident block tables (bit-identical outputs to
the per-step flatten across block growth, copy on write, reordering and a
refused swapped-out sequence, no table rows uploaded on steady steps),
KVAppendBatch (appended K/V land byte-exact in their slots) and
PagedPrefillBatch (within the bf16 tolerance of per-position decodes).

Not collected yet (no test_ prefix): run it on a GPU with
`python -m pytest tests/host_layer_gpu_checks.py -q`, then rename it to
test_host_layer_gpu.py."""
import ctypes as C
import os

import pytest

LIB = os.path.join(os.path.dirname(__file__), "native", "libqvp_hostlayer_checks.so")


def _names():
    if not os.path.exists(LIB):
        return []
    buf = C.create_string_buffer(1 << 16)
    C.CDLL(LIB).qvp_hostlayerchecks_list(buf, len(buf))
    return [n for n in buf.value.decode().splitlines() if n]


@pytest.mark.gpu
@pytest.mark.parametrize("name", _names())
def test_host_layer_check(name):
    msg = C.create_string_buffer(4096)
    rc = C.CDLL(LIB).qvp_hostlayerchecks_run(name.encode(), msg, len(msg))
    assert rc == 0, msg.value.decode()
