"""GPU checks of the host layer's additions (tests/native/host_layer_gpu_checks.cpp):
PagedDecodeBatch with device-resident block tables (bit-identical outputs to
the per-step flatten across block growth, copy on write, reordering and a
refused swapped-out sequence, no table rows uploaded on steady steps),
KVAppendBatch (appended K/V land byte-exact in their slots) and
PagedPrefillBatch (within the bf16 tolerance of per-position decodes)."""
import os

import pytest

from helpers import NativeCases

CASES = NativeCases(os.path.join(os.path.dirname(__file__), "native", "libqvp_hostlayer_checks.so"), "qvp_hostlayerchecks")

@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES.names())
def test_host_layer_check(name):
    rc, msg = CASES.run(name)
    assert rc == 0, msg
