"""The reference's nine test files, unmodified, against libqvp.so on a GPU
with host-visible pools (QVP_HOST_VISIBLE_POOLS=1, CUDA managed memory), so
that the cases which write and read block bytes through PhysicalBlock::data()
and CacheView::slot<T>() run too: all 131 cases must pass. The binaries are
built by oracle/Makefile where the reference sources are present and travel
prebuilt."""
import glob
import os
import re
import subprocess

import pytest

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")
SUITES = sorted(os.path.basename(p)[len("suite_qvp_"):] for p in glob.glob(os.path.join(REF, "suite_qvp_*")))


@pytest.mark.gpu
@pytest.mark.parametrize("suite", SUITES)
def test_reference_suite_on_gpu(suite):
    r = subprocess.run([os.path.join(REF, f"suite_qvp_{suite}")], capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, QVP_HOST_VISIBLE_POOLS="1"))
    verdicts = re.findall(r"^(PASS|FAIL|CRASH) ", r.stdout, flags=re.M)
    assert verdicts and all(v == "PASS" for v in verdicts), r.stdout + r.stderr
    assert r.returncode == 0
