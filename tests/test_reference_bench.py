"""The reference's own benchmark program (bench/benchmark_main.cpp), compiled
unmodified against this project's C++ headers and linked to libqvp.so,
must build and run its four benchmarks to the end, like the same file built
on the reference's sources (both built by oracle/Makefile when the reference
sources are present). On a machine without a GPU the pool holds no device
bytes, so the copy-on-write row times the bookkeeping and the queued copy."""
import os
import subprocess

import pytest

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")
ROWS = ("allocate + release", "fork sequence (8 blocks)", "copy-on-write (1 block)",
        "scheduler admit + retire request")


def _run(name):
    exe = os.path.join(REF, name)
    if not os.path.exists(exe):
        pytest.skip(f"{name} not built (reference sources absent)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    return r.returncode, r.stdout, r.stderr


def _rows(stdout):
    got = {}
    for line in stdout.splitlines():
        for name in ROWS:
            if line.startswith(name):
                ops, ns, _ = line[len(name):].split()
                got[name] = (int(ops), float(ns))
    return got


@pytest.mark.parametrize("name", ["refbench_qvp", "refbench_ref"])
def test_reference_benchmark_runs_to_the_end(name):
    rc, out, err = _run(name)
    assert rc == 0, err
    assert "failed" not in out + err
    rows = _rows(out)
    assert set(rows) == set(ROWS)
    assert all(ops > 0 and ns > 0 for ops, ns in rows.values())
