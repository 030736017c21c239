"""Bit-exact host bookkeeping: the C++ host layer (allocator, block tables,
copy-on-write, swap slots, scheduler) against the reference's own classes.

Each script of tests/replay_scripts.py is replayed by tests/native/replay_ops.h
compiled against this library; the trace (every return value, then every
block's state / ref count / generation, the stats, every table entry and the
scheduler's request states) must hash to what the reference produced
(tests/golden/replay_golden.json, made by make_replay_golden.py). Where the
reference is built here, further random scripts are compared live.
"""
import json
import os

import pytest

import oracle
import replay_scripts as R

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "replay_golden.json")))


@pytest.mark.parametrize("name", sorted(R.golden_cases()))
def test_trace_matches_the_reference_golden(name):
    script = R.golden_cases()[name]
    trace = R.replay_qvp(script)
    assert trace.count("\n") > script.count("\n")
    assert R.digest(trace) == GOLD[name]["sha256"], name


@pytest.mark.skipif(not oracle.ref_available(), reason="reference not built here")
@pytest.mark.parametrize("seed", range(1000, 1040))
def test_trace_matches_the_reference_live(seed):
    script = R.random_script(seed, n_ops=300, scheduler=seed % 2 == 0)
    ours, theirs = R.replay_qvp(script), R.replay_ref(script)
    if ours != theirs:
        for a, b in zip(ours.splitlines(), theirs.splitlines()):
            assert a == b
    assert ours == theirs
