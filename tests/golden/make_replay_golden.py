"""Regenerates tests/golden/replay_golden.json: the sha256 of the trace the
reference's own classes (oracle/_ref/libqvp_ref.so, built from the reference
sources by oracle/Makefile) produce for every bookkeeping script of
tests/replay_scripts.py. Usage: make -C oracle REF=<reference checkout> && python tests/golden/make_replay_golden.py
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "tests"), os.path.join(ROOT, "oracle")]

import replay_scripts as R  # noqa: E402


def main():
    out = {}
    for name, script in sorted(R.golden_cases().items()):
        trace = R.replay_ref(script)
        out[name] = {"sha256": R.digest(trace), "ops": script.count("\n"), "trace_bytes": len(trace)}
    with open(os.path.join(HERE, "replay_golden.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
