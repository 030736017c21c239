"""Regenerates the golden decode fixtures from the reference itself.

Runs the reference's paged_attention_decode<T> (phhuang191129/QwenVL-Paged
include/qwenvl_paged/PagedAttention.h:53-127, compiled from its own sources
into oracle/_ref/libqvp_ref.so by oracle/Makefile) on the seeded workloads of
qwenvl-paged_b200/workloads.py and stores the outputs with a hash of the
inputs they were computed from. Usage (where the reference sources exist):

    make -C oracle REF=<reference checkout> && python tests/golden/make_golden.py
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "qwenvl-paged_b200"), os.path.join(ROOT, "oracle")]

import oracle  # noqa: E402
import workloads as W  # noqa: E402


def input_hash(pool, q, w):
    h = hashlib.sha256()
    for a in (pool, q, w.context_lens, w.tables):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def cases():
    yield "cfg1_ref_out", W.cfg1()
    yield "bf16_small_ref_out", W.small(101, batch=4, ctx_lo=1, ctx_hi=100, hq=28, hkv=4, head_dim=128,
                                        dtype="bf16")


def main():
    meta = {}
    for name, w in cases():
        pool, q = W.host_inputs(w)
        r = oracle.RefDecoder(w, pool)
        out, status = r.decode(q)
        r.close()
        assert status.all(), name
        np.save(os.path.join(HERE, name + ".npy"), out)
        meta[name] = {"workload": w.name, "seed": w.seed, "inputs_sha256": input_hash(pool, q, w),
                      "dtype": w.dtype, "shape": list(out.shape)}
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
