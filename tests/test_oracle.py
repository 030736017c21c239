"""Pins the C oracle: against the golden outputs the reference produced
(tests/golden/, made by make_golden.py from the reference's own sources) and,
where the reference is built here, against the reference directly."""
import json
import os

import numpy as np
import pytest

import oracle
import workloads as W
from helpers import max_rel_err

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _gold(name):
    meta = json.load(open(os.path.join(GOLD, "golden.json")))[name]
    return meta, np.load(os.path.join(GOLD, name + ".npy"))


def _hash(pool, q, w):
    import hashlib
    h = hashlib.sha256()
    for a in (pool, q, w.context_lens, w.tables):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def test_seeded_inputs_are_the_ones_the_golden_outputs_came_from():
    for name, w in (("cfg1_ref_out", W.cfg1()),
                    ("bf16_small_ref_out", W.small(101, batch=4, ctx_lo=1, ctx_hi=100, hq=28, hkv=4,
                                                    head_dim=128, dtype="bf16"))):
        meta, _ = _gold(name)
        pool, q = W.host_inputs(w)
        assert _hash(pool, q, w) == meta["inputs_sha256"], name


def test_oracle_matches_reference_golden_cfg1_fp32():
    meta, gold = _gold("cfg1_ref_out")
    w = W.cfg1()
    pool, q = W.host_inputs(w)
    out, status = oracle.port_decode(w, pool, q)
    assert status.all()
    # same arithmetic order as the reference: bit-identical in practice
    assert max_rel_err(out, gold) < 1e-6
    assert out.shape == (4, 8, 64)


def test_oracle_matches_reference_golden_bf16():
    meta, gold_bits = _gold("bf16_small_ref_out")
    w = W.small(101, batch=4, ctx_lo=1, ctx_hi=100, hq=28, hkv=4, head_dim=128, dtype="bf16")
    pool, q = W.host_inputs(w)
    out, status = oracle.port_decode(w, pool, q)
    assert status.all()
    # the reference stored bf16 (round-to-nearest-even of its fp32 result)
    assert np.array_equal(W.f32_to_bf16_bits(out), gold_bits)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference not built here")
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_oracle_matches_the_reference_on_random_batches(dtype):
    w = W.small(5, batch=6, ctx_lo=1, ctx_hi=70, hq=8, hkv=2, head_dim=32, dtype=dtype, tokens_per_block=4,
                num_layers=2, layer=1)
    pool, q = W.host_inputs(w)
    out, status = oracle.port_decode(w, pool, q)
    r = oracle.RefDecoder(w, pool)
    rout, rstatus = r.decode(q, threads=2)
    r.close()
    assert status.all() and rstatus.all()
    if dtype == "f32":
        assert np.array_equal(out, rout)
    else:
        assert np.array_equal(W.f32_to_bf16_bits(out), rout)


def test_oracle_threads_do_not_change_results():
    w = W.small(6, batch=9, ctx_lo=1, ctx_hi=300, hq=28, hkv=4, head_dim=128, dtype="bf16")
    pool, q = W.host_inputs(w)
    a, _ = oracle.port_decode(w, pool, q, threads=1)
    b, _ = oracle.port_decode(w, pool, q, threads=4)
    assert np.array_equal(a, b)


def test_oracle_copy_blocks_matches_memcpy():
    pool = np.arange(8 * 256, dtype=np.uint32).astype(np.uint8)
    expect = pool.copy().reshape(8, 256)
    expect[5] = expect[2]
    expect[1] = expect[7]
    oracle.port_copy_blocks(pool, 256, 8, 256, np.array([2, 5, 7, 1, 9, 0], dtype=np.int32))
    assert np.array_equal(pool.reshape(8, 256), expect)


def _swap_block_256():
    """128 bf16 values with low byte i: high bytes 0x3F/0xBF/0x40 by i % 3 for
    i < 112, then 0x50..0x5F once each (16 singles: 4 escapes)."""
    hi = [[0x3F, 0xBF, 0x40][i % 3] for i in range(112)] + [0x50 + j for j in range(16)]
    vals = np.array([(h << 8) | i for i, h in enumerate(hi)], dtype=np.uint16)
    return vals.view(np.uint8).copy()


def test_swap_slot_format_known_answer():
    block = _swap_block_256()
    slot, esc = oracle.port_compress_block(block)
    assert len(slot) == oracle.swap_slot_bytes(256) == 272
    head = slot[:16].view(np.uint32)
    # counts 38 (0x3F), 37 (0x40), 37 (0xBF): ties go to the smaller byte
    assert list(head) == [oracle.SLOT_CODED, 4, 32 + 192 + 16, 0]
    assert list(slot[16:32]) == [0x3F, 0x40, 0xBF] + list(range(0x50, 0x5C)) + [0]
    codes = [{0: 0, 1: 2, 2: 1}[i % 3] for i in range(112)] + list(range(3, 15)) + [15] * 4
    packed = [codes[2 * k] | (codes[2 * k + 1] << 4) for k in range(64)]
    assert list(slot[32:96]) == packed
    assert list(slot[96:224]) == list(range(128))
    assert esc == {(124 + j) << 8 | (0x5C + j) for j in range(4)}
    assert np.array_equal(oracle.port_decompress_slot(slot, 256), block)


def test_swap_slot_raw_fallback_and_round_trips():
    rng = np.random.default_rng(2)
    for nb in (16, 48, 64, 256, 4096, 32768):
        for kind in ("random", "gauss", "const"):
            if kind == "random":
                b = rng.integers(0, 256, nb, dtype=np.uint8)
            elif kind == "gauss":
                f = rng.normal(size=nb // 2).astype(np.float32)
                b = (f.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)  # truncated to bf16
            else:
                b = np.full(nb, 7, dtype=np.uint8)
            slot, _ = oracle.port_compress_block(b)
            head = slot[:16].view(np.uint32)
            if nb <= 64 or kind == "random":
                assert head[0] == oracle.SLOT_RAW and head[2] == 16 + nb
            else:
                assert head[0] == oracle.SLOT_CODED and head[2] < 16 + nb
            assert np.array_equal(oracle.port_decompress_slot(slot, nb), b)
