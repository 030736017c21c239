"""Parity of the CUDA decode kernels against the CPU oracle on seeded inputs.

fp32: within 1e-5 of max |oracle| (the north-star "1e-5 relative").
bf16: within 2e-2 absolute of the oracle run in fp32 over the same
bf16-rounded K/V/Q values.
"""
import os

import numpy as np
import pytest

import oracle
import workloads as W
from helpers import bf16_f32, gpu_decode, max_rel_err

pytestmark = pytest.mark.gpu

F32_REL = 1e-5
BF16_ABS = 2e-2


def check(w, *, split_tokens=0, expect_fast=None, threads=8):
    pool, q = W.host_inputs(w)
    ref, status = oracle.port_decode(w, pool, q, threads=threads)
    assert status.all()
    st, out, err, plan = gpu_decode(w, pool, q, split_tokens=split_tokens)
    assert st == 0 and err == 0, (st, err)
    if expect_fast is not None:
        assert plan["fast"] == expect_fast, plan
    if w.dtype == "f32":
        assert max_rel_err(out, ref) < F32_REL, max_rel_err(out, ref)
    else:
        assert np.max(np.abs(out - ref)) < BF16_ABS, np.max(np.abs(out - ref))
    return out, ref, plan


def test_cfg1_fp32_matches_the_oracle():
    w = W.cfg1()
    out, ref, plan = check(w)
    assert out.shape == (4, 8, 64)


@pytest.mark.parametrize("split", [0, 16, 48, 256])
def test_cfg1_fp32_split_k(split):
    check(W.cfg1(), split_tokens=split)


def test_cfg1_matches_the_golden_fixture():
    import os
    gold = os.path.join(os.path.dirname(__file__), "golden", "cfg1_ref_out.npy")
    w = W.cfg1()
    pool, q = W.host_inputs(w)
    st, out, err, _ = gpu_decode(w, pool, q)
    assert st == 0 and err == 0
    assert max_rel_err(out, np.load(gold)) < F32_REL


@pytest.mark.parametrize("hq,hkv,d", [(28, 4, 128), (8, 1, 128), (16, 2, 64), (64, 8, 128), (32, 2, 128),
                                      (12, 3, 128), (4, 4, 64), (16, 1, 64)])
def test_bf16_fast_path_group_shapes(hq, hkv, d):
    w = W.small(10 + hq + hkv + d, batch=5, ctx_lo=1, ctx_hi=300, hq=hq, hkv=hkv, head_dim=d, dtype="bf16")
    check(w, expect_fast=True)


@pytest.mark.parametrize("split", [16, 32, 64, 112, 512])
def test_bf16_fast_path_split_k(split):
    w = W.small(7, batch=6, ctx_lo=200, ctx_hi=1500, hq=28, hkv=4, head_dim=128, dtype="bf16")
    check(w, split_tokens=split, expect_fast=True)


def test_bf16_fast_path_partial_last_blocks_and_tiny_contexts():
    w = W.small(8, batch=12, ctx_lo=1, ctx_hi=40, hq=28, hkv=4, head_dim=128, dtype="bf16")
    ctx = w.context_lens.copy()
    ctx[:4] = [1, 15, 16, 17]
    w = W.with_contexts(w, ctx)
    check(w, expect_fast=True)


def test_bf16_padded_slots_hold_nan_without_leaking():
    # slots past each context inside the last block hold NaN; the kernel
    # must neither read them into the softmax nor let 0 * NaN reach out
    w = W.small(9, batch=4, ctx_lo=3, ctx_hi=60, hq=28, hkv=4, head_dim=128, dtype="bf16")
    w = W.with_contexts(w, [3, 17, 33, 60])
    pool, q = W.host_inputs(w)
    poolv = pool.reshape(w.num_blocks, w.block_stride)
    row = w.num_kv_heads * w.head_dim * 2
    for b, c in enumerate(w.context_lens):
        last = w.tables[b, (c - 1) // 16]
        for t in range(c % 16 or 16, 16):
            for s in range(2):
                off = (s * 16 + t) * row
                poolv[last, off:off + row] = np.frombuffer(np.full(row // 2, 0x7FC0, np.uint16).tobytes(), np.uint8)
    ref, status = oracle.port_decode(w, pool, q)
    st, out, err, _ = gpu_decode(w, pool, q)
    assert st == 0 and err == 0
    assert np.isfinite(out).all()
    assert np.max(np.abs(out - ref)) < BF16_ABS


def test_bf16_second_layer_of_a_multi_layer_block():
    w = W.small(11, batch=3, ctx_lo=20, ctx_hi=200, hq=28, hkv=4, head_dim=128, dtype="bf16", num_layers=2,
                layer=1)
    check(w, expect_fast=True)


@pytest.mark.parametrize("kw", [
    dict(hq=8, hkv=2, head_dim=96, dtype="bf16"),                          # head_dim not 64/128
    dict(hq=34, hkv=2, head_dim=128, dtype="bf16"),                        # group of 17 > 16
    dict(hq=8, hkv=2, head_dim=128, dtype="bf16", tokens_per_block=8),     # 8-token blocks
    dict(hq=6, hkv=3, head_dim=32, dtype="f32", tokens_per_block=4),
    dict(hq=4, hkv=1, head_dim=256, dtype="f32", tokens_per_block=32),
])
def test_generic_path_shapes(kw):
    w = W.small(12, batch=4, ctx_lo=1, ctx_hi=200, **kw)
    check(w, expect_fast=False)


def test_generic_path_split_k_fp32():
    w = W.small(13, batch=3, ctx_lo=300, ctx_hi=900, hq=8, hkv=2, head_dim=64, dtype="f32")
    check(w, split_tokens=100)


def test_cfg2_full_size_matches_the_oracle_on_every_sequence():
    # The full 7B-shaped batch through the default (stream-K) plan, every one
    # of its 64 sequences recomputed by the oracle
    # (tests/PagedAttention.test.cpp:460-495: scattered blocks against a flat
    # reference).
    w = W.cfg2()
    pool, q = W.host_inputs(w)
    st, out, err, plan = gpu_decode(w, pool, q)
    assert st == 0 and err == 0 and plan["stream"]
    ref, status = oracle.port_decode(w, pool, q, threads=os.cpu_count() or 8)
    assert status.all()
    assert np.max(np.abs(out - ref)) < BF16_ABS
    assert np.isfinite(out).all()


def test_cfg4_long_contexts_match_the_oracle():
    # Four sequences of the 72B-shaped config: 32,768 tokens each, 64 query /
    # 8 kv heads (G = 8), scattered blocks.
    w = W.cfg4(batch=4)
    pool, q = W.host_inputs(w)
    st, out, err, plan = gpu_decode(w, pool, q)
    assert st == 0 and err == 0 and plan["stream"]
    ref, status = oracle.port_decode(w, pool, q, threads=os.cpu_count() or 8)
    assert status.all()
    assert np.max(np.abs(out - ref)) < BF16_ABS
    assert np.isfinite(out).all()


def test_decode_is_deterministic_across_calls():
    w = W.small(14, batch=8, ctx_lo=100, ctx_hi=2000, hq=28, hkv=4, head_dim=128, dtype="bf16")
    pool, q = W.host_inputs(w)
    a = gpu_decode(w, pool, q, split_tokens=256)[1]
    b = gpu_decode(w, pool, q, split_tokens=256)[1]
    assert np.array_equal(a, b)


# --- persistent stream-K form (the default for split_tokens = 0) -------------

@pytest.mark.parametrize("kw", [
    dict(batch=300, ctx_lo=1, ctx_hi=40, hq=28, hkv=4, head_dim=128),     # many short segments per CTA
    dict(batch=1, ctx_lo=20000, ctx_hi=20000, hq=28, hkv=4, head_dim=128),  # one segment over all CTAs
    dict(batch=3, ctx_lo=1, ctx_hi=5, hq=28, hkv=4, head_dim=128),        # fewer stages than CTAs
    dict(batch=9, ctx_lo=100, ctx_hi=3000, hq=64, hkv=8, head_dim=128),   # two head groups per sequence
    dict(batch=7, ctx_lo=1, ctx_hi=2000, hq=16, hkv=2, head_dim=64),
    dict(batch=5, ctx_lo=50, ctx_hi=900, hq=8, hkv=1, head_dim=128),
    dict(batch=6, ctx_lo=50, ctx_hi=900, hq=6, hkv=3, head_dim=128),
    dict(batch=40, ctx_lo=1, ctx_hi=3000, hq=64, hkv=4, head_dim=128),   # G = 16: 8 outputs per merging thread
    dict(batch=20, ctx_lo=300, ctx_hi=5000, hq=32, hkv=2, head_dim=64),  # two heads per CTA, G = 16
    dict(batch=2, ctx_lo=30000, ctx_hi=40000, hq=7, hkv=1, head_dim=128),  # one head: hundreds of parts per merge
])
def test_stream_k_matches_the_oracle(kw):
    w = W.small(20 + kw["batch"] + kw["hkv"], dtype="bf16", **kw)
    out, ref, plan = check(w)
    assert plan["stream"], plan


def test_stream_k_falls_back_to_the_grid_kernel_past_2048_segments():
    w = W.small(21, batch=2100, ctx_lo=1, ctx_hi=20, hq=28, hkv=4, head_dim=128, dtype="bf16")
    out, ref, plan = check(w)
    assert plan["fast"] and not plan["stream"]


def test_stream_k_reuses_a_dirty_workspace():
    # the records need no zero-fill: a second call over garbage matches
    w = W.small(22, batch=11, ctx_lo=1, ctx_hi=3000, hq=28, hkv=4, head_dim=128, dtype="bf16")
    pool, q = W.host_inputs(w)
    a = gpu_decode(w, pool, q)[1]
    b = gpu_decode(w, pool, q)[1]
    assert np.array_equal(a, b)
