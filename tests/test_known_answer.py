"""Known-answer tests of paged decode, re-expressed from the reference suite
(phhuang191129/QwenVL-Paged tests/PagedAttention.test.cpp:255-566).

Each case runs on three back ends: the C oracle (`port`), the reference
compiled from its sources (`ref`, when built) and the CUDA kernels through
the C ABI (`gpu`, marked gpu). Block ids follow what the reference's LIFO
allocator would hand out, including the spacer-scattered tables.
"""
import numpy as np
import pytest

import oracle
from helpers import HostCache, gpu_decode, max_rel_err, pattern, scattered_ids

TOL = 1e-5  # tests/PagedAttention.test.cpp:38

BACKENDS = [
    "port",
    pytest.param("ref", marks=pytest.mark.skipif(not oracle.ref_available(), reason="reference not built")),
    pytest.param("gpu", marks=pytest.mark.gpu),
]


def run(backend, w, pool, q):
    """(ok, out float32 [B, Hq, D]) for one workload on one back end."""
    if backend == "port":
        out, status = oracle.port_decode(w, pool, q)
        return bool(status.all()), out
    if backend == "ref":
        r = oracle.RefDecoder(w, pool)
        out, status = r.decode(q)
        r.close()
        return bool(status.all()), out.astype(np.float32)
    status, out, err, _ = gpu_decode(w, pool, q)
    return status == 0 and err == 0, out


@pytest.mark.parametrize("backend", BACKENDS)
def test_uniform_keys_average_the_cached_values(backend):
    # tests/PagedAttention.test.cpp:380-411
    c = HostCache(tokens_per_block=4, num_layers=1, num_kv_heads=1, head_dim=4, num_blocks=8)
    ids = [7, 6]  # two reserve calls' worth of LIFO frames
    for t in range(8):
        c.write(ids[t // 4], 0, 0, t % 4, 0, np.ones(4))
        c.write(ids[t // 4], 0, 1, t % 4, 0, np.full(4, t + 1.0))
    w = c.workload(hq=1, scale=1.0, context_lens=[8], tables=ids)
    ok, out = run(backend, w, c.pool, np.full((1, 1, 4), 0.5, dtype=np.float32))
    assert ok
    np.testing.assert_allclose(out.ravel(), np.full(4, 4.5), atol=TOL)


@pytest.mark.parametrize("backend", BACKENDS)
def test_selects_each_logical_token_in_order_across_scattered_blocks(backend):
    # tests/PagedAttention.test.cpp:413-458
    c = HostCache(tokens_per_block=4, num_layers=1, num_kv_heads=1, head_dim=8, num_blocks=8)
    ids = scattered_ids(8, 2)
    assert max(ids) - min(ids) + 1 != len(ids)  # physically scattered
    for t in range(8):
        key = np.zeros(8)
        key[t] = 1.0
        c.write(ids[t // 4], 0, 0, t % 4, 0, key)
        c.write(ids[t // 4], 0, 1, t % 4, 0, np.full(8, (t + 1) * 10.0))
    for target in range(8):
        q = np.zeros((1, 1, 8), dtype=np.float32)
        q[0, 0, target] = 1.0
        w = c.workload(hq=1, scale=50.0, context_lens=[8], tables=ids)
        ok, out = run(backend, w, c.pool, q)
        assert ok, target
        np.testing.assert_allclose(out.ravel(), np.full(8, (target + 1) * 10.0), atol=1e-3)


def flat_reference(shape_T, L, H, D, query, layer, hq, ctx, scale):
    """Textbook attention over the pattern() mirror (PagedAttention.test.cpp:146-190)."""
    group = hq // H
    out = np.zeros((hq, D), dtype=np.float32)
    for qh in range(hq):
        kv = qh // group
        q = query[qh]
        scores = np.zeros(ctx, dtype=np.float32)
        for t in range(ctx):
            dot = np.float32(0)
            for d in range(D):
                dot = np.float32(dot + q[d] * pattern(layer, 0, t, kv, d))
            scores[t] = dot * np.float32(scale)
        m = scores.max()
        den = np.float32(0)
        acc = np.zeros(D, dtype=np.float32)
        for t in range(ctx):
            wgt = np.float32(np.exp(scores[t] - m))
            den += wgt
            for d in range(D):
                acc[d] += wgt * pattern(layer, 1, t, kv, d)
        out[qh] = acc / den
    return out


@pytest.mark.parametrize("backend", BACKENDS)
def test_matches_contiguous_reference_on_scattered_blocks(backend):
    # tests/PagedAttention.test.cpp:460-495: 2 layers, 2 kv heads, partial last block
    T, L, H, D, ctx = 4, 2, 2, 4, 10
    c = HostCache(tokens_per_block=T, num_layers=L, num_kv_heads=H, head_dim=D, num_blocks=12)
    ids = scattered_ids(12, 3)
    for layer in range(L):
        for stream in range(2):
            for t in range(ctx):
                for h in range(H):
                    c.write(ids[t // T], layer, stream, t % T, h, [pattern(layer, stream, t, h, d) for d in range(D)])
    query = (0.25 * np.arange(H * D, dtype=np.float32) - 0.5).reshape(1, H, D)
    for layer in range(L):
        w = c.workload(hq=H, scale=0.5, context_lens=[ctx], tables=ids, layer=layer)
        ok, out = run(backend, w, c.pool, query)
        assert ok
        expect = flat_reference(T, L, H, D, query[0], layer, H, ctx, 0.5)
        np.testing.assert_allclose(out[0], expect, atol=TOL)


@pytest.mark.parametrize("backend", BACKENDS)
def test_grouped_query_heads_read_their_own_kv_head(backend):
    # tests/PagedAttention.test.cpp:497-533
    c = HostCache(tokens_per_block=4, num_layers=1, num_kv_heads=2, head_dim=4, num_blocks=4)
    ids = [3]
    for h, val in enumerate((100.0, 200.0)):
        for t in range(4):
            c.write(3, 0, 0, t, h, np.ones(4))
            c.write(3, 0, 1, t, h, np.full(4, val))
    w = c.workload(hq=4, scale=1.0, context_lens=[4], tables=ids)
    ok, out = run(backend, w, c.pool, np.ones((1, 4, 4), dtype=np.float32))
    assert ok
    for qh in range(4):
        np.testing.assert_allclose(out[0, qh], np.full(4, (100.0, 200.0)[qh // 2]), atol=TOL)


@pytest.mark.parametrize("backend", BACKENDS)
def test_forked_branches_see_their_own_cache_after_copy_on_write(backend):
    # tests/PagedAttention.test.cpp:535-566: after CoW, branch 2 owns a
    # private copy (frame 6) whose values were overwritten with 9.
    c = HostCache(tokens_per_block=4, num_layers=1, num_kv_heads=1, head_dim=4, num_blocks=8)
    for t in range(4):
        for blk, v in ((7, 5.0), (6, 9.0)):
            c.write(blk, 0, 0, t, 0, np.ones(4))
            c.write(blk, 0, 1, t, 0, np.full(4, v))
    w = c.workload(hq=1, scale=1.0, context_lens=[4, 4], tables=[[7], [6]])
    ok, out = run(backend, w, c.pool, np.ones((2, 1, 4), dtype=np.float32))
    assert ok
    np.testing.assert_allclose(out[0, 0], np.full(4, 5.0), atol=TOL)
    np.testing.assert_allclose(out[1, 0], np.full(4, 9.0), atol=TOL)


# --- rejections (tests/PagedAttention.test.cpp:255-376) ----------------------

def _base_cache():
    c = HostCache(tokens_per_block=4, num_layers=1, num_kv_heads=1, head_dim=4, num_blocks=4)
    for t in range(4):
        c.write(3, 0, 0, t, 0, np.ones(4))
        c.write(3, 0, 1, t, 0, np.ones(4))
    return c


def test_oracle_rejects_what_the_reference_rejects():
    c = _base_cache()
    q = np.ones((1, 1, 4), dtype=np.float32)
    w = c.workload(hq=1, scale=1.0, context_lens=[4], tables=[3])
    assert oracle.port_decode(w, c.pool, q)[1][0] == 1
    # zero context
    assert oracle.port_decode(w, c.pool, q, context_lens=[0])[1][0] == 0
    # layer beyond the block shape
    w.layer = 1
    assert oracle.port_decode(w, c.pool, q)[1][0] == 0
    w.layer = 0
    # context longer than the mapped blocks
    assert oracle.port_decode(w, c.pool, q, context_lens=[5])[1][0] == 0
    # unmapped (swapped-out) block
    assert oracle.port_decode(w, c.pool, q, tables=[[-1]])[1][0] == 0
    # query heads that do not group onto kv heads
    c2 = HostCache(tokens_per_block=4, num_layers=1, num_kv_heads=2, head_dim=4, num_blocks=4)
    w2 = c2.workload(hq=3, scale=1.0, context_lens=[4], tables=[3])
    assert oracle.port_decode(w2, c2.pool, np.ones((1, 3, 4), dtype=np.float32))[1][0] == 0


@pytest.mark.gpu
def test_gpu_rejects_inconsistent_arguments_on_the_host():
    import qvp
    c = _base_cache()
    q = np.ones((1, 1, 4), dtype=np.float32)
    w = c.workload(hq=1, scale=1.0, context_lens=[4], tables=[3])
    # layer beyond the shape
    w.layer = 1
    st, out, err, _ = gpu_decode(w, c.pool, q, out_init=-1.0)
    assert st == qvp.ERR_INVALID and (out == -1.0).all()
    w.layer = 0
    # context longer than the table can address
    st, out, err, _ = gpu_decode(w, c.pool, q, max_context_len=5, out_init=-1.0)
    assert st == qvp.ERR_INVALID and (out == -1.0).all()
    # query heads that do not group
    c2 = HostCache(tokens_per_block=4, num_layers=1, num_kv_heads=2, head_dim=4, num_blocks=4)
    w2 = c2.workload(hq=3, scale=1.0, context_lens=[4], tables=[3])
    st, out, err, _ = gpu_decode(w2, c2.pool, np.ones((1, 3, 4), dtype=np.float32), out_init=-1.0)
    assert st == qvp.ERR_INVALID and (out == -1.0).all()


@pytest.mark.gpu
def test_gpu_flags_bad_table_entries_without_faulting():
    # An id outside the pool inside the context: the kernel records the bad
    # id in the error word and reads block 0 instead; nothing faults.
    import qvp
    c = _base_cache()
    q = np.ones((1, 1, 4), dtype=np.float32)
    w = c.workload(hq=1, scale=1.0, context_lens=[4], tables=[3])
    for bad in (-1, 4, 1 << 30):
        st, out, err, _ = gpu_decode(w, c.pool, q, tables=[[bad]])
        assert st == 0 and err & qvp.DEVERR_BAD_BLOCK
    # a device context length above the host bound is flagged, not read
    st, out, err, _ = gpu_decode(w, c.pool, q, context_lens=[4], max_context_len=4)
    assert st == 0 and err == 0
