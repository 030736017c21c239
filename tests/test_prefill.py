"""Causal prefill (qvp_prefill): the CPU side.

The oracle is the reference's own definition of prefill - its decode at every
prompt position (PagedAttention.h:43-44) - checked here against the reference
compiled from its sources and against plain numpy causal attention; the host
argument checks of qvp_prefill run without a GPU.
"""
import numpy as np
import pytest

import oracle
import qvp
import workloads as W


def _case(dtype="f32"):
    w = W.small(61, batch=3, ctx_lo=5, ctx_hi=70, hq=8, hkv=2, head_dim=32, dtype=dtype, tokens_per_block=16)
    ql = np.minimum(w.context_lens, np.array([5, 17, 70][: w.batch]))
    pool, _ = W.host_inputs(w)
    rng = np.random.default_rng(7)
    qf = rng.standard_normal((w.batch, int(ql.max()), w.num_query_heads, w.head_dim), dtype=np.float32)
    q = W.f32_to_bf16_bits(qf) if dtype == "bf16" else qf
    return w, pool, q, ql


def test_prefill_oracle_is_causal_attention_over_the_paged_cache():
    w, pool, q, ql = _case()
    out, status = oracle.port_prefill(w, pool, q, ql)
    assert status.all()
    blocks = pool.reshape(w.num_blocks, w.block_stride)[:, : w.block_bytes].view(np.float32)
    blocks = blocks.reshape(w.num_blocks, 1, 2, 16, w.num_kv_heads, w.head_dim)
    G = w.num_query_heads // w.num_kv_heads
    for b in range(w.batch):
        n = int(w.context_lens[b])
        ids = w.tables[b, : (n + 15) // 16]
        K = blocks[ids, 0, 0].reshape(-1, w.num_kv_heads, w.head_dim)[:n].astype(np.float64)
        V = blocks[ids, 0, 1].reshape(-1, w.num_kv_heads, w.head_dim)[:n].astype(np.float64)
        for t in range(int(ql[b])):
            pos = n - int(ql[b]) + t
            for h in range(w.num_query_heads):
                s = K[: pos + 1, h // G] @ q[b, t, h].astype(np.float64) * w.scale
                p = np.exp(s - s.max())
                ref = (p[:, None] * V[: pos + 1, h // G]).sum(0) / p.sum()
                np.testing.assert_allclose(out[b, t, h], ref, rtol=1e-5, atol=1e-5)
    # rows past each query length are not written
    for b in range(w.batch):
        assert not out[b, int(ql[b]):].any()


@pytest.mark.skipif(not oracle.ref_available(), reason="reference not built here")
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_prefill_oracle_matches_the_reference_per_position_decode(dtype):
    w, pool, q, ql = _case(dtype)
    out, _ = oracle.port_prefill(w, pool, q, ql)
    seq, tok, ctx = oracle.prefill_pairs(w, ql)
    r = oracle.RefDecoder(w, pool)
    r.bind(ctx, np.ascontiguousarray(w.tables[seq]))
    ro, st = r.decode(np.ascontiguousarray(q[seq, tok]))
    r.close()
    assert st.all()
    got = out[seq, tok]
    if dtype == "f32":
        assert np.array_equal(got, ro)
    else:
        assert np.array_equal(W.f32_to_bf16_bits(got), ro)


def _args(**kw):
    base = dict(pool=0x1000, block_stride=256, num_blocks=4, shape=qvp.make_shape(4, 1, 1, 4, 4),
                dtype=qvp.DTYPE_F32, layer=0, num_query_heads=1, scale=1.0, batch=1, max_blocks_per_seq=1,
                max_query_len=4, block_tables=0x2000, context_lens=0x3000, query_lens=0x3100, query=0x4000,
                out=0x5000, error_word=None)
    base.update(kw)
    a = qvp.PrefillArgs()
    for k, v in base.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("bad", [
    dict(shape=qvp.make_shape(4, 1, 1, 4, 8)),                     # element size mismatch
    dict(layer=1),                                                 # layer beyond the block shape
    dict(num_query_heads=0),
    dict(shape=qvp.make_shape(4, 1, 2, 4, 4), num_query_heads=3),  # heads that do not group
    dict(max_query_len=0),
    dict(query=None), dict(out=None), dict(query_lens=None),
    dict(block_stride=64),
])
def test_prefill_rejects_inconsistent_arguments_before_any_launch(bad):
    import ctypes as C
    assert qvp.lib.qvp_prefill(C.byref(_args(**bad)), None) == qvp.ERR_INVALID
    assert qvp.last_error()


def test_prefill_with_an_empty_batch_is_a_no_op():
    import ctypes as C
    assert qvp.lib.qvp_prefill(C.byref(_args(batch=0)), None) == qvp.OK


def test_bench_prefill_flops_count_every_visible_key():
    import bench
    w = W.small(3, batch=3, ctx_lo=5, ctx_hi=60, hq=8, hkv=2, head_dim=16, dtype="bf16")
    ql = np.array([1, 4, min(17, int(w.context_lens[2]))], dtype=np.int32)
    ql = np.minimum(ql, w.context_lens)
    _, _, ctx = oracle.prefill_pairs(w, ql)
    assert bench.prefill_flops(w, ql) == 4 * w.num_query_heads * w.head_dim * int(ctx.astype(np.int64).sum())
