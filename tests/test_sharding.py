"""KV-head sharding on CPU: per-shard oracle outputs, all-gathered across
world-size-2 gloo ranks, reassemble to the unsharded result; replicated
bookkeeping gives every rank identical tables."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import oracle
import sharding
import workloads as W


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_sharded_oracle_reassembles_to_the_full_result_in_process():
    w = W.small(41, batch=4, ctx_lo=1, ctx_hi=200, hq=32, hkv=4, head_dim=64, dtype="bf16")
    pool, q = W.host_inputs(w)
    full, st = oracle.port_decode(w, pool, q)
    for world in (2, 4):
        parts = []
        for r in range(world):
            sw = sharding.shard_workload(w, world)
            parts.append(oracle.port_decode(sw, sharding.shard_pool(pool, w, world, r),
                                            sharding.shard_query(q, w.num_kv_heads, world, r))[0])
        assert np.array_equal(sharding.assemble(parts), full)


def _rank_main(rank, world, port, result):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w = W.small(42, batch=3, ctx_lo=10, ctx_hi=150, hq=16, hkv=2, head_dim=64, dtype="f32")
    pool, q = W.host_inputs(w)
    sw = sharding.shard_workload(w, world)
    out, st = oracle.port_decode(sw, sharding.shard_pool(pool, w, world, rank),
                                 sharding.shard_query(q, w.num_kv_heads, world, rank))
    gathered = sharding.all_gather_heads(torch.from_numpy(out)).numpy()
    full, _ = oracle.port_decode(w, pool, q)
    # replicated bookkeeping: the same script gives every rank the same trace
    import replay_scripts as R
    trace = R.replay_qvp(R.random_script(7))
    digests = [None] * world
    dist.all_gather_object(digests, R.digest(trace))
    result[rank] = bool(np.array_equal(gathered, full)) and len(set(digests)) == 1
    dist.destroy_process_group()


def test_gloo_world_size_2_gather_and_replicated_bookkeeping():
    port = _free_port()
    mgr = mp.Manager()
    result = mgr.dict()
    mp.spawn(_rank_main, args=(2, port, result), nprocs=2, join=True)
    assert result[0] and result[1]


def test_head_range_rejects_uneven_splits():
    assert sharding.head_range(8, 4, 3) == (6, 8)
    with pytest.raises(ValueError):
        sharding.head_range(4, 8, 0)


def test_hybrid_grid_keeps_four_heads_per_gpu_then_splits_sequences():
    assert sharding.hybrid_grid(8, 32, 1) == (1, 1)
    assert sharding.hybrid_grid(8, 32, 2) == (2, 1)
    assert sharding.hybrid_grid(8, 32, 4) == (2, 2)
    assert sharding.hybrid_grid(8, 32, 8) == (2, 4)
    assert sharding.hybrid_grid(4, 64, 8) == (1, 8)


def test_hybrid_assembly_restores_batch_and_head_order():
    import torch
    full = torch.arange(8 * 16 * 4, dtype=torch.float32).reshape(8, 16, 4)
    hp, dp = 2, 4
    parts = []
    for r in range(hp * dp):
        h, d = sharding.hybrid_coords(r, hp)
        parts.append(full[d * 2:(d + 1) * 2, h * 8:(h + 1) * 8])
    assert torch.equal(sharding.assemble_hybrid(parts, hp, dp), full)


def _dying_rank_main(rank, world, port, result):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=4))
    if rank == 1:
        # leaves between steps, with nothing in flight
        os._exit(0)
    try:
        sharding.all_gather_heads(torch.zeros(2, 4, 8))
        result[rank] = "no error"
    except Exception as e:  # the survivor's collective ends with an error, not a hang
        result[rank] = type(e).__name__


def test_a_rank_that_leaves_makes_the_next_gather_fail_instead_of_hanging():
    import multiprocessing as mpx
    import time
    port = _free_port()
    mgr = mp.Manager()
    result = mgr.dict()
    ctx = mpx.get_context("spawn")
    procs = [ctx.Process(target=_dying_rank_main, args=(r, 2, port, result)) for r in range(2)]
    t0 = time.time()
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    assert all(not p.is_alive() for p in procs)
    assert result.get(0) not in (None, "no error")
    assert time.time() - t0 < 60
