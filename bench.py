"""Benchmark of the B200 paged-decode path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg2|cfg1|cfg4] [--split TOKENS]

A step is one batched decode (qvp_decode: the decode kernel plus, when a
context is split, the combine kernel) over the workload's whole batch, with
the block pool, tables and queries resident in HBM. The default workload is
the Qwen2-VL-7B-shaped config (cfg2: 64 sequences, ctx ~ U[512, 8192], 28/4
heads, head_dim 128, bf16), whose K/V (~570 MB) exceeds the 126 MB L2, so no
flush is needed between steps.

Metric: algorithmic bytes per step (K + V of every context token, Q, out and
the table entries used) / step time, in GB/s, plus sequences/s.

Multi-GPU (torchrun, one rank per GPU): cfg2 runs one independent batch per
rank (different seeds, no collective on the data path, weak scaling); cfg4
shards the kv heads of one batch across ranks (strong scaling).

Other workloads (one JSON line each, one GPU): `cfg3` copy-on-write and
`cfg5` swap churn through the C++ host layer; `engine`, cfg2-shaped decode
steps through KVCacheManager + PagedDecodeBatch with per-step and resident
block tables; `prefill`, causal prefill of 16 x 2048-token prompts
(qvp_prefill, TFLOP/s).

`--impl reference` times the reference's own CPU paged_attention_decode<T>
(oracle/_ref, compiled from the reference sources; the C restatement when
that library is absent) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "qwenvl-paged_b200"), os.path.join(ROOT, "oracle")]

import numpy as np  # noqa: E402

import workloads as W  # noqa: E402

METRIC = "paged-decode KV GB/s (% of HBM peak) and seqs/s at 1/2/4/8 B200 vs host CPU"
FALLBACK_HBM_GBS = 6650.0

# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the dominant
# kernel (paged_decode_stream) on the default workload, from the ncu capture
# summarised in profiles/paged_decode_stream_cfg2.md.
NCU_TRAFFIC_BYTES = {"cfg2-qwen2vl-7b-decode": 603_664_128 + 4_811_776}


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def dist_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(
        os.environ.get("LOCAL_RANK", "0"))


def make_workload(name, world, shard_mode="hybrid", emulate=0):
    """(workload this rank holds, scaling, head_parts, batch_parts).

    cfg2 over N GPUs splits by kv head first (head_parts = min(N, 4), the 4
    kv heads), then by sequence (batch_parts = N / head_parts). Every GPU
    keeps cfg2's bytes: a head group of head_parts GPUs decodes 64*head_parts
    sequences, each GPU its 4/head_parts kv heads of them (weak scaling).
    `emulate` = H runs, on one GPU, the workload one GPU of an H-way head split
    holds (no collective), for profiling."""
    if name == "cfg2":
        hp = emulate if (emulate and world == 1) else min(world, 4)
        if world % min(world, 4) != 0:
            raise SystemExit(f"cfg2 runs on 1, 2, 4 or 8 GPUs, not {world}")
        return W.cfg2_shard(hp), "weak", (hp if world > 1 else 1), world // min(world, 4)
    if name == "cfg1":
        return W.cfg1(seed=1), "weak", 1, world
    if name == "cfg4":
        if shard_mode == "heads" or (emulate and world == 1):
            n = emulate if (emulate and world == 1) else max(world, 1)
            return W.cfg4(shards=n), "strong", (n if world > 1 else 1), 1
        # kv heads split while every GPU keeps >= 4 of them, then sequences
        import sharding
        hp, dp = sharding.hybrid_grid(8, 32, max(world, 1))
        w = W.cfg4(shards=hp, batch=32 // dp)
        w.meta.update({"head_parts": hp, "batch_parts": dp})
        return w, "strong", hp, dp
    raise SystemExit(f"unknown workload {name}")


class ClockSampler:
    """nvidia-smi clock / throttle sampling while a region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        self.lines += [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for l in self.lines:
            parts = [p.strip() for p in l.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def _device_bytes(ptr, nbytes, dev):
    """A uint8 torch view of `nbytes` of device memory at `ptr` (memory that
    libqvp owns)."""
    import torch

    class _Raw:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                    "strides": None}

    return torch.as_tensor(_Raw(), device=dev)


def run_ours(args):
    import ctypes

    import torch

    import qvp

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    w, scaling, hp, dp = make_workload(args.workload, world, args.shard, args.emulate_shards)
    head_part, batch_part = rank % hp, rank // hp
    sharded = hp > 1
    torch_dtype = torch.bfloat16 if w.dtype == "bf16" else torch.float32

    # inputs generated on the device from a seed, resident in HBM; every rank
    # holds different K/V/Q values (its own heads, or its own sequences)
    g = torch.Generator(device=dev)
    g.manual_seed(w.seed * 1000 + 7 + 7919 * rank)
    pool = torch.zeros(w.num_blocks * w.block_stride // w.elem, dtype=torch_dtype, device=dev)
    pool.view(w.num_blocks, -1)[:, : w.block_bytes // w.elem].normal_(generator=g)
    q = torch.randn(w.batch, w.num_query_heads, w.head_dim, generator=g, device=dev, dtype=torch.float32).to(
        torch_dtype)
    ctx_d = torch.from_numpy(w.context_lens).to(dev)
    tab_d = torch.from_numpy(w.tables).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    shape = qvp.make_shape(w.tokens_per_block, w.num_layers, w.num_kv_heads, w.head_dim, w.elem)
    a = qvp.decode_args(pool=pool.data_ptr(), block_stride=w.block_stride, num_blocks=w.num_blocks, shape=shape,
                        dtype=qvp.DTYPE_BF16 if w.dtype == "bf16" else qvp.DTYPE_F32, layer=0,
                        num_query_heads=w.num_query_heads, scale=w.scale, batch=w.batch,
                        max_blocks_per_seq=w.pitch, max_context_len=w.max_context_len,
                        block_tables=tab_d.data_ptr(), context_lens=ctx_d.data_ptr(), query=q.data_ptr(),
                        out=0, split_tokens=args.split, error_word=err.data_ptr())
    # `out` is what the step hands its consumer: this GPU's heads when the
    # batch is not split by head, every head of its sequences when it is
    out = torch.empty((w.batch, w.num_query_heads * hp, w.head_dim), dtype=torch_dtype, device=dev)
    a.out = out.data_ptr()
    plan = qvp.decode_plan(a)
    ws = None
    if plan["workspace_bytes"]:
        ws = torch.empty(plan["workspace_bytes"], dtype=torch.uint8, device=dev)
        a.workspace = ws.data_ptr()
        a.workspace_bytes = plan["workspace_bytes"]
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    launches_per_step = 1 if plan["stream"] else 1 + (1 if plan["num_splits"] > 1 else 0)
    kernel_name = ("paged_decode_stream (persistent stream-K, TMA + mma.sync, in-kernel merge of split segments)"
                   if plan["stream"]
                   else "paged_decode_fast (grid split-K, TMA + mma.sync) + combine_partitions" if plan["fast"]
                   else "paged_decode_generic + combine_partitions")

    comm = None
    peer = None
    if sharded and not args.no_gather and args.exchange == "peer":
        # every GPU of a head group stores its output rows into every other
        # GPU's buffer over NVLink (libqvp's peer group); handles travel over
        # torch.distributed
        import torch.distributed as dist
        peer = qvp.PeerGroup(head_part, hp, out.numel() * out.element_size())
        handles = [None] * world
        dist.all_gather_object(handles, peer.handle)
        peer.open(handles[batch_part * hp:(batch_part + 1) * hp])
        launches_per_step += 1  # peer_signal_wait
    elif sharded and not args.no_gather:
        # one NCCL communicator per head group (the hp GPUs that share a batch),
        # made by libqvp; the unique id travels over torch.distributed
        import torch.distributed as dist
        ids = [None] * world
        dist.all_gather_object(ids, qvp.nccl_unique_id() if head_part == 0 else None)
        comm = qvp.nccl_comm_init(ids[batch_part * hp], hp, head_part)
        launches_per_step += 1  # reassemble_kernel (the NCCL all-gather is a library collective, not counted)

    def shard_args(decode_args, out_ptr, gathered_ptr):
        return qvp.shard_decode_args(decode_args, head_part, hp, local, comm, gathered_ptr, out_ptr)

    gathered = []
    sa = None
    if peer is not None:
        sa = shard_args(a, 0, 0)
    elif comm is not None:
        sa = shard_args(a, out.data_ptr(), 0)
        gathered.append(torch.empty(qvp.shard_gather_bytes(sa), dtype=torch.uint8, device=dev))
        sa.gathered = gathered[0].data_ptr()

    peer_step = [0]

    def run_step(decode_args, shard_decode_args, st, copy_to=None):
        if peer is not None:
            rc = peer.decode(shard_decode_args, peer_step[0], err.data_ptr(), st)
            what = "qvp_shard_decode_peer"
            if rc == 0 and copy_to is not None:
                # the step's output (every head) sits in the group buffer of
                # this step's parity; hand it to the download buffer
                nbytes = copy_to.numel() * copy_to.element_size()
                copy_to.view(-1).view(torch.uint8).copy_(
                    _device_bytes(peer.output(peer_step[0]), nbytes, dev), non_blocking=True)
            peer_step[0] += 1
        elif shard_decode_args is not None:
            rc = qvp.lib.qvp_shard_decode(ctypes.byref(shard_decode_args), st)
            what = "qvp_shard_decode"
        else:
            rc = qvp.decode(decode_args, st)
            what = "qvp_decode"
        if rc != 0:
            raise RuntimeError(f"{what} failed: {rc} {qvp.last_error()}")

    def step():
        run_step(a, sa, sh)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def timed(fn, steps):
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms = e0.elapsed_time(e1)
        if world > 1:
            import torch.distributed as dist
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    sampler = ClockSampler(local)
    sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    total_ms = timed(step, args.steps)
    # Clocks: the timed region of a short run can be shorter than the sampling
    # period, so keep the same step running untimed until ~1 s has elapsed
    # (every rank runs the same number of extra steps: the collective matches).
    n_extra = 0
    if not args.profile:
        per = max(total_ms / args.steps, 1e-3)
        n_extra = int(1000.0 / per) + 1
        if world > 1:
            import torch.distributed as dist
            t = torch.tensor([n_extra], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            n_extra = int(t.item())
        for i in range(n_extra):
            step()
            if i % 64 == 63:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
    sampler.stop()
    if int(err.item()) != 0:
        raise RuntimeError(f"decode kernel reported device error bits {int(err.item())}")
    if peer is not None:
        # the device-resident run's output: every head of the last step
        out.view(-1).view(torch.uint8).copy_(_device_bytes(peer.output(peer_step[0] - 1), out.numel() * 2, dev))
        torch.cuda.synchronize()

    ms_step = total_ms / args.steps
    alg = w.algorithmic_bytes()
    # every rank moves its own algorithmic bytes (its batch, or its heads)
    world_bytes = alg * world
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([float(alg)], device=dev, dtype=torch.float64)
        dist.all_reduce(t)  # the bytes every rank actually moved
        world_bytes = int(t.item())
    value = world_bytes / (ms_step * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    achieved = alg / (ms_step * 1e-3) / 1e9  # per GPU

    # e2e through the C ABI with host buffers. Every step copies its own
    # inputs (block tables, context lengths and queries, packed in one pinned
    # buffer) host -> device, runs the decode (and, for kv-head shards, the
    # all-gather of every head) and copies its outputs back to pinned host
    # memory, all inside the timed region. As in a serving engine the copies
    # run on two copy streams, double-buffered, so step k+1's upload and step
    # k's download overlap step k's decode.
    nb_tab, nb_ctx = w.tables.nbytes, w.context_lens.nbytes
    nb_q = q.numel() * q.element_size()
    off_ctx = nb_tab
    off_q = (nb_tab + nb_ctx + 255) // 256 * 256
    host_in = torch.zeros(off_q + nb_q, dtype=torch.uint8).pin_memory()
    host_in[:nb_tab] = torch.from_numpy(w.tables.view(np.uint8).reshape(-1))
    host_in[off_ctx:off_ctx + nb_ctx] = torch.from_numpy(w.context_lens.view(np.uint8).reshape(-1))
    host_in[off_q:] = q.cpu().contiguous().view(torch.uint8).reshape(-1)
    dev_in = [torch.empty_like(host_in, device=dev) for _ in range(2)]
    dev_out = [torch.empty_like(out) for _ in range(2)]
    host_out = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    args2, sargs2 = [], []
    for b in range(2):
        ab = qvp.DecodeArgs()
        ctypes.memmove(ctypes.byref(ab), ctypes.byref(a), ctypes.sizeof(a))
        ab.block_tables = dev_in[b].data_ptr()
        ab.context_lens = dev_in[b].data_ptr() + off_ctx
        ab.query = dev_in[b].data_ptr() + off_q
        ab.out = dev_out[b].data_ptr()
        args2.append(ab)
        if peer is not None:
            sargs2.append(shard_args(ab, 0, 0))
        elif comm is not None:
            gathered.append(torch.empty_like(gathered[0]))
            sargs2.append(shard_args(ab, dev_out[b].data_ptr(), gathered[-1].data_ptr()))
        else:
            sargs2.append(None)
    up_s, down_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_up = [torch.cuda.Event() for _ in range(2)]
    ev_dec = [torch.cuda.Event() for _ in range(2)]
    ev_down = [torch.cuda.Event() for _ in range(2)]

    def e2e_run(n):
        for i in range(n):
            b = i % 2
            up_s.wait_event(ev_dec[b])  # step i-2 has finished reading buffer b
            with torch.cuda.stream(up_s):
                dev_in[b].copy_(host_in, non_blocking=True)
            ev_up[b].record(up_s)
            stream.wait_event(ev_up[b])
            stream.wait_event(ev_down[b])  # step i-2's outputs have left buffer b
            run_step(args2[b], sargs2[b], sh, copy_to=dev_out[b] if peer is not None else None)
            ev_dec[b].record(stream)
            down_s.wait_event(ev_dec[b])
            with torch.cuda.stream(down_s):
                host_out[b].copy_(dev_out[b], non_blocking=True)
            ev_down[b].record(down_s)
        stream.wait_event(ev_down[(n - 1) % 2])  # the timed region ends with the last download

    e2e_ms = float("nan")
    if not args.profile:
        e2e_run(args.warmup)
        torch.cuda.synchronize()
        e2e_ms = timed(lambda: e2e_run(args.steps), 1) / args.steps
        if not torch.equal(host_out[(args.steps - 1) % 2], out.cpu()):
            raise RuntimeError("e2e outputs differ from the device-resident run")
    h2d = q.numel() * q.element_size() + w.tables.nbytes + w.context_lens.nbytes
    d2h = out.numel() * out.element_size()

    cpu = parity = None
    if rank == 0 and world == 1 and not (args.no_cpu or args.profile or args.emulate_shards):
        host_pool = pool.view(torch.uint8).cpu().numpy() if w.elem == 2 else pool.cpu().numpy().view(np.uint8)
        host_q = q.cpu().view(torch.int16).numpy().view(np.uint16) if w.dtype == "bf16" else q.cpu().numpy()
        ref_out, ref_status, cpu = cpu_baseline(w, host_pool.reshape(-1), host_q, budget_s=args.cpu_budget)
        # parity on the bytes that were timed: the GPU output of the measured
        # step against the reference's output for every sequence of the batch
        gpu_out = out.float().cpu().numpy()
        tol = 2e-2 if w.dtype == "bf16" else 1e-5 * max(1.0, float(np.abs(ref_out).max()))
        max_err = float(np.max(np.abs(gpu_out - ref_out)))
        parity = {"max_abs_err": max_err, "tol": tol, "sequences": int(w.batch),
                  "against": cpu["kind"], "reference_ok": bool(ref_status.all()),
                  "pass": bool(max_err <= tol and ref_status.all())}

    if comm is not None:
        torch.cuda.synchronize()
        qvp.nccl_comm_destroy(comm)
    if peer is not None:
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist
            dist.barrier()  # no peer may still store into this GPU's buffers
        peer.close()

    if rank == 0:
        traffic = NCU_TRAFFIC_BYTES.get(w.name)
        global_batch = w.batch * dp
        if sharded:
            exch = ("; per step: decode storing every head's rows into every GPU of the head group over NVLink "
                    "+ a flag exchange (libqvp peer group), inside the timed region" if peer is not None else
                    "; per step: decode + NCCL all-gather (libqvp, in place) + reassemble kernel to [B, Hq, D] "
                    "inside the timed region")
            parallelism = (f"kv-head shards x{hp} (each GPU {w.num_kv_heads} kv / {w.num_query_heads} q heads) "
                           f"x sequence groups x{dp}" + ("" if args.no_gather else exch))
        elif world > 1:
            parallelism = f"sequence groups x{dp} (one batch per GPU, no collective)"
        else:
            parallelism = "1 GPU" + (f" (emulating one GPU of a {args.emulate_shards}-way kv-head split, no "
                                     f"collective)" if args.emulate_shards else "")
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 5),
            "higher_is_better": True,
            "scaling": scaling,
            "vs_baseline": None,
            "dtype": w.dtype,
            "data": "synthetic: seeded N(0,1) K/V/Q, seeded context lengths and scattered block tables",
            "config": {
                "workload": w.name,
                "batch_per_gpu": w.batch,
                "global_batch": global_batch,
                "context_lens": f"{int(w.context_lens.min())}..{int(w.context_lens.max())} "
                                f"(sum {int(w.context_lens.sum())})",
                "heads": f"{w.num_query_heads}q/{w.num_kv_heads}kv per GPU",
                "head_dim": w.head_dim,
                "tokens_per_block": w.tokens_per_block,
                "pool_blocks": w.num_blocks,
                "split_tokens": plan["split_tokens"],
                "num_splits_max": plan["num_splits"],
                "kernel": kernel_name,
                "l2": f"inputs larger than L2 ({w.kv_bytes() / 1e6:.0f} MB of K/V read per step per GPU)",
                "parallelism": parallelism,
            },
            "seqs_per_s": round(global_batch / (ms_step * 1e-3), 1),
            "roofline": {
                "bound": "hbm",
                "achieved": round(achieved, 1),
                "peak": peak,
                "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback 6.65 TB/s",
                "traffic": traffic,
                "kernel": f"decode step = {kernel_name}, CUDA events, mean over steps",
                "algorithmic_bytes_per_step": alg,
            },
            "e2e": {
                "value": round(world_bytes / (e2e_ms * 1e-3) / 1e9, 2),
                "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 5),
                "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h),
                "path": ("C ABI qvp_shard_decode_peer" if peer is not None else
                         "C ABI qvp_shard_decode" if comm is not None else "C ABI qvp_decode") +
                        "; per step one H2D of tables+ctx+q from pinned memory and one D2H of "
                        "out, on two copy streams double-buffered against the decode",
            },
            "gpu_launches": launches_per_step * args.steps,
            "clocks": sampler.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if parity is not None:
            line["parity"] = parity
        print(json.dumps(line), flush=True)
        if parity is not None and not parity["pass"]:
            raise SystemExit(f"parity failure against the reference: {parity}")
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline(w, pool, q, budget_s=15.0, threads=None):
    """Times the reference CPU path (or the C restatement) on a bounded
    sample of the same workload: the first sequences of the batch, repeated
    until about `budget_s` seconds of wall time."""
    import oracle

    threads = threads or cpu_threads()
    kind = "reference" if oracle.ref_available() else "port"
    n = w.batch
    sub = W.DecodeWorkload(w.name, w.tokens_per_block, w.num_layers, w.num_kv_heads, w.head_dim, w.dtype,
                           w.num_query_heads, w.scale, w.context_lens[:n].copy(), w.tables[:n].copy(),
                           w.num_blocks, w.seed)
    if kind == "reference":
        r = oracle.RefDecoder(sub, pool)
        r.bind()
        run = lambda: r.decode(q[:n], threads=threads)  # noqa: E731
    else:
        run = lambda: oracle.port_decode(sub, pool, q[:n], threads=threads)  # noqa: E731
    t0 = time.perf_counter()
    ref_out, status = run()
    first = time.perf_counter() - t0
    reps = max(1, min(50, int(budget_s / max(first, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(reps):
        run()
    dt = (time.perf_counter() - t0) / reps
    if kind == "reference":
        r.close()
        if w.dtype == "bf16":
            ref_out = W.bf16_bits_to_f32(ref_out)
    return ref_out, status, {"value": round(sub.algorithmic_bytes() / dt / 1e9, 4), "unit": "GB/s", "cores": threads,
            "kind": kind, "ms_per_step": round(dt * 1e3, 3), "seqs_per_s": round(n / dt, 2),
            "sample": f"all {n} sequences of {w.name} (same seeded bytes as the GPU run), "
                      f"{reps} repetitions after 1 untimed, {threads} threads, "
                      f"all_ok={bool(status.all())}"}


def run_reference(args):
    """The reference CPU decode on the host cores (rank 0 only)."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import oracle

    w, scaling, _, _ = make_workload(args.workload, 1)
    pool, q = W.host_inputs(w)
    threads = cpu_threads()
    kind = "reference" if oracle.ref_available() else "port"
    if kind == "reference":
        r = oracle.RefDecoder(w, pool)
        r.bind()
        fn = lambda: r.decode(q, threads=threads)  # noqa: E731
    else:
        fn = lambda: oracle.port_decode(w, pool, q, threads=threads)  # noqa: E731
    # size the sample so the whole run stays within a few minutes
    t0 = time.perf_counter()
    _, status = fn()
    one = time.perf_counter() - t0
    n_seq = w.batch
    if one * (args.steps + args.warmup) > 150.0:
        n_seq = max(1, int(w.batch * 150.0 / (one * (args.steps + args.warmup))))
    sub = W.DecodeWorkload(w.name, w.tokens_per_block, w.num_layers, w.num_kv_heads, w.head_dim, w.dtype,
                           w.num_query_heads, w.scale, w.context_lens[:n_seq].copy(), w.tables[:n_seq].copy(),
                           w.num_blocks, w.seed)
    if kind == "reference":
        r.bind(sub.context_lens, sub.tables)
        fn = lambda: r.decode(q[:n_seq], threads=threads)  # noqa: E731
    else:
        fn = lambda: oracle.port_decode(sub, pool, q[:n_seq], threads=threads)  # noqa: E731
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    dt = (time.perf_counter() - t0) / args.steps
    value = sub.algorithmic_bytes() / dt / 1e9
    sample = f"{n_seq} of {w.batch} sequences of {w.name} per step, {threads} threads"
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": w.dtype,
        "data": "synthetic: seeded N(0,1) K/V/Q, seeded context lengths and scattered block tables",
        "config": {"workload": w.name, "batch": n_seq, "heads": f"{w.num_query_heads}q/{w.num_kv_heads}kv",
                   "head_dim": w.head_dim, "tokens_per_block": w.tokens_per_block},
        "seqs_per_s": round(n_seq / dt, 2),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if kind == "reference":
        r.close()
    print(json.dumps(line), flush=True)


def run_scenario(args):
    """cfg3 / cfg5 through the C++ host layer (qwenvl-paged_b200/scenarios),
    one JSON line with the scenario's own measurements."""
    import ctypes as C
    lib = C.CDLL(os.path.join(ROOT, "qwenvl-paged_b200", "lib", "libqvp_scenarios.so"))
    buf = C.create_string_buffer(1 << 16)
    if args.workload == "engine":
        lib.qvp_scenario_engine.argtypes = [C.c_int] * 6 + [C.c_char_p, C.c_size_t]
        rc = lib.qvp_scenario_engine(64, 512, 8192, max(args.steps, 1), args.warmup, 2, buf, len(buf))
        metric, key, unit = ("cfg2-shaped decode step through KVCacheManager + PagedDecodeBatch (resident tables), "
                             "algorithmic GB/s on wall time"), "resident_gbs", "GB/s"
    elif args.workload == "cfg3":
        lib.qvp_scenario_cow.argtypes = [C.c_int] * 6 + [C.c_char_p, C.c_size_t]
        rc = lib.qvp_scenario_cow(16, 8, 2048, 64, 3, max(args.steps, 1), buf, len(buf))
        metric, key, unit = "copy-on-write materialisation, batched copy kernel GB/s (read+write)", "cow_gbs", "GB/s"
    else:
        lib.qvp_scenario_swap.argtypes = [C.c_uint32, C.c_double, C.c_double, C.c_int, C.c_int, C.c_int,
                                          C.c_char_p, C.c_size_t]
        coded = args.swap_coding == "compressed"
        rc = lib.qvp_scenario_swap(args.swap_pool_blocks, 0.9, 0.25, 64, 5, int(coded), buf, len(buf))
        how = ("compress kernel writing coded slots to mapped pinned memory" if coded
               else "gather kernel + cudaMemcpyAsync")
        metric, key, unit = f"swap-out GB/s of block bytes to pinned host memory ({how})", "swap_out_gbs", "GB/s"
    if rc < 0:
        raise SystemExit("scenario output overflow")
    d = json.loads(buf.value.decode())
    line = {"metric": metric, "value": d.get(key), "unit": unit, "n_gpus": 1, "higher_is_better": True,
            "data": "synthetic: seeded context lengths, branch lengths and preemption choices", "config": d}
    print(json.dumps(line), flush=True)


def prefill_flops(w, qlens) -> int:
    """4*Hq*D per (query token, visible key): query token t of sequence b
    sees keys [0, ctx_b - ql_b + t]."""
    tot = 0
    for c, ql in zip(w.context_lens.astype(np.int64), np.asarray(qlens, dtype=np.int64)):
        tot += int(ql * (c - ql) + ql * (ql + 1) // 2)
    return 4 * w.num_query_heads * w.head_dim * tot


def measured_tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def run_prefill(args):
    """Causal prefill (qvp_prefill) of Qwen2-VL-7B-shaped prompts: every
    prompt token attends to the keys up to its own position, which the
    reference computes as its decode at every position. One step = one
    qvp_prefill over the whole batch; L2 is flushed before each timed launch
    (the batch's K/V fit in L2)."""
    import ctypes as C

    import torch

    import qvp

    rank, world, local = dist_env()
    if world > 1:
        raise SystemExit("--workload prefill runs on one GPU")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B, L = args.prefill_batch, args.prompt
    w = W.small(5, batch=B, ctx_lo=L, ctx_hi=L, hq=28, hkv=4, head_dim=128, dtype="bf16", pool_factor=1.25)
    w.name = f"prefill-qwen2vl-7b-{B}x{L}"
    ql = np.full(B, L, dtype=np.int32)
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    pool = torch.zeros(w.num_blocks * w.block_stride // 2, dtype=torch.bfloat16, device=dev)
    pool.view(w.num_blocks, -1)[:, : w.block_bytes // 2].normal_(generator=g)
    q = torch.randn(B, L, w.num_query_heads, w.head_dim, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    tab = torch.from_numpy(w.tables).to(dev)
    ctx = torch.from_numpy(w.context_lens).to(dev)
    qld = torch.from_numpy(ql).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    a = qvp.PrefillArgs()
    a.pool, a.block_stride, a.num_blocks = pool.data_ptr(), w.block_stride, w.num_blocks
    a.shape = qvp.make_shape(16, 1, w.num_kv_heads, w.head_dim, 2)
    a.dtype = qvp.DTYPE_BF16
    a.layer, a.num_query_heads, a.scale, a.batch = 0, w.num_query_heads, w.scale, B
    a.max_blocks_per_seq, a.max_query_len = w.pitch, L
    a.block_tables, a.context_lens, a.query_lens = tab.data_ptr(), ctx.data_ptr(), qld.data_ptr()
    a.query, a.out, a.error_word = q.data_ptr(), out.data_ptr(), err.data_ptr()
    stream = torch.cuda.current_stream()

    def step():
        st = qvp.lib.qvp_prefill(C.byref(a), stream.cuda_stream)
        if st != 0:
            raise RuntimeError(f"qvp_prefill failed: {st} {qvp.last_error()}")

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    sampler = ClockSampler(local)
    sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for e0, e1 in evs:
        flush.zero_()
        e0.record(stream)
        step()
        e1.record(stream)
    torch.cuda.synchronize()
    sampler.stop()
    if int(err.item()) != 0:
        raise RuntimeError(f"prefill kernel reported device error bits {int(err.item())}")
    ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / args.steps
    flops = prefill_flops(w, ql)
    tflops = flops / (ms * 1e-3) / 1e12
    peak, peak_kind = measured_tensor_peak()

    # e2e: queries up from pinned host memory, outputs back, inside the timed region
    host_q = q.cpu().pin_memory()
    host_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        q.copy_(host_q, non_blocking=True)
        step()
        host_out.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps

    cpu = None
    if not args.no_cpu:
        # the reference's prefill is its decode at each position: time it on a
        # bounded sample of positions (the last ones of sequence 0, the most
        # expensive), threads over positions
        import oracle
        host_pool = pool.view(torch.uint8).cpu().numpy().reshape(-1)
        qb = host_q.view(torch.int16).numpy().view(np.uint16)
        n = args.prefill_cpu_positions
        seq = np.zeros(n, dtype=np.int64)
        tok = np.arange(L - n, L, dtype=np.int64)
        ctxs = (tok + 1).astype(np.int32)
        sub = W.DecodeWorkload(w.name, 16, 1, w.num_kv_heads, w.head_dim, "bf16", w.num_query_heads, w.scale,
                               ctxs, np.ascontiguousarray(w.tables[seq]), w.num_blocks, w.seed)
        qq = np.ascontiguousarray(qb[seq, tok])
        threads = cpu_threads()
        kind = "reference" if oracle.ref_available() else "port"
        if kind == "reference":
            r = oracle.RefDecoder(sub, host_pool)
            r.bind()
            run = lambda: r.decode(qq, threads=threads)  # noqa: E731
        else:
            run = lambda: oracle.port_decode(sub, host_pool, qq, threads=threads)  # noqa: E731
        t0 = time.perf_counter()
        run()
        dt = time.perf_counter() - t0
        if kind == "reference":
            r.close()
        cflops = 4 * w.num_query_heads * w.head_dim * int(ctxs.astype(np.int64).sum())
        cpu = {"value": round(cflops / dt / 1e12, 6), "unit": "TFLOP/s", "cores": threads, "kind": kind,
               "sample": f"per-position decode of the last {n} positions of sequence 0 ({cflops / 1e9:.1f} GFLOP)"}

    line = {
        "metric": "causal prefill attention TFLOP/s over the paged cache",
        "value": round(tflops, 2),
        "unit": "TFLOP/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) K/V/Q, seeded scattered block tables",
        "config": {"workload": w.name, "batch": B, "prompt_tokens": L, "heads": "28q/4kv", "head_dim": 128,
                   "kernel": "paged_prefill_tc (TMA + tcgen05.mma, S and O in TMEM, causal per-row limits)",
                   "l2": "flushed (256 MiB write) before each timed launch"},
        "roofline": {"bound": "tensor", "achieved": round(tflops, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(tflops / peak, 4),
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json bf16_tflops)" if peak_kind == "measured"
                     else "fallback 1.59 PFLOP/s", "traffic": None, "flops_per_step": flops},
        "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": int(q.numel() * 2), "d2h_bytes_per_step": int(out.numel() * 2),
                "path": "C ABI qvp_prefill; per step the queries H2D from pinned memory and the outputs D2H"},
        "gpu_launches": args.steps,
        "clocks": sampler.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=["cfg2", "cfg1", "cfg4", "cfg3", "cfg5", "prefill", "engine"],
                   default="cfg2")
    p.add_argument("--prompt", type=int, default=2048, help="prefill: prompt tokens per sequence")
    p.add_argument("--prefill-batch", type=int, default=16, help="prefill: sequences")
    p.add_argument("--prefill-cpu-positions", type=int, default=512,
                   help="prefill: positions in the CPU baseline sample")
    p.add_argument("--swap-pool-blocks", type=int, default=1 << 20, help="cfg5 pool size in 64 KiB blocks")
    p.add_argument("--swap-coding", choices=["raw", "compressed"], default="raw",
                   help="cfg5: swap slots verbatim or coded (lossless) by the device")
    p.add_argument("--split", type=int, default=0, help="split-K partition in tokens (0 = auto)")
    p.add_argument("--cpu-budget", type=float, default=15.0, help="seconds of CPU-baseline timing")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    p.add_argument("--no-gather", action="store_true", help="kv-head shards: skip the output all-gather")
    p.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                   help="kv-head shards: outputs to every GPU by NVLink peer stores (peer) or NCCL all-gather")
    p.add_argument("--emulate-shards", type=int, choices=[0, 2, 4, 8], default=0,
                   help="one GPU: run the workload one GPU of an H-way kv-head split holds (profiling)")
    p.add_argument("--shard", choices=["hybrid", "heads"], default="hybrid",
                   help="cfg4 over N GPUs: kv heads only, or kv heads (>= 4 per GPU) then sequences")
    p.add_argument("--profile", action="store_true",
                   help="for ncu: only warm-up and timed decode steps (no clock probe, e2e or CPU baseline)")
    args = p.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "prefill" and args.impl == "ours":
        run_prefill(args)
    elif args.workload in ("cfg3", "cfg5", "engine") and args.impl == "ours":
        run_scenario(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
