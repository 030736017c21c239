"""Seeded operation scripts for the bookkeeping replay (tests/native/replay_ops.h).

Each script drives allocator, cache-manager and (optionally) scheduler
operations with ids drawn from small ranges, so the interesting edges occur
often: exhausted pools, shared blocks, swapped parents, full swap spaces,
unknown slots and sequences, repeated releases. The hand-written scripts
mirror cases of the reference suite (tests/MemoryAllocator.test.cpp,
tests/KVCacheManager.test.cpp, tests/Scheduler.test.cpp).
"""
import ctypes as C
import hashlib
import os
import random

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
QVP_REPLAY = os.path.join(ROOT, "tests", "native", "libqvp_replay.so")


def random_script(seed: int, n_ops: int = 160, scheduler: bool = False) -> str:
    rng = random.Random(seed)
    T = rng.choice([2, 4, 16])
    blocks = rng.choice([6, 12, 24])
    slots = rng.choice([-1, 0, 3, 8, 64])
    lines = [f"init {T} {rng.choice([1, 2])} {rng.choice([1, 2])} {rng.choice([4, 8])} {rng.choice([2, 4])} "
             f"{blocks} {slots}" + (f" {rng.randint(1, 4)} {rng.randint(T, 6 * T)} {rng.choice([0, 0, 1, 3])}"
                                    if scheduler else "")]
    seqs = list(range(1, 8))
    for _ in range(n_ops):
        if scheduler and rng.random() < 0.45:
            op = rng.choice(["enqueue", "schedule", "schedule", "complete", "cancel", "preempt", "resume"])
            r = rng.randint(1, 6)
            if op == "enqueue":
                lines.append(f"enqueue {r} {100 + r} {rng.randint(1, 5 * T)}")
            elif op == "schedule":
                lines.append("schedule")
            else:
                lines.append(f"{op} {r}")
            continue
        op = rng.choices(["create", "fork", "reserve", "write", "swapout", "swapin", "release", "view", "alloc",
                          "rel", "retain", "copy", "bswapout", "bswapin", "discard", "failstore", "failload"],
                         weights=[8, 6, 12, 12, 5, 5, 5, 3, 4, 4, 3, 2, 3, 3, 2, 1, 1])[0]
        s = rng.choice(seqs)
        if op in ("create", "swapout", "swapin", "release", "view"):
            lines.append(f"{op} {s}")
        elif op == "fork":
            lines.append(f"fork {s} {rng.choice(seqs)}")
        elif op == "reserve":
            lines.append(f"reserve {s} {rng.randint(0, 3 * T)}")
        elif op == "write":
            lines.append(f"write {s} {rng.randint(0, 6 * T)}")
        elif op == "alloc":
            lines.append("alloc")
        elif op in ("failstore", "failload"):
            lines.append(f"{op} {rng.randint(1, 4)}")
        elif op in ("rel", "retain", "bswapout"):
            lines.append(f"{op} {rng.randint(0, blocks)}")
        elif op == "copy":
            lines.append(f"copy {rng.randint(0, blocks)} {rng.randint(0, blocks)}")
        else:
            lines.append(f"{op} {rng.randint(0, 12)}")
    return "\n".join(lines) + "\n"


# Cases of the reference suite, as scripts.
HANDWRITTEN = {
    # ids come out N-1, N-2, ... and a released id is reused first
    "lifo_ids_and_reuse": "init 4 1 1 4 4 4 -1\nalloc\nalloc\nalloc\nalloc\nalloc\nrel 2\nalloc\n",
    # retain needs a matching release; generation advances on recycle
    "retain_release_generation": "init 4 1 1 4 4 4 -1\nalloc\nretain 3\nrel 3\nrel 3\nrel 3\nretain 3\n",
    # fork shares frames, CoW copies the shared block, sole owner writes in place
    "fork_and_copy_on_write": "init 4 1 1 4 4 8 8\ncreate 1\nreserve 1 8\nfork 1 2\nwrite 2 5\nwrite 2 6\n"
                              "write 1 1\nwrite 1 5\nrelease 1\nwrite 2 1\n",
    # swap out skips blocks shared with a fork; fork refuses a swapped parent
    "swap_skips_shared_and_fork_refuses": "init 4 1 1 4 4 8 8\ncreate 1\nreserve 1 12\nfork 1 2\nwrite 2 9\n"
                                          "swapout 2\nfork 2 3\nview 2\nswapin 2\nfork 2 3\n",
    # sequence swap-in is all-or-nothing when the pool cannot back it
    "swap_in_all_or_nothing": "init 4 1 1 4 4 4 8\ncreate 1\nreserve 1 12\nswapout 1\ncreate 2\nreserve 2 8\n"
                              "swapin 1\nrelease 2\nswapin 1\nview 1\n",
    # full swap space, unknown slots, release discards swapped slots
    "swap_space_edges": "init 4 1 1 4 4 6 2\ncreate 1\nreserve 1 16\nswapout 1\nbswapin 99\nrelease 1\n"
                        "alloc\nbswapout 5\nbswapout 4\nbswapin 3\ndiscard 3\n",
    # scheduler: memory pressure keeps requests pending, watermark preempts newest
    "scheduler_watermark": "init 4 1 1 4 4 6 16 3 24 2\nenqueue 1 101 8\nenqueue 2 102 8\nschedule\ncomplete 1\n"
                           "complete 2\nenqueue 3 103 8\nschedule\nschedule\nresume 2\ncancel 1\nresume 2\nschedule\n",
    # fault injection: a store fails in the middle of a sequence swap-out (the
    # rest still move), a load fails in the middle of a swap-in (the frame is
    # released, generation advances, the sequence stays partly swapped)
    "swap_store_failure_mid_sequence": "init 4 1 1 4 4 8 8\ncreate 1\nreserve 1 16\nfailstore 2\nswapout 1\n"
                                       "view 1\nswapin 1\nview 1\n",
    "swap_load_failure_mid_sequence": "init 4 1 1 4 4 8 8\ncreate 1\nreserve 1 16\nswapout 1\nfailload 3\n"
                                      "swapin 1\nview 1\nswapin 1\nview 1\nrelease 1\n",
    "preempt_with_failing_store": "init 4 1 1 4 4 6 16 3 24 0\nenqueue 1 101 8\nenqueue 2 102 8\nschedule\n"
                                  "failstore 1\npreempt 2\nresume 2\nfailload 1\npreempt 1\nresume 1\nresume 1\n",
    "scheduler_no_backend": "init 4 1 1 4 4 4 -1 4 100 1\nenqueue 1 101 12\nenqueue 2 102 8\nschedule\n"
                            "complete 1\nschedule\npreempt 1\nresume 1\ncancel 2\nschedule\n",
}


def golden_cases():
    cases = dict(HANDWRITTEN)
    for seed in range(12):
        cases[f"random_{seed}"] = random_script(seed)
    for seed in range(12, 20):
        cases[f"sched_{seed}"] = random_script(seed, scheduler=True)
    return cases


def _call(path, symbol, script):
    lib = C.CDLL(path)
    fn = getattr(lib, symbol)
    fn.restype = C.c_int
    fn.argtypes = [C.c_char_p, C.c_char_p, C.c_size_t]
    cap = 1 << 22
    while True:
        buf = C.create_string_buffer(cap)
        n = fn(script.encode(), buf, cap)
        if n >= 0:
            return buf.value.decode()
        cap = -n + 16


def replay_qvp(script: str) -> str:
    return _call(QVP_REPLAY, "qvp_replay", script)


def replay_ref(script: str) -> str:
    import oracle
    return _call(oracle.REF_PATH, "ref_replay", script)


def digest(trace: str) -> str:
    return hashlib.sha256(trace.encode()).hexdigest()
