// Benchmark scenarios that exercise the host layer end to end on one GPU:
//   cfg3  copy-on-write parallel sampling (fork a prompt into n branches, let
//         every branch append private tokens, materialise the shared last
//         block with one batched copy launch, decode all branches);
//   cfg5  preemption / swap churn on a 1,048,576-block pool (swap out a
//         seeded quarter of the resident sequences to pinned host memory,
//         decode the rest, swap them back in);
//   engine  cfg2-shaped decode steps through KVCacheManager and
//         PagedDecodeBatch, with per-step and with resident block tables.
// Each returns one JSON object of measurements. Loaded by bench.py
// (--workload cfg3 / cfg5 / engine) from qwenvl-paged_b200/lib/libqvp_scenarios.so.
#include "qwenvl_paged/KVCacheManager.h"
#include "qwenvl_paged/MemoryAllocator.h"
#include "qwenvl_paged/PagedAttention.h"
#include "qwenvl_paged/SwapBackend.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <sstream>
#include <string>
#include <vector>

using namespace qwenvl_paged;

namespace {

BlockShape bf16_shape(std::uint32_t heads) {
    BlockShape s;
    s.tokens_per_block = 16;
    s.num_layers = 1;
    s.num_kv_heads = heads;
    s.head_dim = 128;
    s.bytes_per_element = 2;
    return s;
}

struct Events {
    cudaEvent_t a, b;
    Events() {
        cudaEventCreate(&a);
        cudaEventCreate(&b);
    }
    ~Events() {
        cudaEventDestroy(a);
        cudaEventDestroy(b);
    }
    float ms() {
        float m = 0.f;
        cudaEventSynchronize(b);
        cudaEventElapsedTime(&m, a, b);
        return m;
    }
};

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

int emit(const std::string& s, char* out, size_t cap) {
    if (s.size() + 1 > cap) return -static_cast<int>(s.size() + 1);
    std::memcpy(out, s.c_str(), s.size() + 1);
    return static_cast<int>(s.size());
}

// Random bf16 query for `batch` sequences on the device.
void* device_query(std::size_t elems, std::uint32_t seed) {
    std::vector<bfloat16> h(elems);
    std::mt19937 rng(seed);
    std::normal_distribution<float> nd;
    for (auto& x : h) x = bfloat16(nd(rng));
    void* d = nullptr;
    cudaMalloc(&d, elems * 2);
    cudaMemcpy(d, h.data(), elems * 2, cudaMemcpyHostToDevice);
    return d;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int qvp_scenario_cow(int prompts, int branches, int prompt_tokens,
                                                                        int max_append, int seed, int reps,
                                                                        char* out, size_t cap) {
    const BlockShape sh = bf16_shape(4);
    const std::uint32_t T = sh.tokens_per_block;
    const std::uint32_t per_prompt_blocks = (prompt_tokens + 1 + T - 1) / T;
    const std::uint32_t pool_blocks =
        prompts * (per_prompt_blocks + branches * ((max_append + T - 1) / T + 1)) + 64;
    AllocatorConfig cfg;
    cfg.block_shape = sh;
    cfg.max_blocks = pool_blocks;
    MemoryAllocator alloc(cfg);
    if (!alloc.has_storage()) return emit("{\"error\": \"pool allocation failed\"}", out, cap);
    KVCacheManager cache(alloc);
    std::mt19937 rng(seed);
    std::uniform_int_distribution<int> append(1, max_append);

    // prompts of prompt_tokens (+1 slot so the first decode token shares the
    // prompt's last block, which is what copy-on-write must materialise)
    std::vector<SequenceId> seqs;
    std::vector<std::uint32_t> ctx;
    SequenceId next = 1;
    for (int p = 0; p < prompts; ++p) {
        const SequenceId root = next++;
        cache.create_sequence(SequenceMetadata{root, root, {}, {}});
        cache.reserve_tokens(root, prompt_tokens + 1);
        seqs.push_back(root);
        for (int b = 1; b < branches; ++b) {
            const SequenceId child = next++;
            cache.fork_sequence(root, SequenceMetadata{child, root, {}, {}});
            seqs.push_back(child);
        }
    }
    const std::uint64_t copies_before = alloc.copies_done();
    const double t_host0 = now_s();
    std::size_t cow_tokens = 0;
    for (SequenceId s : seqs) {
        const int n = append(rng);
        for (int t = 0; t < n; ++t) {
            const std::uint32_t pos = static_cast<std::uint32_t>(prompt_tokens + t);
            const auto v = cache.cache_view(s);
            if (pos >= v->block_table->size() * T) cache.reserve_tokens(s, T);
            (void)cache.ensure_token_writable(s, pos);
            ++cow_tokens;
        }
        ctx.push_back(static_cast<std::uint32_t>(prompt_tokens + n));
    }
    const double host_s = now_s() - t_host0;
    // the queued copies: one batched launch, timed on the engine stream
    Events ev;
    cudaEventRecord(ev.a, alloc.stream());
    alloc.flush();
    cudaEventRecord(ev.b, alloc.stream());
    const float first_ms = ev.ms();
    const std::uint64_t copies = alloc.copies_done() - copies_before;
    // the same copies again, `reps` times, for a steady timing
    std::vector<std::pair<PhysicalBlockId, PhysicalBlockId>> pairs;
    for (SequenceId s : seqs) {
        const auto v = cache.cache_view(s);
        const auto& e = v->block_table->entries()[per_prompt_blocks - 1];
        const auto root_view = cache.cache_view(((s - 1) / branches) * branches + 1);
        const PhysicalBlockId src = root_view->block_table->entries()[per_prompt_blocks - 1].physical_id;
        if (e.physical_id != src) pairs.push_back({src, e.physical_id});
    }
    cudaEventRecord(ev.a, alloc.stream());
    for (int r = 0; r < reps; ++r) {
        for (auto& pr : pairs) alloc.copy_block(pr.first, pr.second);
        alloc.flush();
    }
    cudaEventRecord(ev.b, alloc.stream());
    const float copy_ms = ev.ms() / std::max(reps, 1);
    const double copy_bytes = 2.0 * static_cast<double>(pairs.size()) * alloc.block(0)->size_bytes();

    // decode every branch over its (shared-prefix) table
    std::vector<CacheView> views;
    for (SequenceId s : seqs) views.push_back(*cache.cache_view(s));
    const std::uint32_t hq = 28;
    const std::size_t qel = seqs.size() * hq * sh.head_dim;
    void* q = device_query(qel, seed + 1);
    void* o = nullptr;
    cudaMalloc(&o, qel * 2);
    PagedDecodeBatch batch(alloc);
    const float scale = 1.f / std::sqrt(128.f);
    for (int w = 0; w < 3; ++w) batch.run(views, ctx, 0, hq, scale, q, o);
    cudaEventRecord(ev.a, alloc.stream());
    for (int r = 0; r < reps; ++r) batch.run(views, ctx, 0, hq, scale, q, o);
    cudaEventRecord(ev.b, alloc.stream());
    const float dec_ms = ev.ms() / std::max(reps, 1);
    double logical = 0;
    for (std::uint32_t c : ctx) logical += 2.0 * c * sh.num_kv_heads * sh.head_dim * 2;
    const double unique = static_cast<double>(alloc.stats().active_blocks + alloc.stats().shared_blocks) *
                          alloc.block(0)->size_bytes();
    const int derr = batch.device_error();
    cudaFree(q);
    cudaFree(o);

    std::ostringstream js;
    js << "{\"workload\": \"cfg3-cow-parallel-sampling\", \"prompts\": " << prompts << ", \"branches\": " << branches
       << ", \"prompt_tokens\": " << prompt_tokens << ", \"sequences\": " << seqs.size()
       << ", \"cow_copies\": " << copies << ", \"cow_first_flush_us\": " << first_ms * 1e3
       << ", \"cow_launch_us\": " << copy_ms * 1e3 << ", \"cow_bytes_rw\": " << copy_bytes
       << ", \"cow_gbs\": " << copy_bytes / (copy_ms * 1e-3) / 1e9 << ", \"host_bookkeeping_ms\": " << host_s * 1e3
       << ", \"appended_tokens\": " << cow_tokens << ", \"decode_us\": " << dec_ms * 1e3
       << ", \"decode_logical_gbs\": " << logical / (dec_ms * 1e-3) / 1e9
       << ", \"decode_unique_block_gbs\": " << unique / (dec_ms * 1e-3) / 1e9 << ", \"decode_device_error\": " << derr
       << ", \"decode_ok\": " << (batch.last_status() == 0 ? "true" : "false") << "}";
    return emit(js.str(), out, cap);
}

extern "C" __attribute__((visibility("default"))) int qvp_scenario_swap(std::uint32_t pool_blocks, double occupancy,
                                                                         double preempt_fraction, int decode_batch,
                                                                         int seed, int compressed, char* out,
                                                                         size_t cap) {
    const BlockShape sh = bf16_shape(8);
    AllocatorConfig cfg;
    cfg.block_shape = sh;
    cfg.max_blocks = pool_blocks;
    const double t0 = now_s();
    MemoryAllocator alloc(cfg);
    if (!alloc.has_storage()) return emit("{\"error\": \"pool allocation failed: " + alloc.last_error() + "\"}", out, cap);
    const double pool_s = now_s() - t0;
    {
        // K/V-like contents (N(0,1) bf16) in every frame, so the compressed
        // slots code what serving would swap: one 4 MiB tile, repeated
        const std::size_t tile = std::size_t(4) << 20;
        void* t = device_query(tile / 2, seed + 11);
        const std::size_t total = static_cast<std::size_t>(pool_blocks) * alloc.block_stride();
        for (std::size_t off = 0; off < total; off += tile)
            cudaMemcpyAsync(alloc.pool_base() + off, t, std::min(tile, total - off), cudaMemcpyDeviceToDevice,
                            alloc.stream());
        cudaStreamSynchronize(alloc.stream());
        cudaFree(t);
    }
    KVCacheManager cache(alloc);
    std::mt19937 rng(seed);
    std::uniform_int_distribution<int> ctxd(512, 8192);
    std::vector<SequenceId> seqs;
    std::vector<std::uint32_t> ctx;
    const std::uint32_t target = static_cast<std::uint32_t>(occupancy * pool_blocks);
    SequenceId next = 1;
    while (true) {
        const std::uint32_t c = static_cast<std::uint32_t>(ctxd(rng));
        const std::uint32_t need = (c + 15) / 16;
        if (pool_blocks - alloc.stats().free_blocks + need > target) break;
        cache.create_sequence(SequenceMetadata{next, next, {}, {}});
        cache.reserve_tokens(next, c);
        seqs.push_back(next++);
        ctx.push_back(c);
    }
    std::vector<std::size_t> order(seqs.size());
    for (std::size_t i = 0; i < order.size(); ++i) order[i] = i;
    std::shuffle(order.begin(), order.end(), rng);
    const std::size_t n_pre = static_cast<std::size_t>(preempt_fraction * seqs.size());
    std::vector<std::size_t> pre(order.begin(), order.begin() + n_pre);
    std::vector<std::size_t> stay(order.begin() + n_pre, order.end());
    std::size_t pre_blocks = 0;
    for (std::size_t i : pre) pre_blocks += (ctx[i] + 15) / 16;

    const double t1 = now_s();
    DeviceSwapBackend swap(alloc, pre_blocks + 16, compressed ? SwapCoding::compressed : SwapCoding::raw);
    const double pin_s = now_s() - t1;
    if (!swap.ready()) return emit("{\"error\": \"pinned slab allocation failed\"}", out, cap);
    alloc.set_swap_backend(&swap);

    // link peak probe: one 1 GiB pinned copy each way
    const std::size_t probe = std::min<std::size_t>(std::size_t(1) << 30, pre_blocks * 65536);
    Events ev;
    void* hbuf = nullptr;
    cudaHostAlloc(&hbuf, probe, cudaHostAllocDefault);
    cudaEventRecord(ev.a, alloc.stream());
    cudaMemcpyAsync(hbuf, alloc.pool_base(), probe, cudaMemcpyDeviceToHost, alloc.stream());
    cudaEventRecord(ev.b, alloc.stream());
    const double d2h_peak = probe / (ev.ms() * 1e-3) / 1e9;
    cudaEventRecord(ev.a, alloc.stream());
    cudaMemcpyAsync(alloc.pool_base(), hbuf, probe, cudaMemcpyHostToDevice, alloc.stream());
    cudaEventRecord(ev.b, alloc.stream());
    const double h2d_peak = probe / (ev.ms() * 1e-3) / 1e9;
    cudaFreeHost(hbuf);

    // decode batch over sequences that stay resident
    const std::uint32_t hq = 64;
    const int B = std::min<int>(decode_batch, static_cast<int>(stay.size()));
    std::vector<CacheView> views;
    std::vector<std::uint32_t> bctx;
    for (int b = 0; b < B; ++b) bctx.push_back(ctx[stay[b]]);
    const std::size_t qel = static_cast<std::size_t>(B) * hq * sh.head_dim;
    void* q = device_query(qel, seed + 3);
    void* o = nullptr;
    cudaMalloc(&o, qel * 2);
    PagedDecodeBatch batch(alloc);
    auto refresh = [&]() {
        views.clear();
        for (int b = 0; b < B; ++b) views.push_back(*cache.cache_view(seqs[stay[b]]));
    };
    refresh();
    for (int w = 0; w < 3; ++w) batch.run(views, bctx, 0, hq, 0.0884f, q, o);
    cudaEventRecord(ev.a, alloc.stream());
    for (int r = 0; r < 10; ++r) batch.run(views, bctx, 0, hq, 0.0884f, q, o);
    cudaEventRecord(ev.b, alloc.stream());
    const double decode_ms = ev.ms() / 10;

    // swap out: host bookkeeping, then one flush of all moves
    const double h0 = now_s();
    std::uint64_t swapped = 0;
    for (std::size_t i : pre) swapped += cache.swap_out_sequence(seqs[i]);
    const double out_host_s = now_s() - h0;
    // the moves run on the backend's copy stream, after the engine's work
    cudaStream_t cs = swap.copy_stream();
    cudaEventRecord(ev.a, alloc.stream());
    const double f0 = now_s();
    alloc.flush();
    const double out_wall = now_s() - f0;
    cudaEventRecord(ev.b, cs);
    const double out_ms = ev.ms();
    // a decode step while the swapped quarter is away
    refresh();
    batch.run(views, bctx, 0, hq, 0.0884f, q, o);
    // swap in: bookkeeping, then the flush; then a decode that needs them
    const double h1 = now_s();
    bool all_in = true;
    for (std::size_t i : pre) all_in = cache.swap_in_sequence(seqs[i]) && all_in;
    const double in_host_s = now_s() - h1;
    cudaEventRecord(ev.a, alloc.stream());
    alloc.flush();
    cudaEventRecord(ev.b, cs);
    const double in_ms = ev.ms();
    // decode stall: a step over resumed sequences issued right after their
    // swap-in waits for it on the stream; measure issue -> done
    std::vector<CacheView> rviews;
    std::vector<std::uint32_t> rctx;
    for (int b = 0; b < std::min<int>(B, static_cast<int>(pre.size())); ++b) {
        rviews.push_back(*cache.cache_view(seqs[pre[b]]));
        rctx.push_back(ctx[pre[b]]);
    }
    const double moved = static_cast<double>(swapped) * alloc.block(0)->size_bytes();
    // decode stall: swap the first resumed batch out again, then issue its
    // swap-in and a decode over it back to back; the decode waits for the
    // swap-in on the stream. stall = (swap-in + decode) - decode alone.
    bool dec_ok = true;
    float stall_ms = 0.f, rdecode_ms = 0.f;
    if (!rviews.empty()) {
        const int R = static_cast<int>(rviews.size());
        for (int b = 0; b < R; ++b) rviews[b] = *cache.cache_view(seqs[pre[b]]);
        for (int w = 0; w < 3; ++w) batch.run(rviews, rctx, 0, hq, 0.0884f, q, o);
        cudaEventRecord(ev.a, alloc.stream());
        for (int r = 0; r < 10; ++r) batch.run(rviews, rctx, 0, hq, 0.0884f, q, o);
        cudaEventRecord(ev.b, alloc.stream());
        rdecode_ms = ev.ms() / 10;
        for (int b = 0; b < R; ++b) cache.swap_out_sequence(seqs[pre[b]]);
        alloc.synchronize();
        cudaEventRecord(ev.a, alloc.stream());
        for (int b = 0; b < R; ++b) cache.swap_in_sequence(seqs[pre[b]]);
        for (int b = 0; b < R; ++b) rviews[b] = *cache.cache_view(seqs[pre[b]]);
        dec_ok = batch.run(rviews, rctx, 0, hq, 0.0884f, q, o);  // waits for the swap-in of its frames
        cudaEventRecord(ev.b, alloc.stream());
        stall_ms = ev.ms() - rdecode_ms;
    }
    // Decode of the resident batch while the resumed batch moves over PCIe on
    // the copy stream: first while it swaps out, then while it swaps in. The
    // resident batch reads no frame being moved, so it need not wait.
    float overlap_out_ms = 0.f, overlap_in_ms = 0.f;
    bool out_still_moving = false, in_still_moving = false;
    if (!rviews.empty()) {
        const int R = static_cast<int>(rviews.size());
        cudaEvent_t moved_ev;
        cudaEventCreateWithFlags(&moved_ev, cudaEventDisableTiming);
        alloc.synchronize();
        for (int b = 0; b < R; ++b) cache.swap_out_sequence(seqs[pre[b]]);
        alloc.flush();
        cudaEventRecord(moved_ev, cs);
        cudaEventRecord(ev.a, alloc.stream());
        dec_ok = batch.run(views, bctx, 0, hq, 0.0884f, q, o) && dec_ok;
        cudaEventRecord(ev.b, alloc.stream());
        overlap_out_ms = ev.ms();
        out_still_moving = cudaEventQuery(moved_ev) == cudaErrorNotReady;
        alloc.synchronize();
        for (int b = 0; b < R; ++b) cache.swap_in_sequence(seqs[pre[b]]);
        alloc.flush();
        cudaEventRecord(moved_ev, cs);
        cudaEventRecord(ev.a, alloc.stream());
        dec_ok = batch.run(views, bctx, 0, hq, 0.0884f, q, o) && dec_ok;
        cudaEventRecord(ev.b, alloc.stream());
        overlap_in_ms = ev.ms();
        in_still_moving = cudaEventQuery(moved_ev) == cudaErrorNotReady;
        cudaGetLastError();
        alloc.synchronize();
        cudaEventDestroy(moved_ev);
    }
    const int derr = batch.device_error();
    const auto link = swap.link_bytes();  // every pass above, both directions
    cudaFree(q);
    cudaFree(o);
    std::ostringstream js;
    js << "{\"workload\": \"cfg5-swap-churn\", \"coding\": \"" << (compressed ? "compressed" : "raw")
       << "\", \"link_bytes_out\": " << link.first << ", \"link_bytes_in\": " << link.second
       << ", \"block_bytes_out\": " << swap.bytes_out() << ", \"link_fraction\": "
       << (swap.bytes_out() ? static_cast<double>(link.first) / swap.bytes_out() : 0.0)
       << ", \"pool_blocks\": " << pool_blocks << ", \"block_bytes\": 65536"
       << ", \"pool_gib\": " << pool_blocks * 65536.0 / (1 << 30) << ", \"sequences\": " << seqs.size()
       << ", \"occupied_blocks\": " << pool_blocks - alloc.stats().free_blocks << ", \"preempted_sequences\": "
       << pre.size() << ", \"swapped_blocks\": " << swapped << ", \"swap_bytes_each_way\": " << moved
       << ", \"swap_out_ms\": " << out_ms << ", \"swap_out_gbs\": " << moved / (out_ms * 1e-3) / 1e9
       << ", \"swap_out_flush_wall_ms\": " << out_wall * 1e3 << ", \"swap_out_host_bookkeeping_ms\": "
       << out_host_s * 1e3 << ", \"swap_in_ms\": " << in_ms << ", \"swap_in_gbs\": " << moved / (in_ms * 1e-3) / 1e9
       << ", \"swap_in_host_bookkeeping_ms\": " << in_host_s * 1e3 << ", \"all_resumed\": "
       << (all_in ? "true" : "false") << ", \"pcie_d2h_peak_gbs\": " << d2h_peak << ", \"pcie_h2d_peak_gbs\": "
       << h2d_peak << ", \"decode_batch\": " << B << ", \"decode_ms\": " << decode_ms
       << ", \"resume_batch_decode_ms\": " << rdecode_ms << ", \"resume_batch_stall_ms\": " << stall_ms
       << ", \"resume_batch_sequences\": " << rviews.size()
       << ", \"resident_decode_during_swap_out_ms\": " << overlap_out_ms
       << ", \"swap_out_still_moving_after_that_decode\": " << (out_still_moving ? "true" : "false")
       << ", \"resident_decode_during_swap_in_ms\": " << overlap_in_ms
       << ", \"swap_in_still_moving_after_that_decode\": " << (in_still_moving ? "true" : "false")
       << ", \"pool_alloc_s\": " << pool_s << ", \"slab_pin_s\": " << pin_s << ", \"decode_ok\": "
       << (dec_ok ? "true" : "false") << ", \"decode_device_error\": " << derr << "}";
    return emit(js.str(), out, cap);
}

// cfg2-shaped engine loop through the C++ API: `batch` sequences with seeded
// contexts in [lo, hi]. A step gives every sequence one more token (reserve
// at a block boundary, ensure_token_writable, KVAppendBatch writes the
// token's K and V) and decodes the batch with PagedDecodeBatch. The loop runs twice, with the block tables flattened and
// uploaded every step and with resident tables, each over `steps` timed steps
// after `warmup`. Per mode it reports the wall time of a step (host
// bookkeeping and decode, pipelined; the clock stops after the last decode
// finishes), the host time inside the step calls, the device time (CUDA
// events on the engine stream), GB/s on the decode's algorithmic bytes, and
// the table rows and bytes uploaded. Both modes then decode the final state
// once more and the outputs are compared byte for byte.
extern "C" __attribute__((visibility("default"))) int qvp_scenario_engine(int batch, int lo, int hi, int steps,
                                                                           int warmup, int seed, char* out,
                                                                           size_t cap) {
    const BlockShape sh = bf16_shape(4);
    const std::uint32_t T = sh.tokens_per_block, hq = 28;
    std::mt19937 rng(seed);
    std::uniform_int_distribution<int> len(lo, hi);
    std::vector<std::uint32_t> ctx(batch);
    std::uint64_t need = 64;
    const int grow = 2 * (steps + warmup) + 2;  // both modes advance every sequence
    for (int b = 0; b < batch; ++b) {
        ctx[b] = static_cast<std::uint32_t>(len(rng));
        need += (ctx[b] + grow + T - 1) / T + 1;
    }
    AllocatorConfig cfg;
    cfg.block_shape = sh;
    cfg.max_blocks = static_cast<std::uint32_t>(need + need / 10);
    MemoryAllocator alloc(cfg);
    if (!alloc.has_storage()) return emit("{\"error\": \"pool allocation failed\"}", out, cap);
    KVCacheManager cache(alloc);
    std::vector<SequenceId> seqs;
    for (int b = 0; b < batch; ++b) {
        const SequenceId s = static_cast<SequenceId>(b + 1);
        if (!cache.create_sequence(SequenceMetadata{s, s, {}, {}}) || !cache.reserve_tokens(s, ctx[b]))
            return emit("{\"error\": \"could not reserve the contexts\"}", out, cap);
        seqs.push_back(s);
    }
    // seeded bf16 values over the whole pool, 64 blocks per copy
    {
        const std::size_t stride = alloc.block_stride(), chunk = 64;
        std::vector<bfloat16> h(2 * chunk * stride / 2);  // chunks start at rotating offsets
        std::normal_distribution<float> nd;
        for (auto& x : h) x = bfloat16(nd(rng));
        auto* base = reinterpret_cast<std::uint8_t*>(alloc.pool_base());
        for (std::size_t b0 = 0; b0 < cfg.max_blocks; b0 += chunk) {
            const std::size_t n = std::min<std::size_t>(chunk, cfg.max_blocks - b0);
            const std::size_t rot = (b0 / chunk * 4099) % (h.size() - n * stride / 2 + 1);
            cudaMemcpy(base + b0 * stride, h.data() + rot, n * stride, cudaMemcpyHostToDevice);
        }
    }
    const std::size_t qel = static_cast<std::size_t>(batch) * hq * sh.head_dim;
    void* q = device_query(qel, seed + 1);
    const std::size_t kvel = static_cast<std::size_t>(batch) * sh.num_kv_heads * sh.head_dim;
    void* kd = device_query(kvel, seed + 2);
    void* vd = device_query(kvel, seed + 3);
    void *o1 = nullptr, *o2 = nullptr;
    cudaMalloc(&o1, qel * 2);
    cudaMalloc(&o2, qel * 2);
    const float scale = 1.f / std::sqrt(128.f);
    bool ok = true;
    KVAppendBatch append(alloc);
    std::vector<std::uint32_t> positions(batch);

    auto views = [&]() {
        std::vector<CacheView> v;
        v.reserve(seqs.size());
        for (SequenceId s : seqs) v.push_back(*cache.cache_view(s));
        return v;
    };
    // one new token per sequence: map it, make it private, write its K/V
    auto advance = [&]() {
        for (int b = 0; b < batch; ++b) {
            if (ctx[b] % T == 0) ok = cache.reserve_tokens(seqs[b], 1) && ok;
            ok = cache.ensure_token_writable(seqs[b], ctx[b]).has_value() && ok;
            positions[b] = ctx[b]++;
        }
        ok = append.run(views(), positions, 0, kd, vd) && ok;
    };
    auto alg_bytes = [&]() {
        double kv = 0, tbl = 0;
        for (std::uint32_t c : ctx) {
            kv += 2.0 * c * sh.num_kv_heads * sh.head_dim * 2;
            tbl += 4.0 * ((c + T - 1) / T);
        }
        return kv + tbl + 2.0 * qel * 2;
    };

    struct Result {
        double wall_us, host_us, device_us, gbs, device_gbs, rows, upload_bytes;
        int status, device_error;
    };
    PagedDecodeBatch flat(alloc), resident(alloc, true);
    auto run_mode = [&](PagedDecodeBatch& pb, void* o) {
        Result r{};
        for (int i = 0; i < warmup; ++i) {
            advance();
            ok = pb.run(views(), ctx, 0, hq, scale, q, o) && ok;
        }
        cudaStreamSynchronize(alloc.stream());
        Events ev;
        double host = 0, alg = 0, rows = 0, bytes = 0;
        const double t0 = now_s();
        cudaEventRecord(ev.a, alloc.stream());
        for (int i = 0; i < steps; ++i) {
            const double th = now_s();
            advance();
            ok = pb.run(views(), ctx, 0, hq, scale, q, o) && ok;
            host += now_s() - th;
            alg += alg_bytes();
            rows += pb.rows_uploaded();
            bytes += static_cast<double>(pb.bytes_uploaded());
        }
        cudaEventRecord(ev.b, alloc.stream());
        cudaStreamSynchronize(alloc.stream());
        const double wall = now_s() - t0;
        const double dev_s = ev.ms() * 1e-3;
        const int n = std::max(steps, 1);
        r.wall_us = wall / n * 1e6;
        r.host_us = host / n * 1e6;
        r.device_us = dev_s / n * 1e6;
        r.gbs = alg / wall / 1e9;
        r.device_gbs = alg / dev_s / 1e9;
        r.rows = rows / n;
        r.upload_bytes = bytes / n;
        r.status = pb.last_status();
        r.device_error = pb.device_error();
        return r;
    };
    const Result rf = run_mode(flat, o1);
    const Result rr = run_mode(resident, o2);
    // the same final state through both modes
    const std::vector<CacheView> fin = views();
    ok = flat.run(fin, ctx, 0, hq, scale, q, o1) && ok;
    ok = resident.run(fin, ctx, 0, hq, scale, q, o2) && ok;
    cudaStreamSynchronize(alloc.stream());
    std::vector<std::uint8_t> a(qel * 2), b(qel * 2);
    cudaMemcpy(a.data(), o1, a.size(), cudaMemcpyDeviceToHost);
    cudaMemcpy(b.data(), o2, b.size(), cudaMemcpyDeviceToHost);
    const bool same = std::memcmp(a.data(), b.data(), a.size()) == 0;
    const int append_error = append.device_error();
    cudaFree(q);
    cudaFree(kd);
    cudaFree(vd);
    cudaFree(o1);
    cudaFree(o2);

    std::ostringstream js;
    auto mode = [&](const char* name, const Result& r) {
        js << "\"" << name << "\": {\"wall_us_per_step\": " << r.wall_us << ", \"host_us_per_step\": " << r.host_us
           << ", \"device_us_per_step\": " << r.device_us << ", \"gbs\": " << r.gbs
           << ", \"device_gbs\": " << r.device_gbs << ", \"rows_uploaded_per_step\": " << r.rows
           << ", \"upload_bytes_per_step\": " << r.upload_bytes << ", \"status\": " << r.status
           << ", \"device_error\": " << r.device_error << "}";
    };
    js << "{\"workload\": \"engine-cfg2-qwen2vl-7b-decode\", \"batch\": " << batch << ", \"ctx_range\": [" << lo
       << ", " << hi << "], \"steps\": " << steps << ", \"warmup\": " << warmup << ", ";
    mode("flattened_tables", rf);
    js << ", ";
    mode("resident_tables", rr);
    js << ", \"resident_gbs\": " << rr.gbs << ", \"outputs_identical\": " << (same ? "true" : "false")
       << ", \"append_device_error\": " << append_error << ", \"all_ok\": " << (ok ? "true" : "false")
       << ", \"step\": \"reserve + ensure_token_writable + KVAppendBatch + PagedDecodeBatch\"}";
    return emit(js.str(), out, cap);
}
