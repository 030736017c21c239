// TEST INFRASTRUCTURE: host checks of this library's additions to the
// reference interface: the resident block tables (qwenvl_paged/
// ResidentTables.h), host-visible pools (qwenvl_paged/Block.h), the refusal
// rules of PagedPrefillBatch and KVAppendBatch, and LruEvictionPolicy. For the
// tables, each packet the planner emits is applied to a host mirror of the
// device table, the way qvp_scatter_blocks and the copy
// of the context lengths apply it on the device, and after every step the
// mirror must hold, for every sequence, the same ids over its context as a
// full per-step flatten of its BlockTable. Bookkeeping-only pools, so all of
// it runs on the CPU.
#include "qwenvl_paged/EvictionPolicy.h"
#include "qwenvl_paged/KVCacheManager.h"
#include "qwenvl_paged/MemoryAllocator.h"
#include "qwenvl_paged/PagedAttention.h"
#include "qwenvl_paged/ResidentTables.h"
#include "qwenvl_paged/SwapBackend.h"

#include "harness.h"

#include <algorithm>
#include <cstring>
#include <random>
#include <vector>

using namespace qwenvl_paged;

namespace {

constexpr std::uint32_t kT = 16;

AllocatorConfig config(std::uint32_t blocks) {
    AllocatorConfig c;
    c.block_shape.tokens_per_block = kT;
    c.block_shape.num_layers = 1;
    c.block_shape.num_kv_heads = 2;
    c.block_shape.head_dim = 8;
    c.block_shape.bytes_per_element = 2;
    c.max_blocks = blocks;
    return c;
}

SequenceMetadata meta(SequenceId s) {
    SequenceMetadata m;
    m.sequence_id = s;
    m.request_id = s;
    return m;
}

// The device side of the packet: table [rows][pitch] and context lengths.
struct Mirror {
    std::vector<std::int32_t> table;
    std::vector<std::int32_t> ctx;
    std::uint32_t pitch{0};
    std::size_t rows{0};

    void apply(const TableDeltaPlanner& p) {
        if (p.pitch() != pitch) {  // re-laid: old rows are meaningless
            pitch = p.pitch();
            rows = 0;
            table.clear();
        }
        if (p.batch() > rows) {
            rows = p.batch();
            table.resize(rows * pitch, 0x7eadbeef);
        }
        const std::vector<std::int32_t>& pk = p.packet();
        CHECK(p.context_offset() % 4 == 0 && p.rows_offset() % 4 == 0 && pitch % 4 == 0);
        CHECK(pk.size() == p.rows_offset() + static_cast<std::size_t>(p.rows_written()) * pitch);
        for (std::uint32_t i = 0; i < p.rows_written(); ++i) {
            const std::int32_t r = pk[i];
            CHECK(r >= 0 && static_cast<std::size_t>(r) < rows);
            std::memcpy(table.data() + static_cast<std::size_t>(r) * pitch,
                        pk.data() + p.rows_offset() + static_cast<std::size_t>(i) * pitch, pitch * 4);
        }
        ctx.assign(pk.begin() + static_cast<std::ptrdiff_t>(p.context_offset()),
                   pk.begin() + static_cast<std::ptrdiff_t>(p.context_offset() + p.batch()));
    }
};

// What a full flatten gives for one view: the ids of [0, ceil(ctx/T)), or
// false where the per-step path refuses the batch.
bool flatten(const CacheView& v, std::uint32_t ctx, std::uint32_t num_blocks, std::vector<std::int32_t>& ids) {
    ids.clear();
    if (ctx == 0) return false;
    for (std::uint32_t i = 0; i < (ctx + kT - 1) / kT; ++i) {
        const auto id = v.block_table->lookup(i);
        if (!id || *id >= num_blocks) return false;
        ids.push_back(static_cast<std::int32_t>(*id));
    }
    return true;
}

// Plans a step and checks it against the full flatten; returns rows written.
std::uint32_t step(TableDeltaPlanner& p, Mirror& m, const std::vector<CacheView>& views,
                   const std::vector<std::uint32_t>& ctx, std::uint32_t num_blocks) {
    bool expect_ok = true;
    std::vector<std::vector<std::int32_t>> want(views.size());
    for (std::size_t b = 0; b < views.size(); ++b) expect_ok = flatten(views[b], ctx[b], num_blocks, want[b]) && expect_ok;
    std::string why;
    const bool ok = p.plan(views, ctx, &why);
    CHECK(ok == expect_ok);
    if (!ok) {
        CHECK(!why.empty());
        return 0;
    }
    m.apply(p);
    for (std::size_t b = 0; b < views.size(); ++b) {
        CHECK(m.ctx[b] == static_cast<std::int32_t>(ctx[b]));
        CHECK(want[b].size() <= m.pitch);
        for (std::size_t i = 0; i < want[b].size(); ++i) CHECK(m.table[b * m.pitch + i] == want[b][i]);
        // the planner's shadow is the mirror
        CHECK(std::equal(p.shadow().begin() + static_cast<std::ptrdiff_t>(b * p.pitch()),
                         p.shadow().begin() + static_cast<std::ptrdiff_t>((b + 1) * p.pitch()),
                         m.table.begin() + static_cast<std::ptrdiff_t>(b * m.pitch)));
    }
    return p.rows_written();
}

struct Engine {
    explicit Engine(std::uint32_t blocks)
        : alloc(config(blocks), DevicePoolOptions{-1, false, nullptr}), swap(1 << 16), cache(alloc) {
        alloc.set_swap_backend(&swap);
    }
    MemoryAllocator alloc;
    HostSwapBackend swap;
    KVCacheManager cache;
};

NATIVE_TEST(steady_decode_uploads_a_row_only_when_a_sequence_gains_a_block) {
    Engine e(4096);
    TableDeltaPlanner p(4096);
    Mirror m;
    std::vector<SequenceId> ids;
    std::vector<std::uint32_t> ctx;
    for (SequenceId s = 1; s <= 32; ++s) {
        CHECK(e.cache.create_sequence(meta(s)));
        ctx.push_back(100 + 37 * static_cast<std::uint32_t>(s));
        CHECK(e.cache.reserve_tokens(s, ctx.back()));
        ids.push_back(s);
    }
    auto views = [&] {
        std::vector<CacheView> v;
        for (SequenceId s : ids) v.push_back(*e.cache.cache_view(s));
        return v;
    };
    CHECK(step(p, m, views(), ctx, 4096) == 32u);  // first step: every row
    std::uint64_t rows = 0, crossings = 0;
    for (int it = 0; it < 200; ++it) {
        for (std::size_t b = 0; b < ids.size(); ++b) {
            // the engine's per-token path: reserve when the block is full,
            // then make the slot writable (a no-op on a private block)
            if (ctx[b] % kT == 0) {
                CHECK(e.cache.reserve_tokens(ids[b], 1));
                ++crossings;
            }
            CHECK(e.cache.ensure_token_writable(ids[b], ctx[b]).has_value());
            ++ctx[b];
        }
        rows += step(p, m, views(), ctx, 4096);
    }
    // one row per block boundary crossed, plus a full rewrite per pitch growth
    CHECK(rows >= crossings);
    CHECK(rows <= crossings + 2 * 32);
}

NATIVE_TEST(copy_on_write_rewrites_only_the_branches_that_copied) {
    Engine e(1024);
    TableDeltaPlanner p(1024);
    Mirror m;
    CHECK(e.cache.create_sequence(meta(1)) && e.cache.reserve_tokens(1, 3 * kT + 1));
    for (SequenceId s = 2; s <= 4; ++s) CHECK(e.cache.fork_sequence(1, meta(s)));
    auto views = [&] {
        std::vector<CacheView> v;
        for (SequenceId s = 1; s <= 4; ++s) v.push_back(*e.cache.cache_view(s));
        return v;
    };
    std::vector<std::uint32_t> ctx(4, 3 * kT + 1);
    CHECK(step(p, m, views(), ctx, 1024) == 4u);
    CHECK(step(p, m, views(), ctx, 1024) == 0u);
    // branches 2 and 3 write the shared last block: each gets a private copy
    CHECK(e.cache.ensure_token_writable(2, 3 * kT + 1).has_value());
    CHECK(e.cache.ensure_token_writable(3, 3 * kT + 1).has_value());
    CHECK(step(p, m, views(), ctx, 1024) == 2u);
    CHECK(m.table[1 * m.pitch + 3] != m.table[0 * m.pitch + 3] && m.table[2 * m.pitch + 3] != m.table[0 * m.pitch + 3]);
    CHECK(m.table[3 * m.pitch + 3] == m.table[0 * m.pitch + 3]);
}

NATIVE_TEST(a_swapped_sequence_is_refused_and_its_swap_in_is_picked_up) {
    Engine e(256);
    TableDeltaPlanner p(256);
    Mirror m;
    for (SequenceId s = 1; s <= 3; ++s) CHECK(e.cache.create_sequence(meta(s)) && e.cache.reserve_tokens(s, 40));
    auto views = [&] {
        std::vector<CacheView> v;
        for (SequenceId s = 1; s <= 3; ++s) v.push_back(*e.cache.cache_view(s));
        return v;
    };
    const std::vector<std::uint32_t> ctx(3, 40);
    CHECK(step(p, m, views(), ctx, 256) == 3u);
    CHECK(e.cache.swap_out_sequence(2) == 3u);
    CHECK(step(p, m, views(), ctx, 256) == 0u);  // refused, nothing planned
    // the failed plan forgot every row: the next good one rewrites them all
    CHECK(e.cache.swap_in_sequence(2));
    CHECK(step(p, m, views(), ctx, 256) == 3u);
    CHECK(step(p, m, views(), ctx, 256) == 0u);
}

NATIVE_TEST(a_context_past_the_mapped_blocks_is_refused) {
    Engine e(64);
    TableDeltaPlanner p(64);
    Mirror m;
    CHECK(e.cache.create_sequence(meta(1)) && e.cache.reserve_tokens(1, 2 * kT));
    const std::vector<CacheView> v{*e.cache.cache_view(1)};
    CHECK(step(p, m, v, {2 * kT}, 64) == 1u);
    CHECK(step(p, m, v, {2 * kT + 1}, 64) == 0u);
    CHECK(step(p, m, v, {0}, 64) == 0u);
    CHECK(step(p, m, v, {1}, 64) == 1u);
}

NATIVE_TEST(a_replaced_or_reordered_batch_rewrites_the_positions_that_changed) {
    Engine e(1024);
    TableDeltaPlanner p(1024);
    Mirror m;
    for (SequenceId s = 1; s <= 6; ++s) CHECK(e.cache.create_sequence(meta(s)) && e.cache.reserve_tokens(s, 50));
    std::vector<SequenceId> order{1, 2, 3, 4};
    auto views = [&] {
        std::vector<CacheView> v;
        for (SequenceId s : order) v.push_back(*e.cache.cache_view(s));
        return v;
    };
    CHECK(step(p, m, views(), std::vector<std::uint32_t>(4, 50), 1024) == 4u);
    std::swap(order[1], order[2]);
    CHECK(step(p, m, views(), std::vector<std::uint32_t>(4, 50), 1024) == 2u);
    e.cache.release_sequence(order[3]);
    order[3] = 5;  // a new sequence takes the freed position
    CHECK(step(p, m, views(), std::vector<std::uint32_t>(4, 50), 1024) == 1u);
    order.push_back(6);  // the batch grows
    CHECK(step(p, m, views(), std::vector<std::uint32_t>(5, 50), 1024) == 1u);
    order.resize(2);  // and shrinks
    CHECK(step(p, m, views(), std::vector<std::uint32_t>(2, 50), 1024) == 0u);
}

NATIVE_TEST(random_engine_scripts_match_the_full_flatten_every_step) {
    for (std::uint32_t seed = 1; seed <= 12; ++seed) {
        std::mt19937 rng(seed);
        Engine e(512);
        TableDeltaPlanner p(512);
        Mirror m;
        std::vector<SequenceId> batch;  // batch positions
        std::vector<std::uint32_t> ctx;
        SequenceId next = 1;
        for (int it = 0; it < 300; ++it) {
            const std::uint32_t op = rng() % 100;
            if (op < 10 && batch.size() < 24) {  // admit a sequence
                const std::uint32_t n = 1 + rng() % 90;
                if (e.cache.create_sequence(meta(next)) && e.cache.reserve_tokens(next, n)) {
                    batch.push_back(next);
                    ctx.push_back(n);
                } else {
                    e.cache.release_sequence(next);
                }
                ++next;
            } else if (op < 14 && !batch.empty()) {  // fork into a new position
                const std::size_t b = rng() % batch.size();
                if (e.cache.fork_sequence(batch[b], meta(next))) {
                    batch.push_back(next);
                    ctx.push_back(ctx[b]);
                }
                ++next;
            } else if (op < 18 && !batch.empty()) {  // finish one
                const std::size_t b = rng() % batch.size();
                e.cache.release_sequence(batch[b]);
                batch.erase(batch.begin() + static_cast<std::ptrdiff_t>(b));
                ctx.erase(ctx.begin() + static_cast<std::ptrdiff_t>(b));
            } else if (op < 21 && !batch.empty()) {  // preempt and resume
                const std::size_t b = rng() % batch.size();
                (void)e.cache.swap_out_sequence(batch[b]);
                if (rng() % 2) {
                    std::vector<CacheView> v;
                    for (SequenceId s : batch) v.push_back(*e.cache.cache_view(s));
                    (void)step(p, m, v, ctx, 512);  // refused unless nothing was swapped
                }
                (void)e.cache.swap_in_sequence(batch[b]);
            } else if (op < 23 && batch.size() > 1) {  // reorder
                const std::size_t a = rng() % batch.size(), b = rng() % batch.size();
                std::swap(batch[a], batch[b]);
                std::swap(ctx[a], ctx[b]);
            } else {  // decode a token in every sequence
                for (std::size_t b = 0; b < batch.size(); ++b) {
                    if (ctx[b] % kT == 0 && !e.cache.reserve_tokens(batch[b], 1)) continue;
                    if (e.cache.ensure_token_writable(batch[b], ctx[b]).has_value()) ++ctx[b];
                }
            }
            std::vector<CacheView> v;
            for (SequenceId s : batch) v.push_back(*e.cache.cache_view(s));
            (void)step(p, m, v, ctx, 512);
        }
    }
}

// ---- host-visible pools (the other addition to the reference interface) ----

NATIVE_TEST(host_visible_pools_pad_the_stride_and_follow_the_process_setting) {
    const bool before = host_visible_pools();
    set_host_visible_pools(false);
    CHECK(!DevicePoolOptions{}.host_visible);
    MemoryAllocator plain(config(8), DevicePoolOptions{-1, false, nullptr});
    set_host_visible_pools(true);
    CHECK(DevicePoolOptions{}.host_visible);
    MemoryAllocator visible(config(8), DevicePoolOptions{-1, false, nullptr});
    set_host_visible_pools(before);
    CHECK(!plain.host_visible() && visible.host_visible());
    // the padded stride keeps decode off the TMA view of a managed pool
    CHECK(plain.block_stride() == config(8).block_shape.byte_size());
    CHECK(visible.block_stride() > config(8).block_shape.byte_size() && visible.block_stride() % 256 == 0);
    CHECK(visible.block(1)->size_bytes() == plain.block(1)->size_bytes());
}

// ---- prefill and KV-append batches: refusals before any device work -------

void* const kFakeDevicePtr = reinterpret_cast<void*>(0x100000);  // never dereferenced: no storage

NATIVE_TEST(prefill_batch_refuses_bad_query_lengths_and_unmapped_contexts) {
    Engine e(64);
    PagedPrefillBatch pb(e.alloc);
    CHECK(e.cache.create_sequence(meta(1)) && e.cache.reserve_tokens(1, 40));
    const std::vector<CacheView> v{*e.cache.cache_view(1)};
    CHECK(!pb.run(v, {40}, {41}, 0, 4, 1.f, kFakeDevicePtr, kFakeDevicePtr));  // query past the context
    CHECK(pb.last_error().find("query length") != std::string::npos);
    CHECK(!pb.run(v, {40}, {0}, 0, 4, 1.f, kFakeDevicePtr, kFakeDevicePtr));
    CHECK(!pb.run(v, {49}, {1}, 0, 4, 1.f, kFakeDevicePtr, kFakeDevicePtr));  // context past the mapped blocks
    CHECK(pb.last_status() == 2);                                               // QVP_ERR_UNMAPPED
    CHECK(!pb.run(v, {40}, {8}, 1, 4, 1.f, kFakeDevicePtr, kFakeDevicePtr));  // layer outside the shape
    CHECK(!pb.run(v, {40}, {8}, 0, 3, 1.f, kFakeDevicePtr, kFakeDevicePtr));  // heads that do not group
    CHECK(!pb.run(v, {40, 40}, {8}, 0, 4, 1.f, kFakeDevicePtr, kFakeDevicePtr));
    CHECK(pb.run({}, {}, {}, 0, 4, 1.f, kFakeDevicePtr, kFakeDevicePtr));     // empty batch: nothing to do
    // every check passes: stops at the missing device storage
    CHECK(!pb.run(v, {40}, {40}, 0, 4, 1.f, kFakeDevicePtr, kFakeDevicePtr));
    CHECK(pb.last_error().find("no device storage") != std::string::npos);
    CHECK(e.cache.swap_out_sequence(1) == 3u);
    const std::vector<CacheView> swapped{*e.cache.cache_view(1)};
    CHECK(!pb.run(swapped, {40}, {1}, 0, 4, 1.f, kFakeDevicePtr, kFakeDevicePtr));
    CHECK(pb.last_status() == 2);
}

NATIVE_TEST(kv_append_refuses_shared_read_only_and_unmapped_targets) {
    Engine e(64);
    KVAppendBatch ab(e.alloc);
    CHECK(e.cache.create_sequence(meta(1)) && e.cache.reserve_tokens(1, kT + 1));
    CHECK(e.cache.fork_sequence(1, meta(2)));
    auto views = [&](std::initializer_list<SequenceId> ids) {
        std::vector<CacheView> v;
        for (SequenceId s : ids) v.push_back(*e.cache.cache_view(s));
        return v;
    };
    // block 1 is shared by the fork: writing it would change both sequences
    CHECK(!ab.run(views({1}), {kT}, 0, kFakeDevicePtr, kFakeDevicePtr));
    CHECK(ab.last_error().find("shared or read-only") != std::string::npos);
    CHECK(!ab.run(views({2}), {kT}, 0, kFakeDevicePtr, kFakeDevicePtr));
    // position past the mapped blocks
    CHECK(!ab.run(views({1}), {2 * kT}, 0, kFakeDevicePtr, kFakeDevicePtr));
    CHECK(ab.last_status() == 2);
    // layer outside the shape, count mismatch, null K
    CHECK(!ab.run(views({1}), {kT}, 1, kFakeDevicePtr, kFakeDevicePtr));
    CHECK(!ab.run(views({1, 2}), {kT}, 0, kFakeDevicePtr, kFakeDevicePtr));
    CHECK(!ab.run(views({1}), {kT}, 0, nullptr, kFakeDevicePtr));
    // after copy-on-write both targets are private and writable: the checks
    // pass and the call stops at the missing device storage
    CHECK(e.cache.ensure_token_writable(1, kT).has_value() && e.cache.ensure_token_writable(2, kT).has_value());
    CHECK(!ab.run(views({1, 2}), {kT, kT}, 0, kFakeDevicePtr, kFakeDevicePtr));
    CHECK(ab.last_error().find("no device storage") != std::string::npos);
}

// ---- LruEvictionPolicy ------------------------------------------------------

NATIVE_TEST(eviction_policy_names_the_least_recently_decoded_private_block) {
    Engine e(64);
    LruEvictionPolicy policy(e.cache);
    e.alloc.set_eviction_selector(policy.selector());
    for (SequenceId s = 1; s <= 3; ++s) CHECK(e.cache.create_sequence(meta(s)) && e.cache.reserve_tokens(s, 40));
    auto view = [&](SequenceId s) { return *e.cache.cache_view(s); };
    CHECK(!e.alloc.select_eviction_candidate());  // nothing decoded yet
    policy.touch({view(1), view(2)});
    CHECK(!e.alloc.select_eviction_candidate());  // 1 and 2 are in the current batch; 3 never decoded
    policy.touch({view(2), view(3)});
    // 1 is the oldest outside the batch: its last block
    CHECK(e.alloc.select_eviction_candidate() == view(1).block_table->lookup(2));
    policy.touch({view(3)});
    // 1 (step 1) is older than 2 (step 2)
    CHECK(e.alloc.select_eviction_candidate() == view(1).block_table->lookup(2));
    // shared blocks are skipped: fork 1, so its blocks are held twice
    CHECK(e.cache.fork_sequence(1, meta(4)));
    CHECK(e.alloc.select_eviction_candidate() == view(2).block_table->lookup(2));
    // copy-on-write makes 1's last block private again
    CHECK(e.cache.ensure_token_writable(1, 39).has_value());
    CHECK(e.alloc.select_eviction_candidate() == view(1).block_table->lookup(2));
    // a swapped-out sequence has no frame to name; a released one is skipped
    CHECK(e.cache.swap_out_sequence(2) > 0u);
    e.cache.release_sequence(1);
    // left: 2 swapped out, 3 in the current batch, 4 never decoded
    CHECK(!e.alloc.select_eviction_candidate());
}

NATIVE_TEST(eviction_policy_advice_drives_a_swap_out_that_frees_the_block) {
    Engine e(8);
    LruEvictionPolicy policy(e.cache);
    e.alloc.set_eviction_selector(policy.selector());
    for (SequenceId s = 1; s <= 2; ++s) CHECK(e.cache.create_sequence(meta(s)) && e.cache.reserve_tokens(s, 64));
    CHECK(!e.alloc.can_allocate(1));
    policy.touch({*e.cache.cache_view(1)});
    policy.touch({*e.cache.cache_view(2)});
    const auto victim = e.alloc.select_eviction_candidate();
    CHECK(victim.has_value() && *victim == *e.cache.cache_view(1)->block_table->lookup(3));
    CHECK(e.cache.swap_out_sequence(1) == 4u && e.alloc.can_allocate(4));
    CHECK(e.alloc.info(*victim)->state == BlockState::Free);
}

// A swap backend whose buffers could not be allocated refuses every store
// up front, so a swap-out changes nothing: no frame is freed, no generation
// moves, the table keeps its mappings (the moves that were recorded are
// never dropped later, because nothing is recorded).
NATIVE_TEST(a_swap_backend_without_buffers_refuses_before_the_bookkeeping_moves) {
    MemoryAllocator alloc(config(8), DevicePoolOptions{-1, false, nullptr});
    DeviceSwapBackend swap(alloc, 4);  // no device storage: its buffers are never allocated
    CHECK(!swap.ready());
    alloc.set_swap_backend(&swap);
    KVCacheManager cache(alloc);
    CHECK(cache.create_sequence(meta(1)) && cache.reserve_tokens(1, 40));
    std::vector<PhysicalBlockInfo> before;
    for (PhysicalBlockId i = 0; i < 8; ++i) before.push_back(*alloc.info(i));
    const std::vector<BlockTableEntry> table_before = cache.cache_view(1)->block_table->entries();
    const AllocatorStats st_before = alloc.stats();
    CHECK(cache.swap_out_sequence(1) == 0u);
    CHECK(!alloc.swap_out(*cache.cache_view(1)->block_table->lookup(0)).has_value());
    for (PhysicalBlockId i = 0; i < 8; ++i) {
        CHECK(alloc.info(i)->state == before[i].state && alloc.info(i)->ref_count == before[i].ref_count &&
              alloc.info(i)->generation == before[i].generation);
    }
    const std::vector<BlockTableEntry>& after = cache.cache_view(1)->block_table->entries();
    CHECK(after.size() == table_before.size());
    for (std::size_t i = 0; i < after.size(); ++i)
        CHECK(after[i].physical_id == table_before[i].physical_id && !after[i].swap_slot.has_value());
    CHECK(alloc.stats().free_blocks == st_before.free_blocks && alloc.stats().swapped_blocks == 0u);
    // with nothing deferred, every ordering call is a no-op
    CHECK(!alloc.loads_in_flight());
    alloc.order_reads(nullptr, 0);
    alloc.order_writes();
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int qvp_tablecases_list(char* out, size_t cap) {
    return native::list_cases(out, cap);
}

extern "C" __attribute__((visibility("default"))) int qvp_tablecases_run(const char* name, char* msg, size_t cap) {
    return native::run_case(name, msg, cap);
}
