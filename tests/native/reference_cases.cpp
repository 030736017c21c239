// TEST INFRASTRUCTURE: the reference's specification tests, re-expressed
// against this library's host layer (phhuang191129/QwenVL-Paged
// tests/BlockTable.test.cpp, CacheView.test.cpp (layout and view-structure
// cases), MemoryAllocator.test.cpp, KVCacheManager.test.cpp,
// SwapBackend.test.cpp (bookkeeping cases), Scheduler.test.cpp,
// Block.test.cpp (shape cases)). Pools are bookkeeping-only (no device
// bytes), so every case runs on the CPU; the cases that compare block bytes
// or attention outputs run on real device pools in native_tests.cpp.
//
// Run from pytest (tests/test_reference_cases.py): qvp_refcases_list() names
// the cases, qvp_refcases_run(name) runs one.
#include "qwenvl_paged/Block.h"
#include "qwenvl_paged/BlockTable.h"
#include "qwenvl_paged/CacheLayout.h"
#include "qwenvl_paged/KVCacheManager.h"
#include "qwenvl_paged/MemoryAllocator.h"
#include "qwenvl_paged/Scheduler.h"
#include "qwenvl_paged/SwapBackend.h"

#include "harness.h"

#include <optional>
#include <set>
#include <unordered_map>
#include <vector>

using namespace qwenvl_paged;

namespace {

constexpr std::uint32_t kT = 16;  // tokens per block in the allocator, cache and scheduler cases

BlockShape shape16() {
    BlockShape s;
    s.tokens_per_block = kT;
    s.num_layers = 1;
    s.num_kv_heads = 2;
    s.head_dim = 8;
    s.bytes_per_element = 2;
    return s;
}

// A pool of `blocks` blocks with no device bytes (bookkeeping only).
struct Pool {
    explicit Pool(std::uint32_t blocks, BlockShape s = shape16())
        : alloc(config(s, blocks), DevicePoolOptions{-1, false, nullptr}) {}
    static AllocatorConfig config(BlockShape s, std::uint32_t blocks) {
        AllocatorConfig c;
        c.block_shape = s;
        c.max_blocks = blocks;
        return c;
    }
    MemoryAllocator alloc;
};

SequenceMetadata meta(SequenceId s) {
    SequenceMetadata m;
    m.sequence_id = s;
    m.request_id = s;
    return m;
}

LogicalBlock logical(SequenceId s, LogicalBlockIndex i) {
    LogicalBlock b;
    b.sequence_id = s;
    b.index = i;
    b.cache_kind = CacheKind::TextKV;
    b.start_token = i * kT;
    b.token_count = kT;
    return b;
}

// ---- BlockShape / LogicalBlock / PhysicalBlock metadata --------------------

NATIVE_TEST(block_shape_byte_size_counts_k_and_v_and_scales_linearly) {
    BlockShape s = shape16();
    CHECK(s.byte_size() == 2u * 16 * 1 * 2 * 8 * 2);
    BlockShape twice_tokens = s, twice_layers = s;
    twice_tokens.tokens_per_block *= 2;
    twice_layers.num_layers *= 2;
    CHECK(twice_tokens.byte_size() == 2 * s.byte_size());
    CHECK(twice_layers.byte_size() == 2 * s.byte_size());
}

NATIVE_TEST(logical_block_is_empty_until_it_holds_tokens) {
    LogicalBlock b;
    CHECK(b.empty());
    b.token_count = 3;
    CHECK(!b.empty());
}

NATIVE_TEST(pool_blocks_report_id_shape_and_rounded_size) {
    Pool p(3);
    for (PhysicalBlockId i = 0; i < 3; ++i) {
        const PhysicalBlock* b = p.alloc.block(i);
        CHECK(b != nullptr && b->id() == i);
        CHECK(b->shape().byte_size() == shape16().byte_size());
        CHECK(b->size_bytes() >= b->shape().byte_size());
        CHECK(b->size_bytes() % kDefaultBlockAlignmentBytes == 0);
        CHECK(b->alignment_bytes() == kDefaultBlockAlignmentBytes);
    }
}

// ---- BlockTable ----------------------------------------------------------

NATIVE_TEST(table_starts_empty_with_its_identity) {
    BlockTable t(42, CacheKind::VisionKV);
    CHECK(t.sequence_id() == 42u && t.cache_kind() == CacheKind::VisionKV);
    CHECK(t.empty() && t.size() == 0u);
}

NATIVE_TEST(table_map_lookup_replace_and_miss) {
    BlockTable t(1);
    CHECK(!t.lookup(5).has_value());
    t.map(logical(1, 0), 100, true);
    CHECK(t.lookup(0) == std::optional<PhysicalBlockId>(100) && t.size() == 1u && !t.empty());
    t.map(logical(1, 0), 200, true);  // same index: replaced, not added
    CHECK(t.lookup(0) == std::optional<PhysicalBlockId>(200) && t.size() == 1u);
}

NATIVE_TEST(table_unmap_returns_the_frame_or_nothing) {
    BlockTable t(1);
    CHECK(!t.unmap(0).has_value());
    t.map(logical(1, 0), 100, true);
    CHECK(t.unmap(0) == std::optional<PhysicalBlockId>(100));
    CHECK(!t.lookup(0).has_value());
}

NATIVE_TEST(table_entries_expose_and_update_writable_and_frame) {
    BlockTable t(1);
    t.map(logical(1, 0), 100, false);
    CHECK(t.entry(0) != nullptr && t.entry(0)->physical_id == 100u && !t.entry(0)->writable);
    CHECK(t.entry(1) == nullptr && t.mutable_entry(1) == nullptr);
    t.set_writable(0, true);
    CHECK(t.entry(0)->writable);
    t.mutable_entry(0)->physical_id = 555;
    CHECK(t.lookup(0) == std::optional<PhysicalBlockId>(555));
    CHECK(!t.entry(0)->swap_slot.has_value());
}

NATIVE_TEST(table_keeps_entries_sorted_by_logical_index) {
    BlockTable t(1);
    for (LogicalBlockIndex i : {2u, 0u, 1u}) t.map(logical(1, i), 100 + i, true);
    const auto& e = t.entries();
    CHECK(e.size() == 3u);
    for (LogicalBlockIndex i = 0; i < 3; ++i) CHECK(e[i].logical.index == i && e[i].physical_id == 100 + i);
}

NATIVE_TEST(table_lookup_misses_while_an_entry_is_swapped) {
    BlockTable t(1);
    t.map(logical(1, 0), 100, true);
    t.mutable_entry(0)->swap_slot = SwapSlotId{7};
    CHECK(!t.lookup(0).has_value() && t.size() == 1u);
    CHECK(t.entry(0)->swap_slot == std::optional<SwapSlotId>(7));
    t.mutable_entry(0)->physical_id = 200;
    t.mutable_entry(0)->swap_slot.reset();
    CHECK(t.lookup(0) == std::optional<PhysicalBlockId>(200));
}

NATIVE_TEST(table_fork_shares_frames_read_only_under_the_child_id) {
    BlockTable parent(1);
    parent.map(logical(1, 0), 100, true);
    parent.map(logical(1, 1), 101, true);
    const BlockTable child = parent.fork(2);
    CHECK(child.sequence_id() == 2u && child.size() == 2u);
    for (const BlockTableEntry& e : child.entries()) {
        CHECK(!e.writable && e.logical.sequence_id == 2u);
        CHECK(child.lookup(e.logical.index) == parent.lookup(e.logical.index));
    }
}

// ---- KVBlockLayout (CacheView.test.cpp, layout cases) ---------------------

KVBlockLayout layout_2_4_3_5() {  // 2 layers, 4 tokens, 3 heads, head_dim 5
    KVBlockLayout l;
    l.shape.tokens_per_block = 4;
    l.shape.num_layers = 2;
    l.shape.num_kv_heads = 3;
    l.shape.head_dim = 5;
    l.shape.bytes_per_element = 4;
    return l;
}

NATIVE_TEST(layout_strides_follow_layer_stream_token_head_dim) {
    const KVBlockLayout l = layout_2_4_3_5();
    CHECK(l.head_stride() == 5u && l.token_stride() == 15u && l.stream_stride() == 60u && l.layer_stride() == 120u);
    CHECK(l.element_count() * 4 == l.shape.byte_size());
    CHECK(*l.element_offset(0, KVStream::Key, 0, 1) - *l.element_offset(0, KVStream::Key, 0, 0) == 5u);
    CHECK(*l.element_offset(1, KVStream::Value, 2, 1) - *l.element_offset(1, KVStream::Key, 2, 1) ==
          l.stream_stride());
}

NATIVE_TEST(layout_maps_every_coordinate_to_a_distinct_slot_inside_the_block) {
    const KVBlockLayout l = layout_2_4_3_5();
    std::set<std::size_t> used;
    for (std::uint32_t layer = 0; layer < 2; ++layer)
        for (KVStream s : {KVStream::Key, KVStream::Value})
            for (std::uint32_t t = 0; t < 4; ++t)
                for (std::uint32_t h = 0; h < 3; ++h) {
                    const auto off = l.element_offset(layer, s, t, h);
                    CHECK(off.has_value());
                    for (std::size_t d = 0; d < 5; ++d) {
                        CHECK(*off + d < l.element_count());
                        CHECK(used.insert(*off + d).second);
                    }
                }
    CHECK(used.size() == l.element_count());
    CHECK(!l.element_offset(2, KVStream::Key, 0, 0) && !l.element_offset(0, KVStream::Key, 4, 0) &&
          !l.element_offset(0, KVStream::Key, 0, 3));
}

// ---- CacheView structure (CacheView.test.cpp, non-byte cases) -------------

NATIVE_TEST(view_default_is_invalid_and_resolves_nothing) {
    const CacheView v;
    CHECK(!v.valid() && v.block_bytes(0) == nullptr && v.slot<float>(KVStream::Key, 0, 0, 0) == nullptr);
}

NATIVE_TEST(view_carries_table_allocator_and_the_pool_shape) {
    Pool p(4);
    KVCacheManager c(p.alloc);
    CHECK(c.create_sequence(meta(1)) && c.reserve_tokens(1, kT));
    const auto v = c.cache_view(1);
    CHECK(v && v->valid() && v->sequence_id == 1u && v->block_table != nullptr && v->allocator == &p.alloc);
    CHECK(v->layout.shape.tokens_per_block == kT && v->layout.shape.head_dim == 8u);
    CHECK(!c.cache_view(99).has_value());
}

// ---- MemoryAllocator ------------------------------------------------------

NATIVE_TEST(allocator_starts_all_free_and_hands_out_distinct_ids_until_empty) {
    Pool p(4);
    CHECK(p.alloc.stats().total_blocks == 4u && p.alloc.stats().free_blocks == 4u &&
          p.alloc.stats().active_blocks == 0u);
    std::set<PhysicalBlockId> got;
    for (int i = 0; i < 4; ++i) {
        const auto id = p.alloc.allocate();
        CHECK(id && got.insert(*id).second);
    }
    CHECK(!p.alloc.allocate());
}

NATIVE_TEST(allocator_reuses_a_released_frame) {
    Pool p(1);
    const auto a = p.alloc.allocate();
    CHECK(a && !p.alloc.allocate());
    p.alloc.release(*a);
    CHECK(p.alloc.allocate() == a);
}

NATIVE_TEST(allocator_frees_only_after_every_reference_is_released) {
    Pool p(1);
    const auto a = p.alloc.allocate();
    p.alloc.retain(*a);
    CHECK(p.alloc.info(*a)->ref_count == 2u && p.alloc.info(*a)->state == BlockState::Shared);
    p.alloc.release(*a);
    CHECK(!p.alloc.allocate() && p.alloc.info(*a)->state == BlockState::Active);
    p.alloc.release(*a);
    CHECK(p.alloc.allocate().has_value());
}

NATIVE_TEST(allocator_rejects_unknown_ids) {
    Pool p(1);
    CHECK(p.alloc.block(999) == nullptr && p.alloc.info(999) == nullptr);
    p.alloc.release(999);
    p.alloc.retain(999);
    CHECK(p.alloc.stats().free_blocks == 1u);
}

NATIVE_TEST(allocator_stats_and_can_allocate_track_the_free_list) {
    Pool p(4);
    const auto a = p.alloc.allocate(), b = p.alloc.allocate();
    CHECK(a && b && p.alloc.stats().free_blocks == 2u && p.alloc.stats().active_blocks == 2u);
    CHECK(p.alloc.can_allocate(2) && !p.alloc.can_allocate(3));
    p.alloc.release(*a);
    CHECK(p.alloc.stats().free_blocks == 3u && p.alloc.stats().active_blocks == 1u);
}

NATIVE_TEST(swap_out_needs_a_backend_and_a_sole_owner) {
    Pool p(2);
    const auto a = p.alloc.allocate();
    CHECK(!p.alloc.swap_out(*a) && p.alloc.stats().free_blocks == 1u);  // no backend
    HostSwapBackend swap(4);
    p.alloc.set_swap_backend(&swap);
    p.alloc.retain(*a);
    CHECK(!p.alloc.swap_out(*a) && swap.resident_slots() == 0u && p.alloc.info(*a)->ref_count == 2u);
    p.alloc.release(*a);
    p.alloc.release(*a);
    CHECK(!p.alloc.swap_out(*a) && !p.alloc.swap_out(999));  // free and unknown
}

NATIVE_TEST(swap_out_frees_the_frame_and_advances_its_generation) {
    Pool p(1);
    HostSwapBackend swap(4);
    p.alloc.set_swap_backend(&swap);
    const auto a = p.alloc.allocate();
    const std::uint64_t g = p.alloc.info(*a)->generation;
    CHECK(!p.alloc.can_allocate(1));
    CHECK(p.alloc.swap_out(*a).has_value());
    CHECK(swap.resident_slots() == 1u && p.alloc.can_allocate(1) && p.alloc.stats().free_blocks == 1u);
    CHECK(p.alloc.info(*a)->generation > g && p.alloc.info(*a)->ref_count == 0u);
}

NATIVE_TEST(swap_out_fails_when_the_swap_space_is_full) {
    Pool p(2);
    HostSwapBackend swap(1);
    p.alloc.set_swap_backend(&swap);
    const auto a = p.alloc.allocate(), b = p.alloc.allocate();
    CHECK(p.alloc.swap_out(*a).has_value());
    CHECK(!p.alloc.swap_out(*b) && p.alloc.info(*b)->ref_count == 1u);
}

NATIVE_TEST(swap_in_consumes_the_slot_and_allocates_an_active_frame) {
    Pool p(2);
    HostSwapBackend swap(4);
    p.alloc.set_swap_backend(&swap);
    const auto slot = p.alloc.swap_out(*p.alloc.allocate());
    const auto back = p.alloc.swap_in(*slot);
    CHECK(back && p.alloc.info(*back)->ref_count == 1u && p.alloc.info(*back)->state == BlockState::Active);
    CHECK(swap.resident_slots() == 0u && !p.alloc.swap_in(*slot));
}

NATIVE_TEST(swap_in_keeps_the_slot_when_no_frame_is_free_and_refuses_unknown_slots) {
    Pool p(1);
    HostSwapBackend swap(4);
    p.alloc.set_swap_backend(&swap);
    const auto slot = p.alloc.swap_out(*p.alloc.allocate());
    CHECK(p.alloc.allocate().has_value());
    CHECK(!p.alloc.swap_in(*slot) && swap.resident_slots() == 1u);
    CHECK(!p.alloc.swap_in(9999));
}

NATIVE_TEST(stats_count_swapped_blocks_apart_from_frames) {
    Pool p(2);
    HostSwapBackend swap(4);
    p.alloc.set_swap_backend(&swap);
    const auto a = p.alloc.allocate(), b = p.alloc.allocate();
    const auto sa = p.alloc.swap_out(*a);
    CHECK(p.alloc.swap_out(*b).has_value());
    AllocatorStats st = p.alloc.stats();
    CHECK(st.swapped_blocks == 2u && st.free_blocks == 2u && st.active_blocks == 0u);
    CHECK(p.alloc.swap_in(*sa).has_value());
    st = p.alloc.stats();
    CHECK(st.swapped_blocks == 1u && st.active_blocks == 1u);
}

NATIVE_TEST(eviction_selector_is_advisory) {
    Pool p(2);
    const auto victim = p.alloc.allocate();
    CHECK(!p.alloc.select_eviction_candidate());
    std::uint32_t seen_total = 0;
    p.alloc.set_eviction_selector([&](const MemoryAllocator& a) -> std::optional<PhysicalBlockId> {
        seen_total = a.stats().total_blocks;
        return victim;
    });
    CHECK(p.alloc.select_eviction_candidate() == victim && seen_total == 2u);
    // allocation never evicts on its own, even with a selector installed
    CHECK(p.alloc.allocate().has_value() && !p.alloc.allocate());
    p.alloc.set_eviction_selector([](const MemoryAllocator&) { return std::optional<PhysicalBlockId>{}; });
    CHECK(!p.alloc.select_eviction_candidate());
}

// ---- SwapBackend (bookkeeping cases) ---------------------------------------

NATIVE_TEST(host_swap_backend_slots_capacity_and_discard) {
    Pool p(3);
    HostSwapBackend swap(2);
    CHECK(swap.resident_slots() == 0u && swap.capacity_slots() == 2u);
    const auto s1 = swap.store(*p.alloc.block(0));
    const auto s2 = swap.store(*p.alloc.block(1));
    CHECK(s1 && s2 && *s1 != *s2 && swap.resident_slots() == 2u);
    CHECK(!swap.store(*p.alloc.block(2)));  // full
    CHECK(swap.load(*s1, *p.alloc.block(2)) && swap.resident_slots() == 2u);  // load keeps the slot
    CHECK(swap.load(*s1, *p.alloc.block(2)));
    swap.discard(*s1);
    CHECK(swap.resident_slots() == 1u && !swap.load(*s1, *p.alloc.block(2)) && !swap.load(9999, *p.alloc.block(2)));
    const auto s3 = swap.store(*p.alloc.block(2));  // discard made room; ids keep growing
    CHECK(s3 && *s3 > *s2);
}

// ---- KVCacheManager -------------------------------------------------------

NATIVE_TEST(cache_tracks_created_sequences_with_empty_tables) {
    Pool p(8);
    KVCacheManager c(p.alloc);
    CHECK(!c.contains(1) && c.create_sequence(meta(1)) && c.contains(1) && !c.create_sequence(meta(1)));
    const auto v = c.cache_view(1);
    CHECK(v && v->sequence_id == 1u && v->cache_kind == CacheKind::TextKV && v->block_table->empty());
}

NATIVE_TEST(cache_reserve_maps_whole_blocks_and_release_returns_them) {
    Pool p(8);
    KVCacheManager c(p.alloc);
    CHECK(!c.reserve_tokens(99, kT));
    CHECK(c.create_sequence(meta(1)) && c.reserve_tokens(1, 2 * kT));
    CHECK(c.cache_view(1)->block_table->size() == 2u);
    CHECK(c.reserve_tokens(1, 1) && c.cache_view(1)->block_table->size() == 3u);  // a partial block still maps one
    const std::uint32_t free_before = p.alloc.stats().free_blocks;
    c.release_sequence(1);
    CHECK(!c.contains(1) && p.alloc.stats().free_blocks == free_before + 3);
}

NATIVE_TEST(cache_reserve_checks_capacity_up_front) {
    Pool p(2);
    KVCacheManager c(p.alloc);
    CHECK(c.create_sequence(meta(1)) && !c.reserve_tokens(1, 3 * kT));
    CHECK(c.cache_view(1)->block_table->empty() && p.alloc.stats().free_blocks == 2u);
}

NATIVE_TEST(cache_fork_shares_frames_and_counts_references) {
    Pool p(8);
    KVCacheManager c(p.alloc);
    CHECK(!c.fork_sequence(99, meta(2)));
    CHECK(c.create_sequence(meta(1)) && c.reserve_tokens(1, kT));
    const auto shared = c.cache_view(1)->block_table->lookup(0);
    CHECK(c.fork_sequence(1, meta(2)) && c.contains(2));
    CHECK(c.cache_view(2)->block_table->lookup(0) == shared && p.alloc.info(*shared)->ref_count == 2u);
    CHECK(!c.fork_sequence(1, meta(2)));  // child id already taken
}

NATIVE_TEST(copy_on_write_remaps_a_shared_block_and_keeps_a_sole_owner_in_place) {
    Pool p(8);
    KVCacheManager c(p.alloc);
    CHECK(c.create_sequence(meta(1)) && c.reserve_tokens(1, kT) && c.fork_sequence(1, meta(2)));
    const auto shared = c.cache_view(1)->block_table->lookup(0);
    const auto w = c.ensure_token_writable(2, 0);
    CHECK(w && *w != *shared && c.cache_view(2)->block_table->lookup(0) == w);
    CHECK(p.alloc.info(*shared)->ref_count == 1u && c.cache_view(2)->block_table->entry(0)->writable);
    const std::uint32_t free_before = p.alloc.stats().free_blocks;
    CHECK(c.ensure_token_writable(1, 0) == shared && p.alloc.stats().free_blocks == free_before);
    CHECK(!c.ensure_token_writable(99, 0) && !c.ensure_token_writable(1, kT));  // unknown sequence, unmapped token
}

NATIVE_TEST(sequence_swap_out_frees_frames_and_keeps_the_logical_map) {
    Pool p(4);
    HostSwapBackend swap(8);
    p.alloc.set_swap_backend(&swap);
    KVCacheManager c(p.alloc);
    CHECK(c.create_sequence(meta(1)) && c.reserve_tokens(1, 2 * kT) && p.alloc.stats().free_blocks == 2u);
    CHECK(c.swap_out_sequence(1) == 2u && p.alloc.stats().free_blocks == 4u && swap.resident_slots() == 2u);
    const auto v = c.cache_view(1);
    CHECK(v->block_table->size() == 2u);
    for (const BlockTableEntry& e : v->block_table->entries())
        CHECK(e.swap_slot.has_value() && !v->block_table->lookup(e.logical.index));
    CHECK(c.swap_out_sequence(99) == 0u);
}

NATIVE_TEST(sequence_swap_out_skips_shared_blocks_and_needs_a_backend) {
    Pool p(4);
    KVCacheManager c(p.alloc);
    CHECK(c.create_sequence(meta(1)) && c.reserve_tokens(1, kT));
    CHECK(c.swap_out_sequence(1) == 0u && c.cache_view(1)->block_table->lookup(0));
    HostSwapBackend swap(8);
    p.alloc.set_swap_backend(&swap);
    CHECK(c.fork_sequence(1, meta(2)));
    CHECK(c.swap_out_sequence(1) == 0u && swap.resident_slots() == 0u);
    CHECK(c.cache_view(1)->block_table->lookup(0) && c.cache_view(2)->block_table->lookup(0));
}

NATIVE_TEST(sequence_swap_in_is_all_or_nothing_and_a_no_op_when_resident) {
    Pool p(2);
    HostSwapBackend swap(8);
    p.alloc.set_swap_backend(&swap);
    KVCacheManager c(p.alloc);
    CHECK(c.create_sequence(meta(1)) && c.reserve_tokens(1, 2 * kT) && c.swap_out_sequence(1) == 2u);
    const auto hog = p.alloc.allocate();
    CHECK(hog && p.alloc.stats().free_blocks == 1u);
    CHECK(!c.swap_in_sequence(1) && p.alloc.stats().free_blocks == 1u && swap.resident_slots() == 2u);
    for (const BlockTableEntry& e : c.cache_view(1)->block_table->entries()) CHECK(e.swap_slot.has_value());
    p.alloc.release(*hog);
    CHECK(c.swap_in_sequence(1) && swap.resident_slots() == 0u);
    for (const BlockTableEntry& e : c.cache_view(1)->block_table->entries())
        CHECK(!e.swap_slot.has_value() && c.cache_view(1)->block_table->lookup(e.logical.index));
    const std::uint32_t free_before = p.alloc.stats().free_blocks;
    CHECK(c.swap_in_sequence(1) && p.alloc.stats().free_blocks == free_before);
}

NATIVE_TEST(release_discards_swapped_slots_and_fork_refuses_a_swapped_parent) {
    Pool p(4);
    HostSwapBackend swap(8);
    p.alloc.set_swap_backend(&swap);
    KVCacheManager c(p.alloc);
    CHECK(c.create_sequence(meta(1)) && c.reserve_tokens(1, kT) && c.swap_out_sequence(1) == 1u);
    CHECK(!c.fork_sequence(1, meta(2)) && !c.contains(2));
    CHECK(c.swap_in_sequence(1) && c.fork_sequence(1, meta(2)));
    CHECK(c.create_sequence(meta(3)) && c.reserve_tokens(3, 2 * kT) && c.swap_out_sequence(3) == 2u);
    c.release_sequence(3);
    CHECK(!c.contains(3) && swap.resident_slots() == 0u && p.alloc.stats().swapped_blocks == 0u);
}

// ---- Scheduler ------------------------------------------------------------

Request request(RequestId id, std::uint32_t prompt = 32) {
    Request r;
    r.request_id = id;
    r.root_sequence_id = id;
    r.prompt_tokens = prompt;
    r.sampling.num_parallel_samples = 1;
    r.sampling.max_decode_tokens = 8;
    return r;
}

// Allocator, swap space, cache manager and scheduler over a small pool.
struct Engine {
    Engine(std::uint32_t blocks, std::uint32_t watermark, bool with_swap = true, std::uint32_t max_active = 8)
        : pool(blocks), swap(64), cache(pool.alloc), sched(config(watermark, max_active), cache, pool.alloc) {
        if (with_swap) pool.alloc.set_swap_backend(&swap);
    }
    static SchedulerConfig config(std::uint32_t watermark, std::uint32_t max_active) {
        SchedulerConfig c;
        c.max_active_requests = max_active;
        c.max_batch_tokens = 4096;
        c.preemption_watermark_blocks = watermark;
        return c;
    }
    Pool pool;
    HostSwapBackend swap;
    KVCacheManager cache;
    Scheduler sched;
};

NATIVE_TEST(scheduler_lifecycle_pending_prefill_decode_cancel) {
    Engine e(64, 0);
    CHECK(e.sched.active_size() == 0u && !e.sched.state(1));
    e.sched.enqueue(request(1));
    CHECK(e.sched.state(1) == RequestState::Pending && e.sched.active_size() == 0u);
    const BatchPlan p = e.sched.schedule_next();
    CHECK(p.prefill_requests == std::vector<RequestId>{1} && e.sched.state(1) == RequestState::Prefill);
    CHECK(e.sched.active_size() == 1u && !e.sched.preemption_info(1));
    e.sched.complete_step(1, 1);
    CHECK(e.sched.state(1) == RequestState::Decode);
    const BatchPlan d = e.sched.schedule_next();
    CHECK(d.decode_requests == std::vector<RequestId>{1} && d.scheduled_tokens == 1u);
    e.sched.cancel(1);
    CHECK(e.sched.active_size() == 0u && !e.sched.state(1));
}

NATIVE_TEST(scheduler_preempt_and_resume) {
    Engine e(64, 0);
    CHECK(!e.sched.preempt(99, "x"));
    e.sched.enqueue(request(1));
    (void)e.sched.schedule_next();
    CHECK(e.sched.preempt(1, "cache pressure") && e.sched.state(1) == RequestState::Preempted);
    CHECK(e.sched.active_size() == 0u);
    const auto info = e.sched.preemption_info(1);
    CHECK(info && info->reason == "cache pressure" && info->swapped_blocks == 2u);
    CHECK(e.sched.resume(1) && e.sched.state(1) == RequestState::Decode && e.sched.active_size() == 1u);
    CHECK(!e.sched.preemption_info(1));
}

NATIVE_TEST(scheduler_refused_admission_leaves_nothing_behind_until_preemption_frees_room) {
    Engine e(4, 0);
    e.sched.enqueue(request(1, 64));
    e.sched.enqueue(request(2, 32));
    BatchPlan p = e.sched.schedule_next();
    CHECK(p.prefill_requests == std::vector<RequestId>{1});
    CHECK(e.sched.state(2) == RequestState::Pending && !e.cache.contains(2) && e.sched.active_size() == 1u);
    CHECK(e.sched.preempt(1, "cache pressure"));
    p = e.sched.schedule_next();
    CHECK(p.prefill_requests == std::vector<RequestId>{2} && e.sched.state(2) == RequestState::Prefill);
}

NATIVE_TEST(scheduler_resume_fails_while_the_pool_is_full_and_cancel_frees_swap_slots) {
    Engine e(4, 0);
    e.sched.enqueue(request(1, 32));
    e.sched.enqueue(request(2, 64));
    (void)e.sched.schedule_next();
    CHECK(e.sched.preempt(1, "cache pressure") && e.swap.resident_slots() == 2u);
    (void)e.sched.schedule_next();
    CHECK(e.sched.state(2) == RequestState::Prefill && e.pool.alloc.stats().free_blocks == 0u);
    CHECK(!e.sched.resume(1) && e.sched.state(1) == RequestState::Preempted && e.sched.preemption_info(1));
    e.sched.cancel(1);
    CHECK(!e.sched.state(1) && !e.sched.preemption_info(1) && e.swap.resident_slots() == 0u);
}

// Drives requests to completion (two decode steps each): resume a preempted
// request when nothing is pending; with `manual`, preempt the first decoding
// request when admission is blocked. Returns whether the scheduler itself
// preempted anything.
bool drain(Engine& e, const std::vector<std::uint32_t>& prompts, bool manual) {
    std::vector<RequestId> ids;
    for (std::size_t i = 0; i < prompts.size(); ++i) {
        ids.push_back(i + 1);
        e.sched.enqueue(request(i + 1, prompts[i]));
    }
    auto first = [&](RequestState s) -> std::optional<RequestId> {
        for (RequestId id : ids)
            if (e.sched.state(id) == s) return id;
        return std::nullopt;
    };
    std::unordered_map<RequestId, int> steps;
    std::size_t done = 0;
    bool auto_preempted = false;
    for (int it = 0; it < 200 && done < prompts.size(); ++it) {
        if (!first(RequestState::Pending)) {
            if (const auto pre = first(RequestState::Preempted)) (void)e.sched.resume(*pre);
        }
        const BatchPlan p = e.sched.schedule_next();
        if (!manual && first(RequestState::Preempted)) auto_preempted = true;
        for (RequestId id : p.prefill_requests) e.sched.complete_step(id, 1);
        for (RequestId id : p.decode_requests) {
            e.sched.complete_step(id, 1);
            if (++steps[id] >= 2) {
                e.sched.cancel(id);
                ++done;
            }
        }
        if (manual && p.prefill_requests.empty() && first(RequestState::Pending)) {
            if (const auto v = first(RequestState::Decode)) CHECK(e.sched.preempt(*v, "cache pressure"));
        }
    }
    CHECK(done == prompts.size());
    CHECK(e.pool.alloc.stats().free_blocks == e.pool.alloc.stats().total_blocks);
    CHECK(e.pool.alloc.stats().swapped_blocks == 0u && e.swap.resident_slots() == 0u);
    return auto_preempted;
}

NATIVE_TEST(scheduler_drains_nine_blocks_of_demand_through_four_by_manual_preemption) {
    Engine e(4, 0);
    (void)drain(e, {16, 48, 32, 16, 64}, true);
}

NATIVE_TEST(scheduler_watermark_drains_the_same_demand_on_its_own) {
    Engine e(4, 1);
    CHECK(drain(e, {16, 48, 32, 16, 64}, false));
}

NATIVE_TEST(watermark_zero_keeps_preemption_manual) {
    Engine e(4, 0);
    e.sched.enqueue(request(1, 64));
    CHECK(e.sched.schedule_next().prefill_requests.size() == 1u && e.pool.alloc.stats().free_blocks == 0u);
    e.sched.enqueue(request(2, 32));
    CHECK(e.sched.schedule_next().prefill_requests.empty());
    CHECK(e.sched.state(1) == RequestState::Prefill && e.sched.state(2) == RequestState::Pending);
    CHECK(!e.sched.preemption_info(1));
}

NATIVE_TEST(watermark_preempts_the_newest_older_request_to_admit) {
    Engine e(4, 1);
    e.sched.enqueue(request(1, 32));
    CHECK(e.sched.schedule_next().prefill_requests.size() == 1u);
    e.sched.enqueue(request(2, 32));
    const BatchPlan p = e.sched.schedule_next();
    CHECK(p.prefill_requests == std::vector<RequestId>{2});
    CHECK(e.sched.state(1) == RequestState::Preempted && e.sched.state(2) == RequestState::Prefill);
    const auto info = e.sched.preemption_info(1);
    CHECK(info && !info->reason.empty() && info->swapped_blocks == 2u);

    Engine f(4, 1);
    f.sched.enqueue(request(1, 16));
    (void)f.sched.schedule_next();
    f.sched.enqueue(request(2, 16));
    (void)f.sched.schedule_next();
    f.sched.enqueue(request(3, 32));
    CHECK(f.sched.schedule_next().prefill_requests.size() == 1u);
    CHECK(f.sched.state(1) == RequestState::Prefill && f.sched.state(2) == RequestState::Preempted &&
          f.sched.state(3) == RequestState::Prefill);
}

NATIVE_TEST(watermark_reserve_stays_free_but_never_blocks_a_whole_pool_prompt) {
    Engine e(4, 2);
    e.sched.enqueue(request(1, 32));
    CHECK(e.sched.schedule_next().prefill_requests.size() == 1u && e.pool.alloc.stats().free_blocks >= 2u);
    e.sched.enqueue(request(2, 16));
    CHECK(e.sched.schedule_next().prefill_requests.size() == 1u);
    CHECK(e.sched.state(1) == RequestState::Preempted && e.pool.alloc.stats().free_blocks >= 2u);

    Engine f(4, 2);
    f.sched.enqueue(request(1, 16));
    (void)f.sched.schedule_next();
    f.sched.enqueue(request(2, 64));  // the whole pool: the reserve is capped at capacity
    CHECK(f.sched.schedule_next().prefill_requests == std::vector<RequestId>{2});
    CHECK(f.sched.state(1) == RequestState::Preempted && f.pool.alloc.stats().free_blocks == 0u);
}

NATIVE_TEST(watermark_does_not_preempt_for_an_impossible_prompt_or_without_swap) {
    Engine e(4, 1);
    e.sched.enqueue(request(1, 16));
    (void)e.sched.schedule_next();
    e.sched.enqueue(request(2, 80));  // five blocks never fit four
    CHECK(e.sched.schedule_next().prefill_requests.empty());
    CHECK(e.sched.state(1) == RequestState::Prefill && e.sched.state(2) == RequestState::Pending);
    CHECK(!e.cache.contains(2));

    Engine f(4, 1, /*with_swap=*/false);
    for (RequestId id = 1; id <= 3; ++id) {
        f.sched.enqueue(request(id, 16));
        CHECK(f.sched.schedule_next().prefill_requests.size() == 1u);
    }
    f.sched.enqueue(request(4, 32));
    CHECK(f.sched.schedule_next().prefill_requests.empty());
    int preempted = 0;
    for (RequestId id = 1; id <= 4; ++id) preempted += f.sched.state(id) == RequestState::Preempted;
    CHECK(preempted == 1 && f.sched.state(4) == RequestState::Pending);
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int qvp_refcases_list(char* out, size_t cap) {
    return native::list_cases(out, cap);
}

extern "C" __attribute__((visibility("default"))) int qvp_refcases_run(const char* name, char* msg, size_t cap) {
    return native::run_case(name, msg, cap);
}
