// TEST INFRASTRUCTURE: GPU tests of the C++ host layer on real device pools,
// re-expressing cases of the reference suite (phhuang191129/QwenVL-Paged
// tests/Block.test.cpp, MemoryAllocator.test.cpp, KVCacheManager.test.cpp,
// SwapBackend.test.cpp, PagedAttention.test.cpp, EndToEnd.test.cpp). Cache
// bytes move through MemoryAllocator::write_bytes / read_bytes instead of
// host pointer writes; every bookkeeping assertion is the reference's.
//
// Run from pytest (tests/test_native_gpu.py): qvp_native_list() names the
// cases, qvp_native_run(name) runs one and returns 0 or the failure text.
#include "qwenvl_paged/Block.h"
#include "qwenvl_paged/CacheLayout.h"
#include "qwenvl_paged/KVCacheManager.h"
#include "qwenvl_paged/MemoryAllocator.h"
#include "qwenvl_paged/PagedAttention.h"
#include "qwenvl_paged/Scheduler.h"
#include "qwenvl_paged/SwapBackend.h"

#include <cuda_runtime.h>

#include "harness.h"

#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <sstream>
#include <string>
#include <vector>

using namespace qwenvl_paged;

namespace {

BlockShape shape_of(std::uint32_t tpb, std::uint32_t layers, std::uint32_t heads, std::uint32_t dim,
                    std::uint32_t elem = 4) {
    BlockShape s;
    s.tokens_per_block = tpb;
    s.num_layers = layers;
    s.num_kv_heads = heads;
    s.head_dim = dim;
    s.bytes_per_element = elem;
    return s;
}

AllocatorConfig config_of(BlockShape s, std::uint32_t blocks) {
    AllocatorConfig c;
    c.block_shape = s;
    c.max_blocks = blocks;
    return c;
}

// tests/PagedAttention.test.cpp:80-92 style coordinate hash in [-1, 1)
float mix(std::initializer_list<std::uint32_t> parts) {
    std::uint32_t m = 2166136261u;
    for (std::uint32_t p : parts) m = (m ^ p) * 16777619u;
    return static_cast<float>(m % 2000u) / 1000.0f - 1.0f;
}

void fill_bytes(MemoryAllocator& a, PhysicalBlockId id, std::uint8_t seed) {
    std::vector<std::uint8_t> b(a.block(id)->size_bytes());
    for (std::size_t i = 0; i < b.size(); ++i) b[i] = static_cast<std::uint8_t>((i + seed) % 251);
    CHECK(a.write_bytes(id, 0, b.data(), b.size()));
}

bool holds_bytes(MemoryAllocator& a, PhysicalBlockId id, std::uint8_t seed) {
    std::vector<std::uint8_t> b(a.block(id)->size_bytes());
    if (!a.read_bytes(id, 0, b.data(), b.size())) return false;
    for (std::size_t i = 0; i < b.size(); ++i)
        if (b[i] != static_cast<std::uint8_t>((i + seed) % 251)) return false;
    return true;
}

// Writes one head vector of token `pos` through copy-on-write, as the
// reference tests' write_head_vector does (PagedAttention.test.cpp:97-127).
bool write_vec(KVCacheManager& cache, MemoryAllocator& a, SequenceId s, KVStream st, std::uint32_t layer,
               TokenPosition pos, std::uint32_t head, const std::vector<float>& v) {
    const auto id = cache.ensure_token_writable(s, pos);
    if (!id) return false;
    KVBlockLayout lay;
    lay.shape = a.block_shape();
    const auto off = lay.element_offset(layer, st, pos % lay.shape.tokens_per_block, head);
    if (!off) return false;
    return a.write_bytes(*id, *off * sizeof(float), v.data(), v.size() * sizeof(float));
}

std::vector<float> flat_attention(const std::function<float(std::uint32_t, KVStream, std::uint32_t, std::uint32_t,
                                                            std::uint32_t)>& kv,
                                  const std::vector<float>& q, std::uint32_t layer, std::uint32_t hq,
                                  std::uint32_t hkv, std::uint32_t dim, std::uint32_t ctx, float scale) {
    std::vector<float> out(static_cast<std::size_t>(hq) * dim, 0.f);
    const std::uint32_t g = hq / hkv;
    for (std::uint32_t h = 0; h < hq; ++h) {
        std::vector<float> s(ctx);
        float mx = -INFINITY;
        for (std::uint32_t t = 0; t < ctx; ++t) {
            float d = 0.f;
            for (std::uint32_t i = 0; i < dim; ++i) d += q[h * dim + i] * kv(layer, KVStream::Key, t, h / g, i);
            s[t] = d * scale;
            mx = std::max(mx, s[t]);
        }
        float den = 0.f;
        for (std::uint32_t t = 0; t < ctx; ++t) {
            const float w = std::exp(s[t] - mx);
            den += w;
            for (std::uint32_t i = 0; i < dim; ++i) out[h * dim + i] += w * kv(layer, KVStream::Value, t, h / g, i);
        }
        for (std::uint32_t i = 0; i < dim; ++i) out[h * dim + i] /= den;
    }
    return out;
}

// ---- Block (tests/Block.test.cpp) -------------------------------------------

NATIVE_TEST(block_allocation_is_device_memory_aligned_and_rounded) {
    for (int i = 0; i < 16; ++i) {
        PhysicalBlock b(static_cast<PhysicalBlockId>(i), shape_of(3, 1, 1, 5));
        CHECK(b.data() != nullptr);
        CHECK(reinterpret_cast<std::uintptr_t>(b.data()) % kDefaultBlockAlignmentBytes == 0);
        CHECK(b.size_bytes() >= b.shape().byte_size());
        CHECK(b.size_bytes() % kDefaultBlockAlignmentBytes == 0);
        cudaPointerAttributes at{};
        CHECK(cudaPointerGetAttributes(&at, b.data()) == cudaSuccess && at.type == cudaMemoryTypeDevice);
    }
    HostMemoryOptions o;
    o.prefer_pinned_memory = true;
    CHECK(PhysicalBlock(1, shape_of(4, 1, 1, 4), o).pinned_memory_requested());
}

NATIVE_TEST(block_swap_exchanges_contents_for_owning_blocks_and_pool_views) {
    PhysicalBlock a(1, shape_of(4, 1, 1, 4)), b(2, shape_of(4, 1, 1, 4));
    const std::uint8_t x[4] = {0xA0, 0xA1, 0xA2, 0xA3}, y[4] = {0xB0, 0xB1, 0xB2, 0xB3};
    cudaMemcpy(a.data(), x, 4, cudaMemcpyHostToDevice);
    cudaMemcpy(b.data(), y, 4, cudaMemcpyHostToDevice);
    a.swap(b);
    std::uint8_t r[4];
    cudaMemcpy(r, a.data(), 4, cudaMemcpyDeviceToHost);
    CHECK(std::memcmp(r, y, 4) == 0);
    CHECK(a.id() == 1u && b.id() == 2u);

    MemoryAllocator m(config_of(shape_of(4, 1, 1, 4), 4));
    fill_bytes(m, 0, 1);
    fill_bytes(m, 3, 7);
    std::byte* addr0 = m.block(0)->data();
    m.block(0)->swap(*m.block(3));
    CHECK(m.block(0)->data() == addr0);  // pool views keep their address
    CHECK(holds_bytes(m, 0, 7) && holds_bytes(m, 3, 1));
}

// ---- MemoryAllocator (tests/MemoryAllocator.test.cpp) ---------------------

NATIVE_TEST(allocator_pool_is_one_slab_with_block_at_base_plus_id_stride) {
    MemoryAllocator m(config_of(shape_of(16, 1, 4, 128, 2), 10));
    CHECK(m.has_storage());
    CHECK(m.block_stride() == 32768);
    for (PhysicalBlockId i = 0; i < 10; ++i) CHECK(m.block(i)->data() == m.pool_base() + i * m.block_stride());
    CHECK(m.block(10) == nullptr && m.info(10) == nullptr);
    CHECK(m.stats().bytes_reserved == 10u * 32768u);
}

NATIVE_TEST(copy_block_copies_bytes_and_batches_copies_into_one_launch) {
    MemoryAllocator m(config_of(shape_of(16, 1, 4, 128, 2), 16));
    for (PhysicalBlockId i = 0; i < 8; ++i) fill_bytes(m, i, static_cast<std::uint8_t>(10 + i));
    const auto launches = m.copy_launches();
    for (PhysicalBlockId i = 0; i < 8; ++i) m.copy_block(i, 8 + i);
    CHECK(m.synchronize());
    CHECK(m.copy_launches() == launches + 1);  // eight copies, one kernel
    for (PhysicalBlockId i = 0; i < 8; ++i) CHECK(holds_bytes(m, 8 + i, static_cast<std::uint8_t>(10 + i)));
    // a chain a->b, b->c keeps program order
    fill_bytes(m, 0, 99);
    m.copy_block(0, 1);
    m.copy_block(1, 2);
    CHECK(m.synchronize());
    CHECK(holds_bytes(m, 2, 99));
}

void swap_round_trip(bool device_backend, SwapCoding coding = SwapCoding::raw) {
    MemoryAllocator m(config_of(shape_of(16, 1, 8, 128, 2), 6));
    HostSwapBackend host(4);
    DeviceSwapBackend dev(m, 4, coding);
    SwapBackend* backend = device_backend ? static_cast<SwapBackend*>(&dev) : &host;
    m.set_swap_backend(backend);
    const auto id = m.allocate();
    CHECK(id && *id == 5u);
    fill_bytes(m, *id, 42);
    const std::uint64_t gen = m.info(*id)->generation;
    const auto slot = m.swap_out(*id);
    CHECK(slot && *slot == 1u);
    CHECK(m.info(*id)->state == BlockState::Free && m.info(*id)->generation == gen + 1);
    CHECK(m.stats().swapped_blocks == 1u);
    // the frame is recycled and overwritten before the swap-in
    const auto other = m.allocate();
    CHECK(other && *other == *id);
    fill_bytes(m, *other, 3);
    const auto back = m.swap_in(*slot);
    CHECK(back && *back != *id);
    CHECK(holds_bytes(m, *back, 42));
    CHECK(holds_bytes(m, *other, 3));
    CHECK(m.stats().swapped_blocks == 0u);
    CHECK(!m.swap_in(*slot));  // consumed
}

NATIVE_TEST(swap_out_then_in_restores_contents_host_backend) { swap_round_trip(false); }
NATIVE_TEST(swap_out_then_in_restores_contents_device_backend) { swap_round_trip(true); }
NATIVE_TEST(swap_out_then_in_restores_contents_compressed_device_backend) {
    swap_round_trip(true, SwapCoding::compressed);
}

NATIVE_TEST(device_backend_capacity_and_slot_ids_follow_the_reference) {
    MemoryAllocator m(config_of(shape_of(4, 1, 1, 4), 8));
    DeviceSwapBackend dev(m, 2);
    m.set_swap_backend(&dev);
    CHECK(dev.ready() && dev.capacity_slots() == 2u);
    const auto a = m.allocate(), b = m.allocate(), c = m.allocate();
    const auto sa = m.swap_out(*a), sb = m.swap_out(*b);
    CHECK(sa && sb && *sa == 1u && *sb == 2u);
    CHECK(!m.swap_out(*c));  // full
    m.discard_swapped(*sa);
    const auto sc = m.swap_out(*c);
    CHECK(sc && *sc == 3u);  // ids never reused
    CHECK(dev.resident_slots() == 2u);
}

// ---- KVCacheManager (tests/KVCacheManager.test.cpp) ------------------------

NATIVE_TEST(copy_on_write_materialises_a_private_copy_with_the_same_bytes) {
    MemoryAllocator m(config_of(shape_of(4, 1, 1, 4), 8));
    KVCacheManager cache(m);
    CHECK(cache.create_sequence(SequenceMetadata{1, 1, {}, {}}));
    CHECK(cache.reserve_tokens(1, 8));
    const PhysicalBlockId shared = cache.cache_view(1)->block_table->entries()[1].physical_id;
    fill_bytes(m, shared, 77);
    CHECK(cache.fork_sequence(1, SequenceMetadata{2, 1, {}, {}}));
    CHECK(m.info(shared)->ref_count == 2u);
    const auto copy = cache.ensure_token_writable(2, 5);
    CHECK(copy && *copy != shared);
    CHECK(m.info(shared)->ref_count == 1u);
    CHECK(holds_bytes(m, *copy, 77));
    const auto same = cache.ensure_token_writable(1, 5);  // sole owner now: in place
    CHECK(same && *same == shared);
}

NATIVE_TEST(sequence_swap_out_and_in_restores_every_block_through_the_device_backend) {
    MemoryAllocator m(config_of(shape_of(16, 1, 8, 128, 2), 64));
    DeviceSwapBackend dev(m, 64);
    m.set_swap_backend(&dev);
    KVCacheManager cache(m);
    CHECK(cache.create_sequence(SequenceMetadata{1, 1, {}, {}}));
    CHECK(cache.reserve_tokens(1, 16 * 20));
    std::vector<PhysicalBlockId> before;
    for (const auto& e : cache.cache_view(1)->block_table->entries()) {
        fill_bytes(m, e.physical_id, static_cast<std::uint8_t>(e.logical.index * 3 + 1));
        before.push_back(e.physical_id);
    }
    CHECK(cache.swap_out_sequence(1) == 20u);
    CHECK(m.stats().free_blocks == 64u && m.stats().swapped_blocks == 20u);
    // clobber the freed frames
    CHECK(cache.create_sequence(SequenceMetadata{2, 2, {}, {}}));
    CHECK(cache.reserve_tokens(2, 16 * 64));
    for (const auto& e : cache.cache_view(2)->block_table->entries()) fill_bytes(m, e.physical_id, 200);
    CHECK(!cache.swap_in_sequence(1));  // all-or-nothing: no room
    cache.release_sequence(2);
    CHECK(cache.swap_in_sequence(1));
    for (const auto& e : cache.cache_view(1)->block_table->entries())
        CHECK(holds_bytes(m, e.physical_id, static_cast<std::uint8_t>(e.logical.index * 3 + 1)));
    CHECK(dev.bytes_out() == 20u * 65536u && dev.bytes_in() == 20u * 65536u);
    cache.release_sequence(1);
    CHECK(m.stats().free_blocks == 64u && dev.resident_slots() == 0u);
}

// bf16 bit patterns of N(0,1) values (Box-Muller over a fixed LCG)
std::vector<std::uint16_t> normal_bf16(std::size_t n, std::uint32_t seed) {
    std::vector<std::uint16_t> v(n);
    std::uint64_t x = 0x9E3779B97F4A7C15ull ^ seed;
    auto uniform = [&] {
        x = x * 6364136223846793005ull + 1442695040888963407ull;
        return (static_cast<double>(x >> 11) + 0.5) / 9007199254740992.0;
    };
    for (std::size_t i = 0; i < n; ++i) {
        const float f = static_cast<float>(std::sqrt(-2.0 * std::log(uniform())) * std::cos(6.283185307179586 * uniform()));
        std::uint32_t bits;
        std::memcpy(&bits, &f, 4);
        v[i] = static_cast<std::uint16_t>(bits >> 16);
    }
    return v;
}

NATIVE_TEST(compressed_device_backend_restores_kv_bytes_and_sends_fewer_over_the_link) {
    MemoryAllocator m(config_of(shape_of(16, 1, 8, 128, 2), 64));
    DeviceSwapBackend dev(m, 64, SwapCoding::compressed);
    m.set_swap_backend(&dev);
    CHECK(dev.ready() && dev.coding() == SwapCoding::compressed);
    KVCacheManager cache(m);
    CHECK(cache.create_sequence(SequenceMetadata{1, 1, {}, {}}));
    CHECK(cache.reserve_tokens(1, 16 * 20));
    const std::size_t nb = m.block(0)->size_bytes();
    std::map<std::uint32_t, std::vector<std::uint16_t>> want;
    for (const auto& e : cache.cache_view(1)->block_table->entries()) {
        auto v = normal_bf16(nb / 2, e.logical.index + 1);
        if (e.logical.index == 3) std::fill(v.begin(), v.end(), 0);  // a zero block
        if (e.logical.index == 4)                                   // random bytes: stored raw
            for (std::size_t i = 0; i < v.size(); ++i) v[i] = static_cast<std::uint16_t>(i * 2654435761u >> 7);
        CHECK(m.write_bytes(e.physical_id, 0, v.data(), nb));
        want[e.logical.index] = std::move(v);
    }
    CHECK(cache.swap_out_sequence(1) == 20u);
    CHECK(cache.create_sequence(SequenceMetadata{2, 2, {}, {}}));
    CHECK(cache.reserve_tokens(2, 16 * 64));
    for (const auto& e : cache.cache_view(2)->block_table->entries()) fill_bytes(m, e.physical_id, 200);
    cache.release_sequence(2);
    CHECK(cache.swap_in_sequence(1));
    for (const auto& e : cache.cache_view(1)->block_table->entries()) {
        std::vector<std::uint16_t> got(nb / 2);
        CHECK(m.read_bytes(e.physical_id, 0, got.data(), nb));
        CHECK(got == want[e.logical.index]);
    }
    CHECK(dev.bytes_out() == 20u * nb && dev.bytes_in() == 20u * nb);
    const auto link = dev.link_bytes();
    CHECK(link.first == link.second);
    CHECK(link.first < 20u * nb * 8 / 10);  // 18 coded blocks near 0.75, one raw
    CHECK(link.first > 20u * nb * 6 / 10);
    CHECK(dev.last_error().empty());
    cache.release_sequence(1);
}

NATIVE_TEST(cache_view_block_bytes_are_device_addresses_and_null_when_swapped) {
    MemoryAllocator m(config_of(shape_of(4, 1, 1, 4), 8));
    HostSwapBackend swap(8);
    m.set_swap_backend(&swap);
    KVCacheManager cache(m);
    CHECK(cache.create_sequence(SequenceMetadata{1, 1, {}, {}}));
    CHECK(cache.reserve_tokens(1, 8));
    auto v = cache.cache_view(1);
    CHECK(v->block_bytes(0) == m.block(7)->data() && v->block_bytes(1) == m.block(6)->data());
    CHECK(v->block_bytes(2) == nullptr);
    CHECK(v->slot<float>(KVStream::Value, 0, 5, 0) == reinterpret_cast<const float*>(m.block(6)->data()) + 16 + 1 * 4);
    CHECK(cache.swap_out_sequence(1) == 2u);
    v = cache.cache_view(1);
    CHECK(v->block_bytes(0) == nullptr && v->slot<float>(KVStream::Key, 0, 0, 0) == nullptr);
}

// ---- PagedAttention shim (tests/PagedAttention.test.cpp) ------------------

NATIVE_TEST(decode_shim_uniform_keys_average_the_values_with_host_buffers) {
    MemoryAllocator m(config_of(shape_of(4, 1, 1, 4), 8));
    HostSwapBackend swap(64);
    m.set_swap_backend(&swap);
    KVCacheManager cache(m);
    CHECK(cache.create_sequence(SequenceMetadata{1, 1, {}, {}}));
    CHECK(cache.reserve_tokens(1, 8));
    for (std::uint32_t t = 0; t < 8; ++t) {
        CHECK(write_vec(cache, m, 1, KVStream::Key, 0, t, 0, std::vector<float>(4, 1.f)));
        CHECK(write_vec(cache, m, 1, KVStream::Value, 0, t, 0, std::vector<float>(4, t + 1.f)));
    }
    std::vector<float> q(4, 0.5f), out(4, 0.f);
    CHECK(paged_attention_decode<float>(*cache.cache_view(1), q.data(), PagedAttentionParams{0, 1, 8, 1.f}, out.data()));
    for (float v : out) CHECK_NEAR(v, 4.5, 1e-5);
}

NATIVE_TEST(decode_shim_rejects_like_the_reference_and_leaves_out_untouched) {
    MemoryAllocator m(config_of(shape_of(4, 2, 2, 4), 8));
    HostSwapBackend swap(64);
    m.set_swap_backend(&swap);
    KVCacheManager cache(m);
    CHECK(cache.create_sequence(SequenceMetadata{1, 1, {}, {}}));
    CHECK(cache.reserve_tokens(1, 8));
    const CacheView v = *cache.cache_view(1);
    std::vector<float> q(16, 1.f), out(16, -1.f);
    std::vector<double> qd(8, 1.0), od(8, 0.0);
    CHECK(!paged_attention_decode<float>(CacheView{}, q.data(), PagedAttentionParams{0, 2, 4, 1.f}, out.data()));
    CHECK(!paged_attention_decode<double>(v, qd.data(), PagedAttentionParams{0, 2, 4, 1.f}, od.data()));
    CHECK(!paged_attention_decode<float>(v, nullptr, PagedAttentionParams{0, 2, 4, 1.f}, out.data()));
    CHECK(!paged_attention_decode<float>(v, q.data(), PagedAttentionParams{0, 2, 0, 1.f}, out.data()));
    CHECK(!paged_attention_decode<float>(v, q.data(), PagedAttentionParams{2, 2, 4, 1.f}, out.data()));
    CHECK(!paged_attention_decode<float>(v, q.data(), PagedAttentionParams{0, 3, 4, 1.f}, out.data()));
    CHECK(!paged_attention_decode<float>(v, q.data(), PagedAttentionParams{0, 0, 4, 1.f}, out.data()));
    CHECK(!paged_attention_decode<float>(v, q.data(), PagedAttentionParams{0, 2, 9, 1.f}, out.data()));
    CHECK(cache.swap_out_sequence(1) == 2u);
    CHECK(!paged_attention_decode<float>(*cache.cache_view(1), q.data(), PagedAttentionParams{0, 2, 8, 1.f},
                                         out.data()));
    for (float x : out) CHECK(x == -1.f);
}

NATIVE_TEST(decode_shim_matches_flat_attention_on_scattered_blocks_both_layers) {
    constexpr std::uint32_t T = 4, L = 2, H = 2, D = 4, ctx = 10;
    MemoryAllocator m(config_of(shape_of(T, L, H, D), 12));
    KVCacheManager cache(m);
    CHECK(cache.create_sequence(SequenceMetadata{1, 1, {}, {}}));
    CHECK(cache.create_sequence(SequenceMetadata{99, 99, {}, {}}));
    for (int i = 0; i < 3; ++i) {  // spacer interleaving scatters the frames
        CHECK(cache.reserve_tokens(1, T));
        CHECK(cache.reserve_tokens(99, T));
    }
    cache.release_sequence(99);
    auto kv = [](std::uint32_t layer, KVStream s, std::uint32_t t, std::uint32_t h, std::uint32_t d) {
        return mix({layer, s == KVStream::Key ? 0u : 1u, t, h, d});
    };
    for (std::uint32_t l = 0; l < L; ++l)
        for (KVStream s : {KVStream::Key, KVStream::Value})
            for (std::uint32_t t = 0; t < ctx; ++t)
                for (std::uint32_t h = 0; h < H; ++h) {
                    std::vector<float> vec(D);
                    for (std::uint32_t d = 0; d < D; ++d) vec[d] = kv(l, s, t, h, d);
                    CHECK(write_vec(cache, m, 1, s, l, t, h, vec));
                }
    std::vector<float> q(H * D);
    for (std::size_t i = 0; i < q.size(); ++i) q[i] = 0.25f * static_cast<float>(i) - 0.5f;
    for (std::uint32_t l = 0; l < L; ++l) {
        std::vector<float> out(q.size());
        CHECK(paged_attention_decode<float>(*cache.cache_view(1), q.data(), PagedAttentionParams{l, H, ctx, 0.5f},
                                            out.data()));
        const auto want = flat_attention(kv, q, l, H, H, D, ctx, 0.5f);
        for (std::size_t i = 0; i < out.size(); ++i) CHECK_NEAR(out[i], want[i], 1e-5);
    }
}

NATIVE_TEST(batched_decode_matches_the_per_sequence_shim_and_refuses_swapped_sequences) {
    // bf16, 7B-like head shape, several sequences through PagedDecodeBatch
    constexpr std::uint32_t T = 16, H = 4, D = 128, HQ = 28;
    MemoryAllocator m(config_of(shape_of(T, 1, H, D, 2), 256));
    HostSwapBackend swap(256);
    m.set_swap_backend(&swap);
    KVCacheManager cache(m);
    const std::vector<std::uint32_t> ctx = {1, 17, 300, 40, 1000};
    std::vector<CacheView> views;
    for (std::size_t i = 0; i < ctx.size(); ++i) {
        const SequenceId s = 10 + i;
        CHECK(cache.create_sequence(SequenceMetadata{s, s, {}, {}}));
        CHECK(cache.reserve_tokens(s, ctx[i]));
    }
    // random bf16 values in every allocated block
    std::vector<bfloat16> blk(m.block(0)->size_bytes() / 2);
    for (PhysicalBlockId id = 0; id < 256; ++id) {
        if (m.info(id)->state == BlockState::Free) continue;
        for (std::size_t k = 0; k < blk.size(); ++k) blk[k] = bfloat16(mix({id, static_cast<std::uint32_t>(k)}));
        CHECK(m.write_bytes(id, 0, blk.data(), blk.size() * 2));
    }
    for (std::size_t i = 0; i < ctx.size(); ++i) views.push_back(*cache.cache_view(10 + i));
    const std::size_t per = HQ * D;
    std::vector<bfloat16> q(ctx.size() * per);
    for (std::size_t k = 0; k < q.size(); ++k) q[k] = bfloat16(mix({7u, static_cast<std::uint32_t>(k)}));
    void *qd = nullptr, *od = nullptr;
    CHECK(cudaMalloc(&qd, q.size() * 2) == cudaSuccess && cudaMalloc(&od, q.size() * 2) == cudaSuccess);
    cudaMemcpy(qd, q.data(), q.size() * 2, cudaMemcpyHostToDevice);
    PagedDecodeBatch batch(m);
    CHECK(batch.run(views, ctx, 0, HQ, 1.f / std::sqrt(128.f), qd, od));
    CHECK(batch.device_error() == 0);
    std::vector<bfloat16> got(q.size());
    cudaMemcpy(got.data(), od, got.size() * 2, cudaMemcpyDeviceToHost);
    for (std::size_t i = 0; i < ctx.size(); ++i) {
        std::vector<bfloat16> one(per);
        CHECK(paged_attention_decode<bfloat16>(views[i], q.data() + i * per,
                                               PagedAttentionParams{0, HQ, ctx[i], 1.f / std::sqrt(128.f)}, one.data()));
        for (std::size_t k = 0; k < per; ++k)
            CHECK_NEAR(static_cast<float>(got[i * per + k]), static_cast<float>(one[k]), 2e-2);
    }
    // a swapped-out sequence in the batch: refused, nothing written
    CHECK(cache.swap_out_sequence(12) > 0u);
    views[2] = *cache.cache_view(12);
    cudaMemset(od, 0x7f, q.size() * 2);
    CHECK(!batch.run(views, ctx, 0, HQ, 1.f, qd, od));
    std::vector<std::uint8_t> raw(q.size() * 2);
    cudaMemcpy(raw.data(), od, raw.size(), cudaMemcpyDeviceToHost);
    for (std::uint8_t b : raw) CHECK(b == 0x7f);
    cudaFree(qd);
    cudaFree(od);
}

// ---- End to end (tests/EndToEnd.test.cpp) ---------------------------------

NATIVE_TEST(end_to_end_scheduler_prefill_decode_preempt_resume) {
    constexpr std::uint32_t T = 4, L = 2, H = 2, D = 4, HQ = 4, prompt = 6, decode = 3;
    MemoryAllocator m(config_of(shape_of(T, L, H, D), 16));
    DeviceSwapBackend swap(m, 16);
    m.set_swap_backend(&swap);
    KVCacheManager cache(m);
    SchedulerConfig sc;
    sc.max_active_requests = 3;
    sc.max_batch_tokens = 64;
    Scheduler sched(sc, cache, m);
    auto kv = [](SequenceId s, std::uint32_t l, KVStream st, std::uint32_t t, std::uint32_t h, std::uint32_t d) {
        return mix({static_cast<std::uint32_t>(s), l, st == KVStream::Key ? 0u : 1u, t, h, d});
    };
    auto query = [&](SequenceId s, std::uint32_t pos) {
        std::vector<float> q(HQ * D);
        for (std::size_t i = 0; i < q.size(); ++i) q[i] = kv(s, 0, KVStream::Key, pos, 0, static_cast<std::uint32_t>(i));
        return q;
    };
    auto write_token = [&](SequenceId s, std::uint32_t pos) {
        for (std::uint32_t l = 0; l < L; ++l)
            for (KVStream st : {KVStream::Key, KVStream::Value})
                for (std::uint32_t h = 0; h < H; ++h) {
                    std::vector<float> v(D);
                    for (std::uint32_t d = 0; d < D; ++d) v[d] = kv(s, l, st, pos, h, d);
                    CHECK(write_vec(cache, m, s, st, l, pos, h, v));
                }
    };
    auto check_attention = [&](SequenceId s, std::uint32_t ctx) {
        for (std::uint32_t l = 0; l < L; ++l) {
            const auto q = query(s, ctx - 1);
            std::vector<float> out(q.size());
            CHECK(paged_attention_decode<float>(*cache.cache_view(s), q.data(), PagedAttentionParams{l, HQ, ctx, 0.5f},
                                                out.data()));
            auto f = [&](std::uint32_t ll, KVStream st, std::uint32_t t, std::uint32_t h, std::uint32_t d) {
                return kv(s, ll, st, t, h, d);
            };
            const auto want = flat_attention(f, q, l, HQ, H, D, ctx, 0.5f);
            for (std::size_t i = 0; i < out.size(); ++i) CHECK_NEAR(out[i], want[i], 1e-5);
        }
    };
    for (RequestId r = 1; r <= 3; ++r) {
        Request req;
        req.request_id = r;
        req.root_sequence_id = 100 + r;
        req.prompt_tokens = prompt;
        sched.enqueue(req);
    }
    const BatchPlan p = sched.schedule_next();
    CHECK(p.prefill_requests.size() == 3u);
    for (RequestId r = 1; r <= 3; ++r) {
        for (std::uint32_t pos = 0; pos < prompt; ++pos) {
            write_token(100 + r, pos);
            check_attention(100 + r, pos + 1);  // prefill as per-position decode
        }
        sched.complete_step(r, prompt);
    }
    std::uint32_t len = prompt;
    for (std::uint32_t step = 0; step < decode; ++step) {
        const BatchPlan d = sched.schedule_next();
        CHECK(d.decode_requests.size() == 3u);
        for (RequestId r : d.decode_requests) {
            if (len % T == 0) CHECK(cache.reserve_tokens(100 + r, 1));
            write_token(100 + r, len);
            check_attention(100 + r, len + 1);
        }
        ++len;
    }
    // preempt: refuses attention while swapped, resumes with identical output
    CHECK(sched.preempt(2, "test"));
    std::vector<float> q = query(102, len - 1), out(q.size(), -3.f);
    CHECK(!paged_attention_decode<float>(*cache.cache_view(102), q.data(), PagedAttentionParams{0, HQ, len, 0.5f},
                                         out.data()));
    CHECK(sched.resume(2));
    check_attention(102, len);
    for (RequestId r = 1; r <= 3; ++r) sched.cancel(r);
    CHECK(m.stats().free_blocks == 16u && m.stats().swapped_blocks == 0u);
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int qvp_native_list(char* out, size_t cap) {
    return native::list_cases(out, cap);
}

extern "C" __attribute__((visibility("default"))) int qvp_native_run(const char* name, char* msg, size_t cap) {
    return native::run_case(name, msg, cap);
}
