// TEST INFRASTRUCTURE ONLY - C wrappers around the reference compiled from
// its own sources (phhuang191129/QwenVL-Paged, src/*.cpp and the header
// template include/qwenvl_paged/PagedAttention.h:53-127).
//
// Built by oracle/Makefile into oracle/_ref/libqvp_ref.so with the reference
// namespace renamed (-Dqwenvl_paged=qwenvl_paged_ref) so it can share a
// process with libqvp.so. Only tests/, the smoke check and bench.py's
// reference arm load it, as the checker or the timed CPU baseline.
#include "qwenvl_paged/KVCacheManager.h"
#include "qwenvl_paged/MemoryAllocator.h"
#include "qwenvl_paged/PagedAttention.h"

#include <atomic>
#include <cstdint>
#include <cstring>
#include <memory>
#include <thread>
#include <vector>

namespace ref = qwenvl_paged;

namespace {

// 2-byte host bfloat16 so the reference template reads the same bytes the GPU
// reads: exact widening, round-to-nearest-even narrowing.
struct bf16h {
    std::uint16_t bits;
    bf16h() = default;
    explicit bf16h(float f) {
        std::uint32_t u;
        std::memcpy(&u, &f, 4);
        if ((u & 0x7fffffffu) > 0x7f800000u) {
            bits = static_cast<std::uint16_t>((u >> 16) | 0x40u);
        } else {
            u += 0x7fffu + ((u >> 16) & 1u);
            bits = static_cast<std::uint16_t>(u >> 16);
        }
    }
    explicit operator float() const {
        const std::uint32_t u = static_cast<std::uint32_t>(bits) << 16;
        float f;
        std::memcpy(&f, &u, 4);
        return f;
    }
};
static_assert(sizeof(bf16h) == 2, "bf16h must be two bytes");

struct RefPool {
    ref::BlockShape shape{};
    std::unique_ptr<ref::MemoryAllocator> allocator;
};

}  // namespace

extern "C" {

struct ref_shape {
    std::uint32_t tokens_per_block, num_layers, num_kv_heads, head_dim, bytes_per_element;
};

// A reference MemoryAllocator of `num_blocks` blocks whose bytes are copied
// from a flat pool (block i at pool + i*stride).
__attribute__((visibility("default"))) void* ref_pool_create(const ref_shape* s, std::uint32_t num_blocks,
                                                             const std::uint8_t* pool, std::size_t stride) {
    auto* p = new RefPool;
    p->shape.tokens_per_block = s->tokens_per_block;
    p->shape.num_layers = s->num_layers;
    p->shape.num_kv_heads = s->num_kv_heads;
    p->shape.head_dim = s->head_dim;
    p->shape.bytes_per_element = s->bytes_per_element;
    ref::AllocatorConfig cfg;
    cfg.block_shape = p->shape;
    cfg.max_blocks = num_blocks;
    p->allocator = std::make_unique<ref::MemoryAllocator>(cfg);
    if (pool != nullptr) {
        for (std::uint32_t i = 0; i < num_blocks; ++i) {
            ref::PhysicalBlock* b = p->allocator->block(i);
            const std::size_t n = b->size_bytes() < stride ? b->size_bytes() : stride;
            std::memcpy(b->data(), pool + static_cast<std::size_t>(i) * stride, n);
        }
    }
    return p;
}

__attribute__((visibility("default"))) void ref_pool_destroy(void* h) { delete static_cast<RefPool*>(h); }

// Block tables for a batch, built with BlockTable::map (one per sequence,
// negative entries left unmapped) so timing loops do not rebuild them.
__attribute__((visibility("default"))) void* ref_tables_create(void* h, std::uint32_t batch, std::uint32_t pitch,
                                                               const std::int32_t* tables,
                                                               const std::int32_t* context_lens) {
    auto* p = static_cast<RefPool*>(h);
    const std::uint32_t T = p->shape.tokens_per_block;
    auto* tabs = new std::vector<ref::BlockTable>;
    tabs->reserve(batch);
    for (std::uint32_t b = 0; b < batch; ++b) {
        ref::BlockTable t(b + 1);
        const std::int32_t c = context_lens[b];
        const std::uint32_t nblk = c > 0 ? (static_cast<std::uint32_t>(c) + T - 1) / T : 0;
        for (std::uint32_t i = 0; i < nblk && i < pitch; ++i) {
            const std::int32_t id = tables[static_cast<std::size_t>(b) * pitch + i];
            if (id < 0) continue;
            ref::LogicalBlock lb;
            lb.sequence_id = b + 1;
            lb.index = i;
            lb.start_token = i * T;
            lb.token_count = T;
            t.map(lb, static_cast<ref::PhysicalBlockId>(id), true);
        }
        tabs->push_back(std::move(t));
    }
    return tabs;
}

__attribute__((visibility("default"))) void ref_tables_destroy(void* t) {
    delete static_cast<std::vector<ref::BlockTable>*>(t);
}

// Runs the reference paged_attention_decode<T> for every sequence of a batch
// over tables from ref_tables_create. dtype 0: T = float; dtype 1: T = bf16h.
// `out` holds T elements. status[b] receives the template's return value.
// Sequences are spread over `threads` std::threads (the calls only read
// shared state). Returns the number of sequences that succeeded.
__attribute__((visibility("default"))) int ref_decode_bound(void* h, void* tables_handle, int dtype,
                                                            std::uint32_t layer, std::uint32_t num_query_heads,
                                                            float scale, std::uint32_t batch,
                                                            const std::int32_t* context_lens, const void* query,
                                                            void* out, std::int32_t* status, int threads) {
    auto* p = static_cast<RefPool*>(h);
    auto& tabs = *static_cast<std::vector<ref::BlockTable>*>(tables_handle);
    const std::size_t elem = dtype == 0 ? 4 : 2;
    const std::size_t row = static_cast<std::size_t>(num_query_heads) * p->shape.head_dim * elem;
    std::atomic<std::uint32_t> next{0};
    auto work = [&]() {
        for (;;) {
            const std::uint32_t b = next.fetch_add(1);
            if (b >= batch) return;
            ref::CacheView view;
            view.sequence_id = b + 1;
            view.block_table = &tabs[b];
            view.allocator = p->allocator.get();
            view.layout.shape = p->shape;
            ref::PagedAttentionParams params;
            params.layer = layer;
            params.num_query_heads = num_query_heads;
            params.context_len = context_lens[b] > 0 ? static_cast<std::uint32_t>(context_lens[b]) : 0;
            params.scale = scale;
            const auto* q = static_cast<const std::uint8_t*>(query) + b * row;
            auto* o = static_cast<std::uint8_t*>(out) + b * row;
            bool ok;
            if (dtype == 0)
                ok = ref::paged_attention_decode<float>(view, reinterpret_cast<const float*>(q), params,
                                                        reinterpret_cast<float*>(o));
            else
                ok = ref::paged_attention_decode<bf16h>(view, reinterpret_cast<const bf16h*>(q), params,
                                                        reinterpret_cast<bf16h*>(o));
            status[b] = ok ? 1 : 0;
        }
    };
    if (threads < 1) threads = 1;
    std::vector<std::thread> workers;
    for (int i = 1; i < threads; ++i) workers.emplace_back(work);
    work();
    for (auto& t : workers) t.join();
    int ok = 0;
    for (std::uint32_t b = 0; b < batch; ++b) ok += status[b] == 1;
    return ok;
}

// ref_tables_create + ref_decode_bound + ref_tables_destroy in one call.
__attribute__((visibility("default"))) int ref_decode_batch(void* h, int dtype, std::uint32_t layer,
                                                            std::uint32_t num_query_heads, float scale,
                                                            std::uint32_t batch, std::uint32_t pitch,
                                                            const std::int32_t* tables,
                                                            const std::int32_t* context_lens, const void* query,
                                                            void* out, std::int32_t* status, int threads) {
    void* t = ref_tables_create(h, batch, pitch, tables, context_lens);
    const int ok = ref_decode_bound(h, t, dtype, layer, num_query_heads, scale, batch, context_lens, query, out,
                                    status, threads);
    ref_tables_destroy(t);
    return ok;
}

}  // extern "C"
