// TEST INFRASTRUCTURE: GPU checks of the host layer's additions on device
// pools, driven by tests/test_host_layer_gpu.py:
//  * PagedDecodeBatch with device-resident block tables against the per-step
//    flatten: over decode steps that cross block boundaries, copy on write,
//    reorder the batch and refuse a swapped-out sequence, both must write
//    bit-identical outputs;
//  * KVAppendBatch: appended K/V land byte-exact in their block slots;
//  * PagedPrefillBatch: within the bf16 tolerance of per-position decodes.
#include "qwenvl_paged/KVCacheManager.h"
#include "qwenvl_paged/MemoryAllocator.h"
#include "qwenvl_paged/PagedAttention.h"
#include "qwenvl_paged/SwapBackend.h"

#include <cuda_runtime.h>

#include "harness.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

using namespace qwenvl_paged;

namespace {

constexpr std::uint32_t kT = 16, kH = 4, kD = 128, kHQ = 28;

AllocatorConfig config(std::uint32_t blocks) {
    AllocatorConfig c;
    c.block_shape.tokens_per_block = kT;
    c.block_shape.num_layers = 1;
    c.block_shape.num_kv_heads = kH;
    c.block_shape.head_dim = kD;
    c.block_shape.bytes_per_element = 2;
    c.max_blocks = blocks;
    return c;
}

float mix(std::uint32_t a, std::uint32_t b) {
    std::uint32_t m = 2166136261u;
    m = (m ^ a) * 16777619u;
    m = (m ^ b) * 16777619u;
    return static_cast<float>(m % 2000u) / 1000.0f - 1.0f;
}

void fill_block(MemoryAllocator& m, PhysicalBlockId id) {
    std::vector<bfloat16> blk(m.block(id)->shape().byte_size() / 2);
    for (std::size_t k = 0; k < blk.size(); ++k) blk[k] = bfloat16(mix(id, static_cast<std::uint32_t>(k)));
    CHECK(m.write_bytes(id, 0, blk.data(), blk.size() * 2));
}

NATIVE_TEST(resident_tables_decode_bit_identical_to_the_per_step_flatten) {
    constexpr std::uint32_t kBlocks = 2048;
    MemoryAllocator m(config(kBlocks));
    HostSwapBackend swap(kBlocks);
    m.set_swap_backend(&swap);
    KVCacheManager cache(m);
    std::vector<SequenceId> order;
    std::vector<std::uint32_t> ctx;
    for (SequenceId s = 1; s <= 12; ++s) {
        CHECK(cache.create_sequence(SequenceMetadata{s, s, {}, {}}));
        ctx.push_back(15 + 97 * static_cast<std::uint32_t>(s));
        CHECK(cache.reserve_tokens(s, ctx.back()));
        order.push_back(s);
    }
    for (PhysicalBlockId id = 0; id < kBlocks; ++id)
        if (m.info(id)->state != BlockState::Free) fill_block(m, id);
    CHECK(m.synchronize());

    const std::size_t max_batch = 16, per = kHQ * kD;
    std::vector<bfloat16> q(max_batch * per);
    for (std::size_t k = 0; k < q.size(); ++k) q[k] = bfloat16(mix(7u, static_cast<std::uint32_t>(k)));
    void *qd = nullptr, *o1 = nullptr, *o2 = nullptr;
    CHECK(cudaMalloc(&qd, q.size() * 2) == cudaSuccess && cudaMalloc(&o1, q.size() * 2) == cudaSuccess &&
          cudaMalloc(&o2, q.size() * 2) == cudaSuccess);
    cudaMemcpy(qd, q.data(), q.size() * 2, cudaMemcpyHostToDevice);

    PagedDecodeBatch flat(m), resident(m, true);
    const float scale = 1.f / std::sqrt(static_cast<float>(kD));
    std::vector<std::uint8_t> a(q.size() * 2), b(q.size() * 2);
    std::uint64_t steady_rows = 0;
    int steady_steps = 0;
    SequenceId next = 100;
    for (int it = 0; it < 48; ++it) {
        if (it == 10) {  // fork two sequences; their first tokens copy on write
            for (std::size_t i : {2u, 5u}) {
                CHECK(cache.fork_sequence(order[i], SequenceMetadata{next, next, {}, {}}));
                order.push_back(next++);
                ctx.push_back(ctx[i]);
            }
        }
        if (it == 20) {  // reorder
            std::swap(order[0], order[7]);
            std::swap(ctx[0], ctx[7]);
        }
        bool crossed = false;
        for (std::size_t i = 0; i < order.size(); ++i) {
            if (ctx[i] % kT == 0) {
                CHECK(cache.reserve_tokens(order[i], 1));
                crossed = true;
            }
            const auto id = cache.ensure_token_writable(order[i], ctx[i]);
            CHECK(id.has_value());
            ++ctx[i];
        }
        std::vector<CacheView> views;
        for (SequenceId s : order) views.push_back(*cache.cache_view(s));
        cudaMemset(o1, 0, q.size() * 2);
        cudaMemset(o2, 0xff, q.size() * 2);
        CHECK(flat.run(views, ctx, 0, kHQ, scale, qd, o1));
        CHECK(resident.run(views, ctx, 0, kHQ, scale, qd, o2));
        CHECK(flat.device_error() == 0 && resident.device_error() == 0);
        const std::size_t used = order.size() * per * 2;
        cudaMemcpy(a.data(), o1, used, cudaMemcpyDeviceToHost);
        cudaMemcpy(b.data(), o2, used, cudaMemcpyDeviceToHost);
        CHECK(std::memcmp(a.data(), b.data(), used) == 0);
        if (it > 0 && it != 10 && it != 20 && !crossed) {
            steady_rows += resident.rows_uploaded();
            ++steady_steps;
        }
    }
    CHECK(steady_steps > 0 && steady_rows == 0);

    // a swapped-out sequence: both refuse and leave `out` alone
    CHECK(cache.swap_out_sequence(order[3]) > 0u);
    std::vector<CacheView> views;
    for (SequenceId s : order) views.push_back(*cache.cache_view(s));
    cudaMemset(o2, 0x7f, q.size() * 2);
    CHECK(!resident.run(views, ctx, 0, kHQ, scale, qd, o2));
    CHECK(resident.last_status() == 2);  // QVP_ERR_UNMAPPED
    CHECK(!flat.run(views, ctx, 0, kHQ, scale, qd, o2));
    cudaMemcpy(b.data(), o2, b.size(), cudaMemcpyDeviceToHost);
    for (std::uint8_t x : b) CHECK(x == 0x7f);
    // swapped back in (new frames): the next step matches again
    CHECK(cache.swap_in_sequence(order[3]));
    views.clear();
    for (SequenceId s : order) views.push_back(*cache.cache_view(s));
    CHECK(flat.run(views, ctx, 0, kHQ, scale, qd, o1));
    CHECK(resident.run(views, ctx, 0, kHQ, scale, qd, o2));
    CHECK(resident.rows_uploaded() == order.size());  // the refusal forgot every row
    const std::size_t used = order.size() * per * 2;
    cudaMemcpy(a.data(), o1, used, cudaMemcpyDeviceToHost);
    cudaMemcpy(b.data(), o2, used, cudaMemcpyDeviceToHost);
    CHECK(std::memcmp(a.data(), b.data(), used) == 0);
    cudaFree(qd);
    cudaFree(o1);
    cudaFree(o2);
}

// bf16 bits of a seeded value for (sequence, token, stream, head, dim)
bfloat16 kv_value(SequenceId s, std::uint32_t t, std::uint32_t stream, std::uint32_t h, std::uint32_t d) {
    std::uint32_t m = 2166136261u;
    for (std::uint32_t part : {static_cast<std::uint32_t>(s), t, stream, h, d}) m = (m ^ part) * 16777619u;
    return bfloat16(static_cast<float>(m % 2000u) / 1000.0f - 1.0f);
}

// Writes every prompt token's K/V with KVAppendBatch (one launch per token
// position, all sequences that have it), checks the bytes landed in their
// slots, then prefills the prompts with PagedPrefillBatch and compares with
// the single-sequence decode at each position.
NATIVE_TEST(kv_append_places_tokens_and_prefill_matches_per_position_decode) {
    constexpr std::uint32_t kBlocks = 64;
    MemoryAllocator m(config(kBlocks));
    KVCacheManager cache(m);
    const std::vector<std::uint32_t> ctx = {20, 33, 16, 1};
    const std::size_t B = ctx.size();
    for (std::size_t b = 0; b < B; ++b) {
        CHECK(cache.create_sequence(SequenceMetadata{b + 1, b + 1, {}, {}}));
        CHECK(cache.reserve_tokens(b + 1, ctx[b]));
    }
    const std::size_t row = static_cast<std::size_t>(kH) * kD;  // one token of one stream
    void *kd = nullptr, *vd = nullptr;
    CHECK(cudaMalloc(&kd, B * row * 2) == cudaSuccess && cudaMalloc(&vd, B * row * 2) == cudaSuccess);
    KVAppendBatch append(m);
    const std::uint32_t max_ctx = *std::max_element(ctx.begin(), ctx.end());
    for (std::uint32_t t = 0; t < max_ctx; ++t) {
        std::vector<CacheView> views;
        std::vector<std::uint32_t> pos;
        std::vector<bfloat16> kh, vh;
        for (std::size_t b = 0; b < B; ++b) {
            if (t >= ctx[b]) continue;
            CHECK(cache.ensure_token_writable(b + 1, t).has_value());
            views.push_back(*cache.cache_view(b + 1));
            pos.push_back(t);
            for (std::uint32_t h = 0; h < kH; ++h)
                for (std::uint32_t d = 0; d < kD; ++d) {
                    kh.push_back(kv_value(b + 1, t, 0, h, d));
                    vh.push_back(kv_value(b + 1, t, 1, h, d));
                }
        }
        cudaMemcpy(kd, kh.data(), kh.size() * 2, cudaMemcpyHostToDevice);
        cudaMemcpy(vd, vh.data(), vh.size() * 2, cudaMemcpyHostToDevice);
        CHECK(append.run(views, pos, 0, kd, vd));
        CHECK(m.synchronize());  // the host buffers above are reused next token
    }
    CHECK(append.device_error() == 0);

    // every token's K and V sit at their slots
    KVBlockLayout layout;
    layout.shape = m.block_shape();
    std::vector<std::uint16_t> blk(m.block_shape().byte_size() / 2);
    for (std::size_t b = 0; b < B; ++b) {
        const auto v = cache.cache_view(b + 1);
        for (std::uint32_t t = 0; t < ctx[b]; ++t) {
            const PhysicalBlockId id = *v->block_table->lookup(t / kT);
            CHECK(m.read_bytes(id, 0, blk.data(), blk.size() * 2));
            for (std::uint32_t st = 0; st < 2; ++st)
                for (std::uint32_t h = 0; h < kH; ++h) {
                    const std::size_t off =
                        *layout.element_offset(0, st == 0 ? KVStream::Key : KVStream::Value, t % kT, h);
                    for (std::uint32_t d = 0; d < kD; ++d) CHECK(blk[off + d] == kv_value(b + 1, t, st, h, d).bits);
                }
        }
    }

    // prefill of the whole prompts against the decode at each position
    const std::size_t qrow = static_cast<std::size_t>(kHQ) * kD;
    std::vector<bfloat16> q(B * max_ctx * qrow);
    for (std::size_t k = 0; k < q.size(); ++k) q[k] = bfloat16(mix(11u, static_cast<std::uint32_t>(k)));
    void *qd = nullptr, *od = nullptr;
    CHECK(cudaMalloc(&qd, q.size() * 2) == cudaSuccess && cudaMalloc(&od, q.size() * 2) == cudaSuccess);
    cudaMemcpy(qd, q.data(), q.size() * 2, cudaMemcpyHostToDevice);
    std::vector<CacheView> views;
    for (std::size_t b = 0; b < B; ++b) views.push_back(*cache.cache_view(b + 1));
    const float scale = 1.f / std::sqrt(static_cast<float>(kD));
    PagedPrefillBatch prefill(m);
    CHECK(prefill.run(views, ctx, ctx, 0, kHQ, scale, qd, od));
    CHECK(prefill.device_error() == 0);
    std::vector<bfloat16> got(q.size());
    cudaMemcpy(got.data(), od, got.size() * 2, cudaMemcpyDeviceToHost);
    std::vector<bfloat16> want(qrow);
    for (std::size_t b = 0; b < B; ++b)
        for (std::uint32_t t = 0; t < ctx[b]; ++t) {
            const bfloat16* qp = q.data() + (b * max_ctx + t) * qrow;
            CHECK(paged_attention_decode<bfloat16>(views[b], qp, PagedAttentionParams{0, kHQ, t + 1, scale},
                                                   want.data()));
            for (std::size_t k = 0; k < qrow; ++k)
                CHECK_NEAR(static_cast<float>(got[(b * max_ctx + t) * qrow + k]), static_cast<float>(want[k]), 2e-2);
        }
    cudaFree(kd);
    cudaFree(vd);
    cudaFree(qd);
    cudaFree(od);
}

// Copy-on-write ordering on real bytes: a branch appends into the shared
// last block, so ensure_token_writable queues a copy and KVAppendBatch must
// land it before writing the new token. The branch's private block then holds
// the parent's earlier tokens plus its own; the parent's block is unchanged.
NATIVE_TEST(kv_append_after_copy_on_write_keeps_the_parent_block_intact) {
    MemoryAllocator m(config(16));
    KVCacheManager cache(m);
    CHECK(cache.create_sequence(SequenceMetadata{1, 1, {}, {}}) && cache.reserve_tokens(1, 8));
    const std::size_t row = static_cast<std::size_t>(kH) * kD;
    void *kd = nullptr, *vd = nullptr;
    CHECK(cudaMalloc(&kd, 2 * row * 2) == cudaSuccess && cudaMalloc(&vd, 2 * row * 2) == cudaSuccess);
    KVAppendBatch append(m);
    auto put = [&](const std::vector<SequenceId>& seqs, std::uint32_t t) {
        std::vector<CacheView> views;
        std::vector<std::uint32_t> pos;
        std::vector<bfloat16> kh, vh;
        for (SequenceId s : seqs) {
            CHECK(cache.ensure_token_writable(s, t).has_value());
            views.push_back(*cache.cache_view(s));
            pos.push_back(t);
            for (std::uint32_t h = 0; h < kH; ++h)
                for (std::uint32_t d = 0; d < kD; ++d) {
                    kh.push_back(kv_value(s, t, 0, h, d));
                    vh.push_back(kv_value(s, t, 1, h, d));
                }
        }
        cudaMemcpy(kd, kh.data(), kh.size() * 2, cudaMemcpyHostToDevice);
        cudaMemcpy(vd, vh.data(), vh.size() * 2, cudaMemcpyHostToDevice);
        CHECK(append.run(views, pos, 0, kd, vd));
        CHECK(m.synchronize());
    };
    for (std::uint32_t t = 0; t < 7; ++t) put({1}, t);
    CHECK(cache.fork_sequence(1, SequenceMetadata{2, 1, {}, {}}));
    const PhysicalBlockId shared = *cache.cache_view(1)->block_table->lookup(0);
    put({2}, 7);  // the branch copies block 0, then writes token 7 into its copy
    put({1}, 7);  // the parent now holds block 0 alone and writes in place
    const PhysicalBlockId mine = *cache.cache_view(2)->block_table->lookup(0);
    CHECK(mine != shared && *cache.cache_view(1)->block_table->lookup(0) == shared);
    CHECK(append.device_error() == 0);
    KVBlockLayout layout;
    layout.shape = m.block_shape();
    std::vector<std::uint16_t> blk(m.block_shape().byte_size() / 2);
    for (const auto& [id, owner] : {std::pair<PhysicalBlockId, SequenceId>{shared, 1}, {mine, 2}}) {
        CHECK(m.read_bytes(id, 0, blk.data(), blk.size() * 2));
        for (std::uint32_t t = 0; t < 8; ++t)
            for (std::uint32_t st = 0; st < 2; ++st)
                for (std::uint32_t h = 0; h < kH; ++h) {
                    const std::size_t off = *layout.element_offset(0, st == 0 ? KVStream::Key : KVStream::Value, t, h);
                    // tokens 0..6 are the parent's in both blocks; token 7 is each block's own
                    const SequenceId src = t < 7 ? 1 : owner;
                    for (std::uint32_t d = 0; d < kD; ++d) CHECK(blk[off + d] == kv_value(src, t, st, h, d).bits);
                }
    }
    cudaFree(kd);
    cudaFree(vd);
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int qvp_hostlayerchecks_list(char* out, size_t cap) {
    return native::list_cases(out, cap);
}

extern "C" __attribute__((visibility("default"))) int qvp_hostlayerchecks_run(const char* name, char* msg, size_t cap) {
    return native::run_case(name, msg, cap);
}
