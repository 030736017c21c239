// TEST INFRASTRUCTURE: GPU checks of PagedDecodeBatch with device-resident
// block tables against the per-step flatten, on one device pool: over decode
// steps that cross block boundaries, copy on write, reorder the batch and
// refuse a swapped-out sequence, both must write bit-identical outputs.
// Driven by tests/resident_tables_gpu_checks.py.
#include "qwenvl_paged/KVCacheManager.h"
#include "qwenvl_paged/MemoryAllocator.h"
#include "qwenvl_paged/PagedAttention.h"
#include "qwenvl_paged/SwapBackend.h"

#include <cuda_runtime.h>

#include "harness.h"

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

}  // namespace

extern "C" __attribute__((visibility("default"))) int qvp_residentchecks_list(char* out, size_t cap) {
    return native::list_cases(out, cap);
}

extern "C" __attribute__((visibility("default"))) int qvp_residentchecks_run(const char* name, char* msg, size_t cap) {
    return native::run_case(name, msg, cap);
}
