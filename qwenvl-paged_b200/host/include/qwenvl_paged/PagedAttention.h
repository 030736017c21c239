// Paged-decode attention behind the reference's signature.
//
// paged_attention_decode<T>(view, query, params, out) keeps the contract of
// the reference CPU kernel (include/qwenvl_paged/PagedAttention.h:23-127):
// it returns false and leaves `out` untouched when the arguments do not fit
// the cache shape or any block of [0, context_len) is unmapped or swapped
// out. The work runs on the GPU (qvp_decode) on the allocator's stream; T is
// float or a 2-byte bfloat16 type such as qwenvl_paged::bfloat16, and
// `query` / `out` may be host or device pointers (host pointers make the call
// synchronous). PagedDecodeBatch is the batched form an engine step uses.
#pragma once

#include "qwenvl_paged/CacheLayout.h"
#include "qwenvl_paged/KVCacheManager.h"
#include "qwenvl_paged/ResidentTables.h"

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

struct qvp_decode_args;  // include/qvp.h

namespace qwenvl_paged {

struct PagedAttentionParams {
    std::uint32_t layer{0};
    std::uint32_t num_query_heads{0};
    std::uint32_t context_len{0};
    float scale{1.0F};
};

// Host bfloat16: exact widening, round-to-nearest-even narrowing.
struct bfloat16 {
    std::uint16_t bits{0};
    bfloat16() = default;
    explicit bfloat16(float f) noexcept {
        std::uint32_t u;
        std::memcpy(&u, &f, 4);
        if ((u & 0x7fffffffu) > 0x7f800000u)
            bits = static_cast<std::uint16_t>((u >> 16) | 0x40u);
        else
            bits = static_cast<std::uint16_t>((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
    }
    explicit operator float() const noexcept {
        const std::uint32_t u = static_cast<std::uint32_t>(bits) << 16;
        float f;
        std::memcpy(&f, &u, 4);
        return f;
    }
};
static_assert(sizeof(bfloat16) == 2, "bfloat16 is two bytes");

namespace detail {
// Type-erased body of paged_attention_decode<T>; elem_bytes = sizeof(T).
bool decode_one(const CacheView& view, const void* query, std::size_t elem_bytes,
                const PagedAttentionParams& params, void* out);
}  // namespace detail

template <typename T>
[[nodiscard]] bool paged_attention_decode(const CacheView& view, const T* query, const PagedAttentionParams& params,
                                          T* out) {
    return detail::decode_one(view, query, sizeof(T), params, out);
}

// Batched decode of one layer for an engine step. Each call validates every
// view on the host (any failure: false, nothing enqueued, `out` untouched),
// flattens the block tables into a pinned int32 [batch][max_blocks] buffer,
// uploads it and the context lengths with one cudaMemcpyAsync each, and
// launches qvp_decode on the allocator's stream. `query` and `out` are device
// arrays [batch][num_query_heads][head_dim] in the pool's element type.
// Buffers are kept and reused across calls.
//
// With resident_tables the tables stay on the device between calls
// (ResidentBlockTables): a call uploads the context lengths and only the rows
// whose BlockTable changed, which an engine gets by keeping each sequence at
// the same batch position from step to step. The checks and the results are
// the same as without it.
class PagedDecodeBatch {
public:
    explicit PagedDecodeBatch(const MemoryAllocator& allocator, bool resident_tables = false);
    ~PagedDecodeBatch();
    PagedDecodeBatch(const PagedDecodeBatch&) = delete;
    PagedDecodeBatch& operator=(const PagedDecodeBatch&) = delete;

    bool run(const std::vector<CacheView>& views, const std::vector<std::uint32_t>& context_lens,
             std::uint32_t layer, std::uint32_t num_query_heads, float scale, const void* query, void* out);

    // qvp_status of the last run (0 = OK) and its text.
    [[nodiscard]] int last_status() const noexcept { return status_; }
    [[nodiscard]] const std::string& last_error() const noexcept { return error_; }
    // Device error bits (qvp_decode error_word) of the last run; waits for it.
    [[nodiscard]] int device_error();
    // Table rows and bytes the last run sent to the device (all rows unless
    // the tables are resident).
    [[nodiscard]] std::uint32_t rows_uploaded() const noexcept { return rows_uploaded_; }
    [[nodiscard]] std::size_t bytes_uploaded() const noexcept { return bytes_uploaded_; }

private:
    bool grow(std::size_t table_ints, std::size_t batch, std::size_t workspace);
    bool run_resident(const std::vector<CacheView>& views, const std::vector<std::uint32_t>& context_lens,
                      ::qvp_decode_args& a, std::uint32_t max_ctx, const void* query, void* out);

    const MemoryAllocator* allocator_;
    std::int32_t* host_buf_{nullptr};    // pinned: tables then context lengths
    std::int32_t* dev_buf_{nullptr};
    std::size_t buf_ints_{0};
    void* workspace_{nullptr};
    std::size_t workspace_bytes_{0};
    std::int32_t* error_word_{nullptr};
    void* upload_event_{nullptr};
    std::unique_ptr<ResidentBlockTables> resident_;
    std::uint32_t rows_uploaded_{0};
    std::size_t bytes_uploaded_{0};
    int status_{0};
    std::string error_;
};

// Causal prefill of one layer for a batch (no reference counterpart: the
// reference computes prefill as its decode at every prompt position,
// include/qwenvl_paged/PagedAttention.h:43-44; this runs qvp_prefill, which
// gives the same values). For sequence b, the last query_lens[b] of its
// context_lens[b] cached tokens are queries: each attends to every key up to
// its own position. Their K and V must already be in the cache
// (KVAppendBatch, or host writes into a host-visible pool). `query` and
// `out` are device arrays [batch][max(query_lens)][num_query_heads]
// [head_dim] in the pool's element type. The checks and the refusal rules
// are PagedDecodeBatch's, plus query_lens[b] in [1, context_lens[b]].
class PagedPrefillBatch {
public:
    explicit PagedPrefillBatch(const MemoryAllocator& allocator);
    ~PagedPrefillBatch();
    PagedPrefillBatch(const PagedPrefillBatch&) = delete;
    PagedPrefillBatch& operator=(const PagedPrefillBatch&) = delete;

    bool run(const std::vector<CacheView>& views, const std::vector<std::uint32_t>& context_lens,
             const std::vector<std::uint32_t>& query_lens, std::uint32_t layer, std::uint32_t num_query_heads,
             float scale, const void* query, void* out);

    [[nodiscard]] int last_status() const noexcept { return status_; }
    [[nodiscard]] const std::string& last_error() const noexcept { return error_; }
    // Device error bits of the last run (qvp_prefill error word); waits for it.
    [[nodiscard]] int device_error();

private:
    const MemoryAllocator* allocator_;
    std::int32_t* host_buf_{nullptr};  // pinned: tables, context lengths, query lengths
    std::int32_t* dev_buf_{nullptr};
    std::size_t buf_ints_{0};
    std::int32_t* error_word_{nullptr};
    void* upload_event_{nullptr};
    int status_{0};
    std::string error_;
};

// Writes one new token's K and V per sequence (no reference counterpart: the
// reference's tests store them through CacheView::slot<T>() after
// KVCacheManager::ensure_token_writable, tests/PagedAttention.test.cpp:
// 97-127). Token positions[b] of views[b] goes to slot positions[b] %
// tokens_per_block of its block, for layer `layer`. The block must be mapped,
// writable and held by this sequence alone (call ensure_token_writable
// first), otherwise nothing is written and run() returns false. `k` and `v`
// are device arrays [batch][num_kv_heads][head_dim] in the pool's element
// type. Enqueued on the allocator's stream after any queued copy-on-write
// copies, one launch per call; the host work and the upload are one block id
// and one slot per sequence.
class KVAppendBatch {
public:
    explicit KVAppendBatch(const MemoryAllocator& allocator);
    ~KVAppendBatch();
    KVAppendBatch(const KVAppendBatch&) = delete;
    KVAppendBatch& operator=(const KVAppendBatch&) = delete;

    bool run(const std::vector<CacheView>& views, const std::vector<std::uint32_t>& positions, std::uint32_t layer,
             const void* k, const void* v);

    [[nodiscard]] int last_status() const noexcept { return status_; }
    [[nodiscard]] const std::string& last_error() const noexcept { return error_; }
    [[nodiscard]] int device_error();

private:
    const MemoryAllocator* allocator_;
    std::int32_t* host_buf_{nullptr};  // pinned: tables, positions
    std::int32_t* dev_buf_{nullptr};
    std::size_t buf_ints_{0};
    std::int32_t* error_word_{nullptr};
    void* upload_event_{nullptr};
    int status_{0};
    std::string error_;
};

}  // namespace qwenvl_paged
