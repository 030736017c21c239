// Sequence cache lifecycle and the read-only CacheView.
//
// Same types, signatures and semantics as the reference
// (include/qwenvl_paged/KVCacheManager.h:23-253, src/KVCacheManager.cpp):
// reserve maps whole blocks after an up-front capacity check, fork shares
// every frame and clears `writable`, ensure_token_writable materialises a
// private copy of a shared block (copy-on-write), sequence swap-in is
// all-or-nothing, release discards swapped slots. Copy-on-write copies go
// through MemoryAllocator::copy_block, so all CoW copies of a step run as one
// batched device launch.
#pragma once

#include "qwenvl_paged/Block.h"
#include "qwenvl_paged/BlockTable.h"
#include "qwenvl_paged/CacheLayout.h"
#include "qwenvl_paged/MemoryAllocator.h"

#include <cstddef>
#include <cstdint>
#include <optional>
#include <unordered_map>
#include <vector>

namespace qwenvl_paged {

struct MultimodalSpan {
    TokenPosition start_token{0};
    std::uint32_t token_count{0};
    std::uint32_t feature_index{0};
};

enum class PositionEncodingKind : std::uint8_t { Text1D, Image2D, Video3D };

struct Position3D {
    std::int64_t temporal{0};
    std::int64_t height{0};
    std::int64_t width{0};
};

struct PositionalEncodingSpan {
    TokenPosition start_token{0};
    std::uint32_t token_count{0};
    PositionEncodingKind kind{PositionEncodingKind::Text1D};
    Position3D origin{};
    Position3D stride{};
};

struct PositionalEncodingMetadata {
    std::vector<PositionalEncodingSpan> spans;
};

// Carried with each sequence; the decode kernels never read it.
struct SequenceMetadata {
    SequenceId sequence_id{0};
    RequestId request_id{0};
    std::vector<MultimodalSpan> multimodal_spans;
    PositionalEncodingMetadata positional_encoding;
};

// Borrowed view of one sequence's cache: page table, allocator, layout.
// block_bytes() and slot() return DEVICE addresses here; they are null for
// unmapped or swapped blocks exactly where the reference returns null.
struct CacheView {
    SequenceId sequence_id{0};
    CacheKind cache_kind{CacheKind::TextKV};
    const BlockTable* block_table{nullptr};
    const MemoryAllocator* allocator{nullptr};
    KVBlockLayout layout{};

    [[nodiscard]] bool valid() const noexcept;
    [[nodiscard]] const std::byte* block_bytes(LogicalBlockIndex index) const noexcept;

    template <typename T>
    [[nodiscard]] const T* slot(KVStream stream, std::uint32_t layer, TokenPosition token,
                                std::uint32_t kv_head) const noexcept {
        if (!valid() || sizeof(T) != layout.shape.bytes_per_element) return nullptr;
        const std::uint32_t tpb = layout.shape.tokens_per_block;
        const auto off = layout.element_offset(layer, stream, token % tpb, kv_head);
        if (!off) return nullptr;
        const std::byte* base = block_bytes(static_cast<LogicalBlockIndex>(token / tpb));
        return base == nullptr ? nullptr : reinterpret_cast<const T*>(base) + *off;
    }
};

class KVCacheManager {
public:
    explicit KVCacheManager(MemoryAllocator& allocator);
    ~KVCacheManager() = default;
    KVCacheManager(const KVCacheManager&) = delete;
    KVCacheManager& operator=(const KVCacheManager&) = delete;
    KVCacheManager(KVCacheManager&&) noexcept = default;
    KVCacheManager& operator=(KVCacheManager&&) noexcept = default;

    bool create_sequence(SequenceMetadata metadata);
    bool fork_sequence(SequenceId parent_id, SequenceMetadata child_metadata);
    bool reserve_tokens(SequenceId sequence_id, std::uint32_t token_count);
    [[nodiscard]] std::optional<PhysicalBlockId> ensure_token_writable(SequenceId sequence_id,
                                                                       TokenPosition token_position,
                                                                       CacheKind cache_kind = CacheKind::TextKV);
    std::uint32_t swap_out_sequence(SequenceId sequence_id);
    bool swap_in_sequence(SequenceId sequence_id);
    void release_sequence(SequenceId sequence_id);
    [[nodiscard]] std::optional<CacheView> cache_view(SequenceId sequence_id,
                                                      CacheKind cache_kind = CacheKind::TextKV) const;
    [[nodiscard]] bool contains(SequenceId sequence_id) const noexcept;

    // Metadata a sequence was created with (null for an unknown sequence).
    [[nodiscard]] const SequenceMetadata* metadata(SequenceId sequence_id) const noexcept;

private:
    struct SequenceState {
        SequenceMetadata metadata{};
        BlockTable text_table;
    };

    MemoryAllocator* allocator_{nullptr};
    std::unordered_map<SequenceId, SequenceState> sequences_;
};

}  // namespace qwenvl_paged
