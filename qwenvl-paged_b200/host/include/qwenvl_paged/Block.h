// Core ids, block shape and the device-resident physical block.
//
// Same types and signatures as phhuang191129/QwenVL-Paged
// include/qwenvl_paged/Block.h (ids :10-15, CacheKind/BlockState, BlockShape
// :46-57, HostMemoryOptions :67-70, LogicalBlock, PhysicalBlock :99-166), so
// code written against the reference compiles unchanged. What differs is
// where the bytes live: a PhysicalBlock is a view into its allocator's
// cudaMalloc pool (block id i at base + i*stride), so data() returns a device
// address. Use MemoryAllocator::write_bytes / read_bytes to move bytes
// between the host and a block.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <utility>

namespace qwenvl_paged {

using RequestId = std::uint64_t;
using SequenceId = std::uint64_t;
using TokenPosition = std::uint32_t;
using LogicalBlockIndex = std::uint32_t;
using PhysicalBlockId = std::uint32_t;
using SwapSlotId = std::uint64_t;

inline constexpr std::size_t kDefaultBlockAlignmentBytes = 256;

enum class CacheKind : std::uint8_t { TextKV, VisionKV, RopeState, Auxiliary };

enum class BlockState : std::uint8_t { Free, Active, Shared, Swapped };

struct BlockShape {
    std::uint32_t tokens_per_block{0};
    std::uint32_t num_layers{0};
    std::uint32_t num_kv_heads{0};
    std::uint32_t head_dim{0};
    std::uint32_t bytes_per_element{0};

    // K and V of every layer, token slot, head and dimension.
    [[nodiscard]] std::size_t byte_size() const noexcept;
};

// Kept for source compatibility. `alignment_bytes` is honoured (every block
// starts on that boundary inside the pool); `prefer_pinned_memory` is only
// reported back, since block storage is device memory.
struct HostMemoryOptions {
    std::size_t alignment_bytes{kDefaultBlockAlignmentBytes};
    bool prefer_pinned_memory{false};
};

// Host-visible block storage (not part of the reference interface). By
// default block bytes live in device memory, and PhysicalBlock::data() and
// CacheView::slot<T>() are device addresses. With host-visible storage, pools
// and standalone blocks are CUDA managed memory: the same addresses can also
// be read and written from the host, as in the reference, at the cost of page
// migration. Decode over such a pool never uses the TMA view of the pool
// (the pool's block stride is padded), and copy-on-write copies complete
// before MemoryAllocator::copy_block returns. This mode is meant for code
// that touches block bytes from the host, such as the reference's tests; it
// is not for serving. Off unless QVP_HOST_VISIBLE_POOLS=1 is set in the
// environment; set_host_visible_pools() changes it for allocations made
// afterwards.
[[nodiscard]] bool host_visible_pools() noexcept;
void set_host_visible_pools(bool on) noexcept;

struct LogicalBlock {
    SequenceId sequence_id{0};
    LogicalBlockIndex index{0};
    CacheKind cache_kind{CacheKind::TextKV};
    TokenPosition start_token{0};
    std::uint32_t token_count{0};

    [[nodiscard]] bool empty() const noexcept;
};

// Bytes of one physical block in device memory.
//
// A block built with the public constructor owns its own device allocation
// (one cudaMalloc, or cudaMallocManaged with host-visible storage, released
// by the destructor). Blocks handed out by a
// MemoryAllocator are views into the allocator's pool and own nothing.
class PhysicalBlock {
public:
    PhysicalBlock(PhysicalBlockId id, BlockShape shape, HostMemoryOptions memory_options = {});

    // A view of `size_bytes` bytes at device address `storage` (not owned).
    // Used by MemoryAllocator; `storage` may be null for a bookkeeping-only pool.
    PhysicalBlock(PhysicalBlockId id, BlockShape shape, HostMemoryOptions memory_options, std::byte* storage,
                  std::size_t size_bytes) noexcept;

    ~PhysicalBlock();

    PhysicalBlock(const PhysicalBlock&) = delete;
    PhysicalBlock& operator=(const PhysicalBlock&) = delete;
    PhysicalBlock(PhysicalBlock&& other) noexcept;
    PhysicalBlock& operator=(PhysicalBlock&& other) noexcept;

    [[nodiscard]] PhysicalBlockId id() const noexcept;
    [[nodiscard]] const BlockShape& shape() const noexcept;
    // Device address of the block's first byte (null without storage).
    [[nodiscard]] std::byte* data() noexcept;
    [[nodiscard]] const std::byte* data() const noexcept;
    [[nodiscard]] std::size_t size_bytes() const noexcept;
    [[nodiscard]] std::size_t alignment_bytes() const noexcept;
    [[nodiscard]] bool pinned_memory_requested() const noexcept;

    // Exchanges the two blocks' contents. Identity stays; shape and options
    // follow the bytes, as in the reference (Block.cpp:74-81). Two owning
    // blocks swap their allocations; a pool view keeps its address (the
    // device tables depend on base + id*stride) and the bytes are exchanged.
    void swap(PhysicalBlock& other) noexcept;

private:
    PhysicalBlockId id_{0};
    BlockShape shape_{};
    HostMemoryOptions memory_options_{};
    std::size_t size_bytes_{0};
    std::byte* storage_{nullptr};
    bool owns_storage_{false};
};

}  // namespace qwenvl_paged
