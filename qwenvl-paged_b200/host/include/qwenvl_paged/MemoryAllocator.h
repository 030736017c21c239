// Physical block allocator over one device pool.
//
// Interface and bookkeeping are the reference's (include/qwenvl_paged/
// MemoryAllocator.h:18-198, src/MemoryAllocator.cpp): a LIFO free list
// initialised 0..N-1 (so the first allocate returns N-1), non-atomic
// reference counts, a generation that advances on recycle, swap through a
// SwapBackend, an advisory eviction selector, stats by scan. Block storage
// is one cudaMalloc slab on the allocator's device; copy_block is deferred
// and batched: copies queued during a step run as one kernel launch, in
// order, before any later device work of this allocator.
#pragma once

#include "qwenvl_paged/Block.h"
#include "qwenvl_paged/SwapBackend.h"

#include <cstddef>
#include <cstdint>
#include <functional>
#include <memory>
#include <optional>
#include <string>
#include <unordered_set>
#include <vector>

struct CUstream_st;

namespace qwenvl_paged {

struct AllocatorConfig {
    BlockShape block_shape{};
    HostMemoryOptions memory_options{};
    std::uint32_t max_blocks{0};
};

// Device placement of the pool; not part of the reference (new struct, the
// reference's AllocatorConfig is unchanged).
struct DevicePoolOptions {
    int device{-1};                  // CUDA ordinal; -1 = the current device
    bool allocate_storage{true};     // false: bookkeeping only, no device bytes
    CUstream_st* stream{nullptr};    // engine stream for copies and swaps (null = legacy default)
    bool host_visible{host_visible_pools()};  // managed memory; see host_visible_pools()
};

struct AllocatorStats {
    std::uint32_t total_blocks{0};
    std::uint32_t free_blocks{0};
    std::uint32_t active_blocks{0};
    std::uint32_t shared_blocks{0};
    std::uint32_t swapped_blocks{0};
    std::size_t bytes_reserved{0};
};

struct PhysicalBlockInfo {
    PhysicalBlockId id{0};
    BlockState state{BlockState::Free};
    std::uint32_t ref_count{0};
    std::uint64_t generation{0};
};

class MemoryAllocator;

using EvictionCandidateSelector = std::function<std::optional<PhysicalBlockId>(const MemoryAllocator&)>;

class MemoryAllocator {
public:
    // A pool of config.max_blocks blocks on the current device.
    explicit MemoryAllocator(AllocatorConfig config);
    MemoryAllocator(AllocatorConfig config, DevicePoolOptions options);
    ~MemoryAllocator();

    MemoryAllocator(const MemoryAllocator&) = delete;
    MemoryAllocator& operator=(const MemoryAllocator&) = delete;
    MemoryAllocator(MemoryAllocator&&) noexcept;
    MemoryAllocator& operator=(MemoryAllocator&&) noexcept;

    [[nodiscard]] std::optional<PhysicalBlockId> allocate();
    void release(PhysicalBlockId id);
    void retain(PhysicalBlockId id);
    // Queues a device copy of min(size) bytes; it runs, in order, at the next
    // flush (before any later device work of this allocator).
    void copy_block(PhysicalBlockId source, PhysicalBlockId destination);
    [[nodiscard]] PhysicalBlock* block(PhysicalBlockId id) noexcept;
    [[nodiscard]] const PhysicalBlock* block(PhysicalBlockId id) const noexcept;
    [[nodiscard]] const PhysicalBlockInfo* info(PhysicalBlockId id) const noexcept;
    void set_swap_backend(SwapBackend* backend) noexcept;
    [[nodiscard]] std::optional<SwapSlotId> swap_out(PhysicalBlockId id);
    [[nodiscard]] std::optional<PhysicalBlockId> swap_in(SwapSlotId slot);
    void discard_swapped(SwapSlotId slot);
    void set_eviction_selector(EvictionCandidateSelector selector);
    [[nodiscard]] std::optional<PhysicalBlockId> select_eviction_candidate() const;
    [[nodiscard]] AllocatorStats stats() const noexcept;
    [[nodiscard]] bool can_allocate(std::uint32_t block_count) const noexcept;

    // ---- device-pool additions (no counterpart in the reference) ----------
    // Enqueues all deferred copies and swap moves on the engine stream.
    void flush();
    // flush() and wait (bounded) for the engine stream and the swap moves.
    bool synchronize();
    // Make the engine stream wait for enqueued swap moves that device work
    // about to be enqueued on it depends on: order_reads for work that reads
    // the `n` listed frames (null: any frame; entries < 0 ignored) and waits
    // only for loads into them; order_writes for work that writes the pool,
    // which waits for every enqueued move. Both are no-ops without a swap
    // backend that defers moves.
    void order_reads(const std::int32_t* frames, std::size_t n);
    void order_writes();
    // True while a swap-in enqueued by flush() may not have landed yet.
    [[nodiscard]] bool loads_in_flight() const;
    // Synchronous host <-> block byte moves for set-up and tests.
    bool write_bytes(PhysicalBlockId id, std::size_t offset, const void* host, std::size_t bytes);
    bool read_bytes(PhysicalBlockId id, std::size_t offset, void* host, std::size_t bytes);
    [[nodiscard]] bool has_storage() const noexcept { return pool_ != nullptr; }
    [[nodiscard]] bool host_visible() const noexcept { return host_visible_; }
    [[nodiscard]] std::byte* pool_base() const noexcept { return pool_; }
    [[nodiscard]] std::size_t block_stride() const noexcept { return stride_; }
    [[nodiscard]] std::uint32_t num_blocks() const noexcept { return config_.max_blocks; }
    [[nodiscard]] int device() const noexcept { return device_; }
    [[nodiscard]] CUstream_st* stream() const noexcept { return stream_; }
    [[nodiscard]] const BlockShape& block_shape() const noexcept { return config_.block_shape; }
    [[nodiscard]] SwapBackend* swap_backend() const noexcept { return swap_backend_; }
    // Text of the last device error (cudaMalloc failure, launch error...).
    [[nodiscard]] const std::string& last_error() const noexcept { return error_; }
    // Number of copy launches issued and copies they carried (for tests).
    [[nodiscard]] std::uint64_t copy_launches() const noexcept { return copy_launches_; }
    [[nodiscard]] std::uint64_t copies_done() const noexcept { return copies_done_; }

private:
    void flush_copies();
    void release_storage() noexcept;

    AllocatorConfig config_{};
    int device_{-1};
    CUstream_st* stream_{nullptr};
    bool host_visible_{false};
    std::byte* pool_{nullptr};
    std::size_t stride_{0};
    std::vector<std::unique_ptr<PhysicalBlock>> blocks_;
    std::vector<PhysicalBlockInfo> infos_;
    std::vector<PhysicalBlockId> free_list_;
    SwapBackend* swap_backend_{nullptr};
    EvictionCandidateSelector eviction_selector_{};
    // deferred copy-on-write copies: (src, dst) pairs in program order
    std::vector<std::int32_t> pending_pairs_;
    std::unordered_set<PhysicalBlockId> pending_src_, pending_dst_;
    std::int32_t* pairs_host_{nullptr};   // pinned
    std::int32_t* pairs_dev_{nullptr};
    std::size_t pairs_capacity_{0};
    void* pairs_event_{nullptr};          // cudaEvent_t: the last pairs upload
    std::string error_;
    std::uint64_t copy_launches_{0};
    std::uint64_t copies_done_{0};
};

}  // namespace qwenvl_paged
