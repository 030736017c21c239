// Stores for the bytes of evicted blocks.
//
// `SwapBackend` and `HostSwapBackend` keep the reference's interface and
// semantics (include/qwenvl_paged/SwapBackend.h:27-93, src/SwapBackend.cpp):
// slot ids start at 1 and only grow, at most `max_slots` slots are resident,
// `load` keeps the slot and `discard` drops it. `DeviceSwapBackend` is the
// B200 form: a fixed pinned-host slab, with the block <-> slab moves of many
// store/load calls batched into one gather or scatter kernel plus
// cudaMemcpyAsync on the allocator's stream.
#pragma once

#include "qwenvl_paged/Block.h"

#include <cstddef>
#include <cstdint>
#include <map>
#include <optional>
#include <set>
#include <string>
#include <unordered_map>
#include <vector>

namespace qwenvl_paged {

class MemoryAllocator;

class SwapBackend {
public:
    virtual ~SwapBackend() = default;
    [[nodiscard]] virtual std::optional<SwapSlotId> store(const PhysicalBlock& block) = 0;
    [[nodiscard]] virtual bool load(SwapSlotId slot, PhysicalBlock& block) = 0;
    virtual void discard(SwapSlotId slot) = 0;
    [[nodiscard]] virtual std::size_t resident_slots() const noexcept = 0;
    // Enqueues any store/load data movement the backend has deferred, on the
    // allocator's stream. The allocator calls it before it enqueues other
    // device work, so deferred moves keep program order. Backends that move
    // bytes eagerly need not override it.
    virtual void flush() {}
};

// Host-heap swap space with the reference's behaviour: each store copies the
// block's device bytes to a host vector (synchronously), each load copies
// them back.
class HostSwapBackend final : public SwapBackend {
public:
    explicit HostSwapBackend(std::size_t max_slots);
    ~HostSwapBackend() override = default;
    HostSwapBackend(const HostSwapBackend&) = delete;
    HostSwapBackend& operator=(const HostSwapBackend&) = delete;
    HostSwapBackend(HostSwapBackend&&) noexcept = default;
    HostSwapBackend& operator=(HostSwapBackend&&) noexcept = default;

    [[nodiscard]] std::optional<SwapSlotId> store(const PhysicalBlock& block) override;
    [[nodiscard]] bool load(SwapSlotId slot, PhysicalBlock& block) override;
    void discard(SwapSlotId slot) override;
    [[nodiscard]] std::size_t resident_slots() const noexcept override;
    [[nodiscard]] std::size_t capacity_slots() const noexcept;

private:
    std::size_t max_slots_{0};
    SwapSlotId next_slot_{1};
    std::unordered_map<SwapSlotId, std::vector<std::byte>> slots_;
};

// Pinned-host swap space for a device pool. `store` and `load` only record
// the move (slot bookkeeping is immediate, so the allocator's frame and slot
// decisions are exactly the reference's); `flush` turns all recorded stores
// into one gather kernel into device staging plus one cudaMemcpyAsync per
// contiguous run of slab slots, and all recorded loads into the reverse.
// The slab holds `max_slots` blocks of the allocator's block stride and is
// allocated once (cudaHostAlloc) at construction.
class DeviceSwapBackend final : public SwapBackend {
public:
    DeviceSwapBackend(MemoryAllocator& allocator, std::size_t max_slots);
    ~DeviceSwapBackend() override;
    DeviceSwapBackend(const DeviceSwapBackend&) = delete;
    DeviceSwapBackend& operator=(const DeviceSwapBackend&) = delete;

    [[nodiscard]] std::optional<SwapSlotId> store(const PhysicalBlock& block) override;
    [[nodiscard]] bool load(SwapSlotId slot, PhysicalBlock& block) override;
    void discard(SwapSlotId slot) override;
    [[nodiscard]] std::size_t resident_slots() const noexcept override;
    void flush() override;

    [[nodiscard]] std::size_t capacity_slots() const noexcept;
    // False when the pinned slab could not be allocated (every store fails).
    [[nodiscard]] bool ready() const noexcept;
    // Host address of a resident slot's bytes (for tests), null if unknown.
    // Valid once the stream has passed the flush that filled it.
    [[nodiscard]] const std::byte* slot_bytes(SwapSlotId slot) const noexcept;
    // Bytes moved between pool and slab so far, in each direction.
    [[nodiscard]] std::uint64_t bytes_out() const noexcept { return bytes_out_; }
    [[nodiscard]] std::uint64_t bytes_in() const noexcept { return bytes_in_; }
    // Text of the first failure of a flush (empty when every move was
    // enqueued). A failed store flush loses the bytes of the blocks it held.
    [[nodiscard]] const std::string& last_error() const noexcept { return error_; }

private:
    struct Move {
        std::int32_t block;
        std::uint32_t slab_index;
    };
    void flush_stores();
    void flush_loads();
    bool ensure_staging(std::size_t blocks);
    void note(const std::string& what);  // keeps the first error

    MemoryAllocator* allocator_{nullptr};
    std::size_t max_slots_{0};
    std::size_t slot_bytes_{0};
    std::byte* slab_{nullptr};            // pinned host, max_slots * slot_bytes
    std::byte* staging_{nullptr};         // device, staging_blocks_ * slot_bytes
    std::size_t staging_blocks_{0};
    std::int32_t* ids_host_{nullptr};     // pinned block-id list for one flush
    std::int32_t* ids_dev_{nullptr};
    std::size_t ids_capacity_{0};
    void* ids_event_{nullptr};            // cudaEvent_t: the last id-list upload
    SwapSlotId next_slot_{1};
    std::unordered_map<SwapSlotId, std::uint32_t> slots_;  // resident slot -> slab index
    std::set<std::uint32_t> free_indices_;
    std::vector<Move> pending_stores_;
    std::vector<Move> pending_loads_;
    std::vector<std::uint32_t> release_after_flush_;      // slab indices discarded while a load was pending
    std::uint64_t bytes_out_{0};
    std::uint64_t bytes_in_{0};
    std::string error_;
};

}  // namespace qwenvl_paged
