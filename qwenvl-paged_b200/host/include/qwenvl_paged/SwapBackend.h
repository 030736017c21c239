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
#include <utility>
#include <vector>

struct CUstream_st;
struct CUevent_st;

namespace qwenvl_paged {

class MemoryAllocator;

class SwapBackend {
public:
    virtual ~SwapBackend() = default;
    [[nodiscard]] virtual std::optional<SwapSlotId> store(const PhysicalBlock& block) = 0;
    [[nodiscard]] virtual bool load(SwapSlotId slot, PhysicalBlock& block) = 0;
    virtual void discard(SwapSlotId slot) = 0;
    [[nodiscard]] virtual std::size_t resident_slots() const noexcept = 0;
    // ---- device-pool additions (no counterpart in the reference) ----------
    // Enqueues any store/load data movement the backend has deferred, after
    // all device work already on the allocator's stream. The allocator calls
    // it before it enqueues other device work. Backends that move bytes
    // eagerly need not override these.
    virtual void flush() {}
    // Makes `engine` (the allocator's stream) wait for enqueued moves that
    // device work about to be enqueued there depends on: with `writes`, every
    // enqueued move (a write may land on a frame a store still reads, or on
    // a loaded frame); otherwise only loads into the `n` frames listed
    // (`frames` null: into any frame). Entries < 0 are ignored.
    virtual void order_engine(CUstream_st* /*engine*/, const std::int32_t* /*frames*/, std::size_t /*n*/,
                              bool /*writes*/) {}
    // True while a load enqueued by flush() may not have landed yet.
    [[nodiscard]] virtual bool loads_in_flight() const { return false; }
    // Waits (bounded) until every enqueued move has landed; false on a
    // timeout or a device error.
    virtual bool wait_idle() { return true; }
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
// decisions are exactly the reference's); `flush` enqueues them on a copy
// stream of the backend's own, after the engine work already enqueued:
// recorded stores as gather kernels into device staging plus one
// cudaMemcpyAsync per contiguous run of slab slots, recorded loads as the
// reverse. The engine stream goes on meanwhile: decode of sequences that are
// not being loaded overlaps the PCIe traffic. Work that writes the pool waits
// for every enqueued move first, and work that reads a frame being loaded
// waits for the loads (order_engine, called by the allocator and the decode
// batches). Everything the moves need (the slab, device staging, the block-id
// lists, the copy stream and its events) is allocated at construction, so a
// move once recorded is never dropped; if any of it cannot be had, ready() is
// false and every store is refused, leaving the bookkeeping untouched.
//
// With SwapCoding::compressed a flush codes the stored blocks on the copy
// stream (qvp_compress_blocks) into device staging and the copy engines move
// only each slot's head (the coded form of a K/V block, about 0.755 of its
// bytes) to the slab; the rare slot longer than its head (a block stored raw,
// or one with many escapes) has its tail written by the kernel itself into
// mapped pinned memory. Loads run the same way back (qvp_decompress_blocks).
// The bytes a load gives back are exactly those stored. The coding kernels
// take SM time that plain copies do not; they run one short CTA per block on
// a stream of the lowest priority, so a decode launched meanwhile gets SMs
// first.
enum class SwapCoding { raw, compressed };

class DeviceSwapBackend final : public SwapBackend {
public:
    DeviceSwapBackend(MemoryAllocator& allocator, std::size_t max_slots, SwapCoding coding = SwapCoding::raw);
    ~DeviceSwapBackend() override;
    DeviceSwapBackend(const DeviceSwapBackend&) = delete;
    DeviceSwapBackend& operator=(const DeviceSwapBackend&) = delete;

    [[nodiscard]] std::optional<SwapSlotId> store(const PhysicalBlock& block) override;
    [[nodiscard]] bool load(SwapSlotId slot, PhysicalBlock& block) override;
    void discard(SwapSlotId slot) override;
    [[nodiscard]] std::size_t resident_slots() const noexcept override;
    void flush() override;
    void order_engine(CUstream_st* engine, const std::int32_t* frames, std::size_t n, bool writes) override;
    [[nodiscard]] bool loads_in_flight() const override;
    bool wait_idle() override;

    [[nodiscard]] std::size_t capacity_slots() const noexcept;
    // False when a buffer of the backend could not be allocated (every store
    // is refused).
    [[nodiscard]] bool ready() const noexcept;
    // Host address of a resident slot's bytes (compressed: of its head), null
    // if unknown.
    // Valid once wait_idle() has returned after the flush that filled it.
    [[nodiscard]] const std::byte* slot_bytes(SwapSlotId slot) const noexcept;
    // Block bytes moved between pool and slab so far, in each direction.
    [[nodiscard]] std::uint64_t bytes_out() const noexcept { return bytes_out_; }
    [[nodiscard]] std::uint64_t bytes_in() const noexcept { return bytes_in_; }
    [[nodiscard]] SwapCoding coding() const noexcept { return coding_; }
    // Bytes that crossed the host link so far, {out, in}: the coded slot
    // bytes with SwapCoding::compressed, the block bytes otherwise. Waits
    // (bounded) for the moves enqueued so far.
    [[nodiscard]] std::pair<std::uint64_t, std::uint64_t> link_bytes();
    // The copy stream the moves run on.
    [[nodiscard]] CUstream_st* copy_stream() const noexcept { return copy_; }
    // Text of the first failure (a launch error or a timed-out wait); empty
    // when every move was enqueued.
    [[nodiscard]] const std::string& last_error() const noexcept { return error_; }

private:
    struct Move {
        std::int32_t block;
        std::uint32_t slab_index;
    };
    void flush_moves(std::vector<Move>& moves, bool stores, std::int32_t* ids_dev, std::int32_t* slab_idx_dev);
    void note(const std::string& what);  // keeps the first error
    void refresh_loads() const;

    MemoryAllocator* allocator_{nullptr};
    std::size_t max_slots_{0};
    std::size_t slot_bytes_{0};           // bytes of one block
    SwapCoding coding_{SwapCoding::raw};
    std::size_t slab_stride_{0};          // bytes of one slab slot (compressed: of its head)
    std::size_t tail_stride_{0};          // compressed: bytes of a slot past its head
    std::byte* slab_{nullptr};            // pinned host, max_slots * slab_stride (+ tails)
    std::byte* tails_dev_{nullptr};       // compressed: device address of the mapped tails
    unsigned long long* link_dev_{nullptr};  // compressed: device {out used, out tail, in used, in tail}
    std::uint64_t heads_out_{0};          // compressed: head bytes moved by the copy engines
    std::uint64_t heads_in_{0};
    std::byte* staging_{nullptr};         // device, staging_blocks_ * slab_stride
    std::size_t staging_blocks_{0};
    // two move lists (pinned + device) of 2 * max_slots block ids, followed
    // (compressed) by as many slab indices; flushes alternate between them
    std::int32_t* ids_host_[2]{nullptr, nullptr};
    std::int32_t* ids_dev_[2]{nullptr, nullptr};
    CUevent_st* ids_uploaded_[2]{nullptr, nullptr};  // the list's last upload
    int ids_next_{0};
    CUstream_st* copy_{nullptr};
    CUevent_st* engine_mark_{nullptr};    // the engine stream at the last flush
    CUevent_st* moves_done_{nullptr};     // copy stream after the last flush
    std::uint64_t flush_seq_{0};          // flushes with moves so far
    std::uint64_t engine_waited_{0};      // flushes the engine already waits for
    std::uint64_t last_load_flush_{0};    // newest flush that carried loads
    mutable std::uint64_t done_seq_{0};   // flushes known to have landed
    std::vector<std::uint64_t> frame_load_flush_;  // per frame: flush that loaded it
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
