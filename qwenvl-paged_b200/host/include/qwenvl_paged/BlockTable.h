// Per-sequence logical -> physical page table. Same interface and behaviour
// as the reference (include/qwenvl_paged/BlockTable.h:14-122): entries kept
// sorted by logical index, lookup misses on a swapped entry, fork clears
// `writable`. `entries()` order is what a batch step flattens into the device
// int32 tables.
//
// Beyond the reference interface, revision() stamps the table's contents as
// {instance, count}: {0, 0} for a table with no entries (new or moved from);
// otherwise `instance` is a process-unique id the table takes at its first
// change (or when it is copied) and `count` advances at every call that can
// change a mapping (map, unmap, set_writable, mutable_entry, fork). Two table
// states with the same stamp hold the same entries, so a device-resident copy
// of the table can be refreshed only when the stamp moves. A change costs one
// increment; only a table's first change takes the shared id counter.
#pragma once

#include "qwenvl_paged/Block.h"

#include <cstddef>
#include <cstdint>
#include <optional>
#include <vector>

namespace qwenvl_paged {

struct TableStamp {
    std::uint64_t instance{0};
    std::uint64_t count{0};
    friend bool operator==(const TableStamp& a, const TableStamp& b) noexcept {
        return a.instance == b.instance && a.count == b.count;
    }
    friend bool operator!=(const TableStamp& a, const TableStamp& b) noexcept { return !(a == b); }
};

struct BlockTableEntry {
    LogicalBlock logical{};
    PhysicalBlockId physical_id{0};
    bool writable{true};
    // Engaged while the block's bytes live in the swap backend; physical_id
    // is then stale.
    std::optional<SwapSlotId> swap_slot{};
};

class BlockTable {
public:
    explicit BlockTable(SequenceId sequence_id, CacheKind cache_kind = CacheKind::TextKV);
    BlockTable(const BlockTable& other);
    BlockTable& operator=(const BlockTable& other);
    BlockTable(BlockTable&& other) noexcept;
    BlockTable& operator=(BlockTable&& other) noexcept;

    [[nodiscard]] SequenceId sequence_id() const noexcept;
    [[nodiscard]] CacheKind cache_kind() const noexcept;
    [[nodiscard]] std::size_t size() const noexcept;
    [[nodiscard]] bool empty() const noexcept;

    void map(LogicalBlock logical, PhysicalBlockId physical_id, bool writable);
    [[nodiscard]] std::optional<PhysicalBlockId> unmap(LogicalBlockIndex index);
    [[nodiscard]] std::optional<PhysicalBlockId> lookup(LogicalBlockIndex index) const;
    [[nodiscard]] const BlockTableEntry* entry(LogicalBlockIndex index) const noexcept;
    [[nodiscard]] BlockTableEntry* mutable_entry(LogicalBlockIndex index) noexcept;
    void set_writable(LogicalBlockIndex index, bool writable);
    [[nodiscard]] const std::vector<BlockTableEntry>& entries() const noexcept;
    [[nodiscard]] BlockTable fork(SequenceId child_sequence_id) const;
    [[nodiscard]] TableStamp revision() const noexcept;

private:
    // Position of the first entry whose logical index is >= `index`.
    [[nodiscard]] std::size_t position(LogicalBlockIndex index) const noexcept;

    SequenceId sequence_id_{0};
    CacheKind cache_kind_{CacheKind::TextKV};
    void touch() noexcept;

    std::vector<BlockTableEntry> entries_;
    TableStamp stamp_{};
};

}  // namespace qwenvl_paged
