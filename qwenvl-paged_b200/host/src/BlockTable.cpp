#include "qwenvl_paged/BlockTable.h"

#include <atomic>
#include <utility>

namespace qwenvl_paged {

namespace {
std::uint64_t next_instance() noexcept {
    static std::atomic<std::uint64_t> counter{0};
    return counter.fetch_add(1, std::memory_order_relaxed) + 1;
}
}  // namespace

BlockTable::BlockTable(SequenceId sequence_id, CacheKind cache_kind)
    : sequence_id_(sequence_id), cache_kind_(cache_kind) {}

// A copy holds the same entries under an id of its own, so that the two
// tables can change independently without ever sharing a stamp.
BlockTable::BlockTable(const BlockTable& other)
    : sequence_id_(other.sequence_id_), cache_kind_(other.cache_kind_), entries_(other.entries_) {
    if (!entries_.empty()) stamp_ = TableStamp{next_instance(), 1};
}

BlockTable& BlockTable::operator=(const BlockTable& other) {
    if (this != &other) {
        sequence_id_ = other.sequence_id_;
        cache_kind_ = other.cache_kind_;
        entries_ = other.entries_;
        stamp_ = entries_.empty() ? TableStamp{} : TableStamp{next_instance(), 1};
    }
    return *this;
}

// A moved-from table is left empty, under the stamp of an empty table.
BlockTable::BlockTable(BlockTable&& other) noexcept
    : sequence_id_(other.sequence_id_),
      cache_kind_(other.cache_kind_),
      entries_(std::move(other.entries_)),
      stamp_(other.stamp_) {
    other.entries_.clear();
    other.stamp_ = TableStamp{};
}

BlockTable& BlockTable::operator=(BlockTable&& other) noexcept {
    if (this != &other) {
        sequence_id_ = other.sequence_id_;
        cache_kind_ = other.cache_kind_;
        entries_ = std::move(other.entries_);
        stamp_ = other.stamp_;
        other.entries_.clear();
        other.stamp_ = TableStamp{};
    }
    return *this;
}

void BlockTable::touch() noexcept {
    if (stamp_.instance == 0) stamp_.instance = next_instance();
    ++stamp_.count;
}

TableStamp BlockTable::revision() const noexcept { return stamp_; }

std::size_t BlockTable::position(LogicalBlockIndex index) const noexcept {
    std::size_t lo = 0, hi = entries_.size();
    while (lo < hi) {
        const std::size_t mid = lo + (hi - lo) / 2;
        if (entries_[mid].logical.index < index)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

SequenceId BlockTable::sequence_id() const noexcept { return sequence_id_; }
CacheKind BlockTable::cache_kind() const noexcept { return cache_kind_; }
std::size_t BlockTable::size() const noexcept { return entries_.size(); }
bool BlockTable::empty() const noexcept { return entries_.empty(); }

void BlockTable::map(LogicalBlock logical, PhysicalBlockId physical_id, bool writable) {
    touch();
    const std::size_t at = position(logical.index);
    if (at < entries_.size() && entries_[at].logical.index == logical.index) {
        BlockTableEntry& e = entries_[at];
        e.logical = logical;
        e.physical_id = physical_id;
        e.writable = writable;
        e.swap_slot.reset();
        return;
    }
    BlockTableEntry e;
    e.logical = logical;
    e.physical_id = physical_id;
    e.writable = writable;
    entries_.insert(entries_.begin() + static_cast<std::ptrdiff_t>(at), e);
}

std::optional<PhysicalBlockId> BlockTable::unmap(LogicalBlockIndex index) {
    const std::size_t at = position(index);
    if (at == entries_.size() || entries_[at].logical.index != index) return std::nullopt;
    touch();
    const PhysicalBlockId id = entries_[at].physical_id;
    entries_.erase(entries_.begin() + static_cast<std::ptrdiff_t>(at));
    return id;
}

std::optional<PhysicalBlockId> BlockTable::lookup(LogicalBlockIndex index) const {
    const BlockTableEntry* e = entry(index);
    if (e == nullptr || e->swap_slot.has_value()) return std::nullopt;
    return e->physical_id;
}

const BlockTableEntry* BlockTable::entry(LogicalBlockIndex index) const noexcept {
    const std::size_t at = position(index);
    return (at < entries_.size() && entries_[at].logical.index == index) ? &entries_[at] : nullptr;
}

// The caller may change the entry through the pointer, so the stamp moves.
BlockTableEntry* BlockTable::mutable_entry(LogicalBlockIndex index) noexcept {
    touch();
    return const_cast<BlockTableEntry*>(static_cast<const BlockTable*>(this)->entry(index));
}

void BlockTable::set_writable(LogicalBlockIndex index, bool writable) {
    if (BlockTableEntry* e = mutable_entry(index)) e->writable = writable;
}

const std::vector<BlockTableEntry>& BlockTable::entries() const noexcept { return entries_; }

BlockTable BlockTable::fork(SequenceId child_sequence_id) const {
    BlockTable child = *this;
    child.sequence_id_ = child_sequence_id;
    child.touch();
    for (BlockTableEntry& e : child.entries_) {
        e.writable = false;
        e.logical.sequence_id = child_sequence_id;
    }
    return child;
}

}  // namespace qwenvl_paged
