#include "qwenvl_paged/BlockTable.h"

#include <atomic>
#include <utility>

namespace qwenvl_paged {

namespace {
std::uint64_t next_revision() noexcept {
    static std::atomic<std::uint64_t> counter{0};
    return counter.fetch_add(1, std::memory_order_relaxed) + 1;
}
}  // namespace

BlockTable::BlockTable(SequenceId sequence_id, CacheKind cache_kind)
    : sequence_id_(sequence_id), cache_kind_(cache_kind), revision_(next_revision()) {}

// A moved-from table is left empty under a fresh stamp.
BlockTable::BlockTable(BlockTable&& other) noexcept
    : sequence_id_(other.sequence_id_),
      cache_kind_(other.cache_kind_),
      entries_(std::move(other.entries_)),
      revision_(other.revision_) {
    other.entries_.clear();
    other.revision_ = next_revision();
}

BlockTable& BlockTable::operator=(BlockTable&& other) noexcept {
    if (this != &other) {
        sequence_id_ = other.sequence_id_;
        cache_kind_ = other.cache_kind_;
        entries_ = std::move(other.entries_);
        revision_ = other.revision_;
        other.entries_.clear();
        other.revision_ = next_revision();
    }
    return *this;
}

std::uint64_t BlockTable::revision() const noexcept { return revision_; }

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
    revision_ = next_revision();
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
    revision_ = next_revision();
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
    revision_ = next_revision();
    return const_cast<BlockTableEntry*>(static_cast<const BlockTable*>(this)->entry(index));
}

void BlockTable::set_writable(LogicalBlockIndex index, bool writable) {
    if (BlockTableEntry* e = mutable_entry(index)) e->writable = writable;
}

const std::vector<BlockTableEntry>& BlockTable::entries() const noexcept { return entries_; }

BlockTable BlockTable::fork(SequenceId child_sequence_id) const {
    BlockTable child = *this;
    child.sequence_id_ = child_sequence_id;
    child.revision_ = next_revision();
    for (BlockTableEntry& e : child.entries_) {
        e.writable = false;
        e.logical.sequence_id = child_sequence_id;
    }
    return child;
}

}  // namespace qwenvl_paged
