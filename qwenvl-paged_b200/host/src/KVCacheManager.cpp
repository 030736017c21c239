#include "qwenvl_paged/KVCacheManager.h"

#include <utility>

namespace qwenvl_paged {

bool CacheView::valid() const noexcept {
    return block_table != nullptr && allocator != nullptr && layout.element_count() > 0;
}

const std::byte* CacheView::block_bytes(LogicalBlockIndex index) const noexcept {
    if (!valid()) return nullptr;
    // a swapped entry has no frame: lookup misses and so does this
    const std::optional<PhysicalBlockId> id = block_table->lookup(index);
    if (!id) return nullptr;
    const PhysicalBlock* b = allocator->block(*id);
    return b != nullptr ? b->data() : nullptr;
}

KVCacheManager::KVCacheManager(MemoryAllocator& allocator) : allocator_(&allocator) {}

bool KVCacheManager::create_sequence(SequenceMetadata metadata) {
    const SequenceId id = metadata.sequence_id;
    if (sequences_.count(id) != 0) return false;
    sequences_.emplace(id, SequenceState{std::move(metadata), BlockTable(id)});
    return true;
}

bool KVCacheManager::fork_sequence(SequenceId parent_id, SequenceMetadata child_metadata) {
    const auto parent = sequences_.find(parent_id);
    if (parent == sequences_.end() || sequences_.count(child_metadata.sequence_id) != 0) return false;
    for (const BlockTableEntry& e : parent->second.text_table.entries())
        if (e.swap_slot.has_value()) return false;  // a swapped block has no frame to share
    const SequenceId child_id = child_metadata.sequence_id;
    BlockTable child = parent->second.text_table.fork(child_id);
    for (const BlockTableEntry& e : child.entries()) allocator_->retain(e.physical_id);
    sequences_.emplace(child_id, SequenceState{std::move(child_metadata), std::move(child)});
    return true;
}

bool KVCacheManager::reserve_tokens(SequenceId sequence_id, std::uint32_t token_count) {
    const auto it = sequences_.find(sequence_id);
    if (it == sequences_.end()) return false;
    const PhysicalBlock* b0 = allocator_->block(0);
    const std::uint32_t tpb = b0 != nullptr ? b0->shape().tokens_per_block : 0;
    if (tpb == 0) return false;
    const std::uint32_t need = (token_count + tpb - 1) / tpb;
    if (!allocator_->can_allocate(need)) return false;
    BlockTable& table = it->second.text_table;
    const auto first = static_cast<LogicalBlockIndex>(table.size());
    for (std::uint32_t k = 0; k < need; ++k) {
        const std::optional<PhysicalBlockId> frame = allocator_->allocate();
        if (!frame) return false;
        LogicalBlock lb;
        lb.sequence_id = sequence_id;
        lb.index = first + k;
        lb.cache_kind = table.cache_kind();
        lb.start_token = (first + k) * tpb;
        lb.token_count = tpb;
        table.map(lb, *frame, true);
    }
    return true;
}

std::optional<PhysicalBlockId> KVCacheManager::ensure_token_writable(SequenceId sequence_id,
                                                                     TokenPosition token_position,
                                                                     CacheKind /*cache_kind*/) {
    const auto it = sequences_.find(sequence_id);
    if (it == sequences_.end()) return std::nullopt;
    BlockTable& table = it->second.text_table;
    if (table.empty()) return std::nullopt;
    const std::uint32_t tpb = table.entries().front().logical.token_count;
    if (tpb == 0) return std::nullopt;
    const LogicalBlockIndex index = static_cast<LogicalBlockIndex>(token_position / tpb);
    const BlockTableEntry* seen = table.entry(index);
    if (seen == nullptr || seen->swap_slot.has_value()) return std::nullopt;
    const PhysicalBlockInfo* in = allocator_->info(seen->physical_id);
    if (in == nullptr) return std::nullopt;
    // the common decode case: a private, writable block leaves the table (and
    // its revision stamp) untouched
    if (in->ref_count <= 1 && seen->writable) return seen->physical_id;
    BlockTableEntry* e = table.mutable_entry(index);
    if (in->ref_count <= 1) {
        e->writable = true;
        return e->physical_id;
    }
    // shared: materialise a private copy (queued on the device, batched)
    const std::optional<PhysicalBlockId> copy = allocator_->allocate();
    if (!copy) return std::nullopt;
    allocator_->copy_block(e->physical_id, *copy);
    allocator_->release(e->physical_id);
    e->physical_id = *copy;
    e->writable = true;
    return copy;
}

std::uint32_t KVCacheManager::swap_out_sequence(SequenceId sequence_id) {
    const auto it = sequences_.find(sequence_id);
    if (it == sequences_.end()) return 0;
    BlockTable& table = it->second.text_table;
    std::vector<LogicalBlockIndex> resident;
    for (const BlockTableEntry& e : table.entries())
        if (!e.swap_slot.has_value()) resident.push_back(e.logical.index);
    std::uint32_t moved = 0;
    for (const LogicalBlockIndex idx : resident) {
        BlockTableEntry* e = table.mutable_entry(idx);
        if (e == nullptr) continue;
        const std::optional<SwapSlotId> slot = allocator_->swap_out(e->physical_id);
        if (!slot) continue;  // shared with a fork (or backend full): stays resident
        e->swap_slot = slot;
        moved += 1;
    }
    return moved;
}

bool KVCacheManager::swap_in_sequence(SequenceId sequence_id) {
    const auto it = sequences_.find(sequence_id);
    if (it == sequences_.end()) return false;
    BlockTable& table = it->second.text_table;
    std::vector<LogicalBlockIndex> swapped;
    for (const BlockTableEntry& e : table.entries())
        if (e.swap_slot.has_value()) swapped.push_back(e.logical.index);
    if (swapped.empty()) return true;
    if (!allocator_->can_allocate(static_cast<std::uint32_t>(swapped.size()))) return false;
    for (const LogicalBlockIndex idx : swapped) {
        BlockTableEntry* e = table.mutable_entry(idx);
        if (e == nullptr) continue;
        const std::optional<PhysicalBlockId> frame = allocator_->swap_in(*e->swap_slot);
        if (!frame) return false;
        e->physical_id = *frame;
        e->swap_slot.reset();
    }
    return true;
}

void KVCacheManager::release_sequence(SequenceId sequence_id) {
    const auto it = sequences_.find(sequence_id);
    if (it == sequences_.end()) return;
    for (const BlockTableEntry& e : it->second.text_table.entries()) {
        if (e.swap_slot.has_value())
            allocator_->discard_swapped(*e.swap_slot);
        else
            allocator_->release(e.physical_id);
    }
    sequences_.erase(it);
}

std::optional<CacheView> KVCacheManager::cache_view(SequenceId sequence_id, CacheKind cache_kind) const {
    const auto it = sequences_.find(sequence_id);
    if (it == sequences_.end()) return std::nullopt;
    CacheView v;
    v.sequence_id = sequence_id;
    v.cache_kind = cache_kind;
    v.block_table = &it->second.text_table;
    v.allocator = allocator_;
    if (const PhysicalBlock* b0 = allocator_->block(0)) v.layout.shape = b0->shape();
    return v;
}

bool KVCacheManager::contains(SequenceId sequence_id) const noexcept { return sequences_.count(sequence_id) != 0; }

const SequenceMetadata* KVCacheManager::metadata(SequenceId sequence_id) const noexcept {
    const auto it = sequences_.find(sequence_id);
    return it == sequences_.end() ? nullptr : &it->second.metadata;
}

}  // namespace qwenvl_paged
