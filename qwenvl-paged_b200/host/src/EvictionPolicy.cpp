#include "qwenvl_paged/EvictionPolicy.h"

#include <algorithm>
#include <utility>

namespace qwenvl_paged {

LruEvictionPolicy::LruEvictionPolicy(const KVCacheManager& cache) : cache_(&cache) {}

void LruEvictionPolicy::touch(const std::vector<CacheView>& batch) {
    ++step_;
    for (const CacheView& v : batch) last_used_[v.sequence_id] = step_;
}

void LruEvictionPolicy::forget(SequenceId sequence_id) { last_used_.erase(sequence_id); }

std::optional<PhysicalBlockId> LruEvictionPolicy::choose(const MemoryAllocator& allocator) const {
    // oldest first; ties broken by sequence id so the choice is deterministic
    std::vector<std::pair<std::uint64_t, SequenceId>> order;
    order.reserve(last_used_.size());
    for (const auto& [seq, step] : last_used_)
        if (step < step_) order.emplace_back(step, seq);
    std::sort(order.begin(), order.end());
    for (const auto& entry : order) {
        const std::optional<CacheView> view = cache_->cache_view(entry.second);
        if (!view || view->allocator != &allocator) continue;
        const std::vector<BlockTableEntry>& es = view->block_table->entries();
        for (auto it = es.rbegin(); it != es.rend(); ++it) {
            if (it->swap_slot.has_value()) continue;
            const PhysicalBlockInfo* in = allocator.info(it->physical_id);
            if (in != nullptr && in->ref_count == 1) return it->physical_id;
        }
    }
    return std::nullopt;
}

EvictionCandidateSelector LruEvictionPolicy::selector() const {
    return [this](const MemoryAllocator& allocator) { return choose(allocator); };
}

}  // namespace qwenvl_paged
