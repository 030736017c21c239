// A policy for MemoryAllocator::set_eviction_selector (not part of the
// reference, which defines the hook and leaves the policy to the engine:
// include/qwenvl_paged/MemoryAllocator.h:59-68). It names a block of the
// sequence that has gone longest without being decoded:
//   * sequences in the step's decode batch are never chosen: their blocks may
//     still be read by decode work in flight on the device, and a block whose
//     frame is swapped out and reused under a running kernel would be
//     overwritten while it is read;
//   * a block held by more than one sequence is skipped (swap_out refuses a
//     shared block);
//   * among a sequence's blocks the last mapped one is named first.
// The hook stays advisory, as in the reference: the caller decides whether to
// swap out the owning sequence (KVCacheManager::swap_out_sequence, or
// Scheduler::preempt for its request).
#pragma once

#include "qwenvl_paged/KVCacheManager.h"
#include "qwenvl_paged/MemoryAllocator.h"

#include <cstdint>
#include <optional>
#include <unordered_map>
#include <vector>

namespace qwenvl_paged {

class LruEvictionPolicy {
public:
    explicit LruEvictionPolicy(const KVCacheManager& cache);

    // Call once per engine step with the step's decode batch (before its
    // decode is enqueued): the step counter advances, the batch's sequences
    // are stamped with it and are protected until the next call.
    void touch(const std::vector<CacheView>& batch);
    // Drops a sequence the engine released (optional: sequences the cache
    // manager no longer holds are skipped anyway).
    void forget(SequenceId sequence_id);

    // The choice for `allocator`: nullopt when every known sequence is in the
    // current batch, swapped out, or holds only shared blocks.
    [[nodiscard]] std::optional<PhysicalBlockId> choose(const MemoryAllocator& allocator) const;
    // `choose` bound to this policy, for MemoryAllocator::set_eviction_selector
    // (the policy must outlive the allocator's use of it).
    [[nodiscard]] EvictionCandidateSelector selector() const;

private:
    const KVCacheManager* cache_;
    std::uint64_t step_{0};
    std::unordered_map<SequenceId, std::uint64_t> last_used_;
};

}  // namespace qwenvl_paged
