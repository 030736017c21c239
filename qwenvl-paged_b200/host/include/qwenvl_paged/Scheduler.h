// Continuous-batching scheduler with the reference's frozen semantics
// (include/qwenvl_paged/Scheduler.h:17-199, src/Scheduler.cpp): FIFO
// admission under max_active_requests / max_batch_tokens, a request stays
// pending (leaving nothing behind) when its prompt cannot be reserved,
// watermark-driven preemption newest-first, resume all-or-nothing. It drives
// the device path only through KVCacheManager (swap) and allocator stats.
#pragma once

#include "qwenvl_paged/KVCacheManager.h"
#include "qwenvl_paged/MemoryAllocator.h"

#include <cstdint>
#include <deque>
#include <optional>
#include <string>
#include <unordered_map>
#include <vector>

namespace qwenvl_paged {

enum class RequestState : std::uint8_t { Pending, Prefill, Decode, Preempted, Finished, Cancelled };

struct SamplingConfig {
    std::uint32_t num_parallel_samples{1};
    std::uint32_t max_decode_tokens{0};
};

struct Request {
    RequestId request_id{0};
    SequenceId root_sequence_id{0};
    std::uint32_t prompt_tokens{0};
    SamplingConfig sampling{};
    std::vector<MultimodalSpan> multimodal_spans;
    PositionalEncodingMetadata positional_encoding;
    RequestState state{RequestState::Pending};
};

struct SchedulerConfig {
    std::uint32_t max_active_requests{0};
    std::uint32_t max_batch_tokens{0};
    // 0 disables automatic preemption.
    std::uint32_t preemption_watermark_blocks{0};
};

struct PreemptionInfo {
    std::string reason;
    std::uint32_t swapped_blocks{0};
};

struct BatchPlan {
    std::vector<RequestId> prefill_requests;
    std::vector<RequestId> decode_requests;
    std::uint32_t scheduled_tokens{0};
};

class Scheduler {
public:
    Scheduler(SchedulerConfig config, KVCacheManager& cache_manager, MemoryAllocator& allocator);
    ~Scheduler() = default;
    Scheduler(const Scheduler&) = delete;
    Scheduler& operator=(const Scheduler&) = delete;
    Scheduler(Scheduler&&) noexcept = default;
    Scheduler& operator=(Scheduler&&) noexcept = default;

    void enqueue(Request request);
    [[nodiscard]] BatchPlan schedule_next();
    void complete_step(RequestId request_id, std::uint32_t produced_tokens);
    void cancel(RequestId request_id);
    bool preempt(RequestId request_id, std::string reason);
    bool resume(RequestId request_id);
    [[nodiscard]] std::optional<PreemptionInfo> preemption_info(RequestId request_id) const;
    [[nodiscard]] std::optional<RequestState> state(RequestId request_id) const;
    [[nodiscard]] std::size_t active_size() const noexcept;

private:
    [[nodiscard]] std::uint32_t blocks_for_tokens(std::uint32_t token_count) const noexcept;
    void reclaim_for_admission(std::uint32_t prompt_tokens, std::size_t admitted_this_step);

    SchedulerConfig config_{};
    KVCacheManager* cache_manager_{nullptr};
    MemoryAllocator* allocator_{nullptr};
    std::deque<Request> pending_;
    std::deque<Request> active_;
    std::deque<Request> preempted_;
    std::unordered_map<RequestId, PreemptionInfo> preemption_info_;
};

}  // namespace qwenvl_paged
