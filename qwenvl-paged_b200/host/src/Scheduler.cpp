#include "qwenvl_paged/Scheduler.h"

#include <algorithm>
#include <utility>

namespace qwenvl_paged {

namespace {

template <typename Queue>
auto locate(Queue& q, RequestId id) {
    return std::find_if(q.begin(), q.end(), [id](const Request& r) { return r.request_id == id; });
}

SequenceMetadata sequence_metadata(const Request& r) {
    SequenceMetadata m;
    m.sequence_id = r.root_sequence_id;
    m.request_id = r.request_id;
    m.multimodal_spans = r.multimodal_spans;
    m.positional_encoding = r.positional_encoding;
    return m;
}

}  // namespace

Scheduler::Scheduler(SchedulerConfig config, KVCacheManager& cache_manager, MemoryAllocator& allocator)
    : config_(config), cache_manager_(&cache_manager), allocator_(&allocator) {}

void Scheduler::enqueue(Request request) {
    request.state = RequestState::Pending;
    pending_.push_back(std::move(request));
}

BatchPlan Scheduler::schedule_next() {
    BatchPlan plan;
    while (!pending_.empty() && active_.size() < config_.max_active_requests) {
        Request& next = pending_.front();
        if (plan.scheduled_tokens + next.prompt_tokens > config_.max_batch_tokens) break;
        reclaim_for_admission(next.prompt_tokens, plan.prefill_requests.size());
        if (!cache_manager_->create_sequence(sequence_metadata(next))) break;
        if (!cache_manager_->reserve_tokens(next.root_sequence_id, next.prompt_tokens)) {
            // reference src/Scheduler.cpp:53-56
            cache_manager_->release_sequence(next.root_sequence_id);
            break;
        }
        next.state = RequestState::Prefill;
        plan.prefill_requests.push_back(next.request_id);
        plan.scheduled_tokens += next.prompt_tokens;
        active_.push_back(std::move(next));
        pending_.pop_front();
    }
    for (const Request& r : active_) {
        if (r.state != RequestState::Decode) continue;
        plan.decode_requests.push_back(r.request_id);
        plan.scheduled_tokens += 1;
    }
    return plan;
}

void Scheduler::complete_step(RequestId request_id, std::uint32_t /*produced_tokens*/) {
    const auto it = locate(active_, request_id);
    if (it != active_.end() && it->state == RequestState::Prefill) it->state = RequestState::Decode;
}

void Scheduler::cancel(RequestId request_id) {
    for (std::deque<Request>* q : {&pending_, &active_, &preempted_}) {
        const auto it = locate(*q, request_id);
        if (it == q->end()) continue;
        cache_manager_->release_sequence(it->root_sequence_id);
        q->erase(it);
        preemption_info_.erase(request_id);
        return;
    }
}

bool Scheduler::preempt(RequestId request_id, std::string reason) {
    const auto it = locate(active_, request_id);
    if (it == active_.end()) return false;
    Request r = std::move(*it);
    active_.erase(it);
    r.state = RequestState::Preempted;
    PreemptionInfo info;
    info.reason = std::move(reason);
    info.swapped_blocks = cache_manager_->swap_out_sequence(r.root_sequence_id);
    preemption_info_[r.request_id] = std::move(info);
    preempted_.push_back(std::move(r));
    return true;
}

bool Scheduler::resume(RequestId request_id) {
    const auto it = locate(preempted_, request_id);
    if (it == preempted_.end()) return false;
    if (!cache_manager_->swap_in_sequence(it->root_sequence_id)) return false;
    Request r = std::move(*it);
    preempted_.erase(it);
    r.state = RequestState::Decode;
    preemption_info_.erase(request_id);
    active_.push_back(std::move(r));
    return true;
}

std::optional<PreemptionInfo> Scheduler::preemption_info(RequestId request_id) const {
    const auto it = preemption_info_.find(request_id);
    if (it == preemption_info_.end()) return std::nullopt;
    return it->second;
}

std::optional<RequestState> Scheduler::state(RequestId request_id) const {
    for (const std::deque<Request>* q : {&pending_, &active_, &preempted_})
        for (const Request& r : *q)
            if (r.request_id == request_id) return r.state;
    return std::nullopt;
}

std::size_t Scheduler::active_size() const noexcept { return active_.size(); }

std::uint32_t Scheduler::blocks_for_tokens(std::uint32_t token_count) const noexcept {
    const PhysicalBlock* b0 = allocator_->block(0);
    const std::uint32_t tpb = b0 != nullptr ? b0->shape().tokens_per_block : 0;
    return tpb == 0 ? 0 : (token_count + tpb - 1) / tpb;
}

void Scheduler::reclaim_for_admission(std::uint32_t prompt_tokens, std::size_t admitted_this_step) {
    if (config_.preemption_watermark_blocks == 0) return;
    const AllocatorStats st = allocator_->stats();
    const std::uint32_t need = blocks_for_tokens(prompt_tokens);
    // reference src/Scheduler.cpp:180-185
    if (need == 0 || need > st.total_blocks) return;
    const std::uint32_t target = std::min(need + config_.preemption_watermark_blocks, st.total_blocks);
    while (active_.size() > admitted_this_step && allocator_->stats().free_blocks < target) {
        const std::uint32_t free_before = allocator_->stats().free_blocks;
        // victim order: reference src/Scheduler.cpp:196-199
        const RequestId victim = active_[active_.size() - admitted_this_step - 1].request_id;
        if (!preempt(victim, "cache pressure watermark")) break;
        if (allocator_->stats().free_blocks <= free_before) break;  // reference src/Scheduler.cpp:203-207
    }
}

}  // namespace qwenvl_paged
