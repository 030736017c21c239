#include "qwenvl_paged/SwapBackend.h"

#include "qwenvl_paged/MemoryAllocator.h"
#include "qvp.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>

namespace qwenvl_paged {

// ---- HostSwapBackend: the reference's semantics over device blocks --------

HostSwapBackend::HostSwapBackend(std::size_t max_slots) : max_slots_(max_slots) {}

std::optional<SwapSlotId> HostSwapBackend::store(const PhysicalBlock& block) {
    if (slots_.size() >= max_slots_) return std::nullopt;
    std::vector<std::byte> bytes(block.size_bytes());
    if (!bytes.empty() && block.data() != nullptr) {
        cudaDeviceSynchronize();  // earlier device writes to the block must have landed
        if (cudaMemcpy(bytes.data(), block.data(), bytes.size(), cudaMemcpyDeviceToHost) != cudaSuccess) {
            cudaGetLastError();
            return std::nullopt;
        }
    }
    const SwapSlotId slot = next_slot_++;
    slots_.emplace(slot, std::move(bytes));
    return slot;
}

bool HostSwapBackend::load(SwapSlotId slot, PhysicalBlock& block) {
    const auto it = slots_.find(slot);
    if (it == slots_.end() || block.size_bytes() < it->second.size()) return false;
    if (!it->second.empty() && block.data() != nullptr) {
        cudaDeviceSynchronize();
        if (cudaMemcpy(block.data(), it->second.data(), it->second.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
    }
    return true;
}

void HostSwapBackend::discard(SwapSlotId slot) { slots_.erase(slot); }
std::size_t HostSwapBackend::resident_slots() const noexcept { return slots_.size(); }
std::size_t HostSwapBackend::capacity_slots() const noexcept { return max_slots_; }

// ---- DeviceSwapBackend ------------------------------------------------------

namespace {

constexpr std::size_t kMaxStagingBytes = std::size_t(256) << 20;

struct OnDevice {
    int prev = -1;
    bool switched = false;
    explicit OnDevice(int device) {
        if (device >= 0 && cudaGetDevice(&prev) == cudaSuccess && prev != device &&
            cudaSetDevice(device) == cudaSuccess)
            switched = true;
        cudaGetLastError();
    }
    ~OnDevice() {
        if (switched) cudaSetDevice(prev);
    }
};

}  // namespace

DeviceSwapBackend::DeviceSwapBackend(MemoryAllocator& allocator, std::size_t max_slots)
    : allocator_(&allocator), max_slots_(max_slots) {
    const PhysicalBlock* b0 = allocator.block(0);
    slot_bytes_ = b0 != nullptr ? b0->size_bytes() : 0;
    if (!allocator.has_storage() || slot_bytes_ == 0 || max_slots_ == 0) return;
    OnDevice guard(allocator.device());
    void* p = nullptr;
    if (cudaHostAlloc(&p, max_slots_ * slot_bytes_, cudaHostAllocDefault) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    slab_ = static_cast<std::byte*>(p);
    for (std::uint32_t i = 0; i < max_slots_; ++i) free_indices_.insert(free_indices_.end(), i);
}

DeviceSwapBackend::~DeviceSwapBackend() {
    OnDevice guard(allocator_->device());
    cudaStreamSynchronize(allocator_->stream());
    if (slab_ != nullptr) cudaFreeHost(slab_);
    if (staging_ != nullptr) cudaFree(staging_);
    if (ids_dev_ != nullptr) cudaFree(ids_dev_);
    if (ids_host_ != nullptr) cudaFreeHost(ids_host_);
    if (ids_event_ != nullptr) cudaEventDestroy(static_cast<cudaEvent_t>(ids_event_));
}

void DeviceSwapBackend::note(const std::string& what) {
    if (error_.empty()) error_ = what;
}

bool DeviceSwapBackend::ready() const noexcept { return slab_ != nullptr; }
std::size_t DeviceSwapBackend::capacity_slots() const noexcept { return max_slots_; }
std::size_t DeviceSwapBackend::resident_slots() const noexcept { return slots_.size(); }

const std::byte* DeviceSwapBackend::slot_bytes(SwapSlotId slot) const noexcept {
    const auto it = slots_.find(slot);
    return it == slots_.end() ? nullptr : slab_ + static_cast<std::size_t>(it->second) * slot_bytes_;
}

std::optional<SwapSlotId> DeviceSwapBackend::store(const PhysicalBlock& block) {
    if (!ready() || slots_.size() >= max_slots_) return std::nullopt;
    // capacity counts resident slots, as in the reference; slab slots freed
    // by a discard while moves were queued become usable after a flush
    if (free_indices_.empty() && !release_after_flush_.empty()) flush();
    if (free_indices_.empty()) return std::nullopt;
    if (block.data() != allocator_->pool_base() + static_cast<std::size_t>(block.id()) * allocator_->block_stride())
        return std::nullopt;  // not a block of this backend's pool
    if (!pending_loads_.empty()) flush_loads();
    const std::uint32_t idx = *free_indices_.begin();
    free_indices_.erase(free_indices_.begin());
    const SwapSlotId slot = next_slot_++;
    slots_.emplace(slot, idx);
    pending_stores_.push_back({static_cast<std::int32_t>(block.id()), idx});
    return slot;
}

bool DeviceSwapBackend::load(SwapSlotId slot, PhysicalBlock& block) {
    const auto it = slots_.find(slot);
    if (it == slots_.end() || block.size_bytes() < slot_bytes_) return false;
    if (block.data() != allocator_->pool_base() + static_cast<std::size_t>(block.id()) * allocator_->block_stride())
        return false;
    if (!pending_stores_.empty()) flush_stores();
    pending_loads_.push_back({static_cast<std::int32_t>(block.id()), it->second});
    return true;
}

void DeviceSwapBackend::discard(SwapSlotId slot) {
    const auto it = slots_.find(slot);
    if (it == slots_.end()) return;
    // a slab slot named by a move still queued is freed only after the flush
    if (!pending_stores_.empty() || !pending_loads_.empty())
        release_after_flush_.push_back(it->second);
    else
        free_indices_.insert(it->second);
    slots_.erase(it);
}

void DeviceSwapBackend::flush() {
    flush_stores();
    flush_loads();
    for (std::uint32_t idx : release_after_flush_) free_indices_.insert(idx);
    release_after_flush_.clear();
}

bool DeviceSwapBackend::ensure_staging(std::size_t blocks) {
    // one gather/scatter launch moves at most 65535 blocks
    const std::size_t cap = std::min<std::size_t>(65535, std::max<std::size_t>(1, kMaxStagingBytes / slot_bytes_));
    const std::size_t want = std::min(blocks, cap);
    if (want <= staging_blocks_ && ids_capacity_ >= want) return true;
    cudaStreamSynchronize(allocator_->stream());
    if (staging_ != nullptr) cudaFree(staging_);
    if (ids_dev_ != nullptr) cudaFree(ids_dev_);
    if (ids_host_ != nullptr) cudaFreeHost(ids_host_);
    staging_ = nullptr;
    ids_dev_ = nullptr;
    ids_host_ = nullptr;
    staging_blocks_ = ids_capacity_ = 0;
    if (cudaMalloc(reinterpret_cast<void**>(&staging_), want * slot_bytes_) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&ids_dev_), want * sizeof(std::int32_t)) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void**>(&ids_host_), want * sizeof(std::int32_t)) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (ids_event_ == nullptr) {
        cudaEvent_t ev = nullptr;
        if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        ids_event_ = ev;
    }
    staging_blocks_ = ids_capacity_ = want;
    return true;
}

namespace {

// Calls fn(first, count) for each maximal run of consecutive slab indices.
template <typename Fn>
void for_each_run(const std::uint32_t* idx, std::size_t n, Fn fn) {
    std::size_t i = 0;
    while (i < n) {
        std::size_t j = i + 1;
        while (j < n && idx[j] == idx[j - 1] + 1) ++j;
        fn(i, j - i);
        i = j;
    }
}

}  // namespace

void DeviceSwapBackend::flush_stores() {
    if (pending_stores_.empty()) return;
    OnDevice guard(allocator_->device());
    cudaStream_t st = allocator_->stream();
    if (!ensure_staging(pending_stores_.size())) {
        // the frames were already handed back to the pool: their bytes are lost
        note("swap-out: device staging could not be allocated; " + std::to_string(pending_stores_.size()) +
             " stored blocks were not moved");
        pending_stores_.clear();
        return;
    }
    std::vector<std::uint32_t> idx(staging_blocks_);
    for (std::size_t base = 0; base < pending_stores_.size(); base += staging_blocks_) {
        const std::size_t n = std::min(staging_blocks_, pending_stores_.size() - base);
        cudaEventSynchronize(static_cast<cudaEvent_t>(ids_event_));
        for (std::size_t i = 0; i < n; ++i) {
            ids_host_[i] = pending_stores_[base + i].block;
            idx[i] = pending_stores_[base + i].slab_index;
        }
        cudaMemcpyAsync(ids_dev_, ids_host_, n * sizeof(std::int32_t), cudaMemcpyHostToDevice, st);
        cudaEventRecord(static_cast<cudaEvent_t>(ids_event_), st);
        if (qvp_gather_blocks(allocator_->pool_base(), allocator_->block_stride(), allocator_->num_blocks(), slot_bytes_,
                              ids_dev_, static_cast<std::uint32_t>(n), staging_, nullptr, st) != QVP_OK)
            note(std::string("swap-out gather: ") + qvp_last_error());
        for_each_run(idx.data(), n, [&](std::size_t first, std::size_t count) {
            cudaMemcpyAsync(slab_ + static_cast<std::size_t>(idx[first]) * slot_bytes_, staging_ + first * slot_bytes_,
                            count * slot_bytes_, cudaMemcpyDeviceToHost, st);
        });
        bytes_out_ += n * slot_bytes_;
    }
    pending_stores_.clear();
}

void DeviceSwapBackend::flush_loads() {
    if (pending_loads_.empty()) return;
    OnDevice guard(allocator_->device());
    cudaStream_t st = allocator_->stream();
    if (!ensure_staging(pending_loads_.size())) {
        note("swap-in: device staging could not be allocated; " + std::to_string(pending_loads_.size()) +
             " loaded blocks were not restored");
        pending_loads_.clear();
        return;
    }
    std::vector<std::uint32_t> idx(staging_blocks_);
    for (std::size_t base = 0; base < pending_loads_.size(); base += staging_blocks_) {
        const std::size_t n = std::min(staging_blocks_, pending_loads_.size() - base);
        cudaEventSynchronize(static_cast<cudaEvent_t>(ids_event_));
        for (std::size_t i = 0; i < n; ++i) {
            ids_host_[i] = pending_loads_[base + i].block;
            idx[i] = pending_loads_[base + i].slab_index;
        }
        for_each_run(idx.data(), n, [&](std::size_t first, std::size_t count) {
            cudaMemcpyAsync(staging_ + first * slot_bytes_, slab_ + static_cast<std::size_t>(idx[first]) * slot_bytes_,
                            count * slot_bytes_, cudaMemcpyHostToDevice, st);
        });
        cudaMemcpyAsync(ids_dev_, ids_host_, n * sizeof(std::int32_t), cudaMemcpyHostToDevice, st);
        cudaEventRecord(static_cast<cudaEvent_t>(ids_event_), st);
        if (qvp_scatter_blocks(allocator_->pool_base(), allocator_->block_stride(), allocator_->num_blocks(), slot_bytes_,
                               ids_dev_, static_cast<std::uint32_t>(n), staging_, nullptr, st) != QVP_OK)
            note(std::string("swap-in scatter: ") + qvp_last_error());
        bytes_in_ += n * slot_bytes_;
    }
    pending_loads_.clear();
}

}  // namespace qwenvl_paged
