#include "qwenvl_paged/MemoryAllocator.h"

#include "host_impl.h"
#include "qvp.h"

#include <cuda_runtime.h>

#include <cstring>
#include <utility>

namespace qwenvl_paged {

namespace {

std::size_t round_to(std::size_t v, std::size_t a) { return a == 0 ? v : (v + a - 1) / a * a; }

// Switches to `device` for the lifetime of the guard (no-op for -1).
struct DeviceGuard {
    int prev = -1;
    bool switched = false;
    explicit DeviceGuard(int device) {
        if (device < 0) return;
        if (cudaGetDevice(&prev) == cudaSuccess && prev != device && cudaSetDevice(device) == cudaSuccess)
            switched = true;
        cudaGetLastError();
    }
    ~DeviceGuard() {
        if (switched) cudaSetDevice(prev);
    }
};

}  // namespace

MemoryAllocator::MemoryAllocator(AllocatorConfig config) : MemoryAllocator(config, DevicePoolOptions{}) {}

MemoryAllocator::MemoryAllocator(AllocatorConfig config, DevicePoolOptions options)
    : config_(config), device_(options.device), stream_(options.stream), host_visible_(options.host_visible) {
    const std::size_t alignment =
        config_.memory_options.alignment_bytes == 0 ? kDefaultBlockAlignmentBytes : config_.memory_options.alignment_bytes;
    std::size_t block_size = round_to(config_.block_shape.byte_size(), alignment);
    if (block_size == 0) block_size = alignment;
    stride_ = round_to(block_size, 256);
    // a padded stride keeps decode over managed memory off the TMA view
    if (host_visible_) stride_ += round_to(256, alignment);

    if (options.allocate_storage && config_.max_blocks > 0) {
        DeviceGuard guard(device_);
        if (device_ < 0) cudaGetDevice(&device_);
        void* p = nullptr;
        const std::size_t total = stride_ * config_.max_blocks;
        const cudaError_t e = host_visible_ ? cudaMallocManaged(&p, total, cudaMemAttachGlobal) : cudaMalloc(&p, total);
        // The copy-pair lists are sized for the most copies one flush can
        // carry (pending copies have distinct destinations), so a queued copy
        // never waits on an allocation that could fail.
        const std::size_t pair_ints = 2 * static_cast<std::size_t>(config_.max_blocks);
        cudaEvent_t ev = nullptr;
        const bool ok = e == cudaSuccess &&
                        cudaMalloc(reinterpret_cast<void**>(&pairs_dev_), pair_ints * sizeof(std::int32_t)) ==
                            cudaSuccess &&
                        cudaMallocHost(reinterpret_cast<void**>(&pairs_host_), pair_ints * sizeof(std::int32_t)) ==
                            cudaSuccess &&
                        cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) == cudaSuccess;
        if (ok) {
            pool_ = static_cast<std::byte*>(p);
            pairs_capacity_ = pair_ints;
            pairs_event_ = ev;
            cudaMemset(pool_, 0, total);
            cudaDeviceSynchronize();
        } else {
            const cudaError_t why = e != cudaSuccess ? e : cudaGetLastError();
            cudaGetLastError();
            error_ = std::string("device storage of the block pool could not be allocated: ") +
                     cudaGetErrorString(why);
            if (p != nullptr && e == cudaSuccess) cudaFree(p);
            if (pairs_dev_ != nullptr) cudaFree(pairs_dev_);
            if (pairs_host_ != nullptr) cudaFreeHost(pairs_host_);
            if (ev != nullptr) cudaEventDestroy(ev);
            pairs_dev_ = nullptr;
            pairs_host_ = nullptr;
        }
    }

    blocks_.reserve(config_.max_blocks);
    infos_.resize(config_.max_blocks);
    free_list_.reserve(config_.max_blocks);
    for (std::uint32_t i = 0; i < config_.max_blocks; ++i) {
        std::byte* bytes = pool_ != nullptr ? pool_ + static_cast<std::size_t>(i) * stride_ : nullptr;
        blocks_.push_back(std::make_unique<PhysicalBlock>(i, config_.block_shape, config_.memory_options, bytes,
                                                          block_size));
        infos_[i].id = i;
        free_list_.push_back(i);  // LIFO: the first allocate hands out N-1
    }
}

MemoryAllocator::~MemoryAllocator() { release_storage(); }

void MemoryAllocator::release_storage() noexcept {
    DeviceGuard guard(device_);
    if (pool_ != nullptr || pairs_dev_ != nullptr) host_impl::wait_stream(stream_, "allocator teardown", nullptr);
    if (pool_ != nullptr) cudaFree(pool_);
    if (pairs_dev_ != nullptr) cudaFree(pairs_dev_);
    if (pairs_host_ != nullptr) cudaFreeHost(pairs_host_);
    if (pairs_event_ != nullptr) cudaEventDestroy(static_cast<cudaEvent_t>(pairs_event_));
    pool_ = nullptr;
    pairs_dev_ = nullptr;
    pairs_host_ = nullptr;
    pairs_event_ = nullptr;
    pairs_capacity_ = 0;
}

MemoryAllocator::MemoryAllocator(MemoryAllocator&& o) noexcept { *this = std::move(o); }

MemoryAllocator& MemoryAllocator::operator=(MemoryAllocator&& o) noexcept {
    if (this == &o) return *this;
    release_storage();
    config_ = o.config_;
    device_ = o.device_;
    stream_ = o.stream_;
    host_visible_ = o.host_visible_;
    pool_ = std::exchange(o.pool_, nullptr);
    stride_ = o.stride_;
    blocks_ = std::move(o.blocks_);
    infos_ = std::move(o.infos_);
    free_list_ = std::move(o.free_list_);
    swap_backend_ = std::exchange(o.swap_backend_, nullptr);
    eviction_selector_ = std::move(o.eviction_selector_);
    pending_pairs_ = std::move(o.pending_pairs_);
    pending_src_ = std::move(o.pending_src_);
    pending_dst_ = std::move(o.pending_dst_);
    pairs_host_ = std::exchange(o.pairs_host_, nullptr);
    pairs_dev_ = std::exchange(o.pairs_dev_, nullptr);
    pairs_capacity_ = std::exchange(o.pairs_capacity_, 0);
    pairs_event_ = std::exchange(o.pairs_event_, nullptr);
    error_ = std::move(o.error_);
    copy_launches_ = o.copy_launches_;
    copies_done_ = o.copies_done_;
    return *this;
}

std::optional<PhysicalBlockId> MemoryAllocator::allocate() {
    if (free_list_.empty()) return std::nullopt;
    const PhysicalBlockId id = free_list_.back();
    free_list_.pop_back();
    infos_[id].state = BlockState::Active;
    infos_[id].ref_count = 1;
    return id;
}

void MemoryAllocator::release(PhysicalBlockId id) {
    if (id >= infos_.size() || infos_[id].ref_count == 0) return;
    PhysicalBlockInfo& in = infos_[id];
    in.ref_count -= 1;
    if (in.ref_count == 0) {
        in.state = BlockState::Free;
        in.generation += 1;
        free_list_.push_back(id);
    } else if (in.ref_count == 1) {
        in.state = BlockState::Active;
    }
}

void MemoryAllocator::retain(PhysicalBlockId id) {
    if (id >= infos_.size() || infos_[id].ref_count == 0) return;
    infos_[id].ref_count += 1;
    infos_[id].state = BlockState::Shared;
}

void MemoryAllocator::copy_block(PhysicalBlockId source, PhysicalBlockId destination) {
    if (source >= blocks_.size() || destination >= blocks_.size() || pool_ == nullptr) return;
    if (source == destination) return;  // copying a block onto itself changes nothing
    if (swap_backend_ != nullptr) swap_backend_->flush();
    // A copy that reads a pending destination, or writes a pending source or
    // destination, must wait for the copies already queued.
    if (pending_dst_.count(source) || pending_src_.count(destination) || pending_dst_.count(destination))
        flush_copies();
    pending_pairs_.push_back(static_cast<std::int32_t>(source));
    pending_pairs_.push_back(static_cast<std::int32_t>(destination));
    pending_src_.insert(source);
    pending_dst_.insert(destination);
    if (host_visible_) {
        // host code may read or write either block next: the copy lands now
        flush_copies();
        DeviceGuard guard(device_);
        host_impl::wait_stream(stream_, "copy-on-write copy", &error_);
    }
}

void MemoryAllocator::flush_copies() {
    if (pending_pairs_.empty()) return;
    DeviceGuard guard(device_);
    const std::size_t n = pending_pairs_.size();
    // the copies write frames a swap move may still read, or read frames a
    // swap-in is still filling
    if (swap_backend_ != nullptr) swap_backend_->order_engine(stream_, nullptr, 0, true);
    // the pinned list of the previous flush must have reached the device
    if (!host_impl::wait_event(static_cast<cudaEvent_t>(pairs_event_), "copy-pair upload", &error_)) return;
    std::memcpy(pairs_host_, pending_pairs_.data(), n * sizeof(std::int32_t));
    host_impl::upload_pinned(pairs_dev_, pairs_host_, n * sizeof(std::int32_t), stream_);
    cudaEventRecord(static_cast<cudaEvent_t>(pairs_event_), stream_);
    const int rc = qvp_copy_blocks(pool_, stride_, config_.max_blocks, blocks_.empty() ? 0 : blocks_[0]->size_bytes(),
                                   pairs_dev_, static_cast<std::uint32_t>(n / 2), nullptr, stream_);
    if (rc != QVP_OK) error_ = qvp_last_error();
    copy_launches_ += 1;
    copies_done_ += n / 2;
    pending_pairs_.clear();
    pending_src_.clear();
    pending_dst_.clear();
}

void MemoryAllocator::flush() {
    flush_copies();
    if (swap_backend_ != nullptr) swap_backend_->flush();
}

bool MemoryAllocator::synchronize() {
    flush();
    DeviceGuard guard(device_);
    if (!host_impl::wait_stream(stream_, "engine stream", &error_)) return false;
    if (swap_backend_ != nullptr && !swap_backend_->wait_idle()) {
        if (error_.empty()) error_ = "swap moves did not complete";
        return false;
    }
    return error_.empty();
}

void MemoryAllocator::order_reads(const std::int32_t* frames, std::size_t n) {
    if (swap_backend_ == nullptr) return;
    DeviceGuard guard(device_);
    swap_backend_->order_engine(stream_, frames, n, false);
}

void MemoryAllocator::order_writes() {
    if (swap_backend_ == nullptr) return;
    DeviceGuard guard(device_);
    swap_backend_->order_engine(stream_, nullptr, 0, true);
}

bool MemoryAllocator::loads_in_flight() const {
    return swap_backend_ != nullptr && swap_backend_->loads_in_flight();
}

bool MemoryAllocator::write_bytes(PhysicalBlockId id, std::size_t offset, const void* host, std::size_t bytes) {
    if (pool_ == nullptr || id >= blocks_.size() || offset > blocks_[id]->size_bytes() ||
        bytes > blocks_[id]->size_bytes() - offset)
        return false;
    if (!synchronize()) return false;
    DeviceGuard guard(device_);
    return cudaMemcpy(blocks_[id]->data() + offset, host, bytes, cudaMemcpyHostToDevice) == cudaSuccess;
}

bool MemoryAllocator::read_bytes(PhysicalBlockId id, std::size_t offset, void* host, std::size_t bytes) {
    if (pool_ == nullptr || id >= blocks_.size() || offset > blocks_[id]->size_bytes() ||
        bytes > blocks_[id]->size_bytes() - offset)
        return false;
    if (!synchronize()) return false;
    DeviceGuard guard(device_);
    return cudaMemcpy(host, blocks_[id]->data() + offset, bytes, cudaMemcpyDeviceToHost) == cudaSuccess;
}

PhysicalBlock* MemoryAllocator::block(PhysicalBlockId id) noexcept {
    return id < blocks_.size() ? blocks_[id].get() : nullptr;
}

const PhysicalBlock* MemoryAllocator::block(PhysicalBlockId id) const noexcept {
    return id < blocks_.size() ? blocks_[id].get() : nullptr;
}

const PhysicalBlockInfo* MemoryAllocator::info(PhysicalBlockId id) const noexcept {
    return id < infos_.size() ? &infos_[id] : nullptr;
}

void MemoryAllocator::set_swap_backend(SwapBackend* backend) noexcept { swap_backend_ = backend; }

std::optional<SwapSlotId> MemoryAllocator::swap_out(PhysicalBlockId id) {
    if (swap_backend_ == nullptr || id >= infos_.size()) return std::nullopt;
    PhysicalBlockInfo& in = infos_[id];
    // only a block with exactly one owner can give up its frame
    if (in.ref_count != 1) return std::nullopt;
    flush_copies();
    const std::optional<SwapSlotId> slot = swap_backend_->store(*blocks_[id]);
    if (!slot) return std::nullopt;
    in.ref_count = 0;
    in.state = BlockState::Free;
    in.generation += 1;
    free_list_.push_back(id);
    return slot;
}

std::optional<PhysicalBlockId> MemoryAllocator::swap_in(SwapSlotId slot) {
    if (swap_backend_ == nullptr) return std::nullopt;
    const std::optional<PhysicalBlockId> id = allocate();
    if (!id) return std::nullopt;
    flush_copies();
    if (!swap_backend_->load(slot, *blocks_[*id])) {
        release(*id);
        return std::nullopt;
    }
    swap_backend_->discard(slot);
    return id;
}

void MemoryAllocator::discard_swapped(SwapSlotId slot) {
    if (swap_backend_ != nullptr) swap_backend_->discard(slot);
}

void MemoryAllocator::set_eviction_selector(EvictionCandidateSelector selector) {
    eviction_selector_ = std::move(selector);
}

std::optional<PhysicalBlockId> MemoryAllocator::select_eviction_candidate() const {
    return eviction_selector_ ? eviction_selector_(*this) : std::nullopt;
}

AllocatorStats MemoryAllocator::stats() const noexcept {
    AllocatorStats st;
    st.total_blocks = static_cast<std::uint32_t>(infos_.size());
    for (const PhysicalBlockInfo& in : infos_) {
        if (in.state == BlockState::Free) st.free_blocks += 1;
        else if (in.state == BlockState::Active) st.active_blocks += 1;
        else if (in.state == BlockState::Shared) st.shared_blocks += 1;
    }
    if (swap_backend_ != nullptr) st.swapped_blocks = static_cast<std::uint32_t>(swap_backend_->resident_slots());
    for (const auto& b : blocks_) st.bytes_reserved += b->size_bytes();
    return st;
}

bool MemoryAllocator::can_allocate(std::uint32_t block_count) const noexcept {
    return free_list_.size() >= block_count;
}

}  // namespace qwenvl_paged
