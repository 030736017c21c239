#include "qwenvl_paged/SwapBackend.h"

#include "qwenvl_paged/MemoryAllocator.h"
#include "host_impl.h"
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
// Largest single PCIe copy: a small copy the engine stream enqueues meanwhile
// (a decode's table upload) may queue on the same copy engine behind one.
// Smaller pieces mean more calls per flush, and past about a thousand queued
// copies the host call itself blocks (8 MiB pieces held a 15 GB swap-out's
// flush on the host for 130 ms).
constexpr std::size_t kMaxCopyBytes = std::size_t(64) << 20;

// cudaMemcpyAsync of `bytes` in pieces of at most kMaxCopyBytes.
void copy_in_pieces(void* dst, const void* src, std::size_t bytes, cudaMemcpyKind kind, cudaStream_t st) {
    for (std::size_t off = 0; off < bytes; off += kMaxCopyBytes)
        cudaMemcpyAsync(static_cast<std::byte*>(dst) + off, static_cast<const std::byte*>(src) + off,
                        std::min(kMaxCopyBytes, bytes - off), kind, st);
}

using host_impl::OnDevice;

cudaEvent_t ev(CUevent_st* e) { return reinterpret_cast<cudaEvent_t>(e); }

bool make_event(CUevent_st*& e) {
    cudaEvent_t x = nullptr;
    if (cudaEventCreateWithFlags(&x, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    e = reinterpret_cast<CUevent_st*>(x);
    return true;
}

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

DeviceSwapBackend::DeviceSwapBackend(MemoryAllocator& allocator, std::size_t max_slots, SwapCoding coding)
    : allocator_(&allocator), max_slots_(max_slots), coding_(coding) {
    const PhysicalBlock* b0 = allocator.block(0);
    slot_bytes_ = b0 != nullptr ? b0->size_bytes() : 0;
    if (!allocator.has_storage() || slot_bytes_ == 0 || max_slots_ == 0) return;
    OnDevice guard(allocator.device());
    const bool coded = coding_ == SwapCoding::compressed;
    if (coded && slot_bytes_ % 16 != 0) {
        note("swap backend: compressed slots need blocks of a multiple of 16 bytes; every store is refused");
        return;
    }
    if (coded) {
        // a slot's head holds a coded block with up to one escape per 512
        // values; longer slots spill into the mapped tail
        const std::size_t full = qvp_swap_slot_bytes(slot_bytes_);
        const std::size_t head = (32 + slot_bytes_ / 4 * 3 + slot_bytes_ / 256 + 15) / 16 * 16;
        slab_stride_ = slot_bytes_ % 32 == 0 ? std::min(head, full) : full;
        tail_stride_ = full - slab_stride_;
    } else {
        slab_stride_ = slot_bytes_;
    }
    // Everything a flush needs is allocated here, so recorded moves always run.
    const std::size_t staging = std::min<std::size_t>(
        max_slots_, std::min<std::size_t>(65535, std::max<std::size_t>(1, kMaxStagingBytes / slab_stride_)));
    const std::size_t id_entries = (coded ? 4 : 2) * max_slots_;
    void* p = nullptr;
    bool ok = cudaHostAlloc(&p, max_slots_ * (slab_stride_ + tail_stride_),
                            coded ? cudaHostAllocMapped : cudaHostAllocDefault) == cudaSuccess;
    if (ok) slab_ = static_cast<std::byte*>(p);
    if (coded) {
        void* d = nullptr;
        ok = ok && cudaHostGetDevicePointer(&d, slab_, 0) == cudaSuccess;
        tails_dev_ = static_cast<std::byte*>(d) + max_slots_ * slab_stride_;
        ok = ok && cudaMalloc(reinterpret_cast<void**>(&link_dev_), 4 * sizeof(unsigned long long)) == cudaSuccess &&
             cudaMemset(link_dev_, 0, 4 * sizeof(unsigned long long)) == cudaSuccess;
    }
    ok = ok && cudaMalloc(reinterpret_cast<void**>(&staging_), staging * slab_stride_) == cudaSuccess;
    for (int b = 0; ok && b < 2; ++b) {
        ok = cudaMallocHost(reinterpret_cast<void**>(&ids_host_[b]), id_entries * sizeof(std::int32_t)) ==
                 cudaSuccess &&
             cudaMalloc(reinterpret_cast<void**>(&ids_dev_[b]), id_entries * sizeof(std::int32_t)) == cudaSuccess &&
             make_event(ids_uploaded_[b]);
    }
    // the lowest priority: the block scheduler serves a decode launched
    // meanwhile before the swap's gather, scatter or coding CTAs
    int least = 0, greatest = 0;
    cudaDeviceGetStreamPriorityRange(&least, &greatest);
    cudaStream_t cs = nullptr;
    ok = ok && cudaStreamCreateWithPriority(&cs, cudaStreamNonBlocking, least) == cudaSuccess;
    if (ok) copy_ = cs;
    ok = ok && make_event(engine_mark_) && make_event(moves_done_);
    if (!ok) {
        cudaGetLastError();
        note("swap backend: a buffer, stream or event could not be allocated; every store is refused");
        if (slab_ != nullptr) cudaFreeHost(slab_);
        slab_ = nullptr;
        return;
    }
    staging_blocks_ = staging;
    for (std::uint32_t i = 0; i < max_slots_; ++i) free_indices_.insert(free_indices_.end(), i);
}

DeviceSwapBackend::~DeviceSwapBackend() {
    OnDevice guard(allocator_->device());
    if (copy_ != nullptr) host_impl::wait_stream(copy_, "swap backend teardown", nullptr);
    if (slab_ != nullptr) cudaFreeHost(slab_);
    if (staging_ != nullptr) cudaFree(staging_);
    if (link_dev_ != nullptr) cudaFree(link_dev_);
    for (int b = 0; b < 2; ++b) {
        if (ids_dev_[b] != nullptr) cudaFree(ids_dev_[b]);
        if (ids_host_[b] != nullptr) cudaFreeHost(ids_host_[b]);
        if (ids_uploaded_[b] != nullptr) cudaEventDestroy(ev(ids_uploaded_[b]));
    }
    if (engine_mark_ != nullptr) cudaEventDestroy(ev(engine_mark_));
    if (moves_done_ != nullptr) cudaEventDestroy(ev(moves_done_));
    if (copy_ != nullptr) cudaStreamDestroy(copy_);
}

void DeviceSwapBackend::note(const std::string& what) {
    if (error_.empty()) error_ = what;
}

bool DeviceSwapBackend::ready() const noexcept { return slab_ != nullptr; }
std::size_t DeviceSwapBackend::capacity_slots() const noexcept { return max_slots_; }
std::size_t DeviceSwapBackend::resident_slots() const noexcept { return slots_.size(); }

const std::byte* DeviceSwapBackend::slot_bytes(SwapSlotId slot) const noexcept {
    const auto it = slots_.find(slot);
    return it == slots_.end() ? nullptr : slab_ + static_cast<std::size_t>(it->second) * slab_stride_;
}

std::pair<std::uint64_t, std::uint64_t> DeviceSwapBackend::link_bytes() {
    if (coding_ != SwapCoding::compressed || link_dev_ == nullptr) return {bytes_out_, bytes_in_};
    unsigned long long v[4] = {0, 0, 0, 0};
    if (!wait_idle()) return {0, 0};
    OnDevice guard(allocator_->device());
    if (cudaMemcpyAsync(v, link_dev_, sizeof v, cudaMemcpyDeviceToHost, copy_) != cudaSuccess ||
        !host_impl::wait_stream(copy_, "swap link byte counters", &error_)) {
        cudaGetLastError();
        return {0, 0};
    }
    return {heads_out_ + v[1], heads_in_ + v[3]};
}

std::optional<SwapSlotId> DeviceSwapBackend::store(const PhysicalBlock& block) {
    if (!ready() || slots_.size() >= max_slots_) return std::nullopt;
    // capacity counts resident slots, as in the reference; slab slots freed
    // by a discard while moves were queued become usable after a flush
    if (free_indices_.empty() && !release_after_flush_.empty()) flush();
    if (free_indices_.empty()) return std::nullopt;
    if (block.data() != allocator_->pool_base() + static_cast<std::size_t>(block.id()) * allocator_->block_stride())
        return std::nullopt;  // not a block of this backend's pool
    if (!pending_loads_.empty()) flush();  // stores and loads keep their program order
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
    // stores and loads keep their program order; a flush carries at most
    // max_slots moves, the size of its id lists
    if (!pending_stores_.empty() || pending_loads_.size() >= max_slots_) flush();
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
    if (pending_stores_.empty() && pending_loads_.empty()) {
        for (std::uint32_t idx : release_after_flush_) free_indices_.insert(idx);
        release_after_flush_.clear();
        return;
    }
    OnDevice guard(allocator_->device());
    // The moves follow every piece of engine work already enqueued (earlier
    // writes into a stored frame, earlier reads of a frame a load refills).
    cudaEventRecord(ev(engine_mark_), allocator_->stream());
    cudaStreamWaitEvent(copy_, ev(engine_mark_), 0);
    // one upload of the whole block-id list, into the list not used by the
    // previous flush (whose upload is long done unless flushes run back to back)
    const int b = ids_next_;
    ids_next_ ^= 1;
    if (!host_impl::wait_event(ev(ids_uploaded_[b]), "swap flush: id list still uploading", &error_)) return;
    const bool coded = coding_ == SwapCoding::compressed;
    const std::size_t n = pending_stores_.size() + pending_loads_.size();
    std::size_t k = 0;
    for (const Move& m : pending_stores_) {
        if (coded) ids_host_[b][n + k] = static_cast<std::int32_t>(m.slab_index);
        ids_host_[b][k++] = m.block;
    }
    for (const Move& m : pending_loads_) {
        if (coded) ids_host_[b][n + k] = static_cast<std::int32_t>(m.slab_index);
        ids_host_[b][k++] = m.block;
    }
    cudaMemcpyAsync(ids_dev_[b], ids_host_[b], (coded ? 2 * n : n) * sizeof(std::int32_t), cudaMemcpyHostToDevice,
                    copy_);
    cudaEventRecord(ev(ids_uploaded_[b]), copy_);
    ++flush_seq_;
    const bool loads = !pending_loads_.empty();
    const std::size_t ns = pending_stores_.size();
    flush_moves(pending_stores_, true, ids_dev_[b], ids_dev_[b] + n);
    flush_moves(pending_loads_, false, ids_dev_[b] + ns, ids_dev_[b] + n + ns);
    cudaEventRecord(ev(moves_done_), copy_);
    if (loads) last_load_flush_ = flush_seq_;
    pending_stores_.clear();
    pending_loads_.clear();
    for (std::uint32_t idx : release_after_flush_) free_indices_.insert(idx);
    release_after_flush_.clear();
}

// Enqueues `moves` on the copy stream in chunks of the staging size; ids_dev
// already holds their block ids in order and slab_idx_dev (compressed) their
// slab indices. A chunk is a gather (or coding) kernel into staging plus one
// copy per run of consecutive slab slots; loads the reverse.
void DeviceSwapBackend::flush_moves(std::vector<Move>& moves, bool stores, std::int32_t* ids_dev,
                                    std::int32_t* slab_idx_dev) {
    if (moves.empty()) return;
    std::vector<std::uint32_t> idx(moves.size());
    for (std::size_t i = 0; i < moves.size(); ++i) idx[i] = moves[i].slab_index;
    if (!stores) {
        if (frame_load_flush_.size() < allocator_->num_blocks()) frame_load_flush_.resize(allocator_->num_blocks(), 0);
        for (const Move& m : moves) frame_load_flush_[static_cast<std::size_t>(m.block)] = flush_seq_;
    }
    const bool coded = coding_ == SwapCoding::compressed;
    const auto slots = static_cast<std::uint32_t>(max_slots_);
    for (std::size_t base = 0; base < moves.size(); base += staging_blocks_) {
        const std::size_t n = std::min(staging_blocks_, moves.size() - base);
        const auto n32 = static_cast<std::uint32_t>(n);
        if (stores) {
            const int rc =
                coded ? qvp_compress_blocks(allocator_->pool_base(), allocator_->block_stride(),
                                            allocator_->num_blocks(), slot_bytes_, ids_dev + base,
                                            slab_idx_dev + base, n32, staging_, slab_stride_, tails_dev_,
                                            tail_stride_, slots, link_dev_, nullptr, copy_)
                      : qvp_gather_blocks(allocator_->pool_base(), allocator_->block_stride(),
                                          allocator_->num_blocks(), slot_bytes_, ids_dev + base, n32, staging_,
                                          nullptr, copy_);
            if (rc != QVP_OK) note(std::string(coded ? "swap-out compress: " : "swap-out gather: ") + qvp_last_error());
            for_each_run(idx.data() + base, n, [&](std::size_t first, std::size_t count) {
                copy_in_pieces(slab_ + static_cast<std::size_t>(idx[base + first]) * slab_stride_,
                               staging_ + first * slab_stride_, count * slab_stride_, cudaMemcpyDeviceToHost, copy_);
            });
            bytes_out_ += n * slot_bytes_;
            if (coded) heads_out_ += n * slab_stride_;
        } else {
            for_each_run(idx.data() + base, n, [&](std::size_t first, std::size_t count) {
                copy_in_pieces(staging_ + first * slab_stride_,
                               slab_ + static_cast<std::size_t>(idx[base + first]) * slab_stride_,
                               count * slab_stride_, cudaMemcpyHostToDevice, copy_);
            });
            const int rc =
                coded ? qvp_decompress_blocks(allocator_->pool_base(), allocator_->block_stride(),
                                              allocator_->num_blocks(), slot_bytes_, ids_dev + base,
                                              slab_idx_dev + base, n32, staging_, slab_stride_, tails_dev_,
                                              tail_stride_, slots, link_dev_ + 2, nullptr, copy_)
                      : qvp_scatter_blocks(allocator_->pool_base(), allocator_->block_stride(),
                                           allocator_->num_blocks(), slot_bytes_, ids_dev + base, n32, staging_,
                                           nullptr, copy_);
            if (rc != QVP_OK) note(std::string(coded ? "swap-in decompress: " : "swap-in scatter: ") + qvp_last_error());
            bytes_in_ += n * slot_bytes_;
            if (coded) heads_in_ += n * slab_stride_;
        }
    }
}

void DeviceSwapBackend::refresh_loads() const {
    if (done_seq_ < flush_seq_ && cudaEventQuery(ev(moves_done_)) == cudaSuccess) done_seq_ = flush_seq_;
    cudaGetLastError();
}

bool DeviceSwapBackend::loads_in_flight() const {
    if (last_load_flush_ <= std::max(done_seq_, engine_waited_)) return false;
    refresh_loads();
    return last_load_flush_ > std::max(done_seq_, engine_waited_);
}

void DeviceSwapBackend::order_engine(CUstream_st* engine, const std::int32_t* frames, std::size_t n, bool writes) {
    if (flush_seq_ <= engine_waited_) return;
    refresh_loads();
    const std::uint64_t settled = std::max(done_seq_, engine_waited_);
    if (flush_seq_ <= settled) return;
    const bool loads = last_load_flush_ > settled;
    bool wait = writes || (frames == nullptr && loads);
    if (!wait && loads && frames != nullptr) {
        const std::size_t nf = frame_load_flush_.size();
        for (std::size_t i = 0; i < n && !wait; ++i) {
            const std::int32_t f = frames[i];
            wait = f >= 0 && static_cast<std::size_t>(f) < nf && frame_load_flush_[static_cast<std::size_t>(f)] > settled;
        }
    }
    if (!wait) return;
    OnDevice guard(allocator_->device());
    cudaStreamWaitEvent(engine, ev(moves_done_), 0);
    engine_waited_ = flush_seq_;
}

bool DeviceSwapBackend::wait_idle() {
    if (copy_ == nullptr) return error_.empty();
    OnDevice guard(allocator_->device());
    const bool ok = host_impl::wait_stream(copy_, "swap moves", &error_);
    if (ok) done_seq_ = flush_seq_;
    return ok && error_.empty();
}

}  // namespace qwenvl_paged
