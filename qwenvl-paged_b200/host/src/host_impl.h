// Helpers shared by the host layer's device-facing classes
// (PagedAttention.cpp, ResidentTables.cpp): device switching, view checks and
// table-row flattening with the reference kernel's refusal rules.
#pragma once

#include "qwenvl_paged/KVCacheManager.h"
#include "qwenvl_paged/MemoryAllocator.h"

#include "qvp.h"

#include <cuda_runtime.h>

#include <chrono>
#include <cstddef>
#include <cstdint>
#include <optional>
#include <string>
#include <thread>
#include <vector>

namespace qwenvl_paged {
namespace host_impl {

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

// Uploads a small pinned host buffer to the device on `st`. Up to
// kFetchLimit bytes the SMs read it over PCIe (qvp_fetch_host), so the upload
// does not queue behind swap copies on the copy engines; larger ones go by
// cudaMemcpyAsync.
constexpr std::size_t kFetchLimit = std::size_t(4) << 20;
inline bool upload_pinned(void* dev, const void* pinned, std::size_t bytes, cudaStream_t st) {
    if (bytes <= kFetchLimit) return qvp_fetch_host(dev, pinned, bytes, st) == QVP_OK;
    return cudaMemcpyAsync(dev, pinned, bytes, cudaMemcpyHostToDevice, st) == cudaSuccess;
}

// How long a host-side wait for device work may last before it gives up
// with an error (a healthy wait here is milliseconds; a device that stopped
// answering must not hang the engine thread).
constexpr double kHostWaitLimitSeconds = 60.0;

// Polls `ev` until it completes; false (with `err` set) on a device error or
// after kHostWaitLimitSeconds.
inline bool wait_event(cudaEvent_t ev, const char* what, std::string* err) {
    if (ev == nullptr) return true;
    const auto start = std::chrono::steady_clock::now();
    for (unsigned spins = 0;; ++spins) {
        const cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return true;
        if (e != cudaErrorNotReady) {
            cudaGetLastError();
            if (err != nullptr && err->empty()) *err = std::string(what) + ": " + cudaGetErrorString(e);
            return false;
        }
        if (spins > 64) {
            if (std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count() >
                kHostWaitLimitSeconds) {
                if (err != nullptr && err->empty()) *err = std::string(what) + ": timed out";
                return false;
            }
            std::this_thread::sleep_for(std::chrono::microseconds(spins > 1024 ? 200 : 20));
        }
    }
}

// Waits (bounded, as wait_event) for everything enqueued on `stream` so far.
inline bool wait_stream(cudaStream_t stream, const char* what, std::string* err) {
    cudaEvent_t ev = nullptr;
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        if (err != nullptr && err->empty()) *err = std::string(what) + ": could not create an event";
        return false;
    }
    bool ok = cudaEventRecord(ev, stream) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        if (err != nullptr && err->empty()) *err = std::string(what) + ": could not record an event";
    } else {
        ok = wait_event(ev, what, err);
    }
    cudaEventDestroy(ev);
    return ok;
}

inline bool is_device_pointer(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// The host-side checks of the reference kernel (PagedAttention.h:59-89):
// shape/argument consistency, then every block of [0, context_len) must be
// resolvable. Appends the physical ids of those blocks to `ids`.
inline bool resolve(const CacheView& view, std::size_t elem_bytes, std::uint32_t layer, std::uint32_t num_query_heads,
             std::uint32_t context_len, std::vector<std::int32_t>& ids) {
    if (!view.valid()) return false;
    const BlockShape& sh = view.layout.shape;
    if (elem_bytes != sh.bytes_per_element || context_len == 0 || layer >= sh.num_layers ||
        num_query_heads == 0 || num_query_heads % sh.num_kv_heads != 0)
        return false;
    const std::uint32_t tpb = sh.tokens_per_block;
    const std::uint32_t nblk = (context_len + tpb - 1) / tpb;
    for (std::uint32_t i = 0; i < nblk; ++i) {
        const std::optional<PhysicalBlockId> id = view.block_table->lookup(i);
        if (!id || view.allocator->block(*id) == nullptr) return false;
        ids.push_back(static_cast<std::int32_t>(*id));
    }
    return true;
}

// The arguments part of resolve(), without walking the table.
inline bool arguments_fit(const CacheView& view, std::size_t elem_bytes, std::uint32_t layer, std::uint32_t num_query_heads,
                   std::uint32_t context_len) {
    if (!view.valid()) return false;
    const BlockShape& sh = view.layout.shape;
    return elem_bytes == sh.bytes_per_element && context_len != 0 && layer < sh.num_layers && num_query_heads != 0 &&
           num_query_heads % sh.num_kv_heads == 0;
}

// Writes the physical ids of blocks [0, nblk) into `row` by one pass over the
// table's sorted entries; false if any of them is unmapped or swapped (the
// same blocks resolve() would refuse).
inline bool write_row(const CacheView& view, std::uint32_t nblk, std::int32_t* row) {
    const std::vector<BlockTableEntry>& es = view.block_table->entries();
    const std::uint32_t limit = view.allocator->num_blocks();
    if (es.size() < nblk) return false;
    for (std::uint32_t i = 0; i < nblk; ++i) {
        const BlockTableEntry& e = es[i];
        // sorted and unique: entry i maps logical block i iff its index is i
        if (e.logical.index != i || e.swap_slot.has_value() || e.physical_id >= limit) return false;
        row[i] = static_cast<std::int32_t>(e.physical_id);
    }
    return true;
}

inline int dtype_for(std::size_t elem_bytes) {
    return elem_bytes == 4 ? QVP_DTYPE_F32 : elem_bytes == 2 ? QVP_DTYPE_BF16 : -1;
}

inline qvp_decode_args base_args(const MemoryAllocator& alloc, std::size_t elem_bytes, std::uint32_t layer,
                          std::uint32_t num_query_heads, float scale) {
    qvp_decode_args a{};
    const BlockShape& sh = alloc.block_shape();
    a.pool = alloc.pool_base();
    a.block_stride = alloc.block_stride();
    a.num_blocks = alloc.num_blocks();
    a.shape = {sh.tokens_per_block, sh.num_layers, sh.num_kv_heads, sh.head_dim, sh.bytes_per_element};
    a.dtype = dtype_for(elem_bytes);
    a.layer = layer;
    a.num_query_heads = num_query_heads;
    a.scale = scale;
    return a;
}

}  // namespace host_impl
}  // namespace qwenvl_paged
