#include "qwenvl_paged/Block.h"

#include <atomic>
#include <cstdlib>

#include <cuda_runtime.h>

namespace qwenvl_paged {

namespace {

std::size_t rounded(std::size_t bytes, std::size_t alignment) noexcept {
    if (alignment == 0) alignment = kDefaultBlockAlignmentBytes;
    const std::size_t n = (bytes + alignment - 1) / alignment * alignment;
    return n == 0 ? alignment : n;
}

}  // namespace

std::size_t BlockShape::byte_size() const noexcept {
    return std::size_t{2} * tokens_per_block * num_layers * num_kv_heads * head_dim * bytes_per_element;
}

bool LogicalBlock::empty() const noexcept { return token_count == 0; }

namespace {
std::atomic<int>& host_visible_flag() {
    static std::atomic<int> flag{[] {
        const char* v = std::getenv("QVP_HOST_VISIBLE_POOLS");
        return (v != nullptr && v[0] == '1') ? 1 : 0;
    }()};
    return flag;
}
}  // namespace

bool host_visible_pools() noexcept { return host_visible_flag().load(std::memory_order_relaxed) != 0; }
void set_host_visible_pools(bool on) noexcept { host_visible_flag().store(on ? 1 : 0, std::memory_order_relaxed); }

PhysicalBlock::PhysicalBlock(PhysicalBlockId id, BlockShape shape, HostMemoryOptions memory_options)
    : id_(id), shape_(shape), memory_options_(memory_options) {
    size_bytes_ = rounded(shape_.byte_size(), memory_options_.alignment_bytes);
    void* p = nullptr;
    // cudaMalloc and cudaMallocManaged return addresses aligned to at least
    // 256 bytes, the reference's default block alignment.
    const cudaError_t e = host_visible_pools() ? cudaMallocManaged(&p, size_bytes_, cudaMemAttachGlobal)
                                               : cudaMalloc(&p, size_bytes_);
    if (e == cudaSuccess) {
        storage_ = static_cast<std::byte*>(p);
        owns_storage_ = true;
    } else {
        cudaGetLastError();
        storage_ = nullptr;
    }
}

PhysicalBlock::PhysicalBlock(PhysicalBlockId id, BlockShape shape, HostMemoryOptions memory_options,
                             std::byte* storage, std::size_t size_bytes) noexcept
    : id_(id), shape_(shape), memory_options_(memory_options), size_bytes_(size_bytes), storage_(storage) {}

PhysicalBlock::~PhysicalBlock() {
    if (owns_storage_ && storage_ != nullptr) cudaFree(storage_);
}

PhysicalBlock::PhysicalBlock(PhysicalBlock&& o) noexcept
    : id_(o.id_), shape_(o.shape_), memory_options_(o.memory_options_), size_bytes_(o.size_bytes_),
      storage_(o.storage_), owns_storage_(o.owns_storage_) {
    o.storage_ = nullptr;
    o.owns_storage_ = false;
}

PhysicalBlock& PhysicalBlock::operator=(PhysicalBlock&& o) noexcept {
    if (this != &o) {
        if (owns_storage_ && storage_ != nullptr) cudaFree(storage_);
        id_ = o.id_;
        shape_ = o.shape_;
        memory_options_ = o.memory_options_;
        size_bytes_ = o.size_bytes_;
        storage_ = o.storage_;
        owns_storage_ = o.owns_storage_;
        o.storage_ = nullptr;
        o.owns_storage_ = false;
    }
    return *this;
}

PhysicalBlockId PhysicalBlock::id() const noexcept { return id_; }
const BlockShape& PhysicalBlock::shape() const noexcept { return shape_; }
std::byte* PhysicalBlock::data() noexcept { return storage_; }
const std::byte* PhysicalBlock::data() const noexcept { return storage_; }
std::size_t PhysicalBlock::size_bytes() const noexcept { return size_bytes_; }
std::size_t PhysicalBlock::alignment_bytes() const noexcept { return memory_options_.alignment_bytes; }
bool PhysicalBlock::pinned_memory_requested() const noexcept { return memory_options_.prefer_pinned_memory; }

void PhysicalBlock::swap(PhysicalBlock& other) noexcept {
    if (this == &other) return;
    if (owns_storage_ && other.owns_storage_) {
        std::swap(storage_, other.storage_);
        std::swap(size_bytes_, other.size_bytes_);
    } else if (storage_ != nullptr && other.storage_ != nullptr) {
        // Pool views keep their addresses; exchange the bytes (the common
        // prefix when sizes differ) through a temporary device buffer.
        const std::size_t n = size_bytes_ < other.size_bytes_ ? size_bytes_ : other.size_bytes_;
        void* tmp = nullptr;
        if (cudaMalloc(&tmp, n) == cudaSuccess) {
            cudaMemcpy(tmp, storage_, n, cudaMemcpyDeviceToDevice);
            cudaMemcpy(storage_, other.storage_, n, cudaMemcpyDeviceToDevice);
            cudaMemcpy(other.storage_, tmp, n, cudaMemcpyDeviceToDevice);
            cudaFree(tmp);
        } else {
            cudaGetLastError();
        }
    }
    std::swap(shape_, other.shape_);
    std::swap(memory_options_, other.memory_options_);
}

}  // namespace qwenvl_paged
