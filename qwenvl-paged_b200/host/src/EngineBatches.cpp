// PagedPrefillBatch and KVAppendBatch: the engine-step callers of
// qvp_prefill and qvp_kv_append over the allocator's device pool.
#include "qwenvl_paged/PagedAttention.h"

#include "host_impl.h"
#include "qvp.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

namespace qwenvl_paged {

namespace {

using namespace host_impl;

// Pinned host and device buffers of `ints` int32 each (grown, never shrunk),
// the upload event and the device error word. Synchronizes the stream before
// freeing anything.
bool reserve_upload(std::int32_t*& host, std::int32_t*& dev, std::size_t& cap, void*& event, std::int32_t*& err,
                    std::size_t ints, cudaStream_t st) {
    if (event == nullptr) {
        cudaEvent_t ev = nullptr;
        if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        event = ev;
    }
    if (err == nullptr) {
        if (cudaMalloc(reinterpret_cast<void**>(&err), sizeof(std::int32_t)) != cudaSuccess) {
            cudaGetLastError();
            err = nullptr;
            return false;
        }
        cudaMemset(err, 0, sizeof(std::int32_t));
    }
    if (ints > cap) {
        cudaStreamSynchronize(st);
        if (host != nullptr) cudaFreeHost(host);
        if (dev != nullptr) cudaFree(dev);
        host = nullptr;
        dev = nullptr;
        cap = 0;
        const std::size_t n = std::max<std::size_t>(ints * 2, 4096);
        if (cudaMallocHost(reinterpret_cast<void**>(&host), n * sizeof(std::int32_t)) != cudaSuccess ||
            cudaMalloc(reinterpret_cast<void**>(&dev), n * sizeof(std::int32_t)) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        cap = n;
    }
    return true;
}

void release_upload(const MemoryAllocator& alloc, std::int32_t* host, std::int32_t* dev, void* event,
                    std::int32_t* err) {
    OnDevice guard(alloc.device());
    cudaStreamSynchronize(alloc.stream());
    if (host != nullptr) cudaFreeHost(host);
    if (dev != nullptr) cudaFree(dev);
    if (err != nullptr) cudaFree(err);
    if (event != nullptr) cudaEventDestroy(static_cast<cudaEvent_t>(event));
}

int read_error_word(const MemoryAllocator& alloc, const std::int32_t* err) {
    if (err == nullptr) return 0;
    OnDevice guard(alloc.device());
    std::int32_t v = 0;
    cudaStreamSynchronize(alloc.stream());
    cudaMemcpy(&v, err, sizeof(v), cudaMemcpyDeviceToHost);
    return v;
}

// Copies `staged` into the pinned buffer (once the previous upload has left
// it), lands queued copy-on-write copies and swap moves (the kernel that
// follows waits for every enqueued swap move), then uploads.
void upload(MemoryAllocator& alloc, const std::vector<std::int32_t>& staged, std::int32_t* host, std::int32_t* dev,
            void* event) {
    host_impl::wait_event(static_cast<cudaEvent_t>(event), "index upload", nullptr);
    std::memcpy(host, staged.data(), staged.size() * sizeof(std::int32_t));
    alloc.flush();
    alloc.order_writes();
    host_impl::upload_pinned(dev, host, staged.size() * sizeof(std::int32_t), alloc.stream());
    cudaEventRecord(static_cast<cudaEvent_t>(event), alloc.stream());
}

}  // namespace

// ---- PagedPrefillBatch -----------------------------------------------------

PagedPrefillBatch::PagedPrefillBatch(const MemoryAllocator& allocator) : allocator_(&allocator) {}

PagedPrefillBatch::~PagedPrefillBatch() { release_upload(*allocator_, host_buf_, dev_buf_, upload_event_, error_word_); }

int PagedPrefillBatch::device_error() { return read_error_word(*allocator_, error_word_); }

bool PagedPrefillBatch::run(const std::vector<CacheView>& views, const std::vector<std::uint32_t>& context_lens,
                            const std::vector<std::uint32_t>& query_lens, std::uint32_t layer,
                            std::uint32_t num_query_heads, float scale, const void* query, void* out) {
    status_ = QVP_ERR_INVALID;
    error_.clear();
    const std::size_t B = views.size();
    if (context_lens.size() != B || query_lens.size() != B || query == nullptr || out == nullptr) {
        error_ = "views, context lengths and query lengths differ in count, or a null buffer";
        return false;
    }
    if (B == 0) {
        status_ = QVP_OK;
        return true;
    }
    const std::size_t elem = allocator_->block_shape().bytes_per_element;
    const std::uint32_t tpb = allocator_->block_shape().tokens_per_block;
    std::uint32_t pitch = 1, max_q = 1;
    for (std::size_t b = 0; b < B; ++b) {
        if (views[b].allocator != allocator_ ||
            !arguments_fit(views[b], elem, layer, num_query_heads, context_lens[b])) {
            error_ = "sequence " + std::to_string(b) + " does not fit the cache shape";
            return false;
        }
        if (query_lens[b] == 0 || query_lens[b] > context_lens[b]) {
            error_ = "sequence " + std::to_string(b) + ": query length outside [1, context length]";
            return false;
        }
        pitch = std::max<std::uint32_t>(pitch, (context_lens[b] + tpb - 1) / tpb);
        max_q = std::max(max_q, query_lens[b]);
    }
    // [tables B x pitch][context lengths B][query lengths B]
    std::vector<std::int32_t> staged(B * pitch + 2 * B, -1);
    for (std::size_t b = 0; b < B; ++b) {
        const std::uint32_t nblk = (context_lens[b] + tpb - 1) / tpb;
        if (!write_row(views[b], nblk, staged.data() + b * pitch)) {
            status_ = QVP_ERR_UNMAPPED;
            error_ = "sequence " + std::to_string(b) + " has an unmapped or swapped-out block inside its context";
            return false;
        }
        staged[B * pitch + b] = static_cast<std::int32_t>(context_lens[b]);
        staged[B * pitch + B + b] = static_cast<std::int32_t>(query_lens[b]);
    }
    MemoryAllocator& alloc = const_cast<MemoryAllocator&>(*allocator_);
    if (!alloc.has_storage()) {
        error_ = "the pool has no device storage";
        return false;
    }
    OnDevice guard(alloc.device());
    if (!reserve_upload(host_buf_, dev_buf_, buf_ints_, upload_event_, error_word_, staged.size(), alloc.stream())) {
        status_ = QVP_ERR_NOMEM;
        error_ = "could not allocate prefill buffers";
        return false;
    }
    upload(alloc, staged, host_buf_, dev_buf_, upload_event_);
    const BlockShape& sh = alloc.block_shape();
    qvp_prefill_args a{};
    a.pool = alloc.pool_base();
    a.block_stride = alloc.block_stride();
    a.num_blocks = alloc.num_blocks();
    a.shape = {sh.tokens_per_block, sh.num_layers, sh.num_kv_heads, sh.head_dim, sh.bytes_per_element};
    a.dtype = dtype_for(elem);
    a.layer = layer;
    a.num_query_heads = num_query_heads;
    a.scale = scale;
    a.batch = static_cast<std::uint32_t>(B);
    a.max_blocks_per_seq = pitch;
    a.max_query_len = max_q;
    a.block_tables = dev_buf_;
    a.context_lens = dev_buf_ + B * pitch;
    a.query_lens = dev_buf_ + B * pitch + B;
    a.query = query;
    a.out = out;
    a.error_word = error_word_;
    status_ = qvp_prefill(&a, alloc.stream());
    if (status_ != QVP_OK) error_ = qvp_last_error();
    return status_ == QVP_OK;
}

// ---- KVAppendBatch ---------------------------------------------------------

KVAppendBatch::KVAppendBatch(const MemoryAllocator& allocator) : allocator_(&allocator) {}

KVAppendBatch::~KVAppendBatch() { release_upload(*allocator_, host_buf_, dev_buf_, upload_event_, error_word_); }

int KVAppendBatch::device_error() { return read_error_word(*allocator_, error_word_); }

bool KVAppendBatch::run(const std::vector<CacheView>& views, const std::vector<std::uint32_t>& positions,
                        std::uint32_t layer, const void* k, const void* v) {
    status_ = QVP_ERR_INVALID;
    error_.clear();
    const std::size_t B = views.size();
    if (positions.size() != B || k == nullptr || v == nullptr) {
        error_ = "views and positions differ in count, or a null buffer";
        return false;
    }
    if (B == 0) {
        status_ = QVP_OK;
        return true;
    }
    const BlockShape& sh = allocator_->block_shape();
    const std::uint32_t tpb = sh.tokens_per_block;
    if (tpb == 0 || layer >= sh.num_layers) {
        error_ = "layer outside the block shape";
        return false;
    }
    // The kernel needs only each target block: a one-column table holding it,
    // with the slot inside the block as the position. [ids B][slots B]
    std::vector<std::int32_t> staged(2 * B);
    for (std::size_t b = 0; b < B; ++b) {
        if (views[b].allocator != allocator_ || !views[b].valid()) {
            error_ = "sequence " + std::to_string(b) + " is not a view of this allocator";
            return false;
        }
        const BlockTableEntry* e = views[b].block_table->entry(positions[b] / tpb);
        if (e == nullptr || e->swap_slot.has_value() || e->physical_id >= allocator_->num_blocks()) {
            status_ = QVP_ERR_UNMAPPED;
            error_ = "sequence " + std::to_string(b) + ": the target block is not mapped";
            return false;
        }
        // a shared or read-only block would change every sequence that maps it
        const PhysicalBlockInfo* in = allocator_->info(e->physical_id);
        if (!e->writable || in == nullptr || in->ref_count != 1) {
            error_ = "sequence " + std::to_string(b) +
                     ": the target block is shared or read-only (call ensure_token_writable first)";
            return false;
        }
        staged[b] = static_cast<std::int32_t>(e->physical_id);
        staged[B + b] = static_cast<std::int32_t>(positions[b] % tpb);
    }
    MemoryAllocator& alloc = const_cast<MemoryAllocator&>(*allocator_);
    if (!alloc.has_storage()) {
        error_ = "the pool has no device storage";
        return false;
    }
    OnDevice guard(alloc.device());
    if (!reserve_upload(host_buf_, dev_buf_, buf_ints_, upload_event_, error_word_, staged.size(), alloc.stream())) {
        status_ = QVP_ERR_NOMEM;
        error_ = "could not allocate append buffers";
        return false;
    }
    upload(alloc, staged, host_buf_, dev_buf_, upload_event_);
    const qvp_block_shape shape{sh.tokens_per_block, sh.num_layers, sh.num_kv_heads, sh.head_dim,
                                sh.bytes_per_element};
    status_ = qvp_kv_append(alloc.pool_base(), alloc.block_stride(), alloc.num_blocks(), &shape, layer,
                            static_cast<std::uint32_t>(B), 1, dev_buf_, dev_buf_ + B, k, v, error_word_,
                            alloc.stream());
    if (status_ != QVP_OK) error_ = qvp_last_error();
    return status_ == QVP_OK;
}

}  // namespace qwenvl_paged
