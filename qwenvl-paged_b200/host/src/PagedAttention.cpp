#include "qwenvl_paged/PagedAttention.h"

#include "qvp.h"
#include "host_impl.h"

#include <cuda_runtime.h>

#include <algorithm>

namespace qwenvl_paged {

namespace {

using namespace host_impl;

// Device scratch of the single-sequence shim, grown on demand.
struct ShimBuffers {
    int device = -1;
    void* mem = nullptr;
    std::size_t bytes = 0;
    ~ShimBuffers() {
        if (mem != nullptr) cudaFree(mem);
    }
    std::byte* get(std::size_t need, int dev) {
        if (mem != nullptr && (need > bytes || dev != device)) {
            cudaFree(mem);
            mem = nullptr;
            bytes = 0;
        }
        if (mem == nullptr) {
            const std::size_t n = std::max<std::size_t>(need, 1 << 20);
            if (cudaMalloc(&mem, n) != cudaSuccess) {
                cudaGetLastError();
                return nullptr;
            }
            bytes = n;
            device = dev;
        }
        return static_cast<std::byte*>(mem);
    }
};

std::size_t align256(std::size_t v) { return (v + 255) / 256 * 256; }

}  // namespace

namespace detail {

bool decode_one(const CacheView& view, const void* query, std::size_t elem_bytes, const PagedAttentionParams& params,
                void* out) {
    if (query == nullptr || out == nullptr) return false;
    std::vector<std::int32_t> ids;
    if (!resolve(view, elem_bytes, params.layer, params.num_query_heads, params.context_len, ids)) return false;
    MemoryAllocator& alloc = const_cast<MemoryAllocator&>(*view.allocator);
    if (!alloc.has_storage() || dtype_for(elem_bytes) < 0) return false;
    OnDevice guard(alloc.device());
    alloc.flush();  // queued copy-on-write copies land before the decode reads
    alloc.order_reads(ids.data(), ids.size());  // and swap-ins into its frames

    const BlockShape& sh = view.layout.shape;
    const std::size_t qo_bytes = static_cast<std::size_t>(params.num_query_heads) * sh.head_dim * elem_bytes;
    qvp_decode_args a = base_args(alloc, elem_bytes, params.layer, params.num_query_heads, params.scale);
    a.batch = 1;
    a.max_blocks_per_seq = static_cast<std::uint32_t>(ids.size());
    a.max_context_len = params.context_len;
    a.block_tables = reinterpret_cast<const std::int32_t*>(0x10);  // placeholders for the size query
    a.context_lens = reinterpret_cast<const std::int32_t*>(0x10);
    a.query = query;
    a.out = out;
    std::size_t ws = 0;
    if (qvp_decode_workspace_size(&a, &ws) != QVP_OK) return false;

    const bool q_dev = is_device_pointer(query);
    const bool o_dev = is_device_pointer(out);
    const std::size_t tab_off = 0;
    const std::size_t q_off = align256(tab_off + (ids.size() + 1) * sizeof(std::int32_t));
    const std::size_t o_off = align256(q_off + qo_bytes);
    const std::size_t ws_off = align256(o_off + qo_bytes);
    static thread_local ShimBuffers buffers;
    std::byte* base = buffers.get(ws_off + ws, alloc.device());
    if (base == nullptr) return false;

    cudaStream_t st = alloc.stream();
    ids.push_back(static_cast<std::int32_t>(params.context_len));  // the context length follows the table row
    cudaMemcpyAsync(base + tab_off, ids.data(), ids.size() * sizeof(std::int32_t), cudaMemcpyHostToDevice, st);
    a.block_tables = reinterpret_cast<const std::int32_t*>(base + tab_off);
    a.context_lens = reinterpret_cast<const std::int32_t*>(base + tab_off) + (ids.size() - 1);
    if (!q_dev) {
        cudaMemcpyAsync(base + q_off, query, qo_bytes, cudaMemcpyHostToDevice, st);
        a.query = base + q_off;
    }
    a.out = o_dev ? out : static_cast<void*>(base + o_off);
    a.workspace = ws ? base + ws_off : nullptr;
    a.workspace_bytes = ws;
    if (qvp_decode(&a, st) != QVP_OK) return false;
    // One sequence per call: wait for it, so the caller's host buffers are
    // free to reuse on return. A host `out` is written only after success.
    if (cudaStreamSynchronize(st) != cudaSuccess) return false;
    if (!o_dev && cudaMemcpy(out, base + o_off, qo_bytes, cudaMemcpyDeviceToHost) != cudaSuccess) return false;
    return true;
}

}  // namespace detail

PagedDecodeBatch::PagedDecodeBatch(const MemoryAllocator& allocator, bool resident_tables)
    : allocator_(&allocator),
      resident_(resident_tables ? std::make_unique<ResidentBlockTables>(allocator) : nullptr) {}

PagedDecodeBatch::~PagedDecodeBatch() {
    OnDevice guard(allocator_->device());
    cudaStreamSynchronize(allocator_->stream());
    if (host_buf_ != nullptr) cudaFreeHost(host_buf_);
    if (dev_buf_ != nullptr) cudaFree(dev_buf_);
    if (workspace_ != nullptr) cudaFree(workspace_);
    if (error_word_ != nullptr) cudaFree(error_word_);
    if (upload_event_ != nullptr) cudaEventDestroy(static_cast<cudaEvent_t>(upload_event_));
}

bool PagedDecodeBatch::grow(std::size_t ints, std::size_t /*batch*/, std::size_t workspace) {
    if (upload_event_ == nullptr) {
        cudaEvent_t ev;
        if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return false;
        upload_event_ = ev;
    }
    if (error_word_ == nullptr) {
        if (cudaMalloc(reinterpret_cast<void**>(&error_word_), sizeof(std::int32_t)) != cudaSuccess) return false;
        cudaMemset(error_word_, 0, sizeof(std::int32_t));
    }
    if (ints > buf_ints_) {
        cudaStreamSynchronize(allocator_->stream());
        if (host_buf_ != nullptr) cudaFreeHost(host_buf_);
        if (dev_buf_ != nullptr) cudaFree(dev_buf_);
        host_buf_ = nullptr;
        dev_buf_ = nullptr;
        buf_ints_ = 0;
        const std::size_t n = std::max<std::size_t>(ints * 2, 4096);
        if (cudaMallocHost(reinterpret_cast<void**>(&host_buf_), n * sizeof(std::int32_t)) != cudaSuccess ||
            cudaMalloc(reinterpret_cast<void**>(&dev_buf_), n * sizeof(std::int32_t)) != cudaSuccess)
            return false;
        buf_ints_ = n;
    }
    if (workspace > workspace_bytes_) {
        cudaStreamSynchronize(allocator_->stream());
        if (workspace_ != nullptr) cudaFree(workspace_);
        workspace_ = nullptr;
        workspace_bytes_ = 0;
        if (cudaMalloc(&workspace_, workspace) != cudaSuccess) return false;
        workspace_bytes_ = workspace;
    }
    return true;
}

bool PagedDecodeBatch::run(const std::vector<CacheView>& views, const std::vector<std::uint32_t>& context_lens,
                           std::uint32_t layer, std::uint32_t num_query_heads, float scale, const void* query,
                           void* out) {
    status_ = QVP_ERR_INVALID;
    error_.clear();
    if (views.size() != context_lens.size() || query == nullptr || out == nullptr) {
        error_ = "views and context lengths differ in count, or a null buffer";
        return false;
    }
    const std::size_t B = views.size();
    if (B == 0) {
        status_ = QVP_OK;
        return true;
    }
    const std::size_t elem = allocator_->block_shape().bytes_per_element;
    const std::uint32_t tpb = allocator_->block_shape().tokens_per_block;
    std::uint32_t pitch = 1, max_ctx = 1;
    for (std::size_t b = 0; b < B; ++b) {
        if (views[b].allocator != allocator_ ||
            !arguments_fit(views[b], elem, layer, num_query_heads, context_lens[b])) {
            error_ = "sequence " + std::to_string(b) + " does not fit the cache shape";
            return false;
        }
        pitch = std::max<std::uint32_t>(pitch, (context_lens[b] + tpb - 1) / tpb);
        max_ctx = std::max(max_ctx, context_lens[b]);
    }
    MemoryAllocator& alloc = const_cast<MemoryAllocator&>(*allocator_);
    OnDevice guard(alloc.device());
    qvp_decode_args a = base_args(alloc, elem, layer, num_query_heads, scale);
    a.batch = static_cast<std::uint32_t>(B);
    if (resident_) return run_resident(views, context_lens, a, max_ctx, query, out);
    a.max_blocks_per_seq = pitch;
    a.max_context_len = max_ctx;
    a.block_tables = reinterpret_cast<const std::int32_t*>(0x10);
    a.context_lens = reinterpret_cast<const std::int32_t*>(0x10);
    a.query = query;
    a.out = out;
    std::size_t ws = 0;
    status_ = qvp_decode_workspace_size(&a, &ws);
    if (status_ != QVP_OK) {
        error_ = qvp_last_error();
        return false;
    }
    const std::size_t ints = B * pitch + B;
    if (!grow(ints, B, ws)) {
        status_ = QVP_ERR_NOMEM;
        error_ = "could not allocate decode buffers";
        return false;
    }
    // the previous step's upload must have left the pinned buffer
    if (!host_impl::wait_event(static_cast<cudaEvent_t>(upload_event_), "table upload", &error_)) {
        status_ = QVP_ERR_CUDA;
        return false;
    }
    for (std::size_t b = 0; b < B; ++b) {
        std::int32_t* row = host_buf_ + b * pitch;
        const std::uint32_t nblk = (context_lens[b] + tpb - 1) / tpb;
        if (!write_row(views[b], nblk, row)) {
            status_ = QVP_ERR_UNMAPPED;
            error_ = "sequence " + std::to_string(b) +
                     " has an unmapped or swapped-out block inside its context";
            return false;
        }
        std::fill(row + nblk, row + pitch, -1);
        host_buf_[B * pitch + b] = static_cast<std::int32_t>(context_lens[b]);
    }
    alloc.flush();  // queued copy-on-write copies and swap moves land first
    alloc.order_reads(host_buf_, B * pitch);  // swap-ins still filling a frame of the batch
    cudaStream_t st = alloc.stream();
    host_impl::upload_pinned(dev_buf_, host_buf_, ints * sizeof(std::int32_t), st);
    cudaEventRecord(static_cast<cudaEvent_t>(upload_event_), st);
    rows_uploaded_ = static_cast<std::uint32_t>(B);
    bytes_uploaded_ = ints * sizeof(std::int32_t);
    a.block_tables = dev_buf_;
    a.context_lens = dev_buf_ + B * pitch;
    a.workspace = ws ? workspace_ : nullptr;
    a.workspace_bytes = ws ? workspace_bytes_ : 0;
    a.error_word = error_word_;
    status_ = qvp_decode(&a, st);
    if (status_ != QVP_OK) error_ = qvp_last_error();
    return status_ == QVP_OK;
}

// run() with resident tables: the rows go up first (they fix the pitch the
// workspace size depends on), then copy-on-write copies, then the decode.
bool PagedDecodeBatch::run_resident(const std::vector<CacheView>& views, const std::vector<std::uint32_t>& context_lens,
                                    qvp_decode_args& a, std::uint32_t max_ctx, const void* query, void* out) {
    MemoryAllocator& alloc = const_cast<MemoryAllocator&>(*allocator_);
    if (!grow(0, views.size(), 0)) {
        status_ = QVP_ERR_NOMEM;
        error_ = "could not allocate decode buffers";
        return false;
    }
    if (!resident_->update(views, context_lens, error_word_, &error_)) {
        status_ = resident_->status();
        return false;
    }
    rows_uploaded_ = resident_->rows_written();
    bytes_uploaded_ = resident_->bytes_uploaded();
    a.max_blocks_per_seq = resident_->pitch();
    a.max_context_len = max_ctx;
    a.block_tables = resident_->device_tables();
    a.context_lens = resident_->device_context_lens();
    a.query = query;
    a.out = out;
    std::size_t ws = 0;
    status_ = qvp_decode_workspace_size(&a, &ws);
    if (status_ != QVP_OK) {
        error_ = qvp_last_error();
        return false;
    }
    if (!grow(0, views.size(), ws)) {
        status_ = QVP_ERR_NOMEM;
        error_ = "could not allocate decode workspace";
        return false;
    }
    alloc.flush();  // queued copy-on-write copies and swap moves land first
    if (alloc.loads_in_flight()) {
        // only then: the frames of the batch against swap-ins still landing
        std::vector<std::int32_t> frames;
        const std::uint32_t tpb = alloc.block_shape().tokens_per_block;
        for (std::size_t b = 0; b < views.size(); ++b) {
            const std::uint32_t nblk = (context_lens[b] + tpb - 1) / tpb;
            const std::size_t at = frames.size();
            frames.resize(at + nblk);
            if (!write_row(views[b], nblk, frames.data() + at)) frames.resize(at);
        }
        alloc.order_reads(frames.data(), frames.size());
    }
    a.workspace = ws ? workspace_ : nullptr;
    a.workspace_bytes = ws ? workspace_bytes_ : 0;
    a.error_word = error_word_;
    status_ = qvp_decode(&a, alloc.stream());
    if (status_ != QVP_OK) error_ = qvp_last_error();
    return status_ == QVP_OK;
}

int PagedDecodeBatch::device_error() {
    if (error_word_ == nullptr) return 0;
    OnDevice guard(allocator_->device());
    std::int32_t v = 0;
    cudaStreamSynchronize(allocator_->stream());
    cudaMemcpy(&v, error_word_, sizeof(v), cudaMemcpyDeviceToHost);
    return v;
}

}  // namespace qwenvl_paged
