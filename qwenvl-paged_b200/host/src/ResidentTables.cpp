#include "qwenvl_paged/ResidentTables.h"

#include "qvp.h"
#include "host_impl.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

namespace qwenvl_paged {

namespace {

std::size_t round4(std::size_t n) { return (n + 3) / 4 * 4; }

using host_impl::OnDevice;

}  // namespace

// ---- TableDeltaPlanner -----------------------------------------------------

TableDeltaPlanner::TableDeltaPlanner(std::uint32_t num_blocks) : num_blocks_(num_blocks) {}

void TableDeltaPlanner::invalidate() noexcept {
    for (Row& r : rows_) r = Row{};
}

// Row b of the shadow: entry i of the table lands in column logical.index
// when that index is inside the row (a table has at most size() usable
// leading entries, so the row is size() wide at most). `valid` counts the
// leading columns 0, 1, ... that hold a pool block: the blocks a context may
// cover, the same ones the per-step flatten accepts.
void TableDeltaPlanner::write_row(std::uint32_t b, const BlockTable& table) {
    std::int32_t* row = shadow_.data() + static_cast<std::size_t>(b) * pitch_;
    std::fill(row, row + pitch_, -1);
    std::uint32_t valid = 0;
    bool prefix = true;
    const std::vector<BlockTableEntry>& es = table.entries();
    for (std::size_t i = 0; i < es.size(); ++i) {
        const BlockTableEntry& e = es[i];
        const bool usable = !e.swap_slot.has_value() && e.physical_id < num_blocks_;
        if (e.logical.index < pitch_ && usable) row[e.logical.index] = static_cast<std::int32_t>(e.physical_id);
        // sorted and unique: entry i maps logical block i iff its index is i
        prefix = prefix && usable && e.logical.index == i;
        if (prefix) valid = static_cast<std::uint32_t>(i + 1);
    }
    rows_[b] = Row{&table, table.revision(), valid};
}

bool TableDeltaPlanner::plan(const std::vector<CacheView>& views, const std::vector<std::uint32_t>& context_lens,
                             std::string* why) {
    written_ = 0;
    relaid_ = false;
    packet_.clear();
    const std::size_t B = views.size();
    if (context_lens.size() != B) {
        if (why) *why = "views and context lengths differ in count";
        return false;
    }
    std::size_t need = 1;
    for (const CacheView& v : views) {
        if (v.block_table == nullptr) {
            if (why) *why = "a view without a block table";
            return false;
        }
        need = std::max(need, v.block_table->size());
    }
    if (need > pitch_) {
        // grow by half again so that steady growth re-lays the table rarely
        pitch_ = static_cast<std::uint32_t>(round4(std::max<std::size_t>(need, pitch_ + pitch_ / 2)));
        rows_.assign(B, Row{});
        relaid_ = true;
    }
    rows_.resize(B);
    batch_ = static_cast<std::uint32_t>(B);
    shadow_.resize(B * pitch_);

    std::vector<std::uint32_t> dirty;
    for (std::size_t b = 0; b < B; ++b) {
        const BlockTable* t = views[b].block_table;
        if (rows_[b].table != t || rows_[b].revision != t->revision()) {
            write_row(static_cast<std::uint32_t>(b), *t);
            dirty.push_back(static_cast<std::uint32_t>(b));
        }
    }
    for (std::size_t b = 0; b < B; ++b) {
        const std::uint32_t tpb = views[b].layout.shape.tokens_per_block;
        const std::uint64_t nblk = tpb == 0 ? ~0ull : (static_cast<std::uint64_t>(context_lens[b]) + tpb - 1) / tpb;
        if (context_lens[b] == 0 || nblk > rows_[b].valid) {
            if (why)
                *why = "sequence " + std::to_string(b) + " has an unmapped or swapped-out block inside its context";
            invalidate();
            return false;
        }
    }
    written_ = static_cast<std::uint32_t>(dirty.size());
    ctx_off_ = round4(written_);
    rows_off_ = ctx_off_ + round4(B);
    packet_.resize(rows_off_ + static_cast<std::size_t>(written_) * pitch_, -1);
    for (std::uint32_t i = 0; i < written_; ++i) {
        packet_[i] = static_cast<std::int32_t>(dirty[i]);
        std::memcpy(packet_.data() + rows_off_ + static_cast<std::size_t>(i) * pitch_,
                    shadow_.data() + static_cast<std::size_t>(dirty[i]) * pitch_, pitch_ * sizeof(std::int32_t));
    }
    for (std::size_t b = 0; b < B; ++b) packet_[ctx_off_ + b] = static_cast<std::int32_t>(context_lens[b]);
    return true;
}

// ---- ResidentBlockTables ---------------------------------------------------

ResidentBlockTables::ResidentBlockTables(const MemoryAllocator& allocator)
    : allocator_(&allocator), planner_(allocator.num_blocks()) {}

ResidentBlockTables::~ResidentBlockTables() {
    OnDevice guard(allocator_->device());
    cudaStreamSynchronize(allocator_->stream());
    if (table_ != nullptr) cudaFree(table_);
    if (packet_dev_ != nullptr) cudaFree(packet_dev_);
    if (packet_host_ != nullptr) cudaFreeHost(packet_host_);
    if (upload_event_ != nullptr) cudaEventDestroy(static_cast<cudaEvent_t>(upload_event_));
}

const std::int32_t* ResidentBlockTables::device_context_lens() const noexcept {
    return packet_dev_ == nullptr ? nullptr : packet_dev_ + planner_.context_offset();
}

// Grows the device table (keeping its rows when the pitch is unchanged) and
// the packet buffers. Synchronizes the stream before freeing anything.
bool ResidentBlockTables::reserve(std::size_t rows, std::uint32_t pitch, std::size_t packet_ints, std::string* why) {
    cudaStream_t st = allocator_->stream();
    if (upload_event_ == nullptr) {
        cudaEvent_t ev;
        if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
            if (why) *why = "could not create the upload event";
            return false;
        }
        upload_event_ = ev;
    }
    if (rows > rows_cap_ || pitch != table_pitch_) {
        const std::size_t cap = std::max<std::size_t>({rows, rows_cap_, 64});
        std::int32_t* t = nullptr;
        if (cudaMalloc(reinterpret_cast<void**>(&t), cap * pitch * sizeof(std::int32_t)) != cudaSuccess) {
            cudaGetLastError();
            if (why) *why = "could not allocate the device block table";
            return false;
        }
        if (table_ != nullptr && pitch == table_pitch_)
            cudaMemcpyAsync(t, table_, rows_cap_ * pitch * sizeof(std::int32_t), cudaMemcpyDeviceToDevice, st);
        cudaStreamSynchronize(st);
        if (table_ != nullptr) cudaFree(table_);
        table_ = t;
        rows_cap_ = cap;
        table_pitch_ = pitch;
    }
    if (packet_ints > packet_cap_) {
        cudaStreamSynchronize(st);
        if (packet_dev_ != nullptr) cudaFree(packet_dev_);
        if (packet_host_ != nullptr) cudaFreeHost(packet_host_);
        packet_dev_ = nullptr;
        packet_host_ = nullptr;
        packet_cap_ = 0;
        const std::size_t n = std::max<std::size_t>(packet_ints * 2, 4096);
        if (cudaMallocHost(reinterpret_cast<void**>(&packet_host_), n * sizeof(std::int32_t)) != cudaSuccess ||
            cudaMalloc(reinterpret_cast<void**>(&packet_dev_), n * sizeof(std::int32_t)) != cudaSuccess) {
            cudaGetLastError();
            if (why) *why = "could not allocate the table upload buffers";
            return false;
        }
        packet_cap_ = n;
    }
    return true;
}

bool ResidentBlockTables::update(const std::vector<CacheView>& views, const std::vector<std::uint32_t>& context_lens,
                                 std::int32_t* error_word, std::string* why) {
    uploaded_ = 0;
    status_ = QVP_ERR_INVALID;
    for (const CacheView& v : views) {
        if (v.allocator != allocator_) {
            if (why) *why = "a view of another allocator";
            return false;
        }
    }
    if (!planner_.plan(views, context_lens, why)) {
        status_ = QVP_ERR_UNMAPPED;
        return false;
    }
    OnDevice guard(allocator_->device());
    const std::vector<std::int32_t>& pk = planner_.packet();
    if (!reserve(planner_.batch(), planner_.pitch(), pk.size(), why)) {
        planner_.invalidate();
        status_ = QVP_ERR_NOMEM;
        return false;
    }
    cudaStream_t st = allocator_->stream();
    // the previous step's upload must have left the pinned buffer
    if (!host_impl::wait_event(static_cast<cudaEvent_t>(upload_event_), "resident table upload", why)) {
        planner_.invalidate();
        status_ = QVP_ERR_CUDA;
        return false;
    }
    std::memcpy(packet_host_, pk.data(), pk.size() * sizeof(std::int32_t));
    const std::size_t bytes = pk.size() * sizeof(std::int32_t);
    const std::uint32_t n = planner_.rows_written();
    const std::size_t row_bytes = static_cast<std::size_t>(planner_.pitch()) * sizeof(std::int32_t);
    int status = host_impl::upload_pinned(packet_dev_, packet_host_, bytes, st) ? QVP_OK : QVP_ERR_CUDA;
    cudaEventRecord(static_cast<cudaEvent_t>(upload_event_), st);
    // qvp_scatter_blocks takes at most 65535 rows per launch
    for (std::uint32_t first = 0; status == QVP_OK && first < n; first += 65535u) {
        const std::uint32_t count = std::min<std::uint32_t>(65535u, n - first);
        status = qvp_scatter_blocks(table_, row_bytes, static_cast<std::uint32_t>(rows_cap_), row_bytes,
                                    packet_dev_ + first, count,
                                    packet_dev_ + planner_.rows_offset() + static_cast<std::size_t>(first) * planner_.pitch(),
                                    error_word, st);
    }
    if (status != QVP_OK) {
        cudaGetLastError();
        planner_.invalidate();
        if (why) *why = std::string("table upload: ") + qvp_last_error();
        status_ = QVP_ERR_CUDA;
        return false;
    }
    uploaded_ = bytes;
    status_ = QVP_OK;
    return true;
}

}  // namespace qwenvl_paged
