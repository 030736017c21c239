// Device-resident block tables for batched decode (not part of the reference
// interface; the reference resolves every token through BlockTable::lookup,
// include/qwenvl_paged/PagedAttention.h:77-89).
//
// An engine's decode batch is mostly the same sequences step after step, and
// a sequence's table changes only when it gains a block (every
// tokens_per_block steps), is copied on write, swapped, or replaced. So the
// int32 [batch][pitch] table the decode kernel reads stays on the device and
// a step rewrites only the rows whose table changed:
//
//   * row b belongs to batch position b and holds every mapped entry of
//     views[b]'s table (not only the blocks inside the context), so a context
//     that grows inside mapped blocks needs no table write;
//   * a row is rewritten when the view at position b is another table or its
//     BlockTable::revision() moved since the row was written;
//   * one upload packet [row ids | context lengths | rows] goes host->device
//     with one copy, and one qvp_scatter_blocks launch writes the rows (each
//     row is one pitch*4-byte "block" of the table).
//
// TableDeltaPlanner is the host half (no CUDA calls); ResidentBlockTables
// adds the device buffers and the upload.
#pragma once

#include "qwenvl_paged/KVCacheManager.h"

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

struct CUstream_st;

namespace qwenvl_paged {

class TableDeltaPlanner {
public:
    explicit TableDeltaPlanner(std::uint32_t num_blocks);

    // Plans one step for `views` with their context lengths. False when a
    // block of [0, context_lens[b]) is unmapped, swapped out or outside the
    // pool (the checks of the per-step flatten); the planner then forgets
    // every row so that the next plan rewrites the whole table.
    bool plan(const std::vector<CacheView>& views, const std::vector<std::uint32_t>& context_lens,
              std::string* why = nullptr);

    // Forget every row (after an upload that did not happen).
    void invalidate() noexcept;

    // Layout of the last plan's packet, in int32 units; each part starts on a
    // 16-byte boundary. ids[rows_written()], context_lens[batch()],
    // rows[rows_written()][pitch()].
    [[nodiscard]] const std::vector<std::int32_t>& packet() const noexcept { return packet_; }
    [[nodiscard]] std::size_t context_offset() const noexcept { return ctx_off_; }
    [[nodiscard]] std::size_t rows_offset() const noexcept { return rows_off_; }
    [[nodiscard]] std::uint32_t rows_written() const noexcept { return written_; }
    [[nodiscard]] std::uint32_t batch() const noexcept { return batch_; }
    [[nodiscard]] std::uint32_t pitch() const noexcept { return pitch_; }
    // True when the last plan changed the pitch: every row was rewritten and
    // the device table must be re-laid out.
    [[nodiscard]] bool relaid() const noexcept { return relaid_; }
    // Host copy of the device table after the last successful plan,
    // [batch()][pitch()], -1 where no usable block is mapped.
    [[nodiscard]] const std::vector<std::int32_t>& shadow() const noexcept { return shadow_; }

private:
    struct Row {
        const BlockTable* table{nullptr};
        TableStamp revision{};
        std::uint32_t valid{0};  // leading entries that resolve to a pool block
    };
    void write_row(std::uint32_t b, const BlockTable& table);

    std::uint32_t num_blocks_;
    std::vector<Row> rows_;
    std::vector<std::int32_t> shadow_;
    std::vector<std::int32_t> packet_;
    std::uint32_t pitch_{0};
    std::uint32_t batch_{0};
    std::uint32_t written_{0};
    std::size_t ctx_off_{0};
    std::size_t rows_off_{0};
    bool relaid_{false};
};

class ResidentBlockTables {
public:
    explicit ResidentBlockTables(const MemoryAllocator& allocator);
    ~ResidentBlockTables();
    ResidentBlockTables(const ResidentBlockTables&) = delete;
    ResidentBlockTables& operator=(const ResidentBlockTables&) = delete;

    // Brings the device tables and context lengths up to date for `views`,
    // enqueued on the allocator's stream. On false `why` says what failed and
    // status() is the qvp status (QVP_ERR_UNMAPPED for a block the context
    // cannot use, QVP_ERR_NOMEM, QVP_ERR_CUDA); the next update then rewrites
    // every row.
    bool update(const std::vector<CacheView>& views, const std::vector<std::uint32_t>& context_lens,
                std::int32_t* error_word, std::string* why);

    [[nodiscard]] const std::int32_t* device_tables() const noexcept { return table_; }
    [[nodiscard]] const std::int32_t* device_context_lens() const noexcept;
    [[nodiscard]] std::uint32_t pitch() const noexcept { return planner_.pitch(); }
    // Rows and bytes the last update sent to the device.
    [[nodiscard]] std::uint32_t rows_written() const noexcept { return planner_.rows_written(); }
    [[nodiscard]] std::size_t bytes_uploaded() const noexcept { return uploaded_; }
    [[nodiscard]] int status() const noexcept { return status_; }

private:
    bool reserve(std::size_t rows, std::uint32_t pitch, std::size_t packet_ints, std::string* why);

    const MemoryAllocator* allocator_;
    TableDeltaPlanner planner_;
    std::int32_t* table_{nullptr};      // device [rows_cap_][table_pitch_]
    std::size_t rows_cap_{0};
    std::uint32_t table_pitch_{0};
    std::int32_t* packet_host_{nullptr};  // pinned
    std::int32_t* packet_dev_{nullptr};
    std::size_t packet_cap_{0};
    void* upload_event_{nullptr};
    std::size_t uploaded_{0};
    int status_{0};
};

}  // namespace qwenvl_paged
