// Element order inside a block: [layer][K|V][token_in_block][kv_head][head_dim],
// counted in elements. Same interface as the reference
// (include/qwenvl_paged/CacheLayout.h:14-79); the device kernels address
// blocks with exactly these strides.
#pragma once

#include "qwenvl_paged/Block.h"

#include <cstddef>
#include <cstdint>
#include <optional>

namespace qwenvl_paged {

enum class KVStream : std::uint8_t { Key, Value };

inline constexpr std::uint32_t kKVStreamCount = 2;

struct KVBlockLayout {
    BlockShape shape{};

    [[nodiscard]] std::size_t head_stride() const noexcept;
    [[nodiscard]] std::size_t token_stride() const noexcept;
    [[nodiscard]] std::size_t stream_stride() const noexcept;
    [[nodiscard]] std::size_t layer_stride() const noexcept;
    [[nodiscard]] std::size_t element_count() const noexcept;
    // Offset of one (layer, stream, token, head) vector; nullopt when any
    // coordinate is outside the shape.
    [[nodiscard]] std::optional<std::size_t> element_offset(std::uint32_t layer, KVStream stream,
                                                            std::uint32_t token_in_block,
                                                            std::uint32_t kv_head) const noexcept;
};

}  // namespace qwenvl_paged
