#include "qwenvl_paged/CacheLayout.h"

namespace qwenvl_paged {

std::size_t KVBlockLayout::head_stride() const noexcept { return shape.head_dim; }
std::size_t KVBlockLayout::token_stride() const noexcept { return head_stride() * shape.num_kv_heads; }
std::size_t KVBlockLayout::stream_stride() const noexcept { return token_stride() * shape.tokens_per_block; }
std::size_t KVBlockLayout::layer_stride() const noexcept { return stream_stride() * kKVStreamCount; }
std::size_t KVBlockLayout::element_count() const noexcept { return layer_stride() * shape.num_layers; }

std::optional<std::size_t> KVBlockLayout::element_offset(std::uint32_t layer, KVStream stream,
                                                         std::uint32_t token_in_block,
                                                         std::uint32_t kv_head) const noexcept {
    const bool inside = layer < shape.num_layers && token_in_block < shape.tokens_per_block &&
                        kv_head < shape.num_kv_heads;
    if (!inside) return std::nullopt;
    const std::size_t s = stream == KVStream::Value ? 1u : 0u;
    return layer * layer_stride() + s * stream_stride() + token_in_block * token_stride() + kv_head * head_stride();
}

}  // namespace qwenvl_paged
