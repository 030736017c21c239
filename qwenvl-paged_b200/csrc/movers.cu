// Block movers: batched copy-on-write copies, swap gather/scatter and the
// per-step KV append. All are HBM-bound byte moves: 16-byte vector loads and
// stores, several in flight per thread, grids sized in multiples of the SM
// count. None of them reshapes the work into GEMMs.
//
// Reference operations whose bytes these kernels move
// (phhuang191129/QwenVL-Paged):
//   copy:    MemoryAllocator::copy_block, src/MemoryAllocator.cpp:76-85
//   gather:  HostSwapBackend::store,      src/SwapBackend.cpp:10-23
//   scatter: HostSwapBackend::load,       src/SwapBackend.cpp:25-39
//   append:  the per-token cache writes of tests/PagedAttention.test.cpp:97-127
#include "qvp_device.cuh"
#include "qvp_internal.h"

namespace qvp {

namespace {

constexpr int kMoverThreads = 256;
constexpr int kUnroll = 4;
constexpr size_t kChunkBytes = static_cast<size_t>(kMoverThreads) * kUnroll * 16;  // 16 KiB per CTA step

// Copies `bytes` from src to dst inside one CTA, 16-byte vectors when both
// pointers and the length allow it.
__device__ __forceinline__ void cta_copy(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, size_t bytes,
                                         bool vec) {
    if (vec) {
        const uint4* s = reinterpret_cast<const uint4*>(src);
        uint4* d = reinterpret_cast<uint4*>(dst);
        const size_t n = bytes / 16;
        size_t i = threadIdx.x;
        for (; i + (kUnroll - 1) * kMoverThreads < n; i += kUnroll * kMoverThreads) {
            uint4 r[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) r[u] = __ldcs(s + i + u * kMoverThreads);
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) __stcs(d + i + u * kMoverThreads, r[u]);
        }
        for (; i < n; i += kMoverThreads) __stcs(d + i, __ldcs(s + i));
    } else {
        for (size_t i = threadIdx.x; i < bytes; i += kMoverThreads) dst[i] = src[i];
    }
}

// grid.x = chunks per block, grid.y = block pairs
__global__ void __launch_bounds__(kMoverThreads) copy_blocks_kernel(uint8_t* pool, size_t stride, uint32_t num_blocks,
                                                                    size_t bytes, const int32_t* pairs,
                                                                    int32_t* err, bool vec) {
    const int32_t src = pairs[2 * blockIdx.y];
    const int32_t dst = pairs[2 * blockIdx.y + 1];
    if (static_cast<uint32_t>(src) >= num_blocks || static_cast<uint32_t>(dst) >= num_blocks) {
        if (threadIdx.x == 0 && blockIdx.x == 0) record_error(err, kErrBadBlockId);
        return;
    }
    const size_t off = static_cast<size_t>(blockIdx.x) * kChunkBytes;
    if (off >= bytes) return;
    const size_t len = min(kChunkBytes, bytes - off);
    cta_copy(pool + static_cast<size_t>(dst) * stride + off, pool + static_cast<size_t>(src) * stride + off, len, vec);
}

// to_staging: pool block ids[i] -> staging + i*bytes; otherwise the reverse.
__global__ void __launch_bounds__(kMoverThreads) move_blocks_kernel(uint8_t* pool, size_t stride, uint32_t num_blocks,
                                                                    size_t bytes, const int32_t* ids,
                                                                    uint8_t* staging, int32_t* err, bool vec,
                                                                    bool to_staging) {
    const int32_t id = ids[blockIdx.y];
    if (static_cast<uint32_t>(id) >= num_blocks) {
        if (threadIdx.x == 0 && blockIdx.x == 0) record_error(err, kErrBadBlockId);
        return;
    }
    const size_t off = static_cast<size_t>(blockIdx.x) * kChunkBytes;
    if (off >= bytes) return;
    const size_t len = min(kChunkBytes, bytes - off);
    uint8_t* blk = pool + static_cast<size_t>(id) * stride + off;
    uint8_t* stg = staging + static_cast<size_t>(blockIdx.y) * bytes + off;
    if (to_staging)
        cta_copy(stg, blk, len, vec);
    else
        cta_copy(blk, stg, len, vec);
}

// One CTA per sequence: writes the K row and the V row of the new token.
__global__ void __launch_bounds__(kMoverThreads) kv_append_kernel(uint8_t* pool, size_t stride, uint32_t num_blocks,
                                                                  uint32_t tokens_per_block, size_t row_bytes,
                                                                  size_t stream_bytes, size_t layer_bytes,
                                                                  uint32_t pitch, const int32_t* tables,
                                                                  const int32_t* positions, const uint8_t* k,
                                                                  const uint8_t* v, int32_t* err, bool vec) {
    const int b = blockIdx.x;
    const int32_t pos = positions[b];
    if (pos < 0 || static_cast<uint32_t>(pos) / tokens_per_block >= pitch) {
        if (threadIdx.x == 0) record_error(err, kErrBadContext);
        return;
    }
    const int32_t id = tables[static_cast<size_t>(b) * pitch + pos / tokens_per_block];
    if (static_cast<uint32_t>(id) >= num_blocks) {
        if (threadIdx.x == 0) record_error(err, kErrBadBlockId);
        return;
    }
    uint8_t* kdst = pool + static_cast<size_t>(id) * stride + layer_bytes + (pos % tokens_per_block) * row_bytes;
    cta_copy(kdst, k + static_cast<size_t>(b) * row_bytes, row_bytes, vec);
    cta_copy(kdst + stream_bytes, v + static_cast<size_t>(b) * row_bytes, row_bytes, vec);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Device <- mapped pinned host memory by SM loads over PCIe.
__global__ void __launch_bounds__(kMoverThreads) fetch_host_kernel(uint8_t* __restrict__ dst,
                                                                   const uint8_t* __restrict__ src, size_t bytes,
                                                                   bool vec) {
    const size_t first = static_cast<size_t>(blockIdx.x) * kMoverThreads + threadIdx.x;
    const size_t step = static_cast<size_t>(gridDim.x) * kMoverThreads;
    if (vec) {
        const size_t nv = bytes / 16;
        for (size_t i = first; i < nv; i += step)
            reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
        for (size_t i = nv * 16 + first; i < bytes; i += step) dst[i] = src[i];
    } else {
        for (size_t i = first; i < bytes; i += step) dst[i] = src[i];
    }
}

}  // namespace

}  // namespace qvp

using namespace qvp;

extern "C" int qvp_copy_blocks(void* pool, size_t block_stride, uint32_t num_blocks, size_t bytes,
                               const int32_t* pairs, uint32_t n, int32_t* error_word, qvp_stream_t stream) {
    if (n == 0) return QVP_OK;
    if (pool == nullptr || pairs == nullptr) return fail(QVP_ERR_INVALID, "null pool or pair list");
    if (bytes > block_stride) return fail(QVP_ERR_INVALID, "copy of %zu bytes exceeds the block stride", bytes);
    if (n > 65535u) return fail(QVP_ERR_UNSUPPORTED, "more than 65535 copies in one call");
    if (bytes == 0) return QVP_OK;
    const bool vec = aligned16(pool) && block_stride % 16 == 0 && bytes % 16 == 0;
    dim3 grid(static_cast<unsigned>((bytes + kChunkBytes - 1) / kChunkBytes), n);
    copy_blocks_kernel<<<grid, kMoverThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<uint8_t*>(pool), block_stride, num_blocks, bytes, pairs, error_word, vec);
    return check_cuda(cudaGetLastError(), "launch copy_blocks");
}

static int launch_move(void* pool, size_t block_stride, uint32_t num_blocks, size_t bytes, const int32_t* ids,
                       uint32_t n, void* staging, int32_t* error_word, qvp_stream_t stream, bool to_staging) {
    if (n == 0) return QVP_OK;
    if (pool == nullptr || ids == nullptr || staging == nullptr)
        return fail(QVP_ERR_INVALID, "null pool, id list or staging buffer");
    if (bytes > block_stride) return fail(QVP_ERR_INVALID, "move of %zu bytes exceeds the block stride", bytes);
    if (n > 65535u) return fail(QVP_ERR_UNSUPPORTED, "more than 65535 blocks in one call");
    if (bytes == 0) return QVP_OK;
    const bool vec = aligned16(pool) && aligned16(staging) && block_stride % 16 == 0 && bytes % 16 == 0;
    dim3 grid(static_cast<unsigned>((bytes + kChunkBytes - 1) / kChunkBytes), n);
    move_blocks_kernel<<<grid, kMoverThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<uint8_t*>(pool), block_stride, num_blocks, bytes, ids, static_cast<uint8_t*>(staging),
        error_word, vec, to_staging);
    return check_cuda(cudaGetLastError(), to_staging ? "launch gather_blocks" : "launch scatter_blocks");
}

extern "C" int qvp_gather_blocks(const void* pool, size_t block_stride, uint32_t num_blocks, size_t bytes,
                                 const int32_t* ids, uint32_t n, void* staging, int32_t* error_word,
                                 qvp_stream_t stream) {
    return launch_move(const_cast<void*>(pool), block_stride, num_blocks, bytes, ids, n, staging, error_word,
                       stream, true);
}

extern "C" int qvp_scatter_blocks(void* pool, size_t block_stride, uint32_t num_blocks, size_t bytes,
                                  const int32_t* ids, uint32_t n, const void* staging, int32_t* error_word,
                                  qvp_stream_t stream) {
    return launch_move(pool, block_stride, num_blocks, bytes, ids, n, const_cast<void*>(staging), error_word,
                       stream, false);
}

extern "C" int qvp_fetch_host(void* dst, const void* src, size_t bytes, qvp_stream_t stream) {
    if (bytes == 0) return QVP_OK;
    if (dst == nullptr || src == nullptr) return fail(QVP_ERR_INVALID, "null destination or source");
    const bool vec = aligned16(dst) && aligned16(src);
    const size_t per_cta = static_cast<size_t>(kMoverThreads) * (vec ? 16 : 1) * 4;
    const size_t ctas = std::min<size_t>((bytes + per_cta - 1) / per_cta, 2 * 148);
    fetch_host_kernel<<<static_cast<unsigned>(ctas), kMoverThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<uint8_t*>(dst), static_cast<const uint8_t*>(src), bytes, vec);
    return check_cuda(cudaGetLastError(), "launch fetch_host");
}

extern "C" int qvp_kv_append(void* pool, size_t block_stride, uint32_t num_blocks, const qvp_block_shape* shape,
                             uint32_t layer, uint32_t batch, uint32_t max_blocks_per_seq,
                             const int32_t* block_tables, const int32_t* positions, const void* k,
                             const void* v, int32_t* error_word, qvp_stream_t stream) {
    if (shape == nullptr) return fail(QVP_ERR_INVALID, "null shape");
    if (batch == 0) return QVP_OK;
    if (pool == nullptr || block_tables == nullptr || positions == nullptr || k == nullptr || v == nullptr)
        return fail(QVP_ERR_INVALID, "null pool, table, position or K/V pointer");
    if (shape->tokens_per_block == 0 || shape->num_kv_heads == 0 || shape->head_dim == 0 ||
        shape->bytes_per_element == 0 || shape->num_layers == 0)
        return fail(QVP_ERR_INVALID, "block shape has a zero field");
    if (layer >= shape->num_layers) return fail(QVP_ERR_INVALID, "layer %u >= num_layers", layer);
    if (block_stride < qvp_block_bytes(shape)) return fail(QVP_ERR_INVALID, "block_stride below the block size");
    if (max_blocks_per_seq == 0) return fail(QVP_ERR_INVALID, "empty block table");
    const size_t row = static_cast<size_t>(shape->num_kv_heads) * shape->head_dim * shape->bytes_per_element;
    const size_t stream_bytes = row * shape->tokens_per_block;
    const size_t layer_bytes = stream_bytes * 2 * layer;
    const bool vec = aligned16(pool) && aligned16(k) && aligned16(v) && block_stride % 16 == 0 && row % 16 == 0;
    kv_append_kernel<<<batch, kMoverThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<uint8_t*>(pool), block_stride, num_blocks, shape->tokens_per_block, row, stream_bytes,
        layer_bytes, max_blocks_per_seq, block_tables, positions, static_cast<const uint8_t*>(k),
        static_cast<const uint8_t*>(v), error_word, vec);
    return check_cuda(cudaGetLastError(), "launch kv_append");
}
