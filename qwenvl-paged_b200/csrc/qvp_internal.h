// Host-side internals shared by the qvp translation units: error text,
// CUDA status checks, the decode plan.
#pragma once

#include "qvp.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstddef>
#include <cstdint>

namespace qvp {

// Stores printf-style text as this thread's last error and returns `status`.
int fail(int status, const char* fmt, ...);
// Returns QVP_OK, or QVP_ERR_CUDA with `what` and the CUDA error text recorded.
int check_cuda(cudaError_t err, const char* what);

// Raises `func`'s dynamic shared-memory limit to `bytes` on the current
// device. The attribute belongs to a device, so `done` (one per kernel)
// records the devices already set (bit d for device d < 64; others are set
// on every call).
int set_smem_limit_once(std::atomic<std::uint64_t>& done, const void* func, int bytes, const char* what);

inline bool is_pow2(uint32_t v) { return v != 0 && (v & (v - 1)) == 0; }
inline size_t round_up(size_t v, size_t a) { return a == 0 ? v : (v + a - 1) / a * a; }
inline uint32_t ceil_div(uint32_t a, uint32_t b) { return (a + b - 1) / b; }

// What one qvp_decode call will launch.
struct DecodePlan {
    bool fast = false;          // TMA + tensor-core kernel (bf16, D 64/128, 16-token blocks)
    bool stream = false;        // persistent stream-K form of the fast kernel
    uint32_t grid_ctas = 0;     // stream: CTAs (one per SM)
    uint32_t nseg = 0;          // stream: (sequence, head group) segments
    size_t records = 0;         // stream: partial records in the workspace
    uint32_t group = 0;         // query heads per kv head (G)
    uint32_t heads_per_cta = 0; // kv heads one fast CTA owns (HH)
    uint32_t split_tokens = 0;  // tokens per split-K partition
    uint32_t max_splits = 0;    // partitions of the longest context
    size_t workspace_bytes = 0; // 0 when max_splits == 1
};

// Validates `a` and fills `plan`; returns a qvp_status.
int plan_decode(const qvp_decode_args& a, DecodePlan& plan);
// Where the stream decode kernel writes each output row: the same
// [batch][row_heads][head_dim] slice, at head offset head0, in each of n
// buffers (n > 1: this GPU's buffer and its peers' over NVLink, for kv-head
// shards whose outputs every GPU needs). A plain decode has n = 1, head0 = 0,
// row_heads = num_query_heads.
constexpr int kMaxOutTargets = 8;
struct OutTargets {
    __nv_bfloat16* ptr[kMaxOutTargets];
    uint32_t n;
    uint32_t head0;
    uint32_t row_heads;

#ifdef __CUDACC__
    // Row of query head h of sequence seq in buffer i.
    __device__ __forceinline__ __nv_bfloat16* row(uint32_t i, uint32_t seq, uint32_t h, uint32_t D) const {
        return ptr[i] + (static_cast<size_t>(seq) * row_heads + head0 + h) * D;
    }
#endif
};

// Launches the decode `plan` (from plan_decode on the same arguments, batch
// > 0) after checking the caller's workspace against it. `targets` (stream
// plans only) replaces args.out by several destination buffers.
int run_decode(const qvp_decode_args& a, const DecodePlan& plan, cudaStream_t st,
               const OutTargets* targets = nullptr);

int device_sm_count();

}  // namespace qvp

struct CUtensorMap_st;

namespace qvp {

// Encodes (and caches, per thread) the TMA view of a bf16 pool in which one
// box is the K and V slices of one block for `hh` consecutive kv heads, laid
// out in shared memory as [head_dim/64][hh][16 K rows, 16 V rows][64] with
// 128-byte swizzle. Needs unpadded blocks (stride == byte size).
int encode_pool_map(const void* pool, uint32_t num_blocks, const qvp_block_shape& shape, uint32_t hh,
                    CUtensorMap_st* map);
// The same map with a box of `rows` rows (16 = one K or V slice of a block,
// 32 = both) and `halves` 64-element halves of head_dim.
int encode_pool_map_box(const void* pool, uint32_t num_blocks, const qvp_block_shape& shape, uint32_t hh,
                        uint32_t rows, uint32_t halves, CUtensorMap_st* map);

}  // namespace qvp
