// Host-side internals shared by the qvp translation units: error text,
// CUDA status checks, the decode plan.
#pragma once

#include "qvp.h"

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
// Launches the decode `plan` (from plan_decode on the same arguments, batch
// > 0) after checking the caller's workspace against it.
int run_decode(const qvp_decode_args& a, const DecodePlan& plan, cudaStream_t st);

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

}  // namespace qvp
