// Batched paged-decode attention for B200 (sm_100a).
//
// Computes, for every sequence of a batch and every query head, what the
// reference CPU kernel paged_attention_decode<T> computes for one sequence
// (phhuang191129/QwenVL-Paged include/qwenvl_paged/PagedAttention.h:53-127):
//   kv = h / G;  s_t = scale * <q_h, K_t>;  out_h = sum_t softmax(s)_t V_t
// with fp32 accumulation. The reference takes an exact max and then sums
// exp(s - max) (PagedAttention.h:98-118); here each partition keeps a running
// (max, sum, accumulator) and rescales when the max grows, which is the same
// value in exact arithmetic.
//
// Three kernels:
//  * paged_decode_stream (the default for bf16): the persistent stream-K form
//    of paged_decode_fast below, one CTA per SM over an even share of all
//    (sequence, head group, stage) work; the CTA that completes a segment
//    merges its partial records into the output.
//  * paged_decode_fast: the same tiles as a grid (sequence, partition, head
//    group), partitions merged by `combine_partitions`; used when a
//    partition size is given or a batch has more than 2048 segments.
//    bf16 K/V/Q, 16-token blocks, head_dim 64 or 128,
//    at most 16 query heads per kv head, unpadded blocks. One CTA owns
//    (sequence, partition, group of HH kv heads). A producer warp streams each
//    block's K and V slices for the CTA's heads into shared memory with TMA
//    tensor copies (128-byte swizzle, mbarrier completion, evict-first L2
//    hint); eight consumer warps each own one kv head and every J-th block and
//    run QK^T and PV as m16n8k16 bf16 tensor-core products with the GQA group
//    padded to 16 rows, so one K/V load serves the whole query group.
//  * paged_decode_generic: any element type, block size, head_dim <= 256 and
//    group size; one CTA per (sequence, partition, query head), four warps
//    striding over tokens, lanes over head_dim, exact expf.
#include "attention_tile.cuh"
#include "qvp_device.cuh"
#include "qvp_internal.h"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <chrono>
#include <cmath>
#include <cstring>

namespace qvp {

namespace {

constexpr int kFastComputeWarps = 8;
constexpr int kFastThreads = (kFastComputeWarps + 1) * 32;
constexpr int kGenericWarps = 4;
constexpr int kGenericMaxDimPerLane = 8;  // head_dim <= 256

struct FastParams {
    const int32_t* tables;
    const int32_t* ctx;
    const __nv_bfloat16* q;
    __nv_bfloat16* out;
    float* ws_o;
    float2* ws_ml;
    int32_t* err;
    uint32_t pitch;
    uint32_t num_blocks;
    uint32_t layer;
    uint32_t num_layers;
    uint32_t hq;
    uint32_t group;
    uint32_t split_blocks;
    uint32_t max_splits;
    float scale_log2;
};

template <int D, int HH, int STAGES>
struct FastShape {
    static constexpr int J = kFastComputeWarps / HH;     // blocks in flight per stage
    static constexpr uint32_t kBlock = 2 * HH * 16 * D * 2;  // K and V of one block, HH heads (one TMA box)
    static constexpr uint32_t kStage = J * kBlock;
    static constexpr uint32_t kSmem = STAGES * kStage + 1024 + 2 * STAGES * 8 + 16;
};

// Query rows g and g+8 of the group that reads kv head `kvh` of sequence
// `seq`, as m16n8k16 A fragments; rows >= G are zero.
template <int D>
__device__ __forceinline__ void load_query_fragments(uint32_t (&qa)[D / 16][4], const __nv_bfloat16* q, int seq,
                                                     uint32_t hq, int kvh, int G, int lane) {
    const int g = lane >> 2, c = lane & 3;
    const __nv_bfloat16* qb = q + (static_cast<size_t>(seq) * hq + static_cast<size_t>(kvh) * G) * D;
    const uint32_t* q_lo = reinterpret_cast<const uint32_t*>(qb + g * D);
    const uint32_t* q_hi = reinterpret_cast<const uint32_t*>(qb + (g + 8) * D);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
        const int k0 = (ks * 16 + c * 2) >> 1;
        qa[ks][0] = (g < G) ? __ldg(q_lo + k0) : 0u;
        qa[ks][1] = (g + 8 < G) ? __ldg(q_hi + k0) : 0u;
        qa[ks][2] = (g < G) ? __ldg(q_lo + k0 + 4) : 0u;
        qa[ks][3] = (g + 8 < G) ? __ldg(q_hi + k0 + 4) : 0u;
    }
}

// One 16-token block of one kv head: S = Q K^T on tensor cores, masked to the
// `valid` leading tokens, online-softmax update, O += P V. `blk` is the
// shared-memory box of the block, [head_dim/64][HH][K 16 | V 16 tokens][64]
// (one TMA copy), so the K rows of (dh, head) are row group 2*(dh*HH+head)
// and its V rows the next one; `row_head` picks the head.
template <int D, int HH>
__device__ __forceinline__ void attend_block(WarpState<D>& st, const uint32_t (&qa)[D / 16][4], uint32_t blk,
                                             int row_head, int valid, float scale_log2, int lane) {
    const int c = lane & 3;
    const int mi = lane >> 3;
    const int li = lane & 7;
    float s[2][4];
#pragma unroll
    for (int a = 0; a < 2; ++a) s[a][0] = s[a][1] = s[a][2] = s[a][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
        const int dh = ks >> 2;
        const int chunk = ((ks & 3) << 1) + (mi & 1);
        const int t = ((mi >> 1) << 3) + li;
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4(box_addr(blk, (dh * HH + row_head) * 2, t, chunk), r0, r1, r2, r3);
        mma_bf16_16816(s[0], qa[ks], r0, r1);
        mma_bf16_16816(s[1], qa[ks], r2, r3);
    }
    // scale into the log2 domain and mask tokens past the context
#pragma unroll
    for (int a = 0; a < 2; ++a) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int tok = a * 8 + c * 2 + (e & 1);
            const float v = s[a][e] * scale_log2;
            s[a][e] = (tok < valid) ? v : -INFINITY;
        }
    }
    float r_lo = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
    float r_hi = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
    r_lo = fmaxf(r_lo, __shfl_xor_sync(0xffffffffu, r_lo, 1));
    r_lo = fmaxf(r_lo, __shfl_xor_sync(0xffffffffu, r_lo, 2));
    r_hi = fmaxf(r_hi, __shfl_xor_sync(0xffffffffu, r_hi, 1));
    r_hi = fmaxf(r_hi, __shfl_xor_sync(0xffffffffu, r_hi, 2));
    const float mn0 = fmaxf(st.m0, r_lo);
    const float mn1 = fmaxf(st.m1, r_hi);
    const float corr0 = exp2f(st.m0 - mn0);
    const float corr1 = exp2f(st.m1 - mn1);
    st.m0 = mn0;
    st.m1 = mn1;
#pragma unroll
    for (int a = 0; a < 2; ++a) {
        s[a][0] = exp2f(s[a][0] - mn0);
        s[a][1] = exp2f(s[a][1] - mn0);
        s[a][2] = exp2f(s[a][2] - mn1);
        s[a][3] = exp2f(s[a][3] - mn1);
    }
    st.l0 = st.l0 * corr0 + (s[0][0] + s[0][1] + s[1][0] + s[1][1]);
    st.l1 = st.l1 * corr1 + (s[0][2] + s[0][3] + s[1][2] + s[1][3]);
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
        st.o[n][0] *= corr0;
        st.o[n][1] *= corr0;
        st.o[n][2] *= corr1;
        st.o[n][3] *= corr1;
    }
    const uint32_t pa[4] = {pack_bf16x2(s[0][0], s[0][1]), pack_bf16x2(s[0][2], s[0][3]),
                            pack_bf16x2(s[1][0], s[1][1]), pack_bf16x2(s[1][2], s[1][3])};
#pragma unroll
    for (int np = 0; np < D / 16; ++np) {
        const int dh = np >> 2;
        const int chunk = ((np & 3) << 1) + (mi >> 1);
        const int t = ((mi & 1) << 3) + li;
        uint32_t v0, v1, v2, v3;
        ldmatrix_x4_trans(box_addr(blk, (dh * HH + row_head) * 2 + 1, t, chunk), v0, v1, v2, v3);
        if (valid < 16) {
            // V slots past the context may hold anything (even NaN); zero them
            // so the zero weights cannot turn them into NaN.
            v0 = mask_pair(v0, c * 2, valid);
            v2 = mask_pair(v2, c * 2, valid);
            v1 = mask_pair(v1, 8 + c * 2, valid);
            v3 = mask_pair(v3, 8 + c * 2, valid);
        }
        mma_bf16_16816(st.o[2 * np], pa, v0, v1);
        mma_bf16_16816(st.o[2 * np + 1], pa, v2, v3);
    }
}

template <int D, int HH, int STAGES>
__global__ void __launch_bounds__(kFastThreads, 1)
    paged_decode_fast(const __grid_constant__ CUtensorMap tmap, const FastParams p) {
    using S = FastShape<D, HH, STAGES>;
    constexpr int J = S::J;
    constexpr int KS = D / 16;  // k-steps of QK^T
    constexpr int NT = D / 8;   // n-tiles of the output

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStage);

    const int seq = blockIdx.z;
    const int hg = blockIdx.y;
    const uint32_t split = blockIdx.x;
    const int ctx = p.ctx[seq];
    if (ctx <= 0 || static_cast<uint32_t>(ctx) > p.pitch * 16u) {
        if (threadIdx.x == 0 && split == 0 && hg == 0) record_error(p.err, kErrBadContext);
        return;
    }
    const uint32_t nblk_total = (static_cast<uint32_t>(ctx) + 15u) / 16u;
    const uint32_t nsplits = (nblk_total + p.split_blocks - 1) / p.split_blocks;
    if (nsplits > p.max_splits) {
        if (threadIdx.x == 0 && split == 0 && hg == 0) record_error(p.err, kErrBadContext);
        return;
    }
    const uint32_t b0 = split * p.split_blocks;
    if (b0 >= nblk_total) return;
    const uint32_t b1 = min(b0 + p.split_blocks, nblk_total);
    const uint32_t nblk = b1 - b0;
    const uint32_t iters = (nblk + J - 1) / J;

    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + STAGES);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, kFastComputeWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kFastComputeWarps) {
        // Producer: one elected lane streams K and V slices of each block.
        if (lane == 0) {
            prefetch_tensormap(&tmap);
            const uint64_t policy = l2_policy_evict_first();
            const int32_t* row = p.tables + static_cast<size_t>(seq) * p.pitch;
            for (uint32_t it = 0; it < iters; ++it) {
                const uint32_t slot = it % STAGES;
                if (it >= STAGES &&
                    !mbar_wait_bounded(empty0 + 8 * slot, ((it / STAGES) - 1) & 1u)) {
                    record_error(p.err, kErrWaitTimeout);
                    break;
                }
                const uint32_t nb = min(static_cast<uint32_t>(J), nblk - it * J);
                mbar_arrive_expect_tx(full0 + 8 * slot, nb * S::kBlock);
                const uint32_t dst = smem_u32(smem + slot * S::kStage);
                for (uint32_t j = 0; j < nb; ++j) {
                    int32_t id = row[b0 + it * J + j];
                    if (static_cast<uint32_t>(id) >= p.num_blocks) {
                        record_error(p.err, kErrBadBlockId);
                        id = 0;
                    }
                    const int r = (id * static_cast<int>(p.num_layers) + static_cast<int>(p.layer)) * 32;
                    tma_load_4d(dst + j * S::kBlock, &tmap, full0 + 8 * slot, 0, r, hg * HH, 0, policy);
                }
            }
        }
        return;
    }

    // Consumers: warp (hh, j) owns kv head hg*HH+hh and blocks j, j+J, ...
    const int hh = warp % HH;
    const int j = warp / HH;
    const int kvh = hg * HH + hh;
    const int g = lane >> 2;
    const int c = lane & 3;
    const int G = static_cast<int>(p.group);

    uint32_t qa[KS][4];
    load_query_fragments<D>(qa, p.q, seq, p.hq, kvh, G, lane);
    WarpState<D> st;
    st.reset();
    bool alive = true;

    for (uint32_t it = 0; it < iters && alive; ++it) {
        const uint32_t slot = it % STAGES;
        if (!mbar_wait_bounded(full0 + 8 * slot, (it / STAGES) & 1u)) {
            record_error(p.err, kErrWaitTimeout);
            alive = false;
            break;
        }
        const uint32_t lb = b0 + it * J + j;
        if (lb < b1) {
            const int valid = min(16, ctx - static_cast<int>(lb) * 16);
            const uint32_t kb = smem_u32(smem + slot * S::kStage + j * S::kBlock);
            attend_block<D, HH>(st, qa, kb, hh, valid, p.scale_log2, lane);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * slot);
    }
    float m0 = st.m0, m1 = st.m1, l0 = st.l0, l1 = st.l1;
    auto& o = st.o;

    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

    // Merge the J warps that share a kv head through shared memory (the stage
    // buffers are free once every consumer has passed the barrier).
    if constexpr (J > 1) {
        named_barrier(1, kFastComputeWarps * 32);
        float* scratch = reinterpret_cast<float*>(smem);
        constexpr int kSlot = 16 * D + 32;
        if (j > 0) {
            float* w = scratch + (hh * J + j) * kSlot;
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const int col = n * 8 + c * 2;
                *reinterpret_cast<float2*>(w + g * D + col) = make_float2(o[n][0], o[n][1]);
                *reinterpret_cast<float2*>(w + (g + 8) * D + col) = make_float2(o[n][2], o[n][3]);
            }
            if (c == 0) {
                w[16 * D + g] = m0;
                w[16 * D + g + 8] = m1;
                w[16 * D + 16 + g] = l0;
                w[16 * D + 16 + g + 8] = l1;
            }
        }
        named_barrier(1, kFastComputeWarps * 32);
        if (j == 0) {
            for (int jj = 1; jj < J; ++jj) {
                const float* w = scratch + (hh * J + jj) * kSlot;
                const float mj0 = w[16 * D + g], mj1 = w[16 * D + g + 8];
                const float lj0 = w[16 * D + 16 + g], lj1 = w[16 * D + 16 + g + 8];
                const float M0 = fmaxf(m0, mj0), M1 = fmaxf(m1, mj1);
                const float a0 = exp2f(m0 - M0), a1 = exp2f(m1 - M1);
                const float e0 = (mj0 == -INFINITY) ? 0.f : exp2f(mj0 - M0);
                const float e1 = (mj1 == -INFINITY) ? 0.f : exp2f(mj1 - M1);
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    // keep the loads next to their use (a full hoist would
                    // hold 2 * NT more registers than the kernel has)
                    asm volatile("" ::: "memory");
                    const int col = n * 8 + c * 2;
                    const float2 lo = *reinterpret_cast<const float2*>(w + g * D + col);
                    const float2 hi = *reinterpret_cast<const float2*>(w + (g + 8) * D + col);
                    o[n][0] = o[n][0] * a0 + lo.x * e0;
                    o[n][1] = o[n][1] * a0 + lo.y * e0;
                    o[n][2] = o[n][2] * a1 + hi.x * e1;
                    o[n][3] = o[n][3] * a1 + hi.y * e1;
                }
                l0 = l0 * a0 + lj0 * e0;
                l1 = l1 * a1 + lj1 * e1;
                m0 = M0;
                m1 = M1;
            }
        }
    }
    if (j != 0 || !alive) return;

    if (nsplits == 1) {
        const float inv0 = 1.f / l0, inv1 = 1.f / l1;
        __nv_bfloat16* ob = p.out + (static_cast<size_t>(seq) * p.hq + static_cast<size_t>(kvh) * G) * D;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const int col = n * 8 + c * 2;
            if (g < G)
                *reinterpret_cast<uint32_t*>(ob + g * D + col) = pack_bf16x2(o[n][0] * inv0, o[n][1] * inv0);
            if (g + 8 < G)
                *reinterpret_cast<uint32_t*>(ob + (g + 8) * D + col) =
                    pack_bf16x2(o[n][2] * inv1, o[n][3] * inv1);
        }
    } else {
        const size_t part = (static_cast<size_t>(seq) * p.max_splits + split) * p.hq + static_cast<size_t>(kvh) * G;
        float* wo = p.ws_o + part * D;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const int col = n * 8 + c * 2;
            if (g < G) *reinterpret_cast<float2*>(wo + g * D + col) = make_float2(o[n][0], o[n][1]);
            if (g + 8 < G) *reinterpret_cast<float2*>(wo + (g + 8) * D + col) = make_float2(o[n][2], o[n][3]);
        }
        if (c == 0) {
            if (g < G) p.ws_ml[part + g] = make_float2(m0, l0);
            if (g + 8 < G) p.ws_ml[part + g + 8] = make_float2(m1, l1);
        }
    }
}

// ---------------------------------------------------------------------------
// Persistent stream-K variant of the fast kernel.
//
// A "segment" is one (sequence, head group) pair; its blocks are cut into
// stages of J blocks (the last stage of a segment may be short). All stages of
// all segments, in sequence order, form one stream that is split evenly over
// a grid of one CTA per SM: CTA c owns stages [c*S/grid, (c+1)*S/grid).
//
// A CTA's range holds at most two "shared" pieces (the segment it starts
// inside, shared with the CTAs before it, and the one it ends inside, shared
// with the CTAs after it) and any number of segments wholly its own. It
// streams the shared pieces first (the one at its end, then the one at its
// start) and its own segments after them, so every segment split between
// CTAs has all its pieces done early in the kernel, and the kernel ends on
// segments that need no merging. At the end of each piece the J warp columns
// that share a kv head are combined in shared memory (a tree of log2 J
// rounds); a segment wholly inside the CTA then writes its output directly,
// while a shared piece writes one partial record per kv head at index
// (segment + CTA) * HH + head (injective: segments and CTA ranges are both
// contiguous in stage order) and counts itself on the segment's arrival
// counter. The CTA whose piece completes the count merges the segment's
// records into the output right away (merge_records), while its producer warp
// keeps streaming. No CTA ever waits for another, so the kernel needs no
// co-resident grid. The counters live in the workspace, which may hold
// anything on entry: each holds (epoch << 32 | count), and a word from
// another epoch (another call) counts as zero.

constexpr int kStreamMaxSegments = 2048;

// Fixed work of a segment, in stages, for 1, 2 and 4 kv heads per CTA
// (per-CTA timings on cfg2-shaped batches: a piece's epilogue costs about
// four stages at 4 heads per CTA; these values minimised the step time).
constexpr uint32_t kSegmentCostStages[3] = {2u, 3u, 5u};

struct StreamParams {
    const int32_t* tables;
    const int32_t* ctx;
    const __nv_bfloat16* q;
    float* rec_acc;       // [records][G][D], records = (nseg + grid) * HH
    float2* rec_ml;       // [records][G]
    unsigned long long* seg_count;  // [nseg] arrival counters (epoch << 32 | pieces)
    OutTargets out;
    int32_t* err;
    uint32_t pitch;
    uint32_t num_blocks;
    uint32_t layer;
    uint32_t num_layers;
    uint32_t hq;
    uint32_t group;
    uint32_t head_groups;  // z = kv heads / HH
    uint32_t nseg;         // batch * z
    uint32_t epoch;        // differs between calls
    uint32_t seg_cost;     // fixed work of a segment, in stages (StreamSplit)
    float scale_log2;
};

// Floats of the per-CTA scratch that combines the J warp columns of a kv
// head (and later holds a merge's weights): HH * J / 2 states of G rows.
__host__ __device__ constexpr uint32_t stream_scratch_floats(uint32_t G, uint32_t D) {
    return 4u * (G * D + 2u * G);  // HH * J = 8 warps, half of them write per round
}

// Dynamic shared memory of the stream kernel: the pipeline (3 stages of
// 512 * head_dim bytes at head_dim 128, 6 at 64: 192 KiB either way, plus
// alignment slack and barriers), the segment prefix and the scratch.
constexpr uint32_t stream_pipeline_smem(uint32_t D) {
    return 196608u + 1024u + 2u * (D == 64 ? 6u : 3u) * 8u + 16u;
}
// 227 KB per block on sm_100, less 1 KB kept for the kernel's static shared
// memory (528 bytes)
constexpr uint32_t kMaxDynamicSmem = 232448u - 1024u;
constexpr size_t stream_smem_bytes(uint32_t nseg, uint32_t G, uint32_t D) {
    return stream_pipeline_smem(D) + (static_cast<size_t>(nseg) + 1u) * 4u + 16u +
           static_cast<size_t>(stream_scratch_floats(G, D)) * 4u;
}

__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Largest sigma in [0, nseg) with prefix[sigma] <= x (prefix non-decreasing).
__device__ __forceinline__ int find_segment(const int32_t* prefix, int nseg, uint32_t x) {
    int lo = 0, hi = nseg - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (static_cast<uint32_t>(prefix[mid]) <= x)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

// How the stage stream is cut into CTA ranges. Every segment costs its
// stages plus `b` stage-equivalents of fixed work (its epilogue and, for a
// piece shared between CTAs, the records and the merge), placed before its
// stages; the total cost C is split evenly, so a CTA whose range holds more
// segment starts gets fewer stages. Stage x of segment sg sits at cost
// x + b * (sg + 1).
struct StreamSplit {
    const int32_t* prefix;  // [nseg + 1] stage prefix (shared memory)
    int nseg;
    uint32_t total, grid, b;
    uint64_t cost;

    // First stage at or after cost position y.
    __device__ uint32_t stage_at(uint64_t y) const {
        if (y >= cost) return total;
        int lo = 0, hi = nseg - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (static_cast<uint64_t>(prefix[mid]) + static_cast<uint64_t>(b) * mid <= y)
                lo = mid;
            else
                hi = mid - 1;
        }
        const uint64_t seg0 = static_cast<uint64_t>(prefix[lo]) + static_cast<uint64_t>(b) * lo + b;
        const uint64_t x = static_cast<uint64_t>(prefix[lo]) + (y > seg0 ? y - seg0 : 0);
        return static_cast<uint32_t>(min(x, static_cast<uint64_t>(prefix[lo + 1])));
    }
    __device__ uint32_t begin(uint32_t c) const { return stage_at(static_cast<uint64_t>(c) * cost / grid); }
    __device__ bool empty(uint32_t c) const { return begin(c) == begin(c + 1); }
    // The CTA whose range holds stage x of segment sg.
    __device__ uint32_t cta_of(uint32_t x, int sg) const {
        const uint64_t y = x + static_cast<uint64_t>(b) * (sg + 1);
        return static_cast<uint32_t>(((y + 1) * grid - 1) / cost);
    }
    // First and last CTA holding a piece of (non-empty) segment sg.
    __device__ void pieces(int sg, uint32_t& cf, uint32_t& cl) const {
        cf = cta_of(static_cast<uint32_t>(prefix[sg]), sg);
        cl = cta_of(static_cast<uint32_t>(prefix[sg + 1]) - 1u, sg);
    }
    // Whether some CTA may get an empty range (its share of the cost is no
    // larger than one segment's fixed cost).
    __device__ bool may_have_empty() const { return cost <= static_cast<uint64_t>(grid) * (b + 1); }
};

// Counts one finished piece of a segment on its arrival counter; true for the
// arrival that completes `expected`. A word whose epoch is not `epoch` (left
// by another call, or never written) counts as zero pieces.
__device__ __forceinline__ bool arrive_last(unsigned long long* counter, uint32_t epoch, uint32_t expected) {
    unsigned long long old = *reinterpret_cast<volatile unsigned long long*>(counter);
    uint32_t done;
    while (true) {
        const uint32_t prev = (static_cast<uint32_t>(old >> 32) == epoch) ? static_cast<uint32_t>(old) : 0u;
        done = prev + 1u;
        const unsigned long long want = (static_cast<unsigned long long>(epoch) << 32) | done;
        const unsigned long long seen = atomicCAS(counter, old, want);
        if (seen == old) break;
        old = seen;
    }
    return done == expected;
}

// The pieces of one CTA's stage range [x0, x1), in the order it streams
// them: the shared piece at its end, the shared piece at its start, then the
// segments wholly inside the range (empty segments are skipped by callers).
struct PieceOrder {
    int first, last;
    uint32_t x0, x1;
    bool head_shared, tail_shared;
    int nshared, count;

    __device__ PieceOrder(const int32_t* prefix, int nseg, uint32_t lo, uint32_t hi) : x0(lo), x1(hi) {
        first = find_segment(prefix, nseg, lo);
        last = find_segment(prefix, nseg, hi - 1);
        head_shared = static_cast<uint32_t>(prefix[first]) < lo;
        tail_shared = static_cast<uint32_t>(prefix[last + 1]) > hi;
        if (first == last) {
            nshared = 0;
            count = 1;
        } else {
            nshared = (tail_shared ? 1 : 0) + (head_shared ? 1 : 0);
            count = last - first + 1;
        }
    }

    // Segment, stage range [b, e) and whether the segment lies wholly in
    // this CTA, for piece i < count.
    __device__ void at(const int32_t* prefix, int i, int& sg, uint32_t& b, uint32_t& e, bool& whole) const {
        if (first == last) {
            sg = first;
            b = x0;
            e = x1;
            whole = !head_shared && !tail_shared;
            return;
        }
        if (i < nshared) {
            if (tail_shared && i == 0) {
                sg = last;
                b = static_cast<uint32_t>(prefix[last]);
                e = x1;
            } else {
                sg = first;
                b = x0;
                e = static_cast<uint32_t>(prefix[first + 1]);
            }
            whole = false;
            return;
        }
        sg = first + (head_shared ? 1 : 0) + (i - nshared);
        b = static_cast<uint32_t>(prefix[sg]);
        e = static_cast<uint32_t>(prefix[sg + 1]);
        whole = true;
    }
};

// Merges the partial records of segment `sg` (HH kv heads of G rows; one
// record per head per piece) into the output. Run by the kFastComputeWarps
// consumer warps (tid < 256) of the CTA whose piece completed the segment.
// Pieces are the non-empty CTAs cf..cl. Per chunk of `chunk` pieces: (A)
// every (piece, row) max and sum into shared memory in one parallel pass,
// (B) per row the running max and sum; once all are in, (C) per chunk the
// normalised weights in place of the maxima, then each thread sums its OPT
// float4 outputs over the chunk, KU pieces' loads in flight at once. The
// order of summation depends on neither the merging CTA nor timing.
template <int D, int HH, int OPT>
__device__ __noinline__ void merge_records(const float* __restrict__ rec_acc, const float2* __restrict__ rec_ml,
                                              const OutTargets out, uint32_t group, uint32_t head_groups,
                                              int sg, uint32_t cf, uint32_t cl, StreamSplit split,
                                              float* s_wm, float* s_wl, int chunk, float* s_stat, int tid) {
    constexpr int D4 = D / 4;
    constexpr int kThreads = kFastComputeWarps * 32;
    constexpr int KU = OPT >= 8 ? 1 : 8 / OPT;
    const int G = static_cast<int>(group);
    const int R = HH * G;
    const int nparts = static_cast<int>(cl - cf + 1);
    const bool may_be_empty = split.may_have_empty();
    auto rec_of = [&](int k, int hh) { return (static_cast<size_t>(sg) + cf + static_cast<uint32_t>(k)) * HH + hh; };
    auto usable = [&](int k) { return !may_be_empty || !split.empty(cf + static_cast<uint32_t>(k)); };
    auto load_stats = [&](int k0, int nk) {
        for (int i = tid; i < nk * R; i += kThreads) {
            const int kk = i / R, rr = i % R;
            float2 ml = make_float2(-INFINITY, 0.f);
            if (usable(k0 + kk)) ml = __ldcg(&rec_ml[rec_of(k0 + kk, rr / G) * G + rr % G]);
            s_wm[i] = ml.x;
            s_wl[i] = ml.y;
        }
    };
    float* s_max = s_stat;
    float* s_inv = s_stat + 64;

    float run_m = -INFINITY, run_l = 0.f;  // thread rr < R
    for (int k0 = 0; k0 < nparts; k0 += chunk) {
        const int nk = min(chunk, nparts - k0);
        load_stats(k0, nk);
        named_barrier(1, kThreads);
        if (tid < R) {
            for (int kk = 0; kk < nk; ++kk) {
                const float mk = s_wm[kk * R + tid];
                if (mk == -INFINITY) continue;
                const float mn = fmaxf(run_m, mk);
                run_l = run_l * exp2f(run_m - mn) + s_wl[kk * R + tid] * exp2f(mk - mn);
                run_m = mn;
            }
        }
        named_barrier(1, kThreads);
    }
    if (tid < R) {
        s_max[tid] = run_m;
        s_inv[tid] = 1.f / run_l;
    }
    named_barrier(1, kThreads);

    const int nout = R * D4;
    float4 acc[OPT];
#pragma unroll
    for (int i = 0; i < OPT; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k0 = 0; k0 < nparts; k0 += chunk) {
        const int nk = min(chunk, nparts - k0);
        if (nparts > chunk) {  // otherwise the only chunk's stats are still in shared memory
            load_stats(k0, nk);
            named_barrier(1, kThreads);
        }
        for (int i = tid; i < nk * R; i += kThreads) {
            const float mk = s_wm[i];
            const int rr = i % R;
            s_wm[i] = mk == -INFINITY ? 0.f : exp2f(mk - s_max[rr]) * s_inv[rr];
        }
        named_barrier(1, kThreads);
        for (int kk0 = 0; kk0 < nk; kk0 += KU) {
            float4 v[KU][OPT];
#pragma unroll
            for (int u = 0; u < KU; ++u) {
#pragma unroll
                for (int i = 0; i < OPT; ++i) {
                    const int o = tid + kThreads * i;
                    const int kk = kk0 + u;
                    v[u][i] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (o < nout && kk < nk) {
                        const int rr = o / D4;
                        if (s_wm[kk * R + rr] != 0.f)
                            v[u][i] = __ldcg(reinterpret_cast<const float4*>(
                                                 rec_acc + (rec_of(k0 + kk, rr / G) * G + rr % G) * D) +
                                             (o % D4));
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < KU; ++u) {
#pragma unroll
                for (int i = 0; i < OPT; ++i) {
                    const int o = tid + kThreads * i;
                    const int kk = kk0 + u;
                    if (o < nout && kk < nk) {
                        const float w = s_wm[kk * R + o / D4];
                        acc[i].x += w * v[u][i].x;
                        acc[i].y += w * v[u][i].y;
                        acc[i].z += w * v[u][i].z;
                        acc[i].w += w * v[u][i].w;
                    }
                }
            }
        }
        named_barrier(1, kThreads);  // the next chunk rewrites the shared arrays
    }
    const uint32_t seq = static_cast<uint32_t>(sg) / head_groups;
    const uint32_t kv0 = (static_cast<uint32_t>(sg) % head_groups) * HH;
#pragma unroll
    for (int i = 0; i < OPT; ++i) {
        const int o = tid + kThreads * i;
        if (o < nout) {
            const int rr = o / D4, hh = rr / G, r = rr % G;
            const uint32_t lo = pack_bf16x2(acc[i].x, acc[i].y), hi = pack_bf16x2(acc[i].z, acc[i].w);
            for (uint32_t t = 0; t < out.n; ++t) {
                __nv_bfloat16* ob = out.row(t, seq, (kv0 + hh) * G + r, D) + (o % D4) * 4;
                reinterpret_cast<uint32_t*>(ob)[0] = lo;
                reinterpret_cast<uint32_t*>(ob)[1] = hi;
            }
        }
    }
}

template <int D, int HH, int STAGES>
__global__ void __launch_bounds__(kFastThreads, 1)
    paged_decode_stream(const __grid_constant__ CUtensorMap tmap, const StreamParams p) {
    using S = FastShape<D, HH, STAGES>;
    constexpr int J = S::J;
    constexpr int KS = D / 16;
    constexpr int NT = D / 8;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStage);
    int32_t* prefix = reinterpret_cast<int32_t*>(bars + 2 * STAGES);  // [nseg + 1]

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int nseg = static_cast<int>(p.nseg);
    const uint32_t cap_tokens = p.pitch * 16u;
    // scratch after the prefix, 16-byte aligned
    float* scratch = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(prefix + nseg + 1) + 15) &
                                              ~static_cast<uintptr_t>(15));

    // Launched as a programmatic dependent of the previous kernel on the
    // stream: everything above ran while it drained; wait for it (and its
    // memory) before reading any input.
    if (tid == 0) prefetch_tensormap(&tmap);
    grid_dependency_wait();

    // 1. stage counts of every segment, then an inclusive scan (warp 0).
    for (int sg = tid; sg < nseg; sg += kFastThreads) {
        const int c = p.ctx[sg / p.head_groups];
        const bool ok = c > 0 && static_cast<uint32_t>(c) <= cap_tokens;
        if (!ok && blockIdx.x == 0 && sg % p.head_groups == 0) record_error(p.err, kErrBadContext);
        const uint32_t units = ok ? (static_cast<uint32_t>(c) + 15u) / 16u : 0u;
        prefix[sg + 1] = static_cast<int32_t>((units + J - 1) / J);
    }
    __syncthreads();
    if (warp == 0) {
        int32_t running = 0;
        for (int base = 0; base < nseg; base += 32) {
            const int i = base + lane;
            int32_t v = i < nseg ? prefix[i + 1] : 0;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int32_t t = __shfl_up_sync(0xffffffffu, v, off);
                if (lane >= off) v += t;
            }
            if (i < nseg) prefix[i + 1] = v + running;
            running += __shfl_sync(0xffffffffu, v, 31);
        }
        if (lane == 0) prefix[0] = 0;
    }
    __syncthreads();
    const uint32_t total = static_cast<uint32_t>(prefix[nseg]);
    // The next decode on the stream may be scheduled from here on; it waits
    // (griddepcontrol.wait) for this whole grid before it touches memory.
    grid_launch_dependents();
    const uint32_t grid = gridDim.x;
    StreamSplit split;
    split.prefix = prefix;
    split.nseg = nseg;
    split.total = total;
    split.grid = grid;
    split.b = p.seg_cost;
    split.cost = static_cast<uint64_t>(total) + static_cast<uint64_t>(p.seg_cost) * nseg;
    const uint32_t x0 = split.begin(blockIdx.x);
    const uint32_t x1 = split.begin(blockIdx.x + 1);
    if (x0 >= x1) return;
    const PieceOrder order(prefix, nseg, x0, x1);

    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + STAGES);
    __shared__ int s_dead;  // a consumer warp's pipeline wait gave up
    __shared__ int s_last;  // this CTA completed the segment it just finished
    __shared__ float s_stat[128];
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, kFastComputeWarps);
        }
        mbar_fence_init();
        s_dead = 0;
    }
    __syncthreads();

    if (warp == kFastComputeWarps) {
        // Producer warp: lane 0 issues; all lanes keep two 32-entry windows of
        // the current segment's block table so entries arrive 32 at a time.
        const uint64_t policy = l2_policy_evict_first();
        uint32_t it = 0;
        bool ok_all = true;
        for (int pi = 0; pi < order.count && ok_all; ++pi) {
            int sg;
            uint32_t pb, pe;
            bool whole;
            order.at(prefix, pi, sg, pb, pe, whole);
            if (pb >= pe) continue;
            const uint32_t seg_begin = static_cast<uint32_t>(prefix[sg]);
            const int seq = sg / p.head_groups, hg = sg % p.head_groups;
            const uint32_t units = (static_cast<uint32_t>(p.ctx[seq]) + 15u) / 16u;
            const int32_t* row = p.tables + static_cast<size_t>(seq) * p.pitch;
            int win = -1;
            int32_t entry = 0, entry_next = 0;
            for (uint32_t x = pb; x < pe; ++x, ++it) {
                const uint32_t slot = it % STAGES;
                const int blk0 = static_cast<int>((x - seg_begin) * J);
                if (win < 0 || blk0 < win || blk0 + J > win + 64) {
                    win = blk0;
                    entry = (static_cast<uint32_t>(win + lane) < units) ? row[win + lane] : 0;
                    entry_next = (static_cast<uint32_t>(win + 32 + lane) < units) ? row[win + 32 + lane] : 0;
                } else if (blk0 + J > win + 32) {
                    win += 32;  // J divides 32, so blk0 == win here
                    entry = entry_next;
                    entry_next = (static_cast<uint32_t>(win + 32 + lane) < units) ? row[win + 32 + lane] : 0;
                }
                int32_t ids[J];
#pragma unroll
                for (int j = 0; j < J; ++j) ids[j] = __shfl_sync(0xffffffffu, entry, blk0 - win + j);
                int ok = 1;
                if (lane == 0) {
                    if (it >= STAGES && !mbar_wait_bounded(empty0 + 8 * slot, ((it / STAGES) - 1) & 1u)) {
                        record_error(p.err, kErrWaitTimeout);
                        ok = 0;
                    } else {
                        const uint32_t nb = min(static_cast<uint32_t>(J), units - static_cast<uint32_t>(blk0));
                        mbar_arrive_expect_tx(full0 + 8 * slot, nb * S::kBlock);
                        const uint32_t dst = smem_u32(smem + slot * S::kStage);
#pragma unroll
                        for (int j = 0; j < J; ++j) {
                            if (static_cast<uint32_t>(j) < nb) {
                                int32_t id = ids[j];
                                if (static_cast<uint32_t>(id) >= p.num_blocks) {
                                    record_error(p.err, kErrBadBlockId);
                                    id = 0;
                                }
                                const int r = (id * static_cast<int>(p.num_layers) + static_cast<int>(p.layer)) * 32;
                                tma_load_4d(dst + j * S::kBlock, &tmap, full0 + 8 * slot, 0, r, hg * HH, 0, policy);
                            }
                        }
                    }
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    ok_all = false;
                    break;
                }
            }
        }
        return;
    }

    // Consumer warps: (hh, j) owns kv head hg*HH + hh and unit j of each stage.
    const int hh = warp % HH;
    const int j = warp / HH;
    const int g = lane >> 2;
    const int c = lane & 3;
    const int G = static_cast<int>(p.group);
    constexpr int kConsumers = kFastComputeWarps * 32;
    const uint32_t state_floats = static_cast<uint32_t>(G * D + 2 * G);

    uint32_t qa[KS][4];
    WarpState<D> st;
    bool alive = true;
    uint32_t it = 0;

    // the first piece's query fragments
    int next_pi = 0;
    int n_sg = 0;
    uint32_t n_b = 0, n_e = 0;
    bool n_whole = false;
    auto find_next = [&](int from) {
        for (int pi = from; pi < order.count; ++pi) {
            order.at(prefix, pi, n_sg, n_b, n_e, n_whole);
            if (n_b < n_e) return pi;
        }
        return order.count;
    };
    next_pi = find_next(0);
    if (next_pi < order.count)
        load_query_fragments<D>(qa, p.q, n_sg / p.head_groups, p.hq, (n_sg % p.head_groups) * HH + hh, G, lane);

    while (next_pi < order.count) {
        const int sg = n_sg;
        const uint32_t pb = n_b, pe = n_e;
        const bool whole = n_whole;
        const uint32_t seg_begin = static_cast<uint32_t>(prefix[sg]);
        const int seq = sg / p.head_groups, hg = sg % p.head_groups;
        const int ctx = p.ctx[seq];
        const uint32_t units = (static_cast<uint32_t>(ctx) + 15u) / 16u;
        st.reset();
        for (uint32_t x = pb; x < pe; ++x, ++it) {
            const uint32_t slot = it % STAGES;
            if (alive && !mbar_wait_bounded(full0 + 8 * slot, (it / STAGES) & 1u)) {
                // the warp stops computing but keeps meeting the CTA's
                // barriers; the host sees the error bit and this CTA writes
                // no output and no record
                record_error(p.err, kErrWaitTimeout);
                alive = false;
                s_dead = 1;
            }
            const uint32_t blk = (x - seg_begin) * J + j;
            if (alive && blk < units) {
                const int valid = min(16, ctx - static_cast<int>(blk) * 16);
                const uint32_t kb = smem_u32(smem + slot * S::kStage + j * S::kBlock);
                attend_block<D, HH>(st, qa, kb, hh, valid, p.scale_log2, lane);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8 * slot);
        }
        // The next piece's query rows: after a whole segment they start
        // loading now and arrive during the epilogue; after a shared piece
        // they load once its record is out (and any merge is done), so that
        // no query registers are live across the merge.
        next_pi = find_next(next_pi + 1);
        auto load_next_query = [&]() {
            if (next_pi < order.count)
                load_query_fragments<D>(qa, p.q, n_sg / p.head_groups, p.hq, (n_sg % p.head_groups) * HH + hh, G,
                                        lane);
        };

        // Epilogue. Row sums over the lane quad first.
        float l0 = st.l0 + __shfl_xor_sync(0xffffffffu, st.l0, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        float l1 = st.l1 + __shfl_xor_sync(0xffffffffu, st.l1, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
        float m0 = st.m0, m1 = st.m1;
        auto& o = st.o;
        // Combine the J warp columns of each head into column 0: a tree of
        // rounds; in each, columns [half, 2*half) hand their state over.
#pragma unroll
        for (int half = J / 2; half >= 1; half >>= 1) {
            if (j >= half && j < 2 * half) {
                float* w = scratch + static_cast<uint32_t>((j - half) * HH + hh) * state_floats;
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    const int col = n * 8 + c * 2;
                    if (g < G) *reinterpret_cast<float2*>(w + g * D + col) = make_float2(o[n][0], o[n][1]);
                    if (g + 8 < G) *reinterpret_cast<float2*>(w + (g + 8) * D + col) = make_float2(o[n][2], o[n][3]);
                }
                if (c == 0) {
                    if (g < G) {
                        w[G * D + g] = m0;
                        w[G * D + G + g] = l0;
                    }
                    if (g + 8 < G) {
                        w[G * D + g + 8] = m1;
                        w[G * D + G + g + 8] = l1;
                    }
                }
            }
            named_barrier(1, kConsumers);
            if (j < half) {
                const float* w = scratch + static_cast<uint32_t>(j * HH + hh) * state_floats;
                const float mj0 = g < G ? w[G * D + g] : -INFINITY;
                const float mj1 = g + 8 < G ? w[G * D + g + 8] : -INFINITY;
                const float lj0 = g < G ? w[G * D + G + g] : 0.f;
                const float lj1 = g + 8 < G ? w[G * D + G + g + 8] : 0.f;
                const float M0 = fmaxf(m0, mj0), M1 = fmaxf(m1, mj1);
                const float a0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - M0);
                const float a1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - M1);
                const float e0 = (mj0 == -INFINITY) ? 0.f : exp2f(mj0 - M0);
                const float e1 = (mj1 == -INFINITY) ? 0.f : exp2f(mj1 - M1);
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    // keep the loads next to their use (a full hoist would
                    // hold 2 * NT more registers than the kernel has)
                    asm volatile("" ::: "memory");
                    const int col = n * 8 + c * 2;
                    const float2 lo = g < G ? *reinterpret_cast<const float2*>(w + g * D + col) : make_float2(0.f, 0.f);
                    const float2 hi =
                        g + 8 < G ? *reinterpret_cast<const float2*>(w + (g + 8) * D + col) : make_float2(0.f, 0.f);
                    o[n][0] = o[n][0] * a0 + lo.x * e0;
                    o[n][1] = o[n][1] * a0 + lo.y * e0;
                    o[n][2] = o[n][2] * a1 + hi.x * e1;
                    o[n][3] = o[n][3] * a1 + hi.y * e1;
                }
                l0 = l0 * a0 + lj0 * e0;
                l1 = l1 * a1 + lj1 * e1;
                m0 = M0;
                m1 = M1;
            }
            named_barrier(1, kConsumers);
        }
        const bool dead = s_dead != 0;
        if (whole) {
            // the segment lies wholly in this CTA: write its output now
            if (j == 0 && !dead) {
                const float inv0 = 1.f / l0, inv1 = 1.f / l1;
                for (uint32_t t = 0; t < p.out.n; ++t) {
                    __nv_bfloat16* ob = p.out.row(t, seq, (hg * HH + hh) * G, D);
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
                        const int col = n * 8 + c * 2;
                        if (g < G)
                            *reinterpret_cast<uint32_t*>(ob + g * D + col) =
                                pack_bf16x2(o[n][0] * inv0, o[n][1] * inv0);
                        if (g + 8 < G)
                            *reinterpret_cast<uint32_t*>(ob + (g + 8) * D + col) =
                                pack_bf16x2(o[n][2] * inv1, o[n][3] * inv1);
                    }
                }
            }
            load_next_query();
            continue;
        }
        // a shared piece: one record per head, then count the piece
        if (j == 0 && !dead) {
            const size_t rec = (static_cast<size_t>(sg) + blockIdx.x) * HH + hh;
            float* wo = p.rec_acc + rec * G * D;
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const int col = n * 8 + c * 2;
                if (g < G) *reinterpret_cast<float2*>(wo + g * D + col) = make_float2(o[n][0], o[n][1]);
                if (g + 8 < G) *reinterpret_cast<float2*>(wo + (g + 8) * D + col) = make_float2(o[n][2], o[n][3]);
            }
            if (c == 0) {
                if (g < G) p.rec_ml[rec * G + g] = make_float2(m0, l0);
                if (g + 8 < G) p.rec_ml[rec * G + g + 8] = make_float2(m1, l1);
            }
            __threadfence();  // the record reaches L2 before the arrival is counted
        }
        named_barrier(1, kConsumers);
        uint32_t cf, cl;
        split.pieces(sg, cf, cl);
        if (tid == 0) {
            uint32_t expected = cl - cf + 1;
            if (split.may_have_empty()) {
                expected = 0;
                for (uint32_t cc = cf; cc <= cl; ++cc) expected += split.empty(cc) ? 0u : 1u;
            }
            const bool last = !dead && arrive_last(p.seg_count + sg, p.epoch, expected);
            if (last) __threadfence();  // the other pieces' records are read after this
            s_last = last ? 1 : 0;
        }
        named_barrier(1, kConsumers);
        if (s_last) {
            // this piece completed the segment: merge it now (the producer
            // warp keeps streaming meanwhile); the scratch holds the weights
            const int R = HH * G;
            const int nout = R * (D / 4);
            const int chunk = min(32, static_cast<int>(4u * state_floats) / (2 * R));
            float* s_wm = scratch;
            float* s_wl = scratch + chunk * R;
#define QVP_MERGE(OPT)                                                                                              \
    merge_records<D, HH, OPT>(p.rec_acc, p.rec_ml, p.out, p.group, p.head_groups, sg, cf, cl, split, s_wm, s_wl, \
                              chunk, s_stat, tid)
            if (nout <= 256)
                QVP_MERGE(1);
            else if (nout <= 512)
                QVP_MERGE(2);
            else if (nout <= 1024)
                QVP_MERGE(4);
            else
                QVP_MERGE(8);
#undef QVP_MERGE
            named_barrier(1, kConsumers);  // the scratch is the next piece's again
        }
        load_next_query();
    }
}

// ---------------------------------------------------------------------------

struct GenericParams {
    const uint8_t* pool;
    size_t block_stride;
    const int32_t* tables;
    const int32_t* ctx;
    const void* q;
    void* out;
    float* ws_o;
    float2* ws_ml;
    int32_t* err;
    uint32_t pitch;
    uint32_t num_blocks;
    uint32_t tokens_per_block;
    uint32_t num_kv_heads;
    uint32_t head_dim;
    uint32_t layer;
    uint32_t hq;
    uint32_t group;
    uint32_t split_tokens;
    uint32_t max_splits;
    float scale;
};

template <typename T>
__global__ void __launch_bounds__(kGenericWarps * 32) paged_decode_generic(const GenericParams p) {
    __shared__ float sm_ml[kGenericWarps][2];
    __shared__ float sm_acc[kGenericWarps][kGenericMaxDimPerLane * 32];

    const int seq = blockIdx.z;
    const int qh = blockIdx.y;
    const uint32_t split = blockIdx.x;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int ctx = p.ctx[seq];
    if (ctx <= 0 || static_cast<uint32_t>(ctx) > p.pitch * p.tokens_per_block) {
        if (threadIdx.x == 0 && split == 0 && qh == 0) record_error(p.err, kErrBadContext);
        return;
    }
    const uint32_t nsplits = (static_cast<uint32_t>(ctx) + p.split_tokens - 1) / p.split_tokens;
    if (nsplits > p.max_splits) {
        if (threadIdx.x == 0 && split == 0 && qh == 0) record_error(p.err, kErrBadContext);
        return;
    }
    const uint32_t t0 = split * p.split_tokens;
    if (t0 >= static_cast<uint32_t>(ctx)) return;
    const uint32_t t1 = min(t0 + p.split_tokens, static_cast<uint32_t>(ctx));

    const uint32_t D = p.head_dim;
    const uint32_t kvh = qh / p.group;
    const T* q = static_cast<const T*>(p.q) + (static_cast<size_t>(seq) * p.hq + qh) * D;
    float qr[kGenericMaxDimPerLane];
    float acc[kGenericMaxDimPerLane];
#pragma unroll
    for (int i = 0; i < kGenericMaxDimPerLane; ++i) {
        const uint32_t d = lane + 32 * i;
        qr[i] = d < D ? to_float<T>(q[d]) : 0.f;
        acc[i] = 0.f;
    }
    float m = -INFINITY, l = 0.f;

    const size_t token_stride = static_cast<size_t>(p.num_kv_heads) * D;
    const size_t stream_stride = token_stride * p.tokens_per_block;
    const size_t layer_off = static_cast<size_t>(p.layer) * 2 * stream_stride + kvh * D;
    const int32_t* row = p.tables + static_cast<size_t>(seq) * p.pitch;

    for (uint32_t t = t0 + warp; t < t1; t += kGenericWarps) {
        int32_t id = row[t / p.tokens_per_block];
        if (static_cast<uint32_t>(id) >= p.num_blocks) {
            if (lane == 0) record_error(p.err, kErrBadBlockId);
            id = 0;
        }
        const T* kp = reinterpret_cast<const T*>(p.pool + static_cast<size_t>(id) * p.block_stride) +
                      layer_off + (t % p.tokens_per_block) * token_stride;
        const T* vp = kp + stream_stride;
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < kGenericMaxDimPerLane; ++i) {
            const uint32_t d = lane + 32 * i;
            if (d < D) dot += qr[i] * to_float<T>(kp[d]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        const float s = dot * p.scale;
        const float mn = fmaxf(m, s);
        const float corr = expf(m - mn);
        const float w = expf(s - mn);
        l = l * corr + w;
#pragma unroll
        for (int i = 0; i < kGenericMaxDimPerLane; ++i) {
            const uint32_t d = lane + 32 * i;
            if (d < D) acc[i] = acc[i] * corr + w * to_float<T>(vp[d]);
        }
        m = mn;
    }

    if (lane == 0) {
        sm_ml[warp][0] = m;
        sm_ml[warp][1] = l;
    }
#pragma unroll
    for (int i = 0; i < kGenericMaxDimPerLane; ++i) sm_acc[warp][lane + 32 * i] = acc[i];
    __syncthreads();
    if (warp != 0) return;

    float M = -INFINITY;
    for (int w = 0; w < kGenericWarps; ++w) M = fmaxf(M, sm_ml[w][0]);
    float L = 0.f;
    float wt[kGenericWarps];
    for (int w = 0; w < kGenericWarps; ++w) {
        wt[w] = (sm_ml[w][0] == -INFINITY) ? 0.f : expf(sm_ml[w][0] - M);
        L += wt[w] * sm_ml[w][1];
    }
    if (nsplits == 1) {
        T* out = static_cast<T*>(p.out) + (static_cast<size_t>(seq) * p.hq + qh) * D;
        for (uint32_t d = lane; d < D; d += 32) {
            float a = 0.f;
            for (int w = 0; w < kGenericWarps; ++w) a += wt[w] * sm_acc[w][d];
            out[d] = from_float<T>(a / L);
        }
    } else {
        const size_t part = (static_cast<size_t>(seq) * p.max_splits + split) * p.hq + qh;
        float* wo = p.ws_o + part * D;
        for (uint32_t d = lane; d < D; d += 32) {
            float a = 0.f;
            for (int w = 0; w < kGenericWarps; ++w) a += wt[w] * sm_acc[w][d];
            wo[d] = a;
        }
        if (lane == 0) p.ws_ml[part] = make_float2(M, L);
    }
}

// Merges the partitions of every (sequence, query head) whose context was
// split. `log2_domain` says whether the partition maxima are base-2 (fast
// kernel) or natural (generic kernel).
template <typename T>
__global__ void combine_partitions(const float* __restrict__ ws_o, const float2* __restrict__ ws_ml,
                                   const int32_t* __restrict__ ctx_lens, T* __restrict__ out,
                                   uint32_t hq, uint32_t D, uint32_t max_splits, uint32_t split_tokens,
                                   int log2_domain) {
    const int seq = blockIdx.y;
    const int h = blockIdx.x;
    const int ctx = ctx_lens[seq];
    if (ctx <= 0) return;
    const uint32_t ns = (static_cast<uint32_t>(ctx) + split_tokens - 1) / split_tokens;
    if (ns <= 1 || ns > max_splits) return;
    const size_t base = static_cast<size_t>(seq) * max_splits * hq + h;
    float M = -INFINITY;
    for (uint32_t s = 0; s < ns; ++s) M = fmaxf(M, ws_ml[base + s * hq].x);
    float L = 0.f;
    for (uint32_t s = 0; s < ns; ++s) {
        const float2 ml = ws_ml[base + s * hq];
        const float w = log2_domain ? exp2f(ml.x - M) : expf(ml.x - M);
        L += w * ml.y;
    }
    const float inv = 1.f / L;
    T* o = out + (static_cast<size_t>(seq) * hq + h) * D;
    for (uint32_t d = threadIdx.x; d < D; d += blockDim.x) {
        float a = 0.f;
        for (uint32_t s = 0; s < ns; ++s) {
            const float2 ml = ws_ml[base + s * hq];
            const float w = log2_domain ? exp2f(ml.x - M) : expf(ml.x - M);
            a += w * ws_o[(base + s * hq) * D + d];
        }
        o[d] = from_float<T>(a * inv);
    }
}

// ---- host side ------------------------------------------------------------

// Looked up once per process (a function-local static is initialised once,
// thread-safely).
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult qres;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                             &qres) == cudaSuccess &&
            qres == cudaDriverEntryPointSuccess)
            return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
        cudaGetLastError();
        return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
    }();
    return fn;
}

}  // namespace

// The pool viewed as a 4-D tensor of bf16 so one TMA box is the K and V
// slices of one block for HH consecutive kv heads, laid out in shared memory
// as [head_dim/64][HH][16 K rows, then 16 V rows][64] (K and V of a block
// are adjacent token rows, so one box carries both: one TMA copy per block):
//   dim0: 64 elements of head_dim        (contiguous)
//   dim1: token rows of the whole pool   (stride kv_heads*head_dim*2 bytes)
//   dim2: kv head                        (stride head_dim*2 bytes)
//   dim3: 64-element half of head_dim    (stride 128 bytes)
// Token row r of block b, layer l, stream s, slot t is ((b*L + l)*2 + s)*16 + t,
// which needs blocks stored back to back (stride == byte_size).

int encode_pool_map(const void* pool, uint32_t num_blocks, const qvp_block_shape& shape, uint32_t hh,
                    CUtensorMap* map) {
    return encode_pool_map_box(pool, num_blocks, shape, hh, 32, shape.head_dim / 64, map);
}

int encode_pool_map_box(const void* pool, uint32_t num_blocks, const qvp_block_shape& shape, uint32_t hh,
                        uint32_t rows, uint32_t halves, CUtensorMap* map) {
    struct Key {
        const void* pool;
        uint32_t num_blocks, layers, heads, dim, hh, rows, halves;
    };
    static thread_local Key last{};
    static thread_local CUtensorMap cached;
    // compared with memcmp, so the padding bytes are zeroed too
    Key key;
    std::memset(&key, 0, sizeof(key));
    key.pool = pool;
    key.num_blocks = num_blocks;
    key.layers = shape.num_layers;
    key.heads = shape.num_kv_heads;
    key.dim = shape.head_dim;
    key.hh = hh;
    key.rows = rows;
    key.halves = halves;
    if (std::memcmp(&key, &last, sizeof(Key)) == 0) {
        *map = cached;
        return QVP_OK;
    }
    auto encode = get_encode_fn();
    if (encode == nullptr) return fail(QVP_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const uint32_t D = shape.head_dim;
    const uint32_t H = shape.num_kv_heads;
    cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(num_blocks) * shape.num_layers * 2 * 16, H, D / 64};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(H) * D * 2, static_cast<cuuint64_t>(D) * 2, 128};
    cuuint32_t box[4] = {64, rows, hh, halves};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(pool), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(QVP_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
    last = key;
    cached = *map;
    return QVP_OK;
}

namespace {

template <int D, int HH, int STAGES>
int launch_fast_t(const qvp_decode_args& a, const DecodePlan& plan, const FastParams& fp, cudaStream_t st) {
    using S = FastShape<D, HH, STAGES>;
    static std::atomic<std::uint64_t> attr_done{0};
    auto kern = paged_decode_fast<D, HH, STAGES>;
    int rc = set_smem_limit_once(attr_done, reinterpret_cast<const void*>(kern), S::kSmem,
                                 "cudaFuncSetAttribute(fast decode)");
    if (rc != QVP_OK) return rc;
    CUtensorMap map;
    rc = encode_pool_map(a.pool, a.num_blocks, a.shape, HH, &map);
    if (rc != QVP_OK) return rc;
    dim3 grid(plan.max_splits, a.shape.num_kv_heads / HH, a.batch);
    kern<<<grid, kFastThreads, S::kSmem, st>>>(map, fp);
    return check_cuda(cudaGetLastError(), "launch fast decode");
}

int launch_fast(const qvp_decode_args& a, const DecodePlan& plan, const FastParams& fp, cudaStream_t st) {
    const uint32_t D = a.shape.head_dim;
    switch (plan.heads_per_cta) {
        case 4: return D == 128 ? launch_fast_t<128, 4, 3>(a, plan, fp, st) : launch_fast_t<64, 4, 6>(a, plan, fp, st);
        case 2: return D == 128 ? launch_fast_t<128, 2, 3>(a, plan, fp, st) : launch_fast_t<64, 2, 6>(a, plan, fp, st);
        default: return D == 128 ? launch_fast_t<128, 1, 3>(a, plan, fp, st) : launch_fast_t<64, 1, 6>(a, plan, fp, st);
    }
}

template <int D, int HH, int STAGES>
int launch_stream_t(const qvp_decode_args& a, const DecodePlan& plan, const StreamParams& sp, cudaStream_t st) {
    using S = FastShape<D, HH, STAGES>;
    static_assert(S::kSmem == stream_pipeline_smem(D), "stream decode pipeline size");
    static std::atomic<std::uint64_t> attr_done{0};
    auto kern = paged_decode_stream<D, HH, STAGES>;
    int rc = set_smem_limit_once(attr_done, reinterpret_cast<const void*>(kern), static_cast<int>(kMaxDynamicSmem),
                                 "cudaFuncSetAttribute(stream decode)");
    if (rc != QVP_OK) return rc;
    CUtensorMap map;
    rc = encode_pool_map(a.pool, a.num_blocks, a.shape, HH, &map);
    if (rc != QVP_OK) return rc;
    const uint32_t smem = static_cast<uint32_t>(stream_smem_bytes(sp.nseg, sp.group, D));
    {
        // programmatic dependent of whatever precedes it on the stream (the
        // previous step's decode): the prologue overlaps that kernel's tail
        cudaLaunchConfig_t dcfg = {};
        dcfg.gridDim = dim3(plan.grid_ctas);
        dcfg.blockDim = dim3(kFastThreads);
        dcfg.dynamicSmemBytes = smem;
        dcfg.stream = st;
        cudaLaunchAttribute dattr[1];
        dattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        dattr[0].val.programmaticStreamSerializationAllowed = 1;
        dcfg.attrs = dattr;
        dcfg.numAttrs = 1;
        return check_cuda(cudaLaunchKernelEx(&dcfg, kern, map, sp), "launch stream decode");
    }
}

int launch_stream(const qvp_decode_args& a, const DecodePlan& plan, const StreamParams& sp, cudaStream_t st) {
    const uint32_t D = a.shape.head_dim;
    switch (plan.heads_per_cta) {
        case 4: return D == 128 ? launch_stream_t<128, 4, 3>(a, plan, sp, st) : launch_stream_t<64, 4, 6>(a, plan, sp, st);
        case 2: return D == 128 ? launch_stream_t<128, 2, 3>(a, plan, sp, st) : launch_stream_t<64, 2, 6>(a, plan, sp, st);
        default: return D == 128 ? launch_stream_t<128, 1, 3>(a, plan, sp, st) : launch_stream_t<64, 1, 6>(a, plan, sp, st);
    }
}

// Epoch of a stream-K launch: distinct for every launch of this process and,
// through the clock seed, unlikely to match a word another process left in
// recycled device memory.
uint32_t next_epoch() {
    static std::atomic<uint32_t> epoch{static_cast<uint32_t>(
        std::chrono::steady_clock::now().time_since_epoch().count() * 2654435761ull)};
    return epoch.fetch_add(1, std::memory_order_relaxed) + 1u;
}

}  // namespace

int plan_decode(const qvp_decode_args& a, DecodePlan& plan) {
    plan = DecodePlan{};
    const qvp_block_shape& sh = a.shape;
    if (sh.tokens_per_block == 0 || sh.num_layers == 0 || sh.num_kv_heads == 0 || sh.head_dim == 0)
        return fail(QVP_ERR_INVALID, "block shape has a zero field");
    const uint32_t elem = a.dtype == QVP_DTYPE_F32 ? 4u : a.dtype == QVP_DTYPE_BF16 ? 2u : 0u;
    if (elem == 0) return fail(QVP_ERR_INVALID, "unknown dtype %d", a.dtype);
    if (sh.bytes_per_element != elem)
        return fail(QVP_ERR_INVALID, "bytes_per_element %u does not match the dtype", sh.bytes_per_element);
    if (a.layer >= sh.num_layers) return fail(QVP_ERR_INVALID, "layer %u >= num_layers %u", a.layer, sh.num_layers);
    if (a.num_query_heads == 0 || a.num_query_heads % sh.num_kv_heads != 0)
        return fail(QVP_ERR_INVALID, "num_query_heads %u is not a positive multiple of num_kv_heads %u",
                    a.num_query_heads, sh.num_kv_heads);
    if (a.batch == 0) return QVP_OK;
    if (a.pool == nullptr || a.block_tables == nullptr || a.context_lens == nullptr || a.query == nullptr ||
        a.out == nullptr)
        return fail(QVP_ERR_INVALID, "null pool, table, context, query or output pointer");
    if (a.batch > 65535 || a.num_query_heads > 65535) return fail(QVP_ERR_UNSUPPORTED, "batch or heads above 65535");
    const size_t block_bytes = qvp_block_bytes(&sh);
    if (a.block_stride < block_bytes) return fail(QVP_ERR_INVALID, "block_stride below the block size");
    if (a.num_blocks == 0) return fail(QVP_ERR_INVALID, "empty pool");
    if (a.max_context_len == 0) return fail(QVP_ERR_INVALID, "max_context_len is zero");
    if (static_cast<uint64_t>(a.max_context_len) >
        static_cast<uint64_t>(a.max_blocks_per_seq) * sh.tokens_per_block)
        return fail(QVP_ERR_INVALID, "max_context_len exceeds the table capacity");
    if (sh.head_dim > 32u * kGenericMaxDimPerLane)
        return fail(QVP_ERR_UNSUPPORTED, "head_dim %u above 256", sh.head_dim);

    plan.group = a.num_query_heads / sh.num_kv_heads;
    const uintptr_t pool_addr = reinterpret_cast<uintptr_t>(a.pool);
    plan.fast = a.dtype == QVP_DTYPE_BF16 && sh.tokens_per_block == 16 &&
                (sh.head_dim == 64 || sh.head_dim == 128) && plan.group <= 16 &&
                a.block_stride == block_bytes && (pool_addr & 15u) == 0 &&
                (reinterpret_cast<uintptr_t>(a.query) & 3u) == 0 &&
                (reinterpret_cast<uintptr_t>(a.out) & 3u) == 0 && sh.num_kv_heads <= 256 &&
                static_cast<uint64_t>(a.num_blocks) * sh.num_layers * 32u < (1ull << 31);
    plan.heads_per_cta = sh.num_kv_heads % 4 == 0 ? 4 : sh.num_kv_heads % 2 == 0 ? 2 : 1;

    if (plan.fast && a.split_tokens == 0) {
        const uint32_t z = sh.num_kv_heads / plan.heads_per_cta;
        const uint64_t nseg = static_cast<uint64_t>(a.batch) * z;
        if (nseg <= static_cast<uint64_t>(kStreamMaxSegments) &&
            stream_smem_bytes(static_cast<uint32_t>(nseg), plan.group, sh.head_dim) <= kMaxDynamicSmem) {
            // Persistent stream-K: one CTA per SM over the whole stage stream.
            plan.stream = true;
            plan.nseg = static_cast<uint32_t>(nseg);
            const int sms = device_sm_count();
            plan.grid_ctas = sms > 0 ? static_cast<uint32_t>(sms) : 148u;
            const size_t records = (static_cast<size_t>(plan.nseg) + plan.grid_ctas) * plan.heads_per_cta;
            plan.records = records;
            plan.split_tokens = 0;
            plan.max_splits = 1;
            plan.workspace_bytes = round_up(records * plan.group * sh.head_dim * sizeof(float), 256) +
                                   round_up(records * plan.group * sizeof(float2), 256) +
                                   static_cast<size_t>(plan.nseg) * sizeof(unsigned long long);
            return QVP_OK;
        }
    }
    uint32_t split = a.split_tokens;
    if (split != 0) {
        if (plan.fast && split % 16 != 0)
            return fail(QVP_ERR_INVALID, "split_tokens %u is not a multiple of 16", split);
    } else {
        // Smallest power-of-two partition (>= 256 tokens) that keeps the grid
        // of the longest context within about eight CTAs per SM.
        const uint32_t ctas_per_part = plan.fast ? sh.num_kv_heads / plan.heads_per_cta : a.num_query_heads;
        const uint64_t target = 8ull * static_cast<uint64_t>(device_sm_count() > 0 ? device_sm_count() : 148);
        split = 256;
        while (static_cast<uint64_t>(a.batch) * ctas_per_part * ceil_div(a.max_context_len, split) > target &&
               split < a.max_context_len)
            split *= 2;
    }
    plan.split_tokens = split;
    plan.max_splits = ceil_div(a.max_context_len, split);
    if (plan.max_splits > 0x7fffffffu) return fail(QVP_ERR_UNSUPPORTED, "too many partitions");
    if (plan.max_splits > 1) {
        const size_t parts = static_cast<size_t>(a.batch) * plan.max_splits * a.num_query_heads;
        plan.workspace_bytes = round_up(parts * sh.head_dim * sizeof(float), 256) + parts * sizeof(float2);
    }
    return QVP_OK;
}

}  // namespace qvp

using namespace qvp;

extern "C" int qvp_decode_workspace_size(const qvp_decode_args* args, size_t* bytes) {
    if (args == nullptr || bytes == nullptr) return fail(QVP_ERR_INVALID, "null argument");
    DecodePlan plan;
    const int rc = plan_decode(*args, plan);
    if (rc != QVP_OK) return rc;
    *bytes = plan.workspace_bytes;
    return QVP_OK;
}

extern "C" int qvp_decode_plan(const qvp_decode_args* args, uint32_t* split_tokens, uint32_t* num_splits,
                               int* fast_path) {
    if (args == nullptr) return fail(QVP_ERR_INVALID, "null argument");
    DecodePlan plan;
    const int rc = plan_decode(*args, plan);
    if (rc != QVP_OK) return rc;
    if (split_tokens) *split_tokens = plan.split_tokens;
    if (num_splits) *num_splits = plan.max_splits;
    if (fast_path) *fast_path = plan.stream ? 2 : plan.fast ? 1 : 0;
    return QVP_OK;
}

extern "C" int qvp_decode(const qvp_decode_args* args, qvp_stream_t stream) {
    if (args == nullptr) return fail(QVP_ERR_INVALID, "null argument");
    DecodePlan plan;
    const int rc = plan_decode(*args, plan);
    if (rc != QVP_OK || args->batch == 0) return rc;
    return run_decode(*args, plan, reinterpret_cast<cudaStream_t>(stream));
}

int qvp::run_decode(const qvp_decode_args& a, const DecodePlan& plan, cudaStream_t st, const OutTargets* targets) {
    if (targets != nullptr && !plan.stream)
        return fail(QVP_ERR_UNSUPPORTED, "writing outputs to several GPUs needs the stream-K plan");
    int rc = QVP_OK;
    if (plan.workspace_bytes > 0 && (a.workspace == nullptr || a.workspace_bytes < plan.workspace_bytes))
        return fail(QVP_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", plan.workspace_bytes,
                    a.workspace == nullptr ? size_t(0) : a.workspace_bytes);
    // partial records are read back as float4
    if (plan.workspace_bytes > 0 && (reinterpret_cast<uintptr_t>(a.workspace) & 15u) != 0)
        return fail(QVP_ERR_WORKSPACE, "workspace is not 16-byte aligned");
    const size_t parts = static_cast<size_t>(a.batch) * plan.max_splits * a.num_query_heads;
    float* ws_o = static_cast<float*>(a.workspace);
    float2* ws_ml = plan.workspace_bytes
                        ? reinterpret_cast<float2*>(static_cast<uint8_t*>(a.workspace) +
                                                    round_up(parts * a.shape.head_dim * sizeof(float), 256))
                        : nullptr;
    const uint32_t D = a.shape.head_dim;

    if (plan.stream) {
        uint8_t* ws = static_cast<uint8_t*>(a.workspace);
        const size_t acc_bytes = round_up(plan.records * plan.group * D * sizeof(float), 256);
        const size_t ml_bytes = round_up(plan.records * plan.group * sizeof(float2), 256);
        StreamParams sp;
        sp.tables = a.block_tables;
        sp.ctx = a.context_lens;
        sp.q = static_cast<const __nv_bfloat16*>(a.query);
        sp.rec_acc = reinterpret_cast<float*>(ws);
        sp.rec_ml = reinterpret_cast<float2*>(ws + acc_bytes);
        sp.seg_count = reinterpret_cast<unsigned long long*>(ws + acc_bytes + ml_bytes);
        if (targets != nullptr) {
            sp.out = *targets;
        } else {
            sp.out.ptr[0] = static_cast<__nv_bfloat16*>(a.out);
            sp.out.n = 1;
            sp.out.head0 = 0;
            sp.out.row_heads = a.num_query_heads;
        }
        sp.epoch = next_epoch();
        // fixed cost of a segment in stage-equivalents: its epilogue combines
        // J warp columns (log2 J rounds) and a shared piece adds a record
        // and, for one CTA, the merge; measured on cfg2-shaped batches
        sp.seg_cost = kSegmentCostStages[plan.heads_per_cta == 4 ? 2 : plan.heads_per_cta == 2 ? 1 : 0];
        sp.err = a.error_word;
        sp.pitch = a.max_blocks_per_seq;
        sp.num_blocks = a.num_blocks;
        sp.layer = a.layer;
        sp.num_layers = a.shape.num_layers;
        sp.hq = a.num_query_heads;
        sp.group = plan.group;
        sp.head_groups = a.shape.num_kv_heads / plan.heads_per_cta;
        sp.nseg = plan.nseg;
        sp.scale_log2 = a.scale * 1.4426950408889634f;  // log2(e)
        return launch_stream(a, plan, sp, st);
    }

    if (plan.fast) {
        FastParams fp;
        fp.tables = a.block_tables;
        fp.ctx = a.context_lens;
        fp.q = static_cast<const __nv_bfloat16*>(a.query);
        fp.out = static_cast<__nv_bfloat16*>(a.out);
        fp.ws_o = ws_o;
        fp.ws_ml = ws_ml;
        fp.err = a.error_word;
        fp.pitch = a.max_blocks_per_seq;
        fp.num_blocks = a.num_blocks;
        fp.layer = a.layer;
        fp.num_layers = a.shape.num_layers;
        fp.hq = a.num_query_heads;
        fp.group = plan.group;
        fp.split_blocks = plan.split_tokens / 16;
        fp.max_splits = plan.max_splits;
        fp.scale_log2 = a.scale * 1.4426950408889634f;  // log2(e)
        rc = launch_fast(a, plan, fp, st);
    } else {
        GenericParams gp;
        gp.pool = static_cast<const uint8_t*>(a.pool);
        gp.block_stride = a.block_stride;
        gp.tables = a.block_tables;
        gp.ctx = a.context_lens;
        gp.q = a.query;
        gp.out = a.out;
        gp.ws_o = ws_o;
        gp.ws_ml = ws_ml;
        gp.err = a.error_word;
        gp.pitch = a.max_blocks_per_seq;
        gp.num_blocks = a.num_blocks;
        gp.tokens_per_block = a.shape.tokens_per_block;
        gp.num_kv_heads = a.shape.num_kv_heads;
        gp.head_dim = D;
        gp.layer = a.layer;
        gp.hq = a.num_query_heads;
        gp.group = plan.group;
        gp.split_tokens = plan.split_tokens;
        gp.max_splits = plan.max_splits;
        gp.scale = a.scale;
        dim3 grid(plan.max_splits, a.num_query_heads, a.batch);
        if (a.dtype == QVP_DTYPE_F32)
            paged_decode_generic<float><<<grid, kGenericWarps * 32, 0, st>>>(gp);
        else
            paged_decode_generic<__nv_bfloat16><<<grid, kGenericWarps * 32, 0, st>>>(gp);
        rc = check_cuda(cudaGetLastError(), "launch generic decode");
    }
    if (rc != QVP_OK || plan.max_splits <= 1) return rc;

    dim3 grid(a.num_query_heads, a.batch);
    const int threads = D >= 128 ? 128 : 64;
    const int log2_domain = plan.fast ? 1 : 0;
    if (a.dtype == QVP_DTYPE_F32)
        combine_partitions<float><<<grid, threads, 0, st>>>(ws_o, ws_ml, a.context_lens, static_cast<float*>(a.out),
                                                            a.num_query_heads, D, plan.max_splits,
                                                            plan.split_tokens, log2_domain);
    else
        combine_partitions<__nv_bfloat16><<<grid, threads, 0, st>>>(
            ws_o, ws_ml, a.context_lens, static_cast<__nv_bfloat16*>(a.out), a.num_query_heads, D,
            plan.max_splits, plan.split_tokens, log2_domain);
    return check_cuda(cudaGetLastError(), "launch combine");
}
