// Causal prefill over the paged cache for B200 (sm_100a).
//
// The reference defines prefill as its decode applied at every prompt
// position p with context_len = p + 1 (phhuang191129/QwenVL-Paged
// include/qwenvl_paged/PagedAttention.h:43-44, tests/EndToEnd.test.cpp:
// 252-256). Computed that way, position p re-reads the K/V of all p earlier
// tokens. These kernels compute the same values with each K/V block read once
// per tile of query positions:
//   for query token t of sequence b (position pos = ctx_b - qlen_b + t):
//     out[b, t, h, :] = softmax_k<=pos(scale * <q[b,t,h], K_k>) V_k
//
//  * paged_prefill_fast: bf16, 16-token blocks, head_dim 64/128, group <= 16,
//    unpadded blocks. CTA = (sequence, kv head, tile of TQ = 128/G query
//    tokens). Its TQ*G (token, query head) rows fill the 16-row tensor-core
//    tiles of eight consumer warps; a producer warp streams the kv head's K
//    and V slices of every block the tile can see with TMA; every consumer
//    warp reads every staged block (the rows of one tile share each load).
//    Rows mask keys past their own position.
//  * paged_prefill_generic: any dtype / block size / head_dim <= 256; one CTA
//    per (query token, query head, sequence), four warps over keys.
#include "attention_tile.cuh"
#include "qvp_device.cuh"
#include "qvp_internal.h"
#include "tcgen05.cuh"

#include <cuda.h>

#include <cmath>

namespace qvp {

namespace {

constexpr int kPrefillWarps = 8;
constexpr int kPrefillThreads = (kPrefillWarps + 1) * 32;
constexpr int kPrefillRows = kPrefillWarps * 16;  // (token, head) rows per CTA

struct PrefillParams {
    const int32_t* tables;
    const int32_t* ctx;
    const int32_t* qlen;
    const __nv_bfloat16* q;
    __nv_bfloat16* out;
    int32_t* err;
    uint32_t pitch;
    uint32_t num_blocks;
    uint32_t layer;
    uint32_t num_layers;
    uint32_t hq;
    uint32_t group;
    uint32_t tile_tokens;  // TQ
    uint32_t max_qlen;     // row pitch (tokens) of q and out
    uint32_t batch;
    uint32_t hkv;
    float scale_log2;
};

template <int D, int NB, int STAGES>
struct PrefillShape {
    static constexpr uint32_t kBlock = 2 * 16 * D * 2;  // K and V of one block, one head (one TMA box)
    static constexpr uint32_t kStage = NB * kBlock;
    static constexpr uint32_t kSmem = STAGES * kStage + 1024 + 2 * STAGES * 8 + 16;
};

// attend_block with a separate causal limit for each of the lane's two rows:
// `va` / `vb` keys of this block are visible to rows g and g+8, and `vctx`
// slots hold real data (V past it is zeroed). `blk` is the block's box
// [head_dim/64][K 16 | V 16 tokens][64]: K rows of dh are row group 2*dh, V
// rows row group 2*dh+1.
template <int D>
__device__ __forceinline__ void attend_block_rows(WarpState<D>& st, const uint32_t (&qa)[D / 16][4], uint32_t blk,
                                                  int va, int vb_rows, int vctx, float scale_log2, int lane) {
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
        ldmatrix_x4(box_addr(blk, 2 * dh, t, chunk), r0, r1, r2, r3);
        mma_bf16_16816(s[0], qa[ks], r0, r1);
        mma_bf16_16816(s[1], qa[ks], r2, r3);
    }
#pragma unroll
    for (int a = 0; a < 2; ++a) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int tok = a * 8 + c * 2 + (e & 1);
            const int lim = (e < 2) ? va : vb_rows;
            const float v = s[a][e] * scale_log2;
            s[a][e] = (tok < lim) ? v : -INFINITY;
        }
    }
    float r_lo = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
    float r_hi = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
    r_lo = fmaxf(r_lo, __shfl_xor_sync(0xffffffffu, r_lo, 1));
    r_lo = fmaxf(r_lo, __shfl_xor_sync(0xffffffffu, r_lo, 2));
    r_hi = fmaxf(r_hi, __shfl_xor_sync(0xffffffffu, r_hi, 1));
    r_hi = fmaxf(r_hi, __shfl_xor_sync(0xffffffffu, r_hi, 2));
    // a row with no visible key in this block keeps its state (its max is
    // finite from block 0, which every row sees)
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
        ldmatrix_x4_trans(box_addr(blk, 2 * dh + 1, t, chunk), v0, v1, v2, v3);
        if (vctx < 16) {
            v0 = mask_pair(v0, c * 2, vctx);
            v2 = mask_pair(v2, c * 2, vctx);
            v1 = mask_pair(v1, 8 + c * 2, vctx);
            v3 = mask_pair(v3, 8 + c * 2, vctx);
        }
        mma_bf16_16816(st.o[2 * np], pa, v0, v1);
        mma_bf16_16816(st.o[2 * np + 1], pa, v2, v3);
    }
}

template <int D, int NB, int STAGES>
__global__ void __launch_bounds__(kPrefillThreads, 1)
    paged_prefill_fast(const __grid_constant__ CUtensorMap tmap, const PrefillParams p) {
    using S = PrefillShape<D, NB, STAGES>;
    constexpr int KS = D / 16;
    constexpr int NT = D / 8;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStage);

    const int b = blockIdx.z;
    const int kvh = blockIdx.y;
    const int tile = blockIdx.x;
    const int ctx = p.ctx[b];
    const int ql = p.qlen[b];
    if (ctx <= 0 || static_cast<uint32_t>(ctx) > p.pitch * 16u || ql <= 0 || ql > ctx ||
        static_cast<uint32_t>(ql) > p.max_qlen) {
        if (threadIdx.x == 0 && tile == 0 && kvh == 0) record_error(p.err, kErrBadContext);
        return;
    }
    const int G = static_cast<int>(p.group);
    const int t0 = tile * static_cast<int>(p.tile_tokens);
    if (t0 >= ql) return;
    const int t1 = min(t0 + static_cast<int>(p.tile_tokens), ql);
    const int rows = (t1 - t0) * G;
    const int first_pos = ctx - ql;                    // position of query token 0
    const int last_pos = first_pos + t1 - 1;
    const uint32_t nblk = static_cast<uint32_t>(last_pos) / 16u + 1u;  // blocks the tile can see
    const uint32_t iters = (nblk + NB - 1) / NB;

    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + STAGES);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, kPrefillWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kPrefillWarps) {
        if (lane == 0) {
            prefetch_tensormap(&tmap);
            const uint64_t policy = l2_policy_evict_first();
            const int32_t* row = p.tables + static_cast<size_t>(b) * p.pitch;
            for (uint32_t it = 0; it < iters; ++it) {
                const uint32_t slot = it % STAGES;
                if (it >= STAGES && !mbar_wait_bounded(empty0 + 8 * slot, ((it / STAGES) - 1) & 1u)) {
                    record_error(p.err, kErrWaitTimeout);
                    break;
                }
                const uint32_t nb = min(static_cast<uint32_t>(NB), nblk - it * NB);
                mbar_arrive_expect_tx(full0 + 8 * slot, nb * S::kBlock);
                const uint32_t dst = smem_u32(smem + slot * S::kStage);
                for (uint32_t j = 0; j < nb; ++j) {
                    int32_t id = row[it * NB + j];
                    if (static_cast<uint32_t>(id) >= p.num_blocks) {
                        record_error(p.err, kErrBadBlockId);
                        id = 0;
                    }
                    const int r = (id * static_cast<int>(p.num_layers) + static_cast<int>(p.layer)) * 32;
                    tma_load_4d(dst + j * S::kBlock, &tmap, full0 + 8 * slot, 0, r, kvh, 0, policy);
                }
            }
        }
        return;
    }

    // Consumer warp w owns rows [16w, 16w+16) of the tile; row r is query
    // token t0 + r / G, query head kvh*G + r % G. Lane rows: g and g+8.
    const int g = lane >> 2;
    const int c = lane & 3;
    const int ra = warp * 16 + g;
    const int rb = ra + 8;
    const bool live = warp * 16 < rows;
    const int rlast = min(warp * 16 + 15, rows - 1);
    const int pos_a = first_pos + t0 + min(ra, rows - 1) / G;
    const int pos_b = first_pos + t0 + min(rb, rows - 1) / G;
    const int pos_max = first_pos + t0 + rlast / G;  // the warp's furthest row

    uint32_t qa[KS][4];
    {
        auto qrow = [&](int r) -> const uint32_t* {
            const int t = t0 + r / G, h = kvh * G + r % G;
            return reinterpret_cast<const uint32_t*>(
                p.q + ((static_cast<size_t>(b) * p.max_qlen + t) * p.hq + h) * D);
        };
        const bool ok_a = live && ra < rows, ok_b = live && rb < rows;
        const uint32_t* q_lo = ok_a ? qrow(ra) : nullptr;
        const uint32_t* q_hi = ok_b ? qrow(rb) : nullptr;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int k0 = (ks * 16 + c * 2) >> 1;
            qa[ks][0] = ok_a ? __ldg(q_lo + k0) : 0u;
            qa[ks][1] = ok_b ? __ldg(q_hi + k0) : 0u;
            qa[ks][2] = ok_a ? __ldg(q_lo + k0 + 4) : 0u;
            qa[ks][3] = ok_b ? __ldg(q_hi + k0 + 4) : 0u;
        }
    }
    WarpState<D> st;
    st.reset();
    bool alive = true;
    for (uint32_t it = 0; it < iters; ++it) {
        const uint32_t slot = it % STAGES;
        if (alive && !mbar_wait_bounded(full0 + 8 * slot, (it / STAGES) & 1u)) {
            record_error(p.err, kErrWaitTimeout);
            alive = false;
        }
        if (alive && live) {
#pragma unroll 1
            for (int j = 0; j < NB; ++j) {
                const int blk = static_cast<int>(it) * NB + j;
                const int k0 = blk * 16;
                if (blk >= static_cast<int>(nblk) || k0 > pos_max) break;  // warp-uniform
                const int va = max(0, min(16, pos_a - k0 + 1));
                const int vbr = max(0, min(16, pos_b - k0 + 1));
                const int vctx = min(16, ctx - k0);
                const uint32_t kb = smem_u32(smem + slot * S::kStage + j * S::kBlock);
                attend_block_rows<D>(st, qa, kb, va, vbr, vctx, p.scale_log2, lane);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * slot);
    }
    if (!alive || !live) return;

    float l0 = st.l0 + __shfl_xor_sync(0xffffffffu, st.l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    float l1 = st.l1 + __shfl_xor_sync(0xffffffffu, st.l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float inv0 = 1.f / l0, inv1 = 1.f / l1;
    auto orow = [&](int r) {
        const int t = t0 + r / G, h = kvh * G + r % G;
        return p.out + ((static_cast<size_t>(b) * p.max_qlen + t) * p.hq + h) * D;
    };
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        const int col = n * 8 + c * 2;
        if (ra < rows)
            *reinterpret_cast<uint32_t*>(orow(ra) + col) = pack_bf16x2(st.o[n][0] * inv0, st.o[n][1] * inv0);
        if (rb < rows)
            *reinterpret_cast<uint32_t*>(orow(rb) + col) = pack_bf16x2(st.o[n][2] * inv1, st.o[n][3] * inv1);
    }
}

// ---------------------------------------------------------------------------
// paged_prefill_tc: the same tiles on the fifth-generation tensor cores.
//
// CTA = (pair of tiles A, B of TQ = 128/G query tokens each, kv head,
// sequence). A tile's 128 rows (token, query head) are the M of two tcgen05
// GEMMs per step of 128 keys (8 blocks):
//   S = Q K^T  (M 128, N 128 keys, K head_dim; Q and K from shared memory)
//   O += P V   (M 128, N head_dim, K 128 keys; P from TMEM, V from shared)
// TMEM: S of tile t in columns [128 t, +128), overwritten by its P as bf16
// pairs in the first 64 of them; O of tile t in [256 + 128 t, +128). Keeping
// P in TMEM keeps it off shared memory, whose bandwidth the GEMM operands
// need. The MMAs of one thread complete in issue order, and the issuer
// runs P V(j) then S(j+1) of a tile back to back, so when a tile's S(j+1)
// has landed its P V(j) has too: the softmax of a step waits for S alone.
// While one tile's softmax runs, the tensor cores work on the other tile.
//
// Warps 0-3 are tile A's softmax, warps 4-7 tile B's: a thread owns one row
// (TMEM lane = row). They stage Q, read S from TMEM, apply the causal mask
// and the online softmax, write P and rescale O in TMEM when a row's running
// maximum grows by more than 2^8 (below that the stale maximum is kept:
// P <= 256, and the final division by the sum of the same bf16 weights is
// exact). Warp 8 streams K and V with TMA (one 16-row, 64-column box per
// block, K or V and head_dim half), each with a ring of its own, so that a
// step's K is [half][128 keys][64]: the K-major B operand of the first GEMM;
// V the same, the MN-major B operand of the second. Warp 9 allocates TMEM
// and one of its threads issues every MMA. Keys past a row's position are
// masked in S; V rows past the context in the last block are zeroed in
// shared memory before the second GEMM reads them (P is 0 there, but 0 * NaN
// would not be).

constexpr int kTcThreads = 320;
constexpr uint32_t kTcRows = 128;
constexpr uint32_t kTcKeys = 128;                  // keys per step (8 blocks)
constexpr uint32_t kTcBlocks = kTcKeys / 16;
constexpr uint32_t kTcQHalf = kTcRows * 128;       // one 64-column half of Q: 16 KiB
constexpr uint32_t kTcQ = 2 * kTcQHalf;            // 128 rows x 128 bf16
constexpr uint32_t kTcKVHalf = kTcKeys * 128;      // one half of a K or V tile: 16 KiB
constexpr uint32_t kTcKV = 2 * kTcKVHalf;          // K (or V) of one step: 32 KiB
constexpr uint32_t kTcBox = 16 * 128;              // one block's rows of one half: 2 KiB
constexpr uint32_t kTcCols = 512;                  // TMEM columns allocated

template <int STAGES>
struct TcLayout {
    static constexpr uint32_t kQ = 0;                              // Q of tile t at kQ + t * kTcQ
    static constexpr uint32_t kK = 2 * kTcQ;                       // K of stage s at kK + s * kTcKV
    static constexpr uint32_t kV = kK + STAGES * kTcKV;            // V of stage s at kV + s * kTcKV
    static constexpr uint32_t kBars = kV + STAGES * kTcKV;
    // k_full[S], k_empty[S], v_full[S], v_empty[S], per tile {s_full, p_full, q_ready}, mma_idle
    static constexpr uint32_t kTileBars = 3;
    static constexpr uint32_t kNumBars = 4 * STAGES + 2 * kTileBars + 1;
    static constexpr uint32_t kTmemSlot = kBars + 8 * kNumBars;
    static constexpr uint32_t kSmem = kTmemSlot + 16 + 1024;
};

// byte offset of 16-byte chunk c of row r in a K-major 128-row tile with
// 128-byte swizzle whose 64-column halves are `half` bytes apart
__device__ __forceinline__ uint32_t tc_chunk(uint32_t r, uint32_t c, uint32_t half) {
    return (c >> 3) * half + r * 128u + (((c & 7u) ^ (r & 7u)) << 4);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// 2^x on the special-function unit (flushes subnormal results to 0; the
// softmax weights it makes are rounded to bf16, whose smallest normal is
// 2^-126 as well)
__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// every lane of the warp agrees whether the wait completed
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity));
}

struct TcTile {
    int t0, rows;          // first query token, valid rows (0: no tile)
    uint32_t nblk, steps;  // blocks the tile sees, steps of kTcKeys
};

__device__ __forceinline__ TcTile tc_tile(int t0, int ql, int tq, int G, int first_pos) {
    TcTile t{t0, 0, 0, 0};
    if (t0 >= ql) return t;
    const int t1 = min(t0 + tq, ql);
    t.rows = (t1 - t0) * G;
    t.nblk = static_cast<uint32_t>(first_pos + t1 - 1) / 16u + 1u;
    t.steps = (t.nblk + kTcBlocks - 1) / kTcBlocks;
    return t;
}

template <int STAGES>
__global__ void __launch_bounds__(kTcThreads, 1)
    paged_prefill_tc(const __grid_constant__ CUtensorMap tmap, const PrefillParams p, uint32_t npairs) {
    using L = TcLayout<STAGES>;
    constexpr uint32_t D = 128;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const uint32_t sb = smem_u32(smem);
    const uint32_t bar0 = sb + L::kBars;
    auto k_full = [&](uint32_t s) { return bar0 + 8u * s; };
    auto k_empty = [&](uint32_t s) { return bar0 + 8u * (STAGES + s); };
    auto v_full = [&](uint32_t s) { return bar0 + 8u * (2 * STAGES + s); };
    auto v_empty = [&](uint32_t s) { return bar0 + 8u * (3 * STAGES + s); };
    auto tbar = [&](uint32_t t, uint32_t k) { return bar0 + 8u * (4 * STAGES + t * L::kTileBars + k); };
    auto s_full = [&](uint32_t t) { return tbar(t, 0); };
    auto p_full = [&](uint32_t t) { return tbar(t, 1); };
    auto q_ready = [&](uint32_t t) { return tbar(t, 2); };
    const uint32_t mma_idle = bar0 + 8u * (L::kNumBars - 1);

    // longest pairs first: the pair index is the slowest-varying one, reversed
    const uint32_t hkv = p.hkv;
    const uint32_t per_pair = hkv * p.batch;
    const uint32_t pair = npairs - 1u - blockIdx.x / per_pair;
    const uint32_t rem = blockIdx.x % per_pair;
    const int kvh = static_cast<int>(rem % hkv);
    const int b = static_cast<int>(rem / hkv);
    const int ctx = p.ctx[b];
    const int ql = p.qlen[b];
    if (ctx <= 0 || static_cast<uint32_t>(ctx) > p.pitch * 16u || ql <= 0 || ql > ctx ||
        static_cast<uint32_t>(ql) > p.max_qlen) {
        if (threadIdx.x == 0 && pair == 0 && kvh == 0) record_error(p.err, kErrBadContext);
        return;
    }
    const int G = static_cast<int>(p.group);
    const int tq = static_cast<int>(p.tile_tokens);
    const int first_pos = ctx - ql;
    const TcTile tA = tc_tile(static_cast<int>(pair) * 2 * tq, ql, tq, G, first_pos);
    if (tA.rows == 0) return;
    const TcTile tB = tc_tile(tA.t0 + tq, ql, tq, G, first_pos);
    const uint32_t nblk = max(tA.nblk, tB.nblk);
    const uint32_t nsteps = max(tA.steps, tB.steps);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(k_full(s), 1);
            mbar_init(k_empty(s), 1);
            mbar_init(v_full(s), 1);
            mbar_init(v_empty(s), 1);
        }
        for (uint32_t t = 0; t < 2; ++t) {
            mbar_init(s_full(t), 1);
            mbar_init(p_full(t), kTcRows);
            mbar_init(q_ready(t), kTcRows);
        }
        mbar_init(mma_idle, 1);
        mbar_fence_init();
    }
    if (warp == 9) {
        tc::alloc(smem_u32(tmem_slot), kTcCols);
        tc::relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 8) {
        // ---- producer (whole warp): K and V of kTcBlocks blocks per step ----
        // K and V have rings of their own (a K slot is free once the step's
        // first GEMMs have run, long before its V slot). The block ids come
        // 32 at a time, one per lane, a window ahead of their use, so no load
        // of the table sits in front of a copy; lane jj issues the copies of
        // block jj of the step.
        if (lane == 0) prefetch_tensormap(&tmap);
        const uint64_t policy = l2_policy_evict_last();  // every tile of the sequence reads the prefix
        const int32_t* row = p.tables + static_cast<size_t>(b) * p.pitch;
        auto window = [&](uint32_t w) -> int32_t {
            const uint32_t k = w * 32u + static_cast<uint32_t>(lane);
            return k < nblk ? __ldg(row + k) : 0;
        };
        int32_t win = window(0), win_next = window(1);
        uint32_t cur = 0;
        uint32_t issued_k = 0, issued_v = 0;
        bool ok = true;
        for (uint32_t j = 0; ok && j < nsteps; ++j) {
            const uint32_t s = j % STAGES;
            const uint32_t first = j * kTcBlocks;
            if (first / 32u != cur) {
                cur = first / 32u;
                win = win_next;
                win_next = window(cur + 1u);
            }
            const uint32_t nb = min(kTcBlocks, nblk - first);
            int32_t id = __shfl_sync(0xffffffffu, win, static_cast<int>((first + static_cast<uint32_t>(lane) % kTcBlocks) % 32u));
            if (static_cast<uint32_t>(id) >= p.num_blocks) {
                if (static_cast<uint32_t>(lane) < nb) record_error(p.err, kErrBadBlockId);
                id = 0;
            }
            const int r = (id * static_cast<int>(p.num_layers) + static_cast<int>(p.layer)) * 32;
            for (uint32_t kv = 0; kv < 2; ++kv) {
                const uint32_t full = kv == 0 ? k_full(s) : v_full(s);
                if (j >= STAGES && !warp_wait(kv == 0 ? k_empty(s) : v_empty(s), ((j / STAGES) - 1u) & 1u)) {
                    ok = false;
                    break;
                }
                if (lane == 0) mbar_arrive_expect_tx(full, nb * 2u * kTcBox);
                __syncwarp();
                if (static_cast<uint32_t>(lane) < nb) {
                    const uint32_t dst = sb + (kv == 0 ? L::kK : L::kV) + s * kTcKV + static_cast<uint32_t>(lane) * kTcBox;
                    for (int dh = 0; dh < 2; ++dh)
                        tma_load_4d(dst + static_cast<uint32_t>(dh) * kTcKVHalf, &tmap, full, 0,
                                    r + 16 * static_cast<int>(kv), kvh, dh, policy);
                }
                if (kv == 0)
                    ++issued_k;
                else
                    ++issued_v;
            }
        }
        if (!ok && lane == 0) record_error(p.err, kErrWaitTimeout);
        // no copy may still be landing when the CTA exits
        for (uint32_t j = issued_k > STAGES ? issued_k - STAGES : 0; j < issued_k; ++j)
            if (!warp_wait(k_full(j % STAGES), (j / STAGES) & 1u) && lane == 0) record_error(p.err, kErrWaitTimeout);
        for (uint32_t j = issued_v > STAGES ? issued_v - STAGES : 0; j < issued_v; ++j)
            if (!warp_wait(v_full(j % STAGES), (j / STAGES) & 1u) && lane == 0) record_error(p.err, kErrWaitTimeout);
    } else if (warp == 9) {
        // ---- MMA issue (one thread): per tile, P V(j) then S(j+1) ----
        if (lane == 0) {
            constexpr uint32_t idesc_s = tc::idesc_bf16_f32(kTcRows, kTcKeys, false, false);
            constexpr uint32_t idesc_o = tc::idesc_bf16_f32(kTcRows, D, false, true);
            const TcTile tiles[2] = {tA, tB};
            const uint32_t ntiles = tB.rows > 0 ? 2u : 1u;
            bool ok = mbar_wait_bounded(q_ready(0), 0) && (ntiles == 1 || mbar_wait_bounded(q_ready(1), 0));
            tc::fence_after_sync();
            // S(j) of tile t; the last tile that reads K(j) releases the slot
            auto gemm1 = [&](uint32_t t, uint32_t j) -> bool {
                const uint32_t s = j % STAGES;
                if (!mbar_wait_bounded(k_full(s), (j / STAGES) & 1u)) return false;
                tc::fence_after_sync();
                const uint32_t kb = sb + L::kK + s * kTcKV;
                const uint32_t qa = sb + L::kQ + t * kTcQ;
                for (uint32_t kk = 0; kk < D / 16; ++kk) {
                    const uint64_t ad = tc::smem_desc_sw128(qa + (kk >> 2) * kTcQHalf + (kk & 3u) * 32u, 16, 1024);
                    const uint64_t bd = tc::smem_desc_sw128(kb + (kk >> 2) * kTcKVHalf + (kk & 3u) * 32u, 16, 1024);
                    tc::mma_ss(tmem + 128u * t, ad, bd, idesc_s, kk > 0);
                }
                tc::commit(s_full(t));
                if (t + 1 == ntiles || j >= tiles[t + 1].steps) tc::commit(k_empty(s));
                return true;
            };
            for (uint32_t t = 0; ok && t < ntiles; ++t) ok = gemm1(t, 0);
            for (uint32_t j = 0; ok && j < nsteps; ++j) {
                const uint32_t s = j % STAGES;
                if (!mbar_wait_bounded(v_full(s), (j / STAGES) & 1u)) {
                    ok = false;
                    break;
                }
                const uint32_t vb = sb + L::kV + s * kTcKV;
                for (uint32_t t = 0; ok && t < ntiles; ++t) {
                    if (j >= tiles[t].steps) continue;
                    if (!mbar_wait_bounded(p_full(t), j & 1u)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t nb = min(kTcBlocks, tiles[t].nblk - j * kTcBlocks);
                    for (uint32_t kk = 0; kk < nb; ++kk) {
                        const uint64_t bd = tc::smem_desc_sw128(vb + kk * kTcBox, kTcKVHalf, 1024);
                        tc::mma_ts(tmem + 256u + 128u * t, tmem + 128u * t + kk * 8u, bd, idesc_o, j > 0 || kk > 0);
                    }
                    // the last tile that reads V(j) releases the slot
                    if (t + 1 == ntiles || j >= tiles[t + 1].steps) tc::commit(v_empty(s));
                    if (j + 1 < tiles[t].steps) ok = gemm1(t, j + 1);
                    else tc::commit(s_full(t));  // the tile's last P V has landed
                }
            }
            if (!ok) record_error(p.err, kErrWaitTimeout);
            // every MMA issued has completed before TMEM is released
            tc::commit(mma_idle);
            if (!mbar_wait_bounded(mma_idle, 0)) record_error(p.err, kErrWaitTimeout);
        }
    } else {
        // ---- softmax: thread = row r of tile t ----
        const uint32_t t = static_cast<uint32_t>(warp) >> 2;
        const TcTile tile = t == 0 ? tA : tB;
        const uint32_t r = static_cast<uint32_t>(threadIdx.x) & 127u;
        const bool have = tile.rows > 0;
        const int rr = have ? min(static_cast<int>(r), tile.rows - 1) : 0;
        const int tok = tile.t0 + rr / G;
        const int head = kvh * G + rr % G;
        const bool live_row = static_cast<int>(r) < tile.rows;
        const uint32_t qs = sb + L::kQ + t * kTcQ;
        if (have) {
            const uint4* qrow = reinterpret_cast<const uint4*>(
                p.q + ((static_cast<size_t>(b) * p.max_qlen + tok) * p.hq + head) * D);
            uint4 qv[16];
#pragma unroll
            for (uint32_t c = 0; c < 16; ++c) qv[c] = live_row ? __ldg(qrow + c) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (uint32_t c = 0; c < 16; ++c) st_shared_v4(qs + tc_chunk(r, c, kTcQHalf), qv[c]);
            tc::fence_async_smem();
            mbar_arrive(q_ready(t));
        }
        const int pos = first_pos + tok;  // position of this row's token
        const uint32_t lane_base = tmem + (((static_cast<uint32_t>(warp) & 3u) * 32u) << 16);
        const uint32_t s_col = 128u * t, o_col = 256u + 128u * t;
        const float sl2 = p.scale_log2;
        const float grow_raw = 8.f / sl2;  // 2^8 in the exp2 domain, in raw score units
        float m_used = -INFINITY, l = 0.f;
        bool ok = true;
        // the block holding the last context key, if this tile reads it and
        // it is partly past the context: its V rows past ctx are zeroed
        const uint32_t partial_blk = static_cast<uint32_t>(ctx - 1) / 16u;
        const bool zero_tail = (ctx & 15) != 0 && partial_blk == tile.nblk - 1u;
        for (uint32_t j = 0; have && ok && j < tile.steps; ++j) {
            // S(j) landed, and with it the P V of step j-1 (issued before it)
            if (!warp_wait(s_full(t), j & 1u)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            uint32_t sv[kTcKeys];
#pragma unroll
            for (uint32_t c = 0; c < kTcKeys / 16; ++c)
                tc::ld16(lane_base + s_col + c * 16u, *reinterpret_cast<uint32_t(*)[16]>(&sv[c * 16]));
            tc::wait_ld();
            tc::reg_fence(sv);
            const int lim = pos - static_cast<int>(j * kTcKeys);  // columns <= lim are visible
            if (lim < static_cast<int>(kTcKeys) - 1) {
#pragma unroll
                for (int c = 0; c < static_cast<int>(kTcKeys); ++c)
                    if (c > lim) sv[c] = __float_as_uint(-INFINITY);
            }
            // eight independent chains, then a tree
            float m8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) m8[e] = __uint_as_float(sv[e]);
#pragma unroll
            for (int c = 8; c < static_cast<int>(kTcKeys); ++c) m8[c & 7] = fmaxf(m8[c & 7], __uint_as_float(sv[c]));
            const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                                   fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
            const bool grow = mx > m_used + grow_raw;
            float factor = 1.f;
            if (grow) {
                factor = exp2f((m_used - mx) * sl2);  // 0 on the first step
                l *= factor;
                m_used = mx;
            }
            if (j > 0 && __any_sync(0xffffffffu, grow)) {
                // O holds steps < j (their P V landed before S(j)): rescale it
#pragma unroll 1
                for (uint32_t c = 0; c < D / 16; ++c) {
                    uint32_t v[16];
                    tc::ld16(lane_base + o_col + c * 16u, v);
                    tc::wait_ld();
                    tc::reg_fence(v);
#pragma unroll
                    for (int e = 0; e < 16; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * factor);
                    tc::st16(lane_base + o_col + c * 16u, v);
                }
            }
            const float msl = m_used * sl2;
            float sum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (uint32_t c = 0; c < kTcKeys / 32; ++c) {
                uint32_t w[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    w[e] = pack_bf16x2(ex2_ftz(fmaf(__uint_as_float(sv[c * 32 + 2 * e]), sl2, -msl)),
                                       ex2_ftz(fmaf(__uint_as_float(sv[c * 32 + 2 * e + 1]), sl2, -msl)));
                    // the sum takes the bf16 values the MMA multiplies, so a
                    // row dominated by one key gives back its V exactly
                    sum[e & 3] += __uint_as_float(w[e] << 16) + __uint_as_float(w[e] & 0xFFFF0000u);
                }
                tc::st16(lane_base + s_col + c * 16u, w);  // P over the S just read
            }
            l += (sum[0] + sum[1]) + (sum[2] + sum[3]);
            if (zero_tail && j == tile.steps - 1u) {
                const uint32_t jj = partial_blk - j * kTcBlocks;
                const uint32_t first = static_cast<uint32_t>(ctx & 15);
                const uint32_t n16 = (16u - first) * 8u;  // 16-byte chunks per half
                const uint32_t vbase = sb + L::kV + (j % STAGES) * kTcKV + jj * kTcBox;
                for (uint32_t u = r; u < 2u * n16; u += kTcRows) {
                    const uint32_t dh = u / n16, wq = u % n16;
                    st_shared_v4(vbase + dh * kTcKVHalf + (first + wq / 8u) * 128u + (wq % 8u) * 16u,
                                 make_uint4(0, 0, 0, 0));
                }
                tc::fence_async_smem();
            }
            tc::wait_st();
            tc::fence_before_sync();
            mbar_arrive(p_full(t));
        }
        if (have && ok) {
            // the tile's last P V: the issuer commits s_full once more after it
            ok = warp_wait(s_full(t), tile.steps & 1u);
            if (!ok) {
                record_error(p.err, kErrWaitTimeout);
            } else {
                tc::fence_after_sync();
                const float inv = 1.f / l;
                uint4* orow = reinterpret_cast<uint4*>(
                    p.out + ((static_cast<size_t>(b) * p.max_qlen + tok) * p.hq + head) * D);
                uint32_t ov[D];
#pragma unroll
                for (uint32_t c = 0; c < D / 16; ++c)
                    tc::ld16(lane_base + o_col + c * 16u, *reinterpret_cast<uint32_t(*)[16]>(&ov[c * 16]));
                tc::wait_ld();
                tc::reg_fence(ov);
                if (live_row) {
#pragma unroll
                    for (uint32_t c = 0; c < D / 8; ++c) {
                        uint32_t w[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            w[e] = pack_bf16x2(__uint_as_float(ov[8 * c + 2 * e]) * inv,
                                               __uint_as_float(ov[8 * c + 2 * e + 1]) * inv);
                        orow[c] = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
        } else if (have) {
            record_error(p.err, kErrWaitTimeout);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 9) tc::dealloc(tmem, kTcCols);
}

// ---------------------------------------------------------------------------

constexpr int kGenWarps = 4;
constexpr int kGenDimPerLane = 8;  // head_dim <= 256

struct PrefillGenericParams {
    const uint8_t* pool;
    size_t block_stride;
    const int32_t* tables;
    const int32_t* ctx;
    const int32_t* qlen;
    const void* q;
    void* out;
    int32_t* err;
    uint32_t pitch, num_blocks, tokens_per_block, num_kv_heads, head_dim, layer, hq, group, max_qlen;
    float scale;
};

template <typename T>
__global__ void __launch_bounds__(kGenWarps * 32) paged_prefill_generic(const PrefillGenericParams p) {
    __shared__ float sm_ml[kGenWarps][2];
    __shared__ float sm_acc[kGenWarps][kGenDimPerLane * 32];
    const int b = blockIdx.z, qh = blockIdx.y, t = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ctx = p.ctx[b], ql = p.qlen[b];
    if (ctx <= 0 || static_cast<uint32_t>(ctx) > p.pitch * p.tokens_per_block || ql <= 0 || ql > ctx ||
        static_cast<uint32_t>(ql) > p.max_qlen) {
        if (threadIdx.x == 0 && t == 0 && qh == 0) record_error(p.err, kErrBadContext);
        return;
    }
    if (t >= ql) return;
    const int visible = ctx - ql + t + 1;  // keys [0, pos]
    const uint32_t D = p.head_dim;
    const uint32_t kvh = qh / p.group;
    const size_t qoff = ((static_cast<size_t>(b) * p.max_qlen + t) * p.hq + qh) * D;
    const T* q = static_cast<const T*>(p.q) + qoff;
    float qr[kGenDimPerLane], acc[kGenDimPerLane];
#pragma unroll
    for (int i = 0; i < kGenDimPerLane; ++i) {
        const uint32_t d = lane + 32 * i;
        qr[i] = d < D ? to_float<T>(q[d]) : 0.f;
        acc[i] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    const size_t token_stride = static_cast<size_t>(p.num_kv_heads) * D;
    const size_t stream_stride = token_stride * p.tokens_per_block;
    const size_t layer_off = static_cast<size_t>(p.layer) * 2 * stream_stride + kvh * D;
    const int32_t* row = p.tables + static_cast<size_t>(b) * p.pitch;
    for (int k = warp; k < visible; k += kGenWarps) {
        int32_t id = row[k / p.tokens_per_block];
        if (static_cast<uint32_t>(id) >= p.num_blocks) {
            if (lane == 0) record_error(p.err, kErrBadBlockId);
            id = 0;
        }
        const T* kp = reinterpret_cast<const T*>(p.pool + static_cast<size_t>(id) * p.block_stride) + layer_off +
                      (k % p.tokens_per_block) * token_stride;
        const T* vp = kp + stream_stride;
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < kGenDimPerLane; ++i) {
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
        for (int i = 0; i < kGenDimPerLane; ++i) {
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
    for (int i = 0; i < kGenDimPerLane; ++i) sm_acc[warp][lane + 32 * i] = acc[i];
    __syncthreads();
    if (warp != 0) return;
    float M = -INFINITY;
    for (int w = 0; w < kGenWarps; ++w) M = fmaxf(M, sm_ml[w][0]);
    float L = 0.f, wt[kGenWarps];
    for (int w = 0; w < kGenWarps; ++w) {
        wt[w] = (sm_ml[w][0] == -INFINITY) ? 0.f : expf(sm_ml[w][0] - M);
        L += wt[w] * sm_ml[w][1];
    }
    T* out = static_cast<T*>(p.out) + qoff;
    for (uint32_t d = lane; d < D; d += 32) {
        float a = 0.f;
        for (int w = 0; w < kGenWarps; ++w) a += wt[w] * sm_acc[w][d];
        out[d] = from_float<T>(a / L);
    }
}

template <int D, int NB, int STAGES>
int launch_prefill_fast(const qvp_prefill_args& a, const PrefillParams& pp, cudaStream_t st) {
    using S = PrefillShape<D, NB, STAGES>;
    static std::atomic<std::uint64_t> attr_done{0};
    auto kern = paged_prefill_fast<D, NB, STAGES>;
    int rc = set_smem_limit_once(attr_done, reinterpret_cast<const void*>(kern), static_cast<int>(S::kSmem),
                                 "cudaFuncSetAttribute(prefill)");
    if (rc != QVP_OK) return rc;
    CUtensorMap map;
    rc = encode_pool_map(a.pool, a.num_blocks, a.shape, 1, &map);
    if (rc != QVP_OK) return rc;
    const dim3 grid(ceil_div(a.max_query_len, pp.tile_tokens), a.shape.num_kv_heads, a.batch);
    kern<<<grid, kPrefillThreads, S::kSmem, st>>>(map, pp);
    return check_cuda(cudaGetLastError(), "launch prefill");
}

template <int STAGES>
int launch_prefill_tc(const qvp_prefill_args& a, const PrefillParams& pp, cudaStream_t st) {
    using L = TcLayout<STAGES>;
    static_assert(L::kSmem <= 232448u - 1024u, "tcgen05 prefill shared memory");
    static std::atomic<std::uint64_t> attr_done{0};
    auto kern = paged_prefill_tc<STAGES>;
    int rc = set_smem_limit_once(attr_done, reinterpret_cast<const void*>(kern), static_cast<int>(L::kSmem),
                                 "cudaFuncSetAttribute(tcgen05 prefill)");
    if (rc != QVP_OK) return rc;
    CUtensorMap map;
    rc = encode_pool_map_box(a.pool, a.num_blocks, a.shape, 1, 16, 1, &map);
    if (rc != QVP_OK) return rc;
    const uint32_t npairs = ceil_div(ceil_div(a.max_query_len, pp.tile_tokens), 2);
    const uint64_t ctas = static_cast<uint64_t>(npairs) * pp.hkv * pp.batch;
    if (ctas > 0x7fffffffull) return fail(QVP_ERR_UNSUPPORTED, "prefill grid of %llu CTAs", (unsigned long long)ctas);
    kern<<<static_cast<unsigned>(ctas), kTcThreads, L::kSmem, st>>>(map, pp, npairs);
    return check_cuda(cudaGetLastError(), "launch tcgen05 prefill");
}

}  // namespace

}  // namespace qvp

using namespace qvp;

extern "C" int qvp_prefill(const qvp_prefill_args* args, qvp_stream_t stream) {
    if (args == nullptr) return fail(QVP_ERR_INVALID, "null argument");
    const qvp_prefill_args& a = *args;
    const qvp_block_shape& sh = a.shape;
    if (sh.tokens_per_block == 0 || sh.num_layers == 0 || sh.num_kv_heads == 0 || sh.head_dim == 0)
        return fail(QVP_ERR_INVALID, "block shape has a zero field");
    const uint32_t elem = a.dtype == QVP_DTYPE_F32 ? 4u : a.dtype == QVP_DTYPE_BF16 ? 2u : 0u;
    if (elem == 0 || sh.bytes_per_element != elem) return fail(QVP_ERR_INVALID, "dtype does not match the shape");
    if (a.layer >= sh.num_layers) return fail(QVP_ERR_INVALID, "layer %u >= num_layers %u", a.layer, sh.num_layers);
    if (a.num_query_heads == 0 || a.num_query_heads % sh.num_kv_heads != 0)
        return fail(QVP_ERR_INVALID, "num_query_heads is not a positive multiple of num_kv_heads");
    if (a.batch == 0) return QVP_OK;
    if (a.pool == nullptr || a.block_tables == nullptr || a.context_lens == nullptr || a.query_lens == nullptr ||
        a.query == nullptr || a.out == nullptr)
        return fail(QVP_ERR_INVALID, "null pool, table, length, query or output pointer");
    if (a.max_query_len == 0 || a.max_blocks_per_seq == 0 || a.num_blocks == 0)
        return fail(QVP_ERR_INVALID, "zero max_query_len, table pitch or pool size");
    const size_t block_bytes = qvp_block_bytes(&sh);
    if (a.block_stride < block_bytes) return fail(QVP_ERR_INVALID, "block_stride below the block size");
    if (sh.head_dim > 256) return fail(QVP_ERR_UNSUPPORTED, "head_dim %u above 256", sh.head_dim);
    if (a.batch > 65535 || a.num_query_heads > 65535 || a.max_query_len > 0x7fffffffu)
        return fail(QVP_ERR_UNSUPPORTED, "batch, heads or query length too large");
    const uint32_t G = a.num_query_heads / sh.num_kv_heads;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const bool fast = a.dtype == QVP_DTYPE_BF16 && sh.tokens_per_block == 16 &&
                      (sh.head_dim == 64 || sh.head_dim == 128) && G <= 16 && a.block_stride == block_bytes &&
                      (reinterpret_cast<uintptr_t>(a.pool) & 15u) == 0 &&
                      (reinterpret_cast<uintptr_t>(a.query) & 3u) == 0 &&
                      (reinterpret_cast<uintptr_t>(a.out) & 3u) == 0 &&
                      static_cast<uint64_t>(a.num_blocks) * sh.num_layers * 32u < (1ull << 31);
    if (fast) {
        PrefillParams pp;
        pp.tables = a.block_tables;
        pp.ctx = a.context_lens;
        pp.qlen = a.query_lens;
        pp.q = static_cast<const __nv_bfloat16*>(a.query);
        pp.out = static_cast<__nv_bfloat16*>(a.out);
        pp.err = a.error_word;
        pp.pitch = a.max_blocks_per_seq;
        pp.num_blocks = a.num_blocks;
        pp.layer = a.layer;
        pp.num_layers = sh.num_layers;
        pp.hq = a.num_query_heads;
        pp.group = G;
        pp.tile_tokens = static_cast<uint32_t>(kPrefillRows) / G;
        pp.max_qlen = a.max_query_len;
        pp.batch = a.batch;
        pp.hkv = sh.num_kv_heads;
        pp.scale_log2 = a.scale * 1.4426950408889634f;  // log2(e)
        // head_dim 128 with 16-byte aligned rows: the tcgen05 kernel
        if (sh.head_dim == 128 && (reinterpret_cast<uintptr_t>(a.query) & 15u) == 0 &&
            (reinterpret_cast<uintptr_t>(a.out) & 15u) == 0)
            return launch_prefill_tc<2>(a, pp, st);
        return sh.head_dim == 128 ? launch_prefill_fast<128, 4, 5>(a, pp, st) : launch_prefill_fast<64, 4, 10>(a, pp, st);
    }
    PrefillGenericParams gp;
    gp.pool = static_cast<const uint8_t*>(a.pool);
    gp.block_stride = a.block_stride;
    gp.tables = a.block_tables;
    gp.ctx = a.context_lens;
    gp.qlen = a.query_lens;
    gp.q = a.query;
    gp.out = a.out;
    gp.err = a.error_word;
    gp.pitch = a.max_blocks_per_seq;
    gp.num_blocks = a.num_blocks;
    gp.tokens_per_block = sh.tokens_per_block;
    gp.num_kv_heads = sh.num_kv_heads;
    gp.head_dim = sh.head_dim;
    gp.layer = a.layer;
    gp.hq = a.num_query_heads;
    gp.group = G;
    gp.max_qlen = a.max_query_len;
    gp.scale = a.scale;
    const dim3 grid(a.max_query_len, a.num_query_heads, a.batch);
    if (a.dtype == QVP_DTYPE_F32)
        paged_prefill_generic<float><<<grid, kGenWarps * 32, 0, st>>>(gp);
    else
        paged_prefill_generic<__nv_bfloat16><<<grid, kGenWarps * 32, 0, st>>>(gp);
    return check_cuda(cudaGetLastError(), "launch generic prefill");
}
