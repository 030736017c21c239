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
        pp.scale_log2 = a.scale * 1.4426950408889634f;  // log2(e)
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
