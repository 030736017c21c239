// Tile helpers shared by the decode and prefill kernels: addressing of the
// 128-byte-swizzled K/V boxes that TMA writes to shared memory, masking of V
// slots past a context, and the online-softmax state of one warp.
#pragma once

#include "qvp_device.cuh"

namespace qvp {

// Byte address of element chunk `chunk` (8 bf16) of token `t` inside the
// swizzled box [dh][hh][t][64] written by TMA with 128-byte swizzle.
__device__ __forceinline__ uint32_t box_addr(uint32_t base, int row_group, int t, int chunk) {
    const int r = row_group * 16 + t;
    return base + static_cast<uint32_t>(r * 128 + ((chunk ^ (t & 7)) << 4));
}

__device__ __forceinline__ uint32_t mask_pair(uint32_t x, int t0, int valid) {
    const uint32_t lo = (t0 < valid) ? 0x0000FFFFu : 0u;
    const uint32_t hi = (t0 + 1 < valid) ? 0xFFFF0000u : 0u;
    return x & (lo | hi);
}

// Online-softmax state of one consumer warp: query rows g and g+8 of its
// GQA group (row max in the log2 domain, lane-partial row sums) and the
// m16n8 accumulator fragments of out[16][D].
template <int D>
struct WarpState {
    float o[D / 8][4];
    float m0, m1, l0, l1;

    __device__ __forceinline__ void reset() {
#pragma unroll
        for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
        m0 = m1 = -INFINITY;
        l0 = l1 = 0.f;
    }
};

}  // namespace qvp
