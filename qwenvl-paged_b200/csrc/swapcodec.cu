// Compressed swap slots: lossless block compression between the device pool
// and swap slots in host memory, so fewer bytes cross PCIe. A slot's first
// bytes (its head: all of a coded block whose escapes are few) go to a
// device staging row that the copy engines move; the rest (the tail of a
// raw block or of one with many escapes) the kernel writes or reads itself
// through mapped pinned memory.
//
// The swap moves the bytes of HostSwapBackend::store / load
// (phhuang191129/QwenVL-Paged src/SwapBackend.cpp:10-39) and the reference
// names compression of swapped blocks as the place to save link time
// (docs/architecture.md:128-130). K and V are bf16: a value's high byte (sign
// and the top seven exponent bits) takes few distinct values in a block,
// while its low byte (the last exponent bit and the mantissa) is close to
// random. The slot format codes the high byte with a per-block dictionary of
// its 15 most frequent values (4 bits per value, code 15 = escape) and keeps
// the low byte as is:
//
//   [ 0,16)  header: u32 format ('QVP1' compressed, 'QVP0' raw), u32 escapes,
//            u32 bytes used (header included), u32 0
//   compressed (n = block_bytes / 2 values):
//   [16,32)  dictionary: code c < 15 -> high byte
//   [32, 32 + n/2)             codes, value i in byte i/2 (even i: low nibble)
//   [32 + n/2, 32 + 3n/2)      low bytes
//   [32 + 3n/2, + 4*escapes)   escapes: u32 (index << 8 | high byte), any order
//   raw: [16, 16 + block_bytes) the block's bytes
//
// A block is stored raw when coding would not make it smaller (more than
// n/8 - 4 escapes) or the block size does not suit the layout. N(0,1) bf16
// blocks code to about 0.75 of their size. Both directions are exact for
// any bytes.
#include "qvp_device.cuh"
#include "qvp_internal.h"

namespace qvp {

namespace {

constexpr int kCodecThreads = 256;
constexpr uint32_t kFormatCompressed = 0x31505651u;  // "QVP1"
constexpr uint32_t kFormatRaw = 0x30505651u;         // "QVP0"

__host__ __device__ constexpr size_t slot_bytes_for(size_t block_bytes) { return (block_bytes + 16 + 15) / 16 * 16; }

// The coded layout needs 16 values per 32-byte unit (8-byte aligned low-byte
// words) and indices that fit 24 bits.
__host__ __device__ constexpr bool codable(size_t block_bytes) {
    return block_bytes % 32 == 0 && block_bytes / 2 < (1u << 24);
}

// Where byte o of a slot lives: the first head_bytes in the list entry's head
// (a staging row the copy engines move), the rest in the slot's tail (mapped
// host memory the kernel reaches over PCIe). head_bytes is a multiple of 16
// and every access is at most 16 bytes at its own alignment, so none
// straddles the two.
struct SlotBytes {
    uint8_t* head;
    uint8_t* tail;
    uint32_t head_bytes;
    __device__ uint8_t* at(uint32_t o) const { return o < head_bytes ? head + o : tail + (o - head_bytes); }
};

// One CTA per block: short CTAs let a decode launched meanwhile (on a stream
// of higher priority) take SMs as soon as blocks finish.
__global__ void __launch_bounds__(kCodecThreads) compress_blocks_kernel(
    const uint8_t* __restrict__ pool, size_t stride, uint32_t num_blocks, uint32_t block_bytes,
    const int32_t* __restrict__ ids, const int32_t* __restrict__ slots, uint8_t* heads, uint32_t head_bytes,
    uint8_t* tails, size_t tail_stride, uint32_t num_slots, unsigned long long* moved, int32_t* err) {
    __shared__ uint32_t hist[256];
    __shared__ uint8_t code_of[256];
    __shared__ uint32_t s_dict[4];
    __shared__ uint32_t s_escapes, s_next_escape;
    const uint32_t tid = threadIdx.x, lane = tid & 31u;
    const uint32_t nval = block_bytes / 2;
    const uint32_t nvec = block_bytes / 16;  // 8 values per uint4
    const uint32_t b = blockIdx.x;
    const int32_t id = ids[b];
    const int32_t slot = slots[b];
    if (static_cast<uint32_t>(id) >= num_blocks || static_cast<uint32_t>(slot) >= num_slots) {
        if (tid == 0) record_error(err, kErrBadBlockId);
        return;
    }
    const uint4* src = reinterpret_cast<const uint4*>(pool + static_cast<size_t>(id) * stride);
    const SlotBytes out{heads + static_cast<size_t>(b) * head_bytes,
                        tails == nullptr ? nullptr : tails + static_cast<size_t>(slot) * tail_stride, head_bytes};
    const bool can_code = codable(block_bytes);
    hist[tid] = 0;
    if (tid == 0) {
        s_escapes = 0;
        s_next_escape = 0;
    }
    if (tid < 4) s_dict[tid] = 0;
    __syncthreads();
    if (can_code) {
        // warp-aggregated histogram: one shared atomic per distinct high byte
        // of a warp's 32 values (a K/V block has few)
        for (uint32_t base = 0; base < nvec; base += kCodecThreads) {
            const uint32_t w = base + tid;
            const bool live = w < nvec;
            const unsigned mask = __ballot_sync(0xffffffffu, live);
            if (!live) continue;
            const uint4 v = src[w];
            const uint32_t x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t hi = (x[k >> 1] >> ((k & 1) ? 24 : 8)) & 0xffu;
                const unsigned peers = __match_any_sync(mask, hi);
                if (lane == static_cast<uint32_t>(__ffs(peers) - 1)) atomicAdd(&hist[hi], __popc(peers));
            }
        }
    }
    __syncthreads();
    // rank of each high byte by frequency (ties: smaller byte first); the 15
    // most frequent present ones get codes 0..14
    {
        const uint32_t c = hist[tid];
        uint32_t r = 0;
        for (uint32_t u = 0; u < 256; ++u) {
            const uint32_t cu = hist[u];
            r += (cu > c || (cu == c && u < tid)) ? 1u : 0u;
        }
        const bool coded = c > 0 && r < 15;
        code_of[tid] = coded ? static_cast<uint8_t>(r) : 15u;
        if (coded) reinterpret_cast<uint8_t*>(s_dict)[r] = static_cast<uint8_t>(tid);
        if (!coded && c > 0) atomicAdd(&s_escapes, c);
    }
    __syncthreads();
    const uint32_t escapes = s_escapes;
    const size_t coded_bytes = 32 + static_cast<size_t>(nval) * 3 / 2 + static_cast<size_t>(escapes) * 4;
    const bool raw = !can_code || coded_bytes >= 16 + static_cast<size_t>(block_bytes);
    const uint32_t used = raw ? 16u + block_bytes : static_cast<uint32_t>(coded_bytes);
    if (raw) {
        if (tid == 0) *reinterpret_cast<uint4*>(out.at(0)) = make_uint4(kFormatRaw, 0u, used, 0u);
        for (uint32_t w = tid; w < nvec; w += kCodecThreads)
            *reinterpret_cast<uint4*>(out.at(16 + 16 * w)) = src[w];
    } else {
        if (tid == 0) {
            *reinterpret_cast<uint4*>(out.at(0)) = make_uint4(kFormatCompressed, escapes, used, 0u);
            *reinterpret_cast<uint4*>(out.at(16)) = make_uint4(s_dict[0], s_dict[1], s_dict[2], s_dict[3]);
        }
        const uint32_t lows_at = 32 + nval / 2, esc_at = 32 + nval / 2 * 3;
        for (uint32_t w = tid; w < nvec; w += kCodecThreads) {
            const uint4 v = src[w];
            const uint32_t x[4] = {v.x, v.y, v.z, v.w};
            uint32_t code_word = 0, lo0 = 0, lo1 = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t val = (x[k >> 1] >> ((k & 1) * 16)) & 0xffffu;
                const uint32_t hi = val >> 8, lo = val & 0xffu;
                const uint32_t cd = code_of[hi];
                code_word |= cd << (4 * k);
                if (k < 4)
                    lo0 |= lo << (8 * k);
                else
                    lo1 |= lo << (8 * (k - 4));
                if (cd == 15u) {
                    const uint32_t e = atomicAdd(&s_next_escape, 1u);
                    *reinterpret_cast<uint32_t*>(out.at(esc_at + 4 * e)) = ((w * 8 + k) << 8) | hi;
                }
            }
            *reinterpret_cast<uint32_t*>(out.at(32 + 4 * w)) = code_word;
            *reinterpret_cast<uint2*>(out.at(lows_at + 8 * w)) = make_uint2(lo0, lo1);
        }
    }
    if (tid == 0 && moved != nullptr) {
        atomicAdd(moved, static_cast<unsigned long long>(used));
        if (used > head_bytes) atomicAdd(moved + 1, static_cast<unsigned long long>(used - head_bytes));
    }
}

__global__ void __launch_bounds__(kCodecThreads) decompress_blocks_kernel(
    uint8_t* __restrict__ pool, size_t stride, uint32_t num_blocks, uint32_t block_bytes,
    const int32_t* __restrict__ ids, const int32_t* __restrict__ slots, const uint8_t* heads, uint32_t head_bytes,
    const uint8_t* tails, size_t tail_stride, uint32_t num_slots, unsigned long long* moved, int32_t* err) {
    __shared__ uint4 s_head;
    __shared__ uint32_t s_dict[4];
    const uint32_t tid = threadIdx.x;
    const uint32_t nval = block_bytes / 2;
    const uint32_t nvec = block_bytes / 16;
    const uint32_t b = blockIdx.x;
    const int32_t id = ids[b];
    const int32_t slot = slots[b];
    if (static_cast<uint32_t>(id) >= num_blocks || static_cast<uint32_t>(slot) >= num_slots) {
        if (tid == 0) record_error(err, kErrBadBlockId);
        return;
    }
    // read-only through the same addressing as the coder
    const SlotBytes in{const_cast<uint8_t*>(heads) + static_cast<size_t>(b) * head_bytes,
                       tails == nullptr ? nullptr
                                        : const_cast<uint8_t*>(tails) + static_cast<size_t>(slot) * tail_stride,
                       head_bytes};
    uint8_t* blk = pool + static_cast<size_t>(id) * stride;
    if (tid == 0) {
        s_head = *reinterpret_cast<const uint4*>(in.at(0));
        const uint4 d = *reinterpret_cast<const uint4*>(in.at(16));
        s_dict[0] = d.x;
        s_dict[1] = d.y;
        s_dict[2] = d.z;
        s_dict[3] = d.w;
    }
    __syncthreads();
    const uint4 head = s_head;
    const uint8_t* dict = reinterpret_cast<const uint8_t*>(s_dict);
    uint4* dst = reinterpret_cast<uint4*>(blk);
    const bool coded = head.x == kFormatCompressed && codable(block_bytes) && head.y <= nval &&
                       head.z == 32 + nval / 2 * 3 + 4 * head.y;
    const bool raw = head.x == kFormatRaw && head.z == 16 + block_bytes;
    if (!coded && !raw) {
        if (tid == 0) record_error(err, kErrBadBlockId);  // not a slot this codec wrote
        return;
    }
    if (tid == 0 && moved != nullptr) {
        atomicAdd(moved, static_cast<unsigned long long>(head.z));
        if (head.z > head_bytes) atomicAdd(moved + 1, static_cast<unsigned long long>(head.z - head_bytes));
    }
    if (raw) {
        for (uint32_t w = tid; w < nvec; w += kCodecThreads)
            dst[w] = *reinterpret_cast<const uint4*>(in.at(16 + 16 * w));
        return;
    }
    const uint32_t lows_at = 32 + nval / 2, esc_at = 32 + nval / 2 * 3;
    for (uint32_t w = tid; w < nvec; w += kCodecThreads) {
        const uint32_t cw = *reinterpret_cast<const uint32_t*>(in.at(32 + 4 * w));
        const uint2 lw = *reinterpret_cast<const uint2*>(in.at(lows_at + 8 * w));
        uint32_t y[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t lword = j < 2 ? lw.x : lw.y;
            const uint32_t c0 = (cw >> (8 * j)) & 15u, c1 = (cw >> (8 * j + 4)) & 15u;
            const uint32_t h0 = c0 < 15u ? dict[c0] : 0u, h1 = c1 < 15u ? dict[c1] : 0u;
            const uint32_t l0 = (lword >> (16 * (j & 1))) & 0xffu, l1 = (lword >> (16 * (j & 1) + 8)) & 0xffu;
            y[j] = (h0 << 8) | l0 | (((h1 << 8) | l1) << 16);
        }
        dst[w] = make_uint4(y[0], y[1], y[2], y[3]);
    }
    __syncthreads();  // every value is written before its escape lands
    for (uint32_t e = tid; e < head.y; e += kCodecThreads) {
        const uint32_t x = *reinterpret_cast<const uint32_t*>(in.at(esc_at + 4 * e));
        const uint32_t idx = x >> 8;
        if (idx < nval) blk[2 * static_cast<size_t>(idx) + 1] = static_cast<uint8_t>(x & 0xffu);
    }
}

int codec_check(const void* pool, size_t block_stride, size_t block_bytes, const int32_t* ids, const int32_t* slots,
                uint32_t n, const void* heads, size_t head_bytes, const void* tails, size_t tail_stride) {
    if (pool == nullptr || ids == nullptr || slots == nullptr)
        return fail(QVP_ERR_INVALID, "null pool, id list or slot list");
    if (block_bytes == 0 || block_bytes % 16 != 0 || block_bytes > 0x7fffffffu)
        return fail(QVP_ERR_INVALID, "block bytes %zu not a positive multiple of 16", block_bytes);
    if (block_bytes > block_stride) return fail(QVP_ERR_INVALID, "block bytes exceed the stride");
    if (head_bytes % 16 != 0 || tail_stride % 16 != 0 || head_bytes > 0x7fffffffu)
        return fail(QVP_ERR_INVALID, "head bytes and tail stride must be multiples of 16");
    const size_t need = slot_bytes_for(block_bytes);
    if (head_bytes + tail_stride < need)
        return fail(QVP_ERR_INVALID, "head bytes + tail stride %zu below qvp_swap_slot_bytes (%zu)",
                    head_bytes + tail_stride, need);
    if (head_bytes > 0 && heads == nullptr) return fail(QVP_ERR_INVALID, "null heads with head bytes > 0");
    if (head_bytes < need && tails == nullptr) return fail(QVP_ERR_INVALID, "null tails for slots longer than a head");
    if (n > 0x7fffffffu) return fail(QVP_ERR_INVALID, "too many blocks in one call");
    if ((reinterpret_cast<uintptr_t>(pool) & 15u) != 0 || block_stride % 16 != 0 ||
        (reinterpret_cast<uintptr_t>(heads) & 15u) != 0 || (reinterpret_cast<uintptr_t>(tails) & 15u) != 0)
        return fail(QVP_ERR_INVALID, "pool, stride, heads or tails not 16-byte aligned");
    return QVP_OK;
}

}  // namespace

}  // namespace qvp

using namespace qvp;

extern "C" size_t qvp_swap_slot_bytes(size_t block_bytes) { return slot_bytes_for(block_bytes); }

extern "C" int qvp_compress_blocks(const void* pool, size_t block_stride, uint32_t num_blocks, size_t block_bytes,
                                   const int32_t* ids, const int32_t* slots, uint32_t n, void* heads,
                                   size_t head_bytes, void* tails, size_t tail_stride, uint32_t num_slots,
                                   unsigned long long* bytes_moved, int32_t* error_word, qvp_stream_t stream) {
    if (n == 0) return QVP_OK;
    int rc = codec_check(pool, block_stride, block_bytes, ids, slots, n, heads, head_bytes, tails, tail_stride);
    if (rc != QVP_OK) return rc;
    compress_blocks_kernel<<<n, kCodecThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(pool), block_stride, num_blocks, static_cast<uint32_t>(block_bytes), ids, slots,
        static_cast<uint8_t*>(heads), static_cast<uint32_t>(head_bytes), static_cast<uint8_t*>(tails), tail_stride,
        num_slots, bytes_moved, error_word);
    return check_cuda(cudaGetLastError(), "launch compress_blocks");
}

extern "C" int qvp_decompress_blocks(void* pool, size_t block_stride, uint32_t num_blocks, size_t block_bytes,
                                     const int32_t* ids, const int32_t* slots, uint32_t n, const void* heads,
                                     size_t head_bytes, const void* tails, size_t tail_stride, uint32_t num_slots,
                                     unsigned long long* bytes_moved, int32_t* error_word, qvp_stream_t stream) {
    if (n == 0) return QVP_OK;
    int rc = codec_check(pool, block_stride, block_bytes, ids, slots, n, heads, head_bytes, tails, tail_stride);
    if (rc != QVP_OK) return rc;
    decompress_blocks_kernel<<<n, kCodecThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<uint8_t*>(pool), block_stride, num_blocks, static_cast<uint32_t>(block_bytes), ids, slots,
        static_cast<const uint8_t*>(heads), static_cast<uint32_t>(head_bytes), static_cast<const uint8_t*>(tails),
        tail_stride, num_slots, bytes_moved, error_word);
    return check_cuda(cudaGetLastError(), "launch decompress_blocks");
}
