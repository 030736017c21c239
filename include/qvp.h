/*
 * qvp.h - C ABI of the B200 paged-decode path (sm_100a).
 *
 * Every entry point takes plain pointers and sizes, never a C++ or torch type,
 * so any FFI (ctypes, cgo, JNI, N-API) can bind it. All device work is enqueued
 * on the caller's stream; no call synchronises the device unless its comment
 * says so. Nothing here is thread-safe: like the C++ API it serves, it is meant
 * to be driven from one engine thread.
 *
 * Status convention: every function returns a qvp_status (0 = success). On a
 * non-zero status that was detected on the host, no device work was enqueued
 * and no output buffer was touched.
 *
 * Reference interfaces each group replaces (paths inside the reference project
 * phhuang191129/QwenVL-Paged):
 *   - decode:      include/qwenvl_paged/PagedAttention.h:53-127
 *                  (paged_attention_decode<T>) and PagedAttention.h:23-28
 *                  (PagedAttentionParams)
 *   - layout:      include/qwenvl_paged/CacheLayout.h:40-79, src/CacheLayout.cpp:5-38
 *   - block bytes: src/Block.cpp:8-13 (BlockShape::byte_size), Block.cpp:30-44
 *                  (size rounded up to the 256-byte alignment)
 *   - block copy:  src/MemoryAllocator.cpp:76-85 (copy_block)
 *   - swap bytes:  src/SwapBackend.cpp:10-39 (HostSwapBackend::store / load)
 */
#ifndef QVP_H
#define QVP_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QVP_API __attribute__((visibility("default")))
#else
#define QVP_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t / CUstream; NULL is the legacy default stream. */
typedef struct CUstream_st* qvp_stream_t;

typedef enum qvp_status {
    QVP_OK = 0,
    QVP_ERR_INVALID = 1,      /* arguments inconsistent with the cache shape     */
    QVP_ERR_UNMAPPED = 2,     /* a block in [0, context) is unmapped or swapped  */
    QVP_ERR_CUDA = 3,         /* a CUDA runtime call failed (see qvp_last_error) */
    QVP_ERR_DEVICE = 4,       /* a kernel reported a bad block id or a timeout   */
    QVP_ERR_NOMEM = 5,        /* device or pinned allocation failed              */
    QVP_ERR_UNSUPPORTED = 6,  /* shape outside what the kernels implement        */
    QVP_ERR_WORKSPACE = 7     /* caller workspace smaller than required          */
} qvp_status;

typedef enum qvp_dtype {
    QVP_DTYPE_F32 = 0,   /* 4-byte IEEE float            */
    QVP_DTYPE_BF16 = 1   /* 2-byte bfloat16, fp32 math   */
} qvp_dtype;

/*
 * Shape of one physical block. Field for field the reference BlockShape
 * (include/qwenvl_paged/Block.h:46-57). Elements inside a block are ordered
 * [layer][K|V][token_in_block][kv_head][head_dim] (src/CacheLayout.cpp:5-19).
 */
typedef struct qvp_block_shape {
    uint32_t tokens_per_block;
    uint32_t num_layers;
    uint32_t num_kv_heads;
    uint32_t head_dim;
    uint32_t bytes_per_element;
} qvp_block_shape;

/* BlockShape::byte_size(): tokens * layers * kv_heads * head_dim * elem * 2. */
QVP_API size_t qvp_block_bytes(const qvp_block_shape* shape);
/* Distance between two physical blocks in a pool: byte_size rounded up to 256
 * (the reference rounds each block allocation the same way, Block.cpp:30-44). */
QVP_API size_t qvp_block_stride(const qvp_block_shape* shape);

/* Human-readable text of the last error raised on this thread. */
QVP_API const char* qvp_last_error(void);
/* Library version string, e.g. "qvp 0.1.0 sm_100a". */
QVP_API const char* qvp_version(void);
/* Number of SMs of the current device, 0 when no device is visible. */
QVP_API int qvp_device_sm_count(void);

/* ---------------------------------------------------------------------------
 * Block pool: one cudaMalloc'd slab per GPU. Block i lives at base + i*stride.
 * Replaces the per-block aligned_alloc of PhysicalBlock (src/Block.cpp:30-44);
 * the whole pool is zero-filled once at creation.
 * ------------------------------------------------------------------------- */
typedef struct qvp_pool qvp_pool;

QVP_API int qvp_pool_create(int device, const qvp_block_shape* shape, uint32_t num_blocks,
                    qvp_pool** out_pool);
QVP_API int qvp_pool_destroy(qvp_pool* pool);
QVP_API void* qvp_pool_base(const qvp_pool* pool);
QVP_API size_t qvp_pool_stride(const qvp_pool* pool);
QVP_API uint32_t qvp_pool_num_blocks(const qvp_pool* pool);
QVP_API int qvp_pool_device(const qvp_pool* pool);
/* Synchronous helpers for tests and set-up: copy `bytes` between host memory
 * and block `block` at byte `offset`. Bounds are checked against the stride. */
QVP_API int qvp_pool_write(qvp_pool* pool, uint32_t block, size_t offset, const void* host,
                   size_t bytes);
QVP_API int qvp_pool_read(const qvp_pool* pool, uint32_t block, size_t offset, void* host,
                  size_t bytes);

/* ---------------------------------------------------------------------------
 * Batched paged decode.
 *
 * For every sequence b in [0, batch) and query head h in [0, num_query_heads):
 *   kv = h / (num_query_heads / num_kv_heads)
 *   s_t = scale * <q[b,h,:], K[b, layer, t, kv, :]>      for t < context_lens[b]
 *   out[b,h,:] = sum_t softmax(s)_t * V[b, layer, t, kv, :]
 * which is paged_attention_decode<T> (PagedAttention.h:94-124) applied to every
 * sequence of the batch at once. Token t of sequence b lives in physical block
 * block_tables[b * max_blocks_per_seq + t / tokens_per_block], slot
 * t % tokens_per_block.
 *
 * Checks done on the host (status returned, nothing enqueued): shape, dtype,
 * layer < num_layers, num_query_heads a positive multiple of num_kv_heads,
 * context lengths bounded by max_context_len <= max_blocks_per_seq*tokens.
 * The device tables are not read on the host: a table entry outside
 * [0, num_blocks) inside a context makes the kernel record a non-zero value in
 * *error_word (when given) and read block 0 instead, so no access leaves the
 * pool; the output of that sequence is then unspecified. Callers that need the
 * reference's "refuse and leave out untouched" behaviour validate the tables
 * on the host first (the C++ layer does).
 *
 * Split-K: contexts longer than split_tokens are cut into partitions whose
 * partial (max, sum, accumulator) go to `workspace` and are merged by a second
 * kernel. split_tokens = 0 picks a size from the batch shape.
 * ------------------------------------------------------------------------- */
typedef struct qvp_decode_args {
    const void* pool;              /* device base of the block pool            */
    size_t block_stride;           /* bytes between physical blocks            */
    uint32_t num_blocks;           /* pool capacity in blocks                  */
    qvp_block_shape shape;         /* shape shared by every block              */
    int32_t dtype;                 /* qvp_dtype of K/V, query and out          */
    uint32_t layer;                /* PagedAttentionParams::layer              */
    uint32_t num_query_heads;      /* PagedAttentionParams::num_query_heads    */
    float scale;                   /* PagedAttentionParams::scale              */
    uint32_t batch;                /* number of sequences                      */
    uint32_t max_blocks_per_seq;   /* row pitch of block_tables                */
    uint32_t max_context_len;      /* host-known upper bound of context_lens   */
    const int32_t* block_tables;   /* device int32 [batch][max_blocks_per_seq] */
    const int32_t* context_lens;   /* device int32 [batch], each in [1, max]   */
    const void* query;             /* device [batch][num_query_heads][head_dim]*/
    void* out;                     /* device [batch][num_query_heads][head_dim]*/
    uint32_t split_tokens;         /* 0 = auto; fast path: a multiple of 16    */
    void* workspace;               /* device scratch, >= qvp_decode_workspace_size,
                                      16-byte aligned                              */
    size_t workspace_bytes;
    int32_t* error_word;           /* device int32 or NULL; never cleared here */
} qvp_decode_args;

/* Scratch bytes `qvp_decode` needs for these arguments (0 when no split). */
QVP_API int qvp_decode_workspace_size(const qvp_decode_args* args, size_t* bytes);
/* The split size `qvp_decode` would use for these arguments. */
QVP_API int qvp_decode_plan(const qvp_decode_args* args, uint32_t* split_tokens,
                    uint32_t* num_splits, int* fast_path);
QVP_API int qvp_decode(const qvp_decode_args* args, qvp_stream_t stream);

/*
 * qvp_decode_noalloc: qvp_decode for callers that cannot allocate device
 * memory. No counterpart in the reference (its CPU kernel needs no scratch).
 *
 * Some callers cannot call cudaMalloc: a host process that owns the whole
 * device-memory budget and gives plugins only the buffers they compute on,
 * an FFI caller without a device allocator, or a step loop where cudaMalloc
 * and cudaFree would synchronise the device. This entry point runs the same
 * kernels as qvp_decode but ignores args->workspace: its scratch is a 16 MiB
 * array compiled into the library (every GPU that loads the library holds
 * it until the process exits). The caller still passes pool, tables,
 * context lengths, queries and output.
 *   - A batch needing more than 16 MiB of scratch (qvp_decode_workspace_size)
 *     is refused with QVP_ERR_WORKSPACE before anything is enqueued.
 *   - It calls no cudaMalloc, cudaFree or other allocating routine. The first
 *     call on each device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture. The address is kept per device ordinal and
 *     belongs to the device's primary context (the runtime API's context):
 *     callers that make another context current through the driver API must
 *     not use this entry point.
 *   - Every call shares the one array, which keeps the last call's contents.
 *     Nothing in it needs to start at zero (the kernels write every scratch
 *     byte they read), but calls that overlap on the GPU (other streams, other
 *     threads) race on it: order them on one stream.
 */
QVP_API int qvp_decode_noalloc(const qvp_decode_args* args, qvp_stream_t stream);

/* ---------------------------------------------------------------------------
 * Causal prefill over the paged cache.
 *
 * The reference defines prefill as paged_attention_decode<T> applied at every
 * prompt position p with context_len = p + 1 (PagedAttention.h:43-44). For
 * each sequence b, the last query_lens[b] tokens of its context_lens[b]-token
 * cache are queries: query token t (position pos = context_lens[b] -
 * query_lens[b] + t) attends keys [0, pos] with the decode's arithmetic. K and
 * V of the new tokens must already be in the cache (qvp_kv_append). query and
 * out are [batch][max_query_len][num_query_heads][head_dim]; rows t >=
 * query_lens[b] are neither read nor written. Device-side problems (bad block
 * ids, lengths outside [1, capacity], query_lens > context_lens or >
 * max_query_len) set bits in *error_word and never fault.
 * ------------------------------------------------------------------------- */
typedef struct qvp_prefill_args {
    const void* pool;              /* device base of the block pool            */
    size_t block_stride;           /* bytes between physical blocks            */
    uint32_t num_blocks;           /* pool capacity in blocks                  */
    qvp_block_shape shape;         /* shape shared by every block              */
    int32_t dtype;                 /* qvp_dtype of K/V, query and out          */
    uint32_t layer;
    uint32_t num_query_heads;
    float scale;
    uint32_t batch;
    uint32_t max_blocks_per_seq;   /* row pitch of block_tables                */
    uint32_t max_query_len;        /* token pitch of query / out               */
    const int32_t* block_tables;   /* device int32 [batch][max_blocks_per_seq] */
    const int32_t* context_lens;   /* device int32 [batch]: tokens in the cache */
    const int32_t* query_lens;     /* device int32 [batch]: new tokens (<= ctx) */
    const void* query;             /* device [batch][max_query_len][Hq][D]     */
    void* out;                     /* device [batch][max_query_len][Hq][D]     */
    int32_t* error_word;           /* device int32 or NULL                      */
} qvp_prefill_args;

QVP_API int qvp_prefill(const qvp_prefill_args* args, qvp_stream_t stream);

/* ---------------------------------------------------------------------------
 * Block movers.
 *
 * qvp_copy_blocks: for i < n, copy `bytes` from block pairs[2i] to block
 * pairs[2i+1] of the same pool (MemoryAllocator::copy_block, called by
 * copy-on-write at src/KVCacheManager.cpp:146). `pairs` is device int32.
 * One launch for the whole batch.
 *
 * qvp_gather_blocks / qvp_scatter_blocks: move the blocks named by the device
 * int32 list `ids` between the pool and a contiguous buffer `staging`
 * (staging + i*bytes). `staging` may be device memory or pinned host memory
 * mapped into the device's address space. These carry the bytes of
 * HostSwapBackend::store / load (src/SwapBackend.cpp:10-39).
 *
 * Ids outside [0, num_blocks) are skipped and recorded in *error_word.
 * ------------------------------------------------------------------------- */
QVP_API int qvp_copy_blocks(void* pool, size_t block_stride, uint32_t num_blocks, size_t bytes,
                    const int32_t* pairs, uint32_t n, int32_t* error_word,
                    qvp_stream_t stream);
QVP_API int qvp_gather_blocks(const void* pool, size_t block_stride, uint32_t num_blocks,
                      size_t bytes, const int32_t* ids, uint32_t n, void* staging,
                      int32_t* error_word, qvp_stream_t stream);
QVP_API int qvp_scatter_blocks(void* pool, size_t block_stride, uint32_t num_blocks,
                       size_t bytes, const int32_t* ids, uint32_t n,
                       const void* staging, int32_t* error_word, qvp_stream_t stream);

/* ---------------------------------------------------------------------------
 * qvp_fetch_host: copy `bytes` from page-locked host memory (mapped into the
 * device's address space, as all page-locked memory is under unified
 * addressing) to device memory with a kernel whose SMs read over PCIe. The
 * engine's small per-step uploads (block tables, copy pairs, append slots)
 * go this way so that they never wait behind a large swap copy queued on the
 * copy engines. The host must not change `src` until the kernel has run.
 * ------------------------------------------------------------------------- */
QVP_API int qvp_fetch_host(void* dst, const void* src, size_t bytes, qvp_stream_t stream);

/* ---------------------------------------------------------------------------
 * Compressed swap slots (lossless). The reference's swap path copies every
 * block's bytes verbatim (src/SwapBackend.cpp:10-39) and names compressing
 * swapped blocks as the way to cut link time (docs/architecture.md:128-130).
 *
 * qvp_compress_blocks codes block ids[i] of the pool, for i < n, into swap
 * slot slots[i]; qvp_decompress_blocks is the inverse. A slot is split in
 * two places: its first head_bytes bytes at heads + i*head_bytes (indexed by
 * list position: a device staging buffer that the caller moves with the copy
 * engines) and the rest at tails + slots[i]*tail_stride (normally pinned
 * host memory mapped into the device, which the kernels reach over PCIe).
 * head_bytes = 0 puts whole slots in the tails. A slot holds a 16-byte
 * header (u32 format 'QVP1' coded / 'QVP0' raw, u32 escapes, u32 bytes used,
 * u32 0) and then either the raw block or, for bf16 blocks: a 16-byte
 * dictionary of the 15 most frequent high bytes, one 4-bit code per value
 * (code 15 = escape), the low bytes, and u32 escapes (value index << 8 |
 * high byte). Blocks that would not shrink are stored raw. Requirements:
 * head_bytes + tail_stride >= qvp_swap_slot_bytes(block_bytes); block_bytes,
 * head_bytes, tail_stride and the stride multiples of 16; pool, heads and
 * tails 16-byte aligned. `bytes_moved` (device u64[2], optional) accumulates
 * the slot bytes used and, of those, the bytes past head_bytes. Ids or slots
 * out of range are skipped and recorded in *error_word (1), as are slots
 * this codec did not write (the frame is left as it was).
 * ------------------------------------------------------------------------- */
QVP_API size_t qvp_swap_slot_bytes(size_t block_bytes);
QVP_API int qvp_compress_blocks(const void* pool, size_t block_stride, uint32_t num_blocks,
                        size_t block_bytes, const int32_t* ids, const int32_t* slots, uint32_t n,
                        void* heads, size_t head_bytes, void* tails, size_t tail_stride,
                        uint32_t num_slots, unsigned long long* bytes_moved, int32_t* error_word,
                        qvp_stream_t stream);
QVP_API int qvp_decompress_blocks(void* pool, size_t block_stride, uint32_t num_blocks,
                          size_t block_bytes, const int32_t* ids, const int32_t* slots, uint32_t n,
                          const void* heads, size_t head_bytes, const void* tails, size_t tail_stride,
                          uint32_t num_slots, unsigned long long* bytes_moved, int32_t* error_word,
                          qvp_stream_t stream);

/* ---------------------------------------------------------------------------
 * KV append: write one new token's K and V for every kv head of every
 * sequence: for b < batch, token position positions[b] of sequence b goes to
 * block block_tables[b*pitch + pos/tokens_per_block], slot pos%tokens_per_block,
 * layer `layer`. k and v are device [batch][num_kv_heads][head_dim] in the
 * pool's element type. This is the device form of the per-token writes that
 * the reference performs through ensure_token_writable and a host store
 * (tests/PagedAttention.test.cpp:97-127); call it only after copy-on-write has
 * made every target block private.
 * ------------------------------------------------------------------------- */
QVP_API int qvp_kv_append(void* pool, size_t block_stride, uint32_t num_blocks,
                  const qvp_block_shape* shape, uint32_t layer, uint32_t batch,
                  uint32_t max_blocks_per_seq, const int32_t* block_tables,
                  const int32_t* positions, const void* k, const void* v,
                  int32_t* error_word, qvp_stream_t stream);

/* ---------------------------------------------------------------------------
 * KV-head sharding across the GPUs of one node (one process per GPU).
 *
 * Each GQA group (a kv head and the num_query_heads/num_kv_heads query heads
 * that read it) is independent (PagedAttention.h:94-96), so a batch splits by
 * kv head with no exchange inside the decode: shard s of n owns kv heads
 * [s*Hkv/n, (s+1)*Hkv/n) and query heads [s*Hq/n, (s+1)*Hq/n). Its pool holds
 * blocks of num_kv_heads = Hkv/n; the host bookkeeping (allocator, tables,
 * copy-on-write, swap) is replicated, so every shard uses the same block ids
 * and tables (the view every shard decodes through is the one
 * KVCacheManager::cache_view builds, src/KVCacheManager.cpp:241-256). Only
 * where a consumer needs every head on every GPU are the outputs reassembled:
 * qvp_shard_decode decodes into its slot of a gather buffer, all-gathers the
 * slots with NCCL over NVLink (in place, on the caller's communicator and
 * stream) and reorders them into [batch][Hq][head_dim].
 *
 * NCCL is loaded at the first call that needs it (dlopen of libnccl.so.2: the
 * copy already in the process if there is one), so the rest of the library
 * does not depend on it. No counterpart in the reference (it runs on one CPU).
 * ------------------------------------------------------------------------- */
typedef struct qvp_shard {
    uint32_t shard;        /* this GPU's shard, in [0, num_shards)            */
    uint32_t num_shards;   /* GPUs sharing the batch by kv head               */
    int device;            /* CUDA device of this shard; must be current      */
} qvp_shard;

typedef struct qvp_shard_decode_args {
    qvp_shard shard;
    /* the decode of this shard: its pool (num_kv_heads = Hkv/num_shards), its
     * queries [batch][Hq/num_shards][head_dim] and num_query_heads =
     * Hq/num_shards; decode.out is ignored (the output goes to `gathered`). */
    qvp_decode_args decode;
    void* nccl_comm;       /* ncclComm_t over the num_shards GPUs, rank = shard */
    void* gathered;        /* device, qvp_shard_gather_bytes: [num_shards][batch]
                              [Hq/num_shards][head_dim]                        */
    void* out;             /* device [batch][Hq][head_dim], every head         */
} qvp_shard_decode_args;

/* Bytes of the `gathered` buffer qvp_shard_decode needs. */
QVP_API int qvp_shard_gather_bytes(const qvp_shard_decode_args* args, size_t* bytes);
/* Decode + in-place NCCL all-gather + reorder, enqueued on `stream`. Every
 * shard of the communicator must make the matching call (the all-gather is a
 * collective). The decode's workspace rules are qvp_decode's. */
QVP_API int qvp_shard_decode(const qvp_shard_decode_args* args, qvp_stream_t stream);
/* The reorder step alone: gathered [num_shards][batch][heads_per_shard]
 * [head_dim] -> out [batch][num_shards * heads_per_shard][head_dim]. */
QVP_API int qvp_shard_reassemble(const void* gathered, void* out, uint32_t num_shards,
                         uint32_t batch, uint32_t heads_per_shard, uint32_t head_dim,
                         uint32_t bytes_per_element, qvp_stream_t stream);

/* ---------------------------------------------------------------------------
 * Output exchange over NVLink peer memory (the fused form of the shard
 * all-gather): each GPU's decode kernel stores its heads' output rows
 * straight into the output buffer of every GPU of the group, then a one-warp
 * kernel raises this GPU's flag on every peer and waits (bounded, about one
 * second, error bit 2 on timeout) for every peer's flag, all on the caller's
 * stream. No NCCL and no reassembly pass.
 *
 * Set-up, once per process: qvp_peer_group_create allocates this GPU's two
 * output buffers (steps alternate between them) and flags, and writes an
 * opaque QVP_PEER_HANDLE_BYTES handle (a CUDA IPC handle); the caller gathers
 * every rank's handle by its own transport and hands all of them, in rank
 * order, to qvp_peer_group_open. Every GPU of the group must be able to reach
 * the others' memory (NVLink / NVSwitch).
 *
 * qvp_shard_decode_peer(step) writes step's output into buffer step % 2 of
 * every GPU; qvp_peer_group_output(group, step) is this GPU's copy, valid on
 * the stream after the call. Steps must be issued in order 0, 1, 2, ... on
 * every rank, and work reading the output of step k must be enqueued on the
 * same stream before the decode of step k + 1 (peers overwrite that buffer
 * in step k + 2). Needs the stream-K plan (bf16, head_dim 64/128, 16-token
 * blocks). No counterpart in the reference.
 * ------------------------------------------------------------------------- */
#define QVP_PEER_HANDLE_BYTES 64
typedef struct qvp_peer_group qvp_peer_group;

QVP_API int qvp_peer_group_create(int rank, int nranks, size_t out_bytes, void* handle,
                          qvp_peer_group** group);
QVP_API int qvp_peer_group_open(qvp_peer_group* group, const void* handles);
QVP_API int qvp_peer_group_destroy(qvp_peer_group* group);
QVP_API void* qvp_peer_group_output(const qvp_peer_group* group, uint64_t step);
/* args->nccl_comm and args->gathered are ignored; args->out is ignored (the
 * output goes to the group's buffers). */
QVP_API int qvp_shard_decode_peer(const qvp_shard_decode_args* args, qvp_peer_group* group,
                          uint64_t step, int32_t* error_word, qvp_stream_t stream);

/* NCCL communicator helpers for callers that have no NCCL binding of their
 * own (FFI callers): the unique id (QVP_NCCL_ID_BYTES opaque bytes) is made
 * on one rank and handed to the others by the caller's own transport. The
 * communicator belongs to the current device. comm_init blocks until every
 * rank has joined; comm_destroy waits for the communicator's work. */
#define QVP_NCCL_ID_BYTES 128
QVP_API int qvp_nccl_unique_id(void* id, size_t bytes);
QVP_API int qvp_nccl_comm_init(const void* id, size_t bytes, int nranks, int rank, void** comm);
QVP_API int qvp_nccl_comm_destroy(void* comm);

#ifdef __cplusplus
}
#endif

#endif /* QVP_H */
