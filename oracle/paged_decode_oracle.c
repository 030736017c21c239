/*
 * TEST INFRASTRUCTURE ONLY - the CPU oracle for the paged-decode path.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may load this file's library, and only as the checker or the timed CPU
 * baseline. The product (libqvp.so) never calls it and has no CPU fallback.
 *
 * A plain-C restatement of phhuang191129/QwenVL-Paged's
 * paged_attention_decode<T> (include/qwenvl_paged/PagedAttention.h:53-127)
 * over a flat block pool addressed the way CacheView::slot does
 * (include/qwenvl_paged/KVCacheManager.h:131-154, src/CacheLayout.cpp:5-38):
 *   - reject (return 0, `out` untouched) on bad arguments (PagedAttention.h:59-68)
 *     or on any unmapped block inside the context (PagedAttention.h:73-89);
 *   - per query head: kv = h / group; scores in fp32 with a sequential dot
 *     over head_dim, times scale (PagedAttention.h:99-107);
 *   - exact max, then weights expf(s - max), denominator and value sum in
 *     token order (PagedAttention.h:109-118); out = acc / denominator
 *     (PagedAttention.h:120-123).
 * bf16 inputs are widened exactly to float; the output is always float (the
 * reference run with T = float over bf16-rounded values).
 *
 * Pinned against: the reference's own known-answer tests (re-expressed in
 * tests/test_oracle.py) and outputs of the reference compiled from its
 * sources (oracle/_ref, tests/golden/).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct oracle_shape {
    uint32_t tokens_per_block, num_layers, num_kv_heads, head_dim, bytes_per_element;
} oracle_shape;

static float bf16_to_float(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

static float load_elem(const uint8_t* p, int dtype) {
    if (dtype == 0) {
        float f;
        memcpy(&f, p, 4);
        return f;
    }
    uint16_t b;
    memcpy(&b, p, 2);
    return bf16_to_float(b);
}

/* Element offset of (layer, stream, token_in_block, kv_head) inside a block,
 * src/CacheLayout.cpp:25-38 (strides :5-19). */
static size_t element_offset(const oracle_shape* s, uint32_t layer, uint32_t stream, uint32_t t, uint32_t h) {
    const size_t head = s->head_dim;
    const size_t token = (size_t)s->num_kv_heads * head;
    const size_t strm = (size_t)s->tokens_per_block * token;
    const size_t lay = 2 * strm;
    return layer * lay + stream * strm + t * token + h * head;
}

/* One sequence. dtype 0 = f32, 1 = bf16. Returns 1 on success, 0 when the
 * reference would return false (out untouched). */
int oracle_paged_decode(const uint8_t* pool, size_t block_stride, uint32_t num_blocks, const oracle_shape* s,
                        int dtype, uint32_t layer, uint32_t num_query_heads, float scale,
                        const int32_t* table_row, uint32_t table_len, uint32_t context_len, const void* query,
                        float* out) {
    const uint32_t elem = dtype == 0 ? 4u : 2u;
    if (pool == NULL || query == NULL || out == NULL || s == NULL) return 0;
    if (s->tokens_per_block == 0 || s->num_layers == 0 || s->num_kv_heads == 0 || s->head_dim == 0) return 0;
    if (s->bytes_per_element != elem || context_len == 0 || layer >= s->num_layers || num_query_heads == 0 ||
        num_query_heads % s->num_kv_heads != 0)
        return 0;
    const uint32_t T = s->tokens_per_block, D = s->head_dim;
    const uint32_t nblk = (context_len + T - 1) / T;
    if (nblk > table_len) return 0;
    for (uint32_t b = 0; b < nblk; ++b)
        if (table_row[b] < 0 || (uint32_t)table_row[b] >= num_blocks) return 0;

    const uint32_t group = num_query_heads / s->num_kv_heads;
    float* scores = (float*)malloc(sizeof(float) * context_len);
    float* acc = (float*)malloc(sizeof(float) * D);
    float* result = (float*)malloc(sizeof(float) * (size_t)num_query_heads * D);
    if (!scores || !acc || !result) {
        free(scores);
        free(acc);
        free(result);
        return 0;
    }
    for (uint32_t qh = 0; qh < num_query_heads; ++qh) {
        const uint32_t kv = qh / group;
        const uint8_t* q = (const uint8_t*)query + (size_t)qh * D * elem;
        float max_score = -INFINITY;
        for (uint32_t t = 0; t < context_len; ++t) {
            const uint8_t* blk = pool + (size_t)table_row[t / T] * block_stride;
            const uint8_t* k = blk + element_offset(s, layer, 0, t % T, kv) * elem;
            float dot = 0.0f;
            for (uint32_t d = 0; d < D; ++d) dot += load_elem(q + d * elem, dtype) * load_elem(k + d * elem, dtype);
            scores[t] = dot * scale;
            if (scores[t] > max_score) max_score = scores[t];
        }
        for (uint32_t d = 0; d < D; ++d) acc[d] = 0.0f;
        float denom = 0.0f;
        for (uint32_t t = 0; t < context_len; ++t) {
            const uint8_t* blk = pool + (size_t)table_row[t / T] * block_stride;
            const uint8_t* v = blk + element_offset(s, layer, 1, t % T, kv) * elem;
            const float w = expf(scores[t] - max_score);
            denom += w;
            for (uint32_t d = 0; d < D; ++d) acc[d] += w * load_elem(v + d * elem, dtype);
        }
        for (uint32_t d = 0; d < D; ++d) result[(size_t)qh * D + d] = acc[d] / denom;
    }
    memcpy(out, result, sizeof(float) * (size_t)num_query_heads * D);
    free(scores);
    free(acc);
    free(result);
    return 1;
}

typedef struct batch_job {
    const uint8_t* pool;
    size_t block_stride;
    uint32_t num_blocks;
    const oracle_shape* s;
    int dtype;
    uint32_t layer, hq;
    float scale;
    uint32_t batch, pitch;
    const int32_t* tables;
    const int32_t* ctx;
    const uint8_t* q;
    float* out;
    int32_t* status;
    uint32_t next;
    pthread_mutex_t lock;
} batch_job;

static void* batch_worker(void* arg) {
    batch_job* j = (batch_job*)arg;
    const size_t qbytes = (size_t)j->hq * j->s->head_dim * (j->dtype == 0 ? 4 : 2);
    for (;;) {
        pthread_mutex_lock(&j->lock);
        const uint32_t b = j->next++;
        pthread_mutex_unlock(&j->lock);
        if (b >= j->batch) break;
        const int32_t c = j->ctx[b];
        j->status[b] = c > 0 ? oracle_paged_decode(j->pool, j->block_stride, j->num_blocks, j->s, j->dtype,
                                                   j->layer, j->hq, j->scale, j->tables + (size_t)b * j->pitch,
                                                   j->pitch, (uint32_t)c, j->q + b * qbytes,
                                                   j->out + (size_t)b * j->hq * j->s->head_dim)
                             : 0;
    }
    return NULL;
}

/* The whole batch, sequences spread over `threads` workers. status[b] = 1
 * when sequence b succeeded. Returns the number of successes. */
int oracle_paged_decode_batch(const uint8_t* pool, size_t block_stride, uint32_t num_blocks, const oracle_shape* s,
                              int dtype, uint32_t layer, uint32_t num_query_heads, float scale, uint32_t batch,
                              uint32_t pitch, const int32_t* tables, const int32_t* context_lens, const void* query,
                              float* out, int32_t* status, int threads) {
    batch_job j;
    j.pool = pool;
    j.block_stride = block_stride;
    j.num_blocks = num_blocks;
    j.s = s;
    j.dtype = dtype;
    j.layer = layer;
    j.hq = num_query_heads;
    j.scale = scale;
    j.batch = batch;
    j.pitch = pitch;
    j.tables = tables;
    j.ctx = context_lens;
    j.q = (const uint8_t*)query;
    j.out = out;
    j.status = status;
    j.next = 0;
    pthread_mutex_init(&j.lock, NULL);
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    for (int i = 1; i < threads; ++i) pthread_create(&tid[i], NULL, batch_worker, &j);
    batch_worker(&j);
    for (int i = 1; i < threads; ++i) pthread_join(tid[i], NULL);
    pthread_mutex_destroy(&j.lock);
    int ok = 0;
    for (uint32_t b = 0; b < batch; ++b) ok += status[b] == 1;
    return ok;
}

/* MemoryAllocator::copy_block restated (src/MemoryAllocator.cpp:76-85):
 * bytes of block src -> block dst for every pair, in order. */
void oracle_copy_blocks(uint8_t* pool, size_t block_stride, uint32_t num_blocks, size_t bytes, const int32_t* pairs,
                        uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) {
        const int32_t src = pairs[2 * i], dst = pairs[2 * i + 1];
        if (src < 0 || dst < 0 || (uint32_t)src >= num_blocks || (uint32_t)dst >= num_blocks) continue;
        memmove(pool + (size_t)dst * block_stride, pool + (size_t)src * block_stride, bytes);
    }
}
