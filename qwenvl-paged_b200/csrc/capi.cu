// C ABI plumbing: error text, the per-GPU block pool, small queries.
#include "qvp_internal.h"

#include <cstdio>
#include <cstring>
#include <new>
#include <string>

namespace qvp {

namespace {
thread_local std::string g_last_error;
}

int fail(int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

int check_cuda(cudaError_t err, const char* what) {
    if (err == cudaSuccess) return QVP_OK;
    return fail(QVP_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

int set_smem_limit_once(std::atomic<std::uint64_t>& done, const void* func, int bytes, const char* what) {
    int dev = 0;
    const int rc = check_cuda(cudaGetDevice(&dev), what);
    if (rc != QVP_OK) return rc;
    const std::uint64_t bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0ull;
    if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return QVP_OK;
    const int set = check_cuda(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what);
    if (set == QVP_OK && bit != 0) done.fetch_or(bit, std::memory_order_release);
    return set;
}

// Cached per thread (a thread's current device rarely changes).
int device_sm_count() {
    static thread_local int cached_dev = -2;
    static thread_local int cached = 0;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (dev != cached_dev) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        cached = n;
        cached_dev = dev;
    }
    return cached;
}

}  // namespace qvp

using namespace qvp;

struct qvp_pool {
    int device = -1;
    qvp_block_shape shape{};
    size_t stride = 0;
    uint32_t num_blocks = 0;
    void* base = nullptr;
};

extern "C" size_t qvp_block_bytes(const qvp_block_shape* s) {
    if (s == nullptr) return 0;
    return static_cast<size_t>(s->tokens_per_block) * s->num_layers * s->num_kv_heads * s->head_dim *
           s->bytes_per_element * 2u;
}

extern "C" size_t qvp_block_stride(const qvp_block_shape* s) {
    size_t bytes = qvp_block_bytes(s);
    if (bytes == 0) bytes = 256;  // the reference never hands out a zero-byte block
    return round_up(bytes, 256);
}

extern "C" const char* qvp_last_error(void) { return g_last_error.c_str(); }

extern "C" const char* qvp_version(void) { return "qvp 0.1.0 sm_100a"; }

extern "C" int qvp_device_sm_count(void) { return device_sm_count(); }

extern "C" int qvp_pool_create(int device, const qvp_block_shape* shape, uint32_t num_blocks, qvp_pool** out_pool) {
    if (shape == nullptr || out_pool == nullptr) return fail(QVP_ERR_INVALID, "null shape or output");
    *out_pool = nullptr;
    int prev = -1;
    int rc = check_cuda(cudaGetDevice(&prev), "cudaGetDevice");
    if (rc != QVP_OK) return rc;
    if (device >= 0 && device != prev) {
        rc = check_cuda(cudaSetDevice(device), "cudaSetDevice");
        if (rc != QVP_OK) return rc;
    }
    auto* pool = new (std::nothrow) qvp_pool;
    if (pool == nullptr) {
        if (device >= 0 && device != prev) cudaSetDevice(prev);
        return fail(QVP_ERR_NOMEM, "out of host memory");
    }
    pool->device = device >= 0 ? device : prev;
    pool->shape = *shape;
    pool->stride = qvp_block_stride(shape);
    pool->num_blocks = num_blocks;
    const size_t total = pool->stride * num_blocks;
    if (total > 0) {
        cudaError_t e = cudaMalloc(&pool->base, total);
        if (e != cudaSuccess) {
            cudaGetLastError();
            delete pool;
            if (device >= 0 && device != prev) cudaSetDevice(prev);
            return fail(QVP_ERR_NOMEM, "cudaMalloc of a %zu-byte block pool: %s", total, cudaGetErrorString(e));
        }
        rc = check_cuda(cudaMemset(pool->base, 0, total), "cudaMemset(pool)");
        if (rc == QVP_OK) rc = check_cuda(cudaDeviceSynchronize(), "pool zero-fill");
        if (rc != QVP_OK) {
            cudaFree(pool->base);
            delete pool;
            if (device >= 0 && device != prev) cudaSetDevice(prev);
            return rc;
        }
    }
    if (device >= 0 && device != prev) cudaSetDevice(prev);
    *out_pool = pool;
    return QVP_OK;
}

extern "C" int qvp_pool_destroy(qvp_pool* pool) {
    if (pool == nullptr) return QVP_OK;
    int rc = QVP_OK;
    if (pool->base != nullptr) {
        int prev = -1;
        cudaGetDevice(&prev);
        if (pool->device != prev) cudaSetDevice(pool->device);
        rc = check_cuda(cudaFree(pool->base), "cudaFree(pool)");
        if (pool->device != prev) cudaSetDevice(prev);
    }
    delete pool;
    return rc;
}

extern "C" void* qvp_pool_base(const qvp_pool* pool) { return pool ? pool->base : nullptr; }
extern "C" size_t qvp_pool_stride(const qvp_pool* pool) { return pool ? pool->stride : 0; }
extern "C" uint32_t qvp_pool_num_blocks(const qvp_pool* pool) { return pool ? pool->num_blocks : 0; }
extern "C" int qvp_pool_device(const qvp_pool* pool) { return pool ? pool->device : -1; }

static int pool_span_ok(const qvp_pool* pool, uint32_t block, size_t offset, size_t bytes) {
    if (pool == nullptr) return fail(QVP_ERR_INVALID, "null pool");
    if (block >= pool->num_blocks) return fail(QVP_ERR_INVALID, "block %u outside the pool", block);
    if (offset > pool->stride || bytes > pool->stride - offset)
        return fail(QVP_ERR_INVALID, "byte range outside the block");
    return QVP_OK;
}

extern "C" int qvp_pool_write(qvp_pool* pool, uint32_t block, size_t offset, const void* host, size_t bytes) {
    int rc = pool_span_ok(pool, block, offset, bytes);
    if (rc != QVP_OK || bytes == 0) return rc;
    char* dst = static_cast<char*>(pool->base) + static_cast<size_t>(block) * pool->stride + offset;
    return check_cuda(cudaMemcpy(dst, host, bytes, cudaMemcpyHostToDevice), "pool write");
}

extern "C" int qvp_pool_read(const qvp_pool* pool, uint32_t block, size_t offset, void* host, size_t bytes) {
    int rc = pool_span_ok(pool, block, offset, bytes);
    if (rc != QVP_OK || bytes == 0) return rc;
    const char* src = static_cast<const char*>(pool->base) + static_cast<size_t>(block) * pool->stride + offset;
    return check_cuda(cudaMemcpy(host, src, bytes, cudaMemcpyDeviceToHost), "pool read");
}
