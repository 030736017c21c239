// qvp_decode_noalloc: the batched decode for callers that cannot allocate
// device memory. It runs exactly the kernels of qvp_decode, with their
// scratch taken from a fixed array compiled into this library instead of a
// caller-provided workspace.
//
// Who needs it: a host process that owns the whole device-memory budget and
// hands plugins only the buffers they compute on (a serving engine that
// reserves HBM up front), an FFI caller with no device allocator of its own,
// and a latency-critical step loop where cudaMalloc / cudaFree would
// synchronise the device. Such a caller still passes the pool, tables,
// queries and output; only the split-K / stream-K scratch comes from here.
#include "qvp_internal.h"

#include <atomic>

namespace {

// 16 MiB of device memory, held by every GPU that loads the library until
// the process exits. Enough for the stream-K records of several thousand
// (sequence, head group) segments at head_dim 128.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device ordinal, looked up once
// with that device current. In host code the symbol itself is only a
// host-side stand-in, never a device address. The address belongs to the
// device's primary context (the one the runtime API makes current). Threads
// making their first call on a device at the same time both look it up and
// store the same pointer; the atomic makes that race well defined.
constexpr int kMaxDevices = 64;
std::atomic<void*> g_scratch_addr[kMaxDevices] = {};

}  // namespace

using namespace qvp;

extern "C" int qvp_decode_noalloc(const qvp_decode_args* args, qvp_stream_t stream) {
    if (args == nullptr) return fail(QVP_ERR_INVALID, "null argument");
    DecodePlan plan;
    int rc = plan_decode(*args, plan);
    if (rc != QVP_OK || args->batch == 0) return rc;
    const size_t need = plan.workspace_bytes;
    if (need > kNoAllocScratchBytes)
        return fail(QVP_ERR_WORKSPACE,
                    "qvp_decode_noalloc: this batch needs %zu bytes of scratch but the static array holds %zu; "
                    "use qvp_decode with a caller workspace",
                    need, kNoAllocScratchBytes);
    int dev = -1;
    rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc != QVP_OK) return rc;
    if (dev < 0 || dev >= kMaxDevices) return fail(QVP_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    void* scratch = g_scratch_addr[dev].load(std::memory_order_relaxed);
    if (scratch == nullptr) {
        rc = check_cuda(cudaGetSymbolAddress(&scratch, g_noalloc_scratch), "cudaGetSymbolAddress(no-alloc scratch)");
        if (rc != QVP_OK) return rc;
        g_scratch_addr[dev].store(scratch, std::memory_order_relaxed);
    }
    qvp_decode_args a = *args;
    a.workspace = scratch;
    a.workspace_bytes = kNoAllocScratchBytes;
    return run_decode(a, plan, reinterpret_cast<cudaStream_t>(stream));
}
