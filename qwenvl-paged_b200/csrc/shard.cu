// KV-head sharding: the reassembly of per-shard decode outputs across GPUs.
//
// A batch splits by kv head with no exchange inside the decode (every GQA
// group is independent, phhuang191129/QwenVL-Paged
// include/qwenvl_paged/PagedAttention.h:94-96). qvp_shard_decode runs the
// shard's decode straight into its slot of a gather buffer
// [num_shards][batch][heads_per_shard][head_dim], all-gathers the slots in
// place with NCCL (NVLink / NVSwitch inside one node) and reorders them into
// [batch][Hq][head_dim] with reassemble_kernel, all on the caller's stream.
//
// NCCL is resolved with dlopen at the first call that needs it. A process
// that already loaded libnccl.so.2 (a torch process, for one) gets that copy,
// so the library never brings a second NCCL into a process.
#include "qvp_internal.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

namespace qvp {

namespace {

// out[b][s][r] = gathered[s][b][r] for rows r of `row_vec` vectors of type V
// (one row = heads_per_shard * head_dim elements). Consecutive threads write
// consecutive vectors of out.
template <typename V>
__global__ void reassemble_kernel(const V* __restrict__ gathered, V* __restrict__ out, uint32_t num_shards,
                                  uint32_t batch, uint32_t row_vec) {
    const size_t total = static_cast<size_t>(num_shards) * batch * row_vec;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t r = i % row_vec;
        const size_t bs = i / row_vec;
        const size_t s = bs % num_shards;
        const size_t b = bs / num_shards;
        out[i] = gathered[(s * batch + b) * row_vec + r];
    }
}

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    decltype(&ncclCommCount) comm_count = nullptr;
    decltype(&ncclCommUserRank) comm_user_rank = nullptr;
    bool ok = false;
    std::string why;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
        if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (h == nullptr) {
            const char* e = dlerror();
            api.why = e != nullptr ? e : "dlopen(libnccl.so.2) failed";
            return;
        }
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.comm_count = reinterpret_cast<decltype(api.comm_count)>(dlsym(h, "ncclCommCount"));
        api.comm_user_rank = reinterpret_cast<decltype(api.comm_user_rank)>(dlsym(h, "ncclCommUserRank"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather && api.error_string &&
                 api.comm_count && api.comm_user_rank;
        if (!api.ok) api.why = "libnccl.so.2 lacks a needed symbol";
    });
    return api;
}

int check_nccl(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return QVP_OK;
    return fail(QVP_ERR_CUDA, "%s: %s", what, nccl().error_string(r));
}

int require_nccl() {
    const NcclApi& api = nccl();
    if (!api.ok) return fail(QVP_ERR_UNSUPPORTED, "NCCL unavailable: %s", api.why.c_str());
    return QVP_OK;
}

size_t elem_bytes(int32_t dtype) { return dtype == QVP_DTYPE_F32 ? 4u : dtype == QVP_DTYPE_BF16 ? 2u : 0u; }

// Bytes of one shard's slot of the gather buffer.
size_t slot_bytes(const qvp_decode_args& d) {
    return static_cast<size_t>(d.batch) * d.num_query_heads * d.shape.head_dim * elem_bytes(d.dtype);
}

int check_shard(const qvp_shard_decode_args& a) {
    const qvp_shard& s = a.shard;
    if (s.num_shards == 0 || s.shard >= s.num_shards)
        return fail(QVP_ERR_INVALID, "shard %u of %u", s.shard, s.num_shards);
    if (elem_bytes(a.decode.dtype) == 0) return fail(QVP_ERR_INVALID, "unknown dtype %d", a.decode.dtype);
    int dev = -1;
    int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc != QVP_OK) return rc;
    if (s.device >= 0 && s.device != dev)
        return fail(QVP_ERR_INVALID, "shard device %d is not the current device %d", s.device, dev);
    return QVP_OK;
}

}  // namespace

int launch_reassemble(const void* gathered, void* out, uint32_t num_shards, uint32_t batch, uint32_t heads,
                      uint32_t head_dim, uint32_t elem, cudaStream_t st) {
    const size_t row = static_cast<size_t>(heads) * head_dim * elem;
    const size_t total = row * num_shards * batch;
    if (total == 0) return QVP_OK;
    const uintptr_t align = reinterpret_cast<uintptr_t>(gathered) | reinterpret_cast<uintptr_t>(out);
    const int sms = device_sm_count() > 0 ? device_sm_count() : 148;
    auto grid = [&](size_t vecs) {
        const size_t want = (vecs + 255) / 256;
        return static_cast<unsigned>(want < static_cast<size_t>(sms) * 8 ? want : static_cast<size_t>(sms) * 8);
    };
    if (row % 16 == 0 && (align & 15u) == 0) {
        const uint32_t rv = static_cast<uint32_t>(row / 16);
        reassemble_kernel<uint4><<<grid(total / 16), 256, 0, st>>>(static_cast<const uint4*>(gathered),
                                                                   static_cast<uint4*>(out), num_shards, batch, rv);
    } else if (row % 4 == 0 && (align & 3u) == 0) {
        const uint32_t rv = static_cast<uint32_t>(row / 4);
        reassemble_kernel<uint32_t><<<grid(total / 4), 256, 0, st>>>(
            static_cast<const uint32_t*>(gathered), static_cast<uint32_t*>(out), num_shards, batch, rv);
    } else {
        if (row > 0xffffffffu) return fail(QVP_ERR_UNSUPPORTED, "row too large");
        reassemble_kernel<uint8_t><<<grid(total), 256, 0, st>>>(static_cast<const uint8_t*>(gathered),
                                                                static_cast<uint8_t*>(out), num_shards, batch,
                                                                static_cast<uint32_t>(row));
    }
    return check_cuda(cudaGetLastError(), "launch reassemble");
}

}  // namespace qvp

using namespace qvp;

extern "C" int qvp_shard_gather_bytes(const qvp_shard_decode_args* args, size_t* bytes) {
    if (args == nullptr || bytes == nullptr) return fail(QVP_ERR_INVALID, "null argument");
    const qvp_shard& s = args->shard;
    if (s.num_shards == 0 || s.shard >= s.num_shards)
        return fail(QVP_ERR_INVALID, "shard %u of %u", s.shard, s.num_shards);
    if (elem_bytes(args->decode.dtype) == 0) return fail(QVP_ERR_INVALID, "unknown dtype %d", args->decode.dtype);
    *bytes = slot_bytes(args->decode) * s.num_shards;
    return QVP_OK;
}

extern "C" int qvp_shard_reassemble(const void* gathered, void* out, uint32_t num_shards, uint32_t batch,
                                    uint32_t heads_per_shard, uint32_t head_dim, uint32_t bytes_per_element,
                                    qvp_stream_t stream) {
    if (num_shards == 0 || bytes_per_element == 0) return fail(QVP_ERR_INVALID, "zero shards or element size");
    if (batch == 0 || heads_per_shard == 0 || head_dim == 0) return QVP_OK;
    if (gathered == nullptr || out == nullptr) return fail(QVP_ERR_INVALID, "null buffer");
    return launch_reassemble(gathered, out, num_shards, batch, heads_per_shard, head_dim, bytes_per_element,
                             reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int qvp_shard_decode(const qvp_shard_decode_args* args, qvp_stream_t stream) {
    if (args == nullptr) return fail(QVP_ERR_INVALID, "null argument");
    const qvp_shard_decode_args& a = *args;
    int rc = check_shard(a);
    if (rc != QVP_OK) return rc;
    const uint32_t n = a.shard.num_shards;
    if (n > 1 && a.nccl_comm == nullptr) return fail(QVP_ERR_INVALID, "null NCCL communicator");
    if (a.gathered == nullptr || a.out == nullptr) return fail(QVP_ERR_INVALID, "null gather or output buffer");
    if (n > 1 && (rc = require_nccl()) != QVP_OK) return rc;
    DecodePlan plan;
    qvp_decode_args d = a.decode;
    const size_t slot = slot_bytes(d);
    d.out = static_cast<uint8_t*>(a.gathered) + slot * a.shard.shard;
    rc = plan_decode(d, plan);
    if (rc != QVP_OK) return rc;
    if (d.batch == 0) return QVP_OK;
    if (n > 1) {
        // a communicator that does not match the shard geometry is refused
        // before anything is enqueued
        int nranks = 0, rank = -1;
        ncclComm_t comm = static_cast<ncclComm_t>(a.nccl_comm);
        if ((rc = check_nccl(nccl().comm_count(comm, &nranks), "ncclCommCount")) != QVP_OK) return rc;
        if ((rc = check_nccl(nccl().comm_user_rank(comm, &rank), "ncclCommUserRank")) != QVP_OK) return rc;
        if (static_cast<uint32_t>(nranks) != n || static_cast<uint32_t>(rank) != a.shard.shard)
            return fail(QVP_ERR_INVALID, "communicator is rank %d of %d, shard is %u of %u", rank, nranks,
                        a.shard.shard, n);
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    rc = run_decode(d, plan, st);
    if (rc != QVP_OK) return rc;
    if (n > 1) {
        const ncclDataType_t type = d.dtype == QVP_DTYPE_F32 ? ncclFloat32 : ncclBfloat16;
        const size_t count = slot / elem_bytes(d.dtype);
        rc = check_nccl(nccl().all_gather(d.out, a.gathered, count, type, static_cast<ncclComm_t>(a.nccl_comm), st),
                        "ncclAllGather");
        if (rc != QVP_OK) return rc;
    }
    return launch_reassemble(a.gathered, a.out, n, d.batch, d.num_query_heads, d.shape.head_dim,
                             static_cast<uint32_t>(elem_bytes(d.dtype)), st);
}

extern "C" int qvp_nccl_unique_id(void* id, size_t bytes) {
    if (id == nullptr || bytes < sizeof(ncclUniqueId)) return fail(QVP_ERR_INVALID, "id buffer below %zu bytes",
                                                                    sizeof(ncclUniqueId));
    int rc = require_nccl();
    if (rc != QVP_OK) return rc;
    ncclUniqueId uid;
    rc = check_nccl(nccl().get_unique_id(&uid), "ncclGetUniqueId");
    if (rc != QVP_OK) return rc;
    std::memcpy(id, &uid, sizeof(uid));
    return QVP_OK;
}

extern "C" int qvp_nccl_comm_init(const void* id, size_t bytes, int nranks, int rank, void** comm) {
    if (id == nullptr || comm == nullptr || bytes < sizeof(ncclUniqueId))
        return fail(QVP_ERR_INVALID, "null id / comm or id below %zu bytes", sizeof(ncclUniqueId));
    if (nranks <= 0 || rank < 0 || rank >= nranks) return fail(QVP_ERR_INVALID, "rank %d of %d", rank, nranks);
    int rc = require_nccl();
    if (rc != QVP_OK) return rc;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclComm_t c = nullptr;
    rc = check_nccl(nccl().comm_init_rank(&c, nranks, uid, rank), "ncclCommInitRank");
    if (rc != QVP_OK) return rc;
    *comm = c;
    return QVP_OK;
}

extern "C" int qvp_nccl_comm_destroy(void* comm) {
    if (comm == nullptr) return QVP_OK;
    int rc = require_nccl();
    if (rc != QVP_OK) return rc;
    return check_nccl(nccl().comm_destroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy");
}

// ---- output exchange over NVLink peer memory -------------------------------

struct qvp_peer_group {
    int rank = 0, nranks = 0, device = -1;
    size_t out_bytes = 0;
    size_t buf_stride = 0;  // out_bytes rounded up to 256
    uint8_t* local = nullptr;  // [2 buffers][flags: 2 parities x kMaxOutTargets sources x u64]
    uint8_t* peer[qvp::kMaxOutTargets] = {};
    bool opened = false;
};

namespace qvp {
namespace {

constexpr uint64_t kPeerWaitLimitNs = 1000000000ull;

size_t flag_offset(const qvp_peer_group& g, uint32_t parity, uint32_t src) {
    return 2 * g.buf_stride + (static_cast<size_t>(parity) * kMaxOutTargets + src) * sizeof(unsigned long long);
}

struct PeerSignal {
    unsigned long long* remote[kMaxOutTargets];       // peer q's flag for (parity, this rank)
    const unsigned long long* local[kMaxOutTargets];  // this GPU's flag for (parity, q)
    uint32_t n, rank;
    unsigned long long target;
    int32_t* err;
};

__device__ __forceinline__ unsigned long long load_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// One warp. Lane q (q != rank) makes this GPU's output stores of the step
// visible system-wide, raises this rank's flag on peer q, then waits until
// peer q has raised its flag here (its rows have landed in this GPU's
// buffer). A wait longer than kPeerWaitLimitNs records error bit 2 and gives
// up, so a missing peer never hangs the GPU.
__global__ void peer_signal_wait(const PeerSignal s) {
    const uint32_t q = threadIdx.x;
    if (q >= s.n || q == s.rank) return;
    __threadfence_system();
    atomicAdd_system(s.remote[q], 1ull);
    const uint64_t start = timer_ns();
    uint32_t spins = 0;
    while (load_acquire_sys(s.local[q]) < s.target) {
        if ((++spins & 63u) == 0u && timer_ns() - start > kPeerWaitLimitNs) {
            if (s.err != nullptr) atomicOr(s.err, 2);
            return;
        }
    }
}

}  // namespace
}  // namespace qvp

extern "C" int qvp_peer_group_create(int rank, int nranks, size_t out_bytes, void* handle, qvp_peer_group** group) {
    if (group == nullptr || handle == nullptr) return fail(QVP_ERR_INVALID, "null argument");
    if (nranks <= 0 || nranks > kMaxOutTargets || rank < 0 || rank >= nranks)
        return fail(QVP_ERR_INVALID, "rank %d of %d (at most %d ranks)", rank, nranks, kMaxOutTargets);
    if (out_bytes == 0) return fail(QVP_ERR_INVALID, "zero output bytes");
    static_assert(sizeof(cudaIpcMemHandle_t) <= QVP_PEER_HANDLE_BYTES, "IPC handle size");
    auto* g = new (std::nothrow) qvp_peer_group;
    if (g == nullptr) return fail(QVP_ERR_NOMEM, "out of host memory");
    g->rank = rank;
    g->nranks = nranks;
    g->out_bytes = out_bytes;
    g->buf_stride = (out_bytes + 255) / 256 * 256;
    int rc = check_cuda(cudaGetDevice(&g->device), "cudaGetDevice");
    const size_t total = 2 * g->buf_stride + 2 * kMaxOutTargets * sizeof(unsigned long long);
    if (rc == QVP_OK) rc = check_cuda(cudaMalloc(reinterpret_cast<void**>(&g->local), total), "cudaMalloc(peer group)");
    if (rc == QVP_OK) rc = check_cuda(cudaMemset(g->local, 0, total), "cudaMemset(peer group)");
    if (rc == QVP_OK) rc = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize(peer group)");
    cudaIpcMemHandle_t h;
    if (rc == QVP_OK) rc = check_cuda(cudaIpcGetMemHandle(&h, g->local), "cudaIpcGetMemHandle");
    if (rc != QVP_OK) {
        if (g->local != nullptr) cudaFree(g->local);
        delete g;
        return rc;
    }
    std::memset(handle, 0, QVP_PEER_HANDLE_BYTES);
    std::memcpy(handle, &h, sizeof(h));
    g->peer[rank] = g->local;
    *group = g;
    return QVP_OK;
}

extern "C" int qvp_peer_group_open(qvp_peer_group* g, const void* handles) {
    if (g == nullptr || handles == nullptr) return fail(QVP_ERR_INVALID, "null argument");
    if (g->opened) return QVP_OK;
    for (int q = 0; q < g->nranks; ++q) {
        if (q == g->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t*>(handles) + static_cast<size_t>(q) * QVP_PEER_HANDLE_BYTES,
                    sizeof(h));
        void* p = nullptr;
        const int rc = check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
        if (rc != QVP_OK) {
            for (int k = 0; k < q; ++k)
                if (k != g->rank && g->peer[k] != nullptr) {
                    cudaIpcCloseMemHandle(g->peer[k]);
                    g->peer[k] = nullptr;
                }
            return rc;
        }
        g->peer[q] = static_cast<uint8_t*>(p);
    }
    g->opened = true;
    return QVP_OK;
}

extern "C" int qvp_peer_group_destroy(qvp_peer_group* g) {
    if (g == nullptr) return QVP_OK;
    cudaDeviceSynchronize();
    for (int q = 0; q < g->nranks; ++q)
        if (q != g->rank && g->peer[q] != nullptr) cudaIpcCloseMemHandle(g->peer[q]);
    if (g->local != nullptr) cudaFree(g->local);
    cudaGetLastError();
    delete g;
    return QVP_OK;
}

extern "C" void* qvp_peer_group_output(const qvp_peer_group* g, uint64_t step) {
    return g == nullptr ? nullptr : g->local + (step & 1u) * g->buf_stride;
}

extern "C" int qvp_shard_decode_peer(const qvp_shard_decode_args* args, qvp_peer_group* g, uint64_t step,
                                     int32_t* error_word, qvp_stream_t stream) {
    if (args == nullptr || g == nullptr) return fail(QVP_ERR_INVALID, "null argument");
    const qvp_shard_decode_args& a = *args;
    int rc = check_shard(a);
    if (rc != QVP_OK) return rc;
    const uint32_t n = a.shard.num_shards;
    if (static_cast<int>(n) != g->nranks || static_cast<int>(a.shard.shard) != g->rank)
        return fail(QVP_ERR_INVALID, "peer group is rank %d of %d, shard is %u of %u", g->rank, g->nranks,
                    a.shard.shard, n);
    if (n > 1 && !g->opened) return fail(QVP_ERR_INVALID, "peer group not opened");
    if (a.decode.dtype != QVP_DTYPE_BF16) return fail(QVP_ERR_UNSUPPORTED, "peer output exchange needs bf16");
    qvp_decode_args d = a.decode;
    const size_t full = slot_bytes(d) * n;
    if (full > g->out_bytes)
        return fail(QVP_ERR_INVALID, "output of %zu bytes does not fit the group's %zu-byte buffers", full,
                    g->out_bytes);
    const uint32_t parity = static_cast<uint32_t>(step & 1u);
    d.out = g->local + parity * g->buf_stride;
    DecodePlan plan;
    rc = plan_decode(d, plan);
    if (rc != QVP_OK || d.batch == 0) return rc;
    if (!plan.stream) return fail(QVP_ERR_UNSUPPORTED, "peer output exchange needs the stream-K plan");
    OutTargets t{};
    t.n = n;
    t.head0 = a.shard.shard * d.num_query_heads;
    t.row_heads = d.num_query_heads * n;
    for (uint32_t q = 0; q < n; ++q)
        t.ptr[q] = reinterpret_cast<__nv_bfloat16*>(g->peer[q] + parity * g->buf_stride);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    rc = run_decode(d, plan, st, &t);
    if (rc != QVP_OK || n == 1) return rc;
    PeerSignal s{};
    s.n = n;
    s.rank = a.shard.shard;
    s.target = step / 2 + 1;
    s.err = error_word;
    for (uint32_t q = 0; q < n; ++q) {
        if (q == s.rank) continue;
        s.remote[q] = reinterpret_cast<unsigned long long*>(g->peer[q] + flag_offset(*g, parity, s.rank));
        s.local[q] = reinterpret_cast<const unsigned long long*>(g->local + flag_offset(*g, parity, q));
    }
    peer_signal_wait<<<1, 32, 0, st>>>(s);
    return check_cuda(cudaGetLastError(), "launch peer_signal_wait");
}
