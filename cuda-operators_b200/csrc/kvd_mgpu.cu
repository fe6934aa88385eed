// kvd_mgpu.cu -- multi-GPU sequence split behind the C ABI (no reference
// counterpart: the reference is single-GPU). One process (or host thread) per
// GPU. Each rank holds its own token range of every sequence; it decodes that
// range into (m, l, o) partial records, the records of all ranks are gathered,
// and every rank merges them with the log-sum-exp combine kernel.
//
// NCCL is loaded at run time (dlopen), so the library has no link-time NCCL
// dependency and shares the copy a host framework (torch) already loaded:
// dlopen by soname returns the loaded object when there is one.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "kvd_common.cuh"
#include "kvd_decode.cuh"

namespace kvd {
namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    bool ok = false;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather;
    });
    return api;
}

cudaError_t from_nccl(ncclResult_t r) { return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown; }

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// The local decode's descriptor: same shard, partial records into the workspace.
kvd_decode_desc record_desc(const kvd_decode_desc& d) {
    kvd_decode_desc r = d;
    r.flags = KVD_FLAG_PARTIAL_OUT | (d.flags & (KVD_FLAG_Q_BF16 | KVD_FLAG_Q_F16 | KVD_FLAG_QK_INT8));
    r.o_stride_h = d.head_dim + 4;
    r.o_stride_b = static_cast<int64_t>(d.num_q_heads) * r.o_stride_h;
    return r;
}

size_t record_bytes(const kvd_decode_desc& d) {
    return align256(static_cast<size_t>(d.batch) * d.num_q_heads * (d.head_dim + 4) * sizeof(float));
}

}  // namespace
}  // namespace kvd

using namespace kvd;

extern "C" int kvd_mgpu_get_unique_id(unsigned char* id) {
    if (!id) return static_cast<int>(ncclInvalidArgument);
    const NcclApi& api = nccl();
    if (!api.ok) return static_cast<int>(ncclSystemError);
    ncclUniqueId u;
    const ncclResult_t r = api.get_unique_id(&u);
    if (r == ncclSuccess) std::memcpy(id, u.internal, sizeof(u.internal));
    return static_cast<int>(r);
}

extern "C" int kvd_mgpu_comm_init(void** comm, int nranks, int rank, const unsigned char* id) {
    if (!comm || !id || nranks < 1 || rank < 0 || rank >= nranks) return static_cast<int>(ncclInvalidArgument);
    const NcclApi& api = nccl();
    if (!api.ok) return static_cast<int>(ncclSystemError);
    ncclUniqueId u;
    std::memcpy(u.internal, id, sizeof(u.internal));
    ncclComm_t c = nullptr;
    const ncclResult_t r = api.comm_init_rank(&c, nranks, u, rank);
    *comm = r == ncclSuccess ? static_cast<void*>(c) : nullptr;
    return static_cast<int>(r);
}

extern "C" int kvd_mgpu_comm_destroy(void* comm) {
    if (!comm) return static_cast<int>(ncclInvalidArgument);
    const NcclApi& api = nccl();
    if (!api.ok) return static_cast<int>(ncclSystemError);
    return static_cast<int>(api.comm_destroy(static_cast<ncclComm_t>(comm)));
}

extern "C" size_t kvd_mgpu_seq_split_workspace_size(const kvd_decode_desc* desc, int nranks) {
    if (!desc || nranks < 1) return 0;
    const kvd_decode_desc& d = *desc;
    if (d.batch < 1 || d.num_q_heads < 1 || d.num_kv_heads < 1 || d.head_dim < 1 || d.max_seq_len < 0 ||
        d.num_q_heads % d.num_kv_heads != 0)
        return 0;
    const kvd_decode_desc r = record_desc(d);
    return record_bytes(r) * (1 + static_cast<size_t>(nranks)) + align256(kvd_workspace_size(&r));
}

extern "C" cudaError_t kvd_mgpu_seq_split_decode(const kvd_decode_desc* desc, const void* Q, const int8_t* K,
                                                 const int8_t* V, const float* k_scale, const float* v_scale,
                                                 void* out, void* workspace, size_t workspace_bytes, void* comm,
                                                 int nranks, cudaStream_t stream) {
    int* launches = launch_counter();
    if (!desc || !out || !workspace || !comm || nranks < 1) return cudaErrorInvalidValue;
    if (desc->flags & KVD_FLAG_PARTIAL_OUT) return cudaErrorInvalidValue;
    const size_t need = kvd_mgpu_seq_split_workspace_size(desc, nranks);
    if (need == 0 || workspace_bytes < need) return cudaErrorInvalidValue;
    const NcclApi& api = nccl();
    if (!api.ok) return cudaErrorSharedObjectInitFailed;
    const kvd_decode_desc r = record_desc(*desc);
    const size_t rec = record_bytes(r);
    char* ws = static_cast<char*>(workspace);
    float* local = reinterpret_cast<float*>(ws);
    float* gathered = reinterpret_cast<float*>(ws + rec);
    char* dws = ws + rec * (1 + static_cast<size_t>(nranks));
    // 1. this rank's token range -> partial records
    cudaError_t e = kvd_decode_launch(&r, Q, K, V, k_scale, v_scale, local, dws, workspace_bytes - (dws - ws), stream);
    if (e != cudaSuccess) return e;
    int n = *launches;
    // 2. every rank's records, over NVLink
    const size_t count = rec / sizeof(float);
    e = from_nccl(api.all_gather(local, gathered, count, ncclFloat32, static_cast<ncclComm_t>(comm), stream));
    if (e != cudaSuccess) return e;
    // 3. log-sum-exp merge into normalised rows (typed as desc->flags asks)
    const int64_t rows = static_cast<int64_t>(desc->batch) * desc->num_q_heads;
    const int64_t rs = desc->head_dim + 4;
    e = launch_combine_records(gathered, nranks, static_cast<int64_t>(count), rs, rows, desc->num_q_heads,
                               desc->head_dim, out, desc->o_stride_b, desc->o_stride_h,
                               desc->flags & kDtypeFlags & ~(KVD_FLAG_Q_BF16 | KVD_FLAG_Q_F16), stream, &n);
    *launches = n;
    return e;
}

// ---------------------------------------------------------------- peer exchange
// The sequence split without NCCL on the hot path: after the local decode, ONE
// kernel pushes this rank's records straight into every rank's gather buffer
// over NVLink (peer stores through CUDA IPC mappings), raises a flag per (rank,
// CTA) in every peer's memory, waits (bounded) for all ranks' flags of its own
// rows and merges them. NCCL is used once, at set-up, to swap the IPC handles.
//
// Epochs: CTA c keeps its own call count in local device memory; every rank
// runs the same calls, so CTA c of every rank uses the same epoch e and writes
// buffer parity e & 1. A rank can be at most one epoch ahead of a peer (its
// step e + 1 waited for the peer's step e flags... which the peer raised after
// finishing step e - 1), so two parities never collide.
namespace kvd {
namespace {

constexpr int kP2PRows = 4;         // record rows per CTA of the exchange kernel
constexpr int kMaxRanks = 8;

struct P2PPeers {
    float* gather[kMaxRanks];        // rank p's gather buffer [2][nranks][rows][D+4]
    unsigned int* flags[kMaxRanks];  // rank p's flags [nranks][ctas]
};

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(128) p2p_exchange_combine_kernel(
    const float* __restrict__ local, const P2PPeers peers, unsigned int* epochs, int nranks, int rank, int rows,
    int D, int rows_per_b, void* out, int64_t o_sb, int64_t o_sh, uint32_t flags) {
    const int c = blockIdx.x, ctas = gridDim.x;
    const int r0 = c * kP2PRows, r1 = min(rows, r0 + kP2PRows);
    const int rs = D + 4;
    __shared__ unsigned int e_sh;
    __shared__ int ok_sh;
    if (threadIdx.x == 0) e_sh = ++epochs[c];
    __syncthreads();
    const unsigned int e = e_sh;
    const int par = static_cast<int>(e & 1u);
    const size_t slab = static_cast<size_t>(rows) * rs;  // one rank's records
    // 1. push this CTA's rows of our records into every rank's buffer
    const float4* src = reinterpret_cast<const float4*>(local + static_cast<size_t>(r0) * rs);
    const int n4 = (r1 - r0) * rs / 4;
    for (int p = 0; p < nranks; ++p) {
        float4* dst = reinterpret_cast<float4*>(peers.gather[p] + (static_cast<size_t>(par) * nranks + rank) * slab +
                                                static_cast<size_t>(r0) * rs);
        for (int i = threadIdx.x; i < n4; i += blockDim.x) dst[i] = __ldg(src + i);
    }
    __syncthreads();
    // 2. publish: one release store per rank, ordered after every thread's stores
    if (threadIdx.x < nranks) {
        __threadfence_system();
        st_release_sys(peers.flags[threadIdx.x] + static_cast<size_t>(rank) * ctas + c, e);
    }
    // 3. wait for every rank's rows of this epoch (bounded)
    if (threadIdx.x == 0) ok_sh = 1;
    __syncthreads();
    if (threadIdx.x < nranks) {
        const unsigned int* f = peers.flags[rank] + static_cast<size_t>(threadIdx.x) * ctas + c;
        if (static_cast<int>(ld_acquire_sys(f) - e) < 0) {
            const uint64_t t0 = globaltimer_ns();
            while (static_cast<int>(ld_acquire_sys(f) - e) < 0) {
                __nanosleep(256);
                if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
                    record_status(KVD_STATUS_WAIT_TIMEOUT);
                    ok_sh = 0;
                    break;
                }
            }
        }
    }
    __syncthreads();
    if (!ok_sh) return;
    // 4. log-sum-exp merge of our rows (records read from L2: peers wrote them)
    const float* mine = peers.gather[rank] + static_cast<size_t>(par) * nranks * slab;
    for (int r = r0; r < r1; ++r) {
        float M = -INFINITY;
        for (int k = 0; k < nranks; ++k) M = fmaxf(M, __ldcg(mine + k * slab + static_cast<size_t>(r) * rs));
        const int b = r / rows_per_b, h = r - b * rows_per_b;
        const int64_t ro = b * o_sb + static_cast<int64_t>(h) * o_sh;
        for (int d = threadIdx.x; d < D; d += blockDim.x) {
            float O = 0.f, L = 0.f;
            if (M != -INFINITY) {
                for (int k = 0; k < nranks; ++k) {
                    const float* rec = mine + k * slab + static_cast<size_t>(r) * rs;
                    const float f = exp2f(__ldcg(rec) - M);
                    O = fmaf(f, __ldcg(rec + 4 + d), O);
                    L = fmaf(f, __ldcg(rec + 1), L);
                }
            }
            store_out(out, ro + d, L > 0.f ? O / L : 0.f, flags);
        }
    }
}

}  // namespace
}  // namespace kvd

struct kvd_mgpu_p2p {
    int nranks, rank, batch, heads, head_dim, rows, ctas;
    size_t slab_floats;
    void* region;             // this rank's gather buffer + flags (IPC-exported)
    unsigned int* epochs;     // local per-CTA epoch counters
    kvd::P2PPeers peers;
    void* opened[kvd::kMaxRanks];  // IPC mappings of the peers' regions
};

extern "C" cudaError_t kvd_mgpu_p2p_create(kvd_mgpu_p2p** out, int batch, int num_q_heads, int head_dim, void* comm,
                                           int nranks, int rank) {
    using namespace kvd;
    if (!out || !comm || batch < 1 || num_q_heads < 1 || head_dim < 1 || (head_dim & 3) != 0 || nranks < 1 ||
        nranks > kMaxRanks || rank < 0 || rank >= nranks)
        return cudaErrorInvalidValue;
    const NcclApi& api = nccl();
    if (!api.ok) return cudaErrorSharedObjectInitFailed;
    kvd_mgpu_p2p* c = new kvd_mgpu_p2p{};
    c->nranks = nranks; c->rank = rank; c->batch = batch; c->heads = num_q_heads; c->head_dim = head_dim;
    c->rows = batch * num_q_heads;
    c->ctas = (c->rows + kP2PRows - 1) / kP2PRows;
    c->slab_floats = static_cast<size_t>(c->rows) * (head_dim + 4);
    const size_t gather_bytes = align256(2 * static_cast<size_t>(nranks) * c->slab_floats * sizeof(float));
    const size_t flag_bytes = align256(static_cast<size_t>(nranks) * c->ctas * sizeof(unsigned int));
    cudaError_t e = cudaMalloc(&c->region, gather_bytes + flag_bytes);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&c->epochs), c->ctas * sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMemset(c->region, 0, gather_bytes + flag_bytes);
    if (e == cudaSuccess) e = cudaMemset(c->epochs, 0, c->ctas * sizeof(unsigned int));
    cudaIpcMemHandle_t mine{};
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&mine, c->region);
    // swap handles through NCCL (the all-gather also orders every rank's zeroing before any push)
    void* dh = nullptr;
    if (e == cudaSuccess) e = cudaMalloc(&dh, sizeof(cudaIpcMemHandle_t) * (nranks + 1));
    std::vector<cudaIpcMemHandle_t> all(nranks);
    if (e == cudaSuccess) e = cudaMemcpy(static_cast<char*>(dh) + sizeof(mine) * nranks, &mine, sizeof(mine),
                                         cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess)
        e = from_nccl(api.all_gather(static_cast<char*>(dh) + sizeof(mine) * nranks, dh, sizeof(mine), ncclUint8,
                                     static_cast<ncclComm_t>(comm), nullptr));
    if (e == cudaSuccess) e = cudaMemcpy(all.data(), dh, sizeof(mine) * nranks, cudaMemcpyDeviceToHost);
    if (dh) cudaFree(dh);
    for (int p = 0; p < nranks && e == cudaSuccess; ++p) {
        void* base = c->region;
        if (p != rank) {
            e = cudaIpcOpenMemHandle(&base, all[p], cudaIpcMemLazyEnablePeerAccess);
            c->opened[p] = e == cudaSuccess ? base : nullptr;
        }
        c->peers.gather[p] = static_cast<float*>(base);
        c->peers.flags[p] = reinterpret_cast<unsigned int*>(static_cast<char*>(base) + gather_bytes);
    }
    if (e != cudaSuccess) {
        kvd_mgpu_p2p_destroy(c);
        return e;
    }
    *out = c;
    return cudaSuccess;
}

extern "C" cudaError_t kvd_mgpu_p2p_destroy(kvd_mgpu_p2p* c) {
    if (!c) return cudaErrorInvalidValue;
    cudaError_t first = cudaDeviceSynchronize();
    for (int p = 0; p < c->nranks; ++p)
        if (c->opened[p]) {
            const cudaError_t e = cudaIpcCloseMemHandle(c->opened[p]);
            if (first == cudaSuccess) first = e;
        }
    if (c->region) cudaFree(c->region);
    if (c->epochs) cudaFree(c->epochs);
    delete c;
    return first;
}

extern "C" size_t kvd_mgpu_p2p_workspace_size(const kvd_decode_desc* desc) {
    if (!desc) return 0;
    return kvd_mgpu_seq_split_workspace_size(desc, 1);
}

extern "C" cudaError_t kvd_mgpu_p2p_seq_split_decode(kvd_mgpu_p2p* c, const kvd_decode_desc* desc, const void* Q,
                                                     const int8_t* K, const int8_t* V, const float* k_scale,
                                                     const float* v_scale, void* out, void* workspace,
                                                     size_t workspace_bytes, cudaStream_t stream) {
    using namespace kvd;
    int* launches = launch_counter();
    if (!c || !desc || !out || !workspace) return cudaErrorInvalidValue;
    if (desc->batch != c->batch || desc->num_q_heads != c->heads || desc->head_dim != c->head_dim ||
        (desc->flags & KVD_FLAG_PARTIAL_OUT))
        return cudaErrorInvalidValue;
    const size_t need = kvd_mgpu_p2p_workspace_size(desc);
    if (need == 0 || workspace_bytes < need) return cudaErrorInvalidValue;
    const kvd_decode_desc r = record_desc(*desc);
    const size_t rec = record_bytes(r);
    char* ws = static_cast<char*>(workspace);
    float* local = reinterpret_cast<float*>(ws);
    char* dws = ws + 2 * rec;
    cudaError_t e = kvd_decode_launch(&r, Q, K, V, k_scale, v_scale, local, dws, workspace_bytes - (dws - ws), stream);
    if (e != cudaSuccess) return e;
    int n = *launches;
    p2p_exchange_combine_kernel<<<c->ctas, 128, 0, stream>>>(
        local, c->peers, c->epochs, c->nranks, c->rank, c->rows, c->head_dim, c->heads, out, desc->o_stride_b,
        desc->o_stride_h, desc->flags & (KVD_FLAG_OUT_BF16 | KVD_FLAG_OUT_F16));
    e = cudaGetLastError();
    if (e == cudaSuccess) ++n;
    *launches = n;
    return e;
}
