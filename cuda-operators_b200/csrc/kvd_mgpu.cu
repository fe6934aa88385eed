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
// kernel merges this rank's split records of each row, pushes the merged
// record straight into every rank's gather buffer over NVLink (peer stores
// through CUDA IPC mappings), raises a flag per (rank, CTA) in every peer's
// memory, waits (bounded) for all ranks' flags and merges the gathered records
// into output rows. NCCL is used at set-up (to swap the IPC handles) and by
// the collective reset only.
//
// Persistent grid: the kernel runs at most as many CTAs as fit on the GPU at
// once, each looping over row blocks (first pushing all of them, then waiting).
// Every CTA therefore runs and pushes before any CTA of this rank has to wait,
// so no CTA waits on a peer CTA that cannot be scheduled, whatever the batch.
//
// Epochs: CTA c keeps its own call count in local device memory; every rank
// runs the same calls, so CTA c of every rank uses the same epoch e and writes
// buffer parity e & 1. A rank can be at most one epoch ahead of a peer (its
// step e + 1 needs the peer's step-e flags, raised after the peer finished
// step e - 1), so two parities never collide. A rank that misses a call breaks
// that agreement: the others time out, and kvd_mgpu_p2p_reset restores it.
namespace kvd {
namespace {

constexpr int kP2PRows = 1;         // record rows per block of the exchange kernel
constexpr int kP2PThreads = 128;
constexpr int kMaxRanks = 8;
constexpr int kMaxMerge = 256;      // records merged per row (split count cap of the planner)

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

// Log-sum-exp weights of the n records of one row (record k at first +
// k*stride, n <= kMaxMerge), computed by the whole CTA: the records' maxima
// and weights wk[k] = 2^(m_k - M) are each computed once, spread over the
// threads and kept in shared memory, so the per-dimension sums that follow
// (sum_k wk[k] * o_k[d]) run over independent loads. Every thread returns M
// and L = sum_k wk[k] * l_k. Ends with a barrier: red is free again, wk holds
// the weights until the caller's next barrier.
template <bool CACHED>
__device__ __forceinline__ void merge_weights(const float* first, int n, size_t stride, float* wk, float* red,
                                              float& M, float& L) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nw = blockDim.x >> 5;
    auto ld = [](const float* x) { return CACHED ? __ldcg(x) : __ldg(x); };
    float m = -INFINITY;
    for (int k = t; k < n; k += blockDim.x) m = fmaxf(m, ld(first + k * stride));
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    M = red[0];
    for (int w = 1; w < nw; ++w) M = fmaxf(M, red[w]);
    float l = 0.f;
    for (int k = t; k < n; k += blockDim.x) {
        const float f = M == -INFINITY ? 0.f : exp2f(ld(first + k * stride) - M);
        wk[k] = f;
        l = fmaf(f, ld(first + k * stride + 1), l);
    }
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    __syncthreads();  // every thread has read the maxima in red
    if (lane == 0) red[warp] = l;
    __syncthreads();  // the sums are in red and the weights in wk
    L = 0.f;
    for (int w = 0; w < nw; ++w) L += red[w];
    __syncthreads();  // red is reused by the next call
}

template <bool CACHED>
__device__ __forceinline__ float merged_dim(const float* first, int n, size_t stride, const float* wk, int d) {
    float acc = 0.f;
#pragma unroll 4
    for (int k = 0; k < n; ++k) acc = fmaf(wk[k], CACHED ? __ldcg(first + k * stride + 4 + d) : __ldg(first + k * stride + 4 + d), acc);
    return acc;
}

// src: this rank's records, P consecutive records of D+4 floats per row (the
// decode's split records; P == 1: one record per row).
__global__ void __launch_bounds__(kP2PThreads) p2p_exchange_combine_kernel(
    const float* __restrict__ src, int P, const P2PPeers peers, unsigned int* epochs, int nranks, int rank,
    int rows, int D, int rows_per_b, void* out, int64_t o_sb, int64_t o_sh, uint32_t flags) {
    const int c = blockIdx.x, ctas = gridDim.x;
    const int rs = D + 4;
    const int nblk = (rows + kP2PRows - 1) / kP2PRows;
    __shared__ unsigned int e_sh;
    __shared__ int ok_sh;
    __shared__ float wk[kMaxMerge];
    __shared__ float red[kP2PThreads / 32];
    grid_dependency_wait();  // launched as a programmatic dependent of the local decode: its records are complete
    if (threadIdx.x == 0) e_sh = ++epochs[c];
    __syncthreads();
    const unsigned int e = e_sh;
    const int par = static_cast<int>(e & 1u);
    const size_t slab = static_cast<size_t>(rows) * rs;  // one rank's records
    // 1. merge this rank's split records of every row of this CTA's blocks and
    //    push the merged record into every rank's gather buffer
    for (int blk = c; blk < nblk; blk += ctas) {
        const int r1 = min(rows, (blk + 1) * kP2PRows);
        for (int r = blk * kP2PRows; r < r1; ++r) {
            const float* rec = src + static_cast<size_t>(r) * P * rs;
            const size_t dst_off = (static_cast<size_t>(par) * nranks + rank) * slab + static_cast<size_t>(r) * rs;
            if (P == 1) {
                for (int i = threadIdx.x; i < rs / 4; i += blockDim.x) {
                    const float4 v = __ldg(reinterpret_cast<const float4*>(rec) + i);
                    for (int p = 0; p < nranks; ++p) reinterpret_cast<float4*>(peers.gather[p] + dst_off)[i] = v;
                }
                continue;
            }
            float M, L;
            merge_weights<false>(rec, P, rs, wk, red, M, L);
            for (int d = threadIdx.x; d < D; d += blockDim.x) {
                const float O = merged_dim<false>(rec, P, rs, wk, d);
                for (int p = 0; p < nranks; ++p) {
                    float* dst = peers.gather[p] + dst_off;
                    dst[4 + d] = O;
                    if (d == 0) { dst[0] = M; dst[1] = L; }
                }
            }
            __syncthreads();  // wk is rewritten by the next row
        }
    }
    __syncthreads();
    // 2. publish: one release store per rank, ordered after every thread's stores
    if (threadIdx.x < nranks) {
        __threadfence_system();
        st_release_sys(peers.flags[threadIdx.x] + static_cast<size_t>(rank) * ctas + c, e);
    }
    // 3. wait for every rank's flag of this CTA and epoch (bounded)
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
    if (!ok_sh) return;  // a rank missed this call: these rows stay unwritten (the status says so)
    // 4. log-sum-exp merge of this CTA's rows (records read from L2: peers wrote them)
    const float* mine = peers.gather[rank] + static_cast<size_t>(par) * nranks * slab;
    for (int blk = c; blk < nblk; blk += ctas) {
        const int r1 = min(rows, (blk + 1) * kP2PRows);
        for (int r = blk * kP2PRows; r < r1; ++r) {
            const float* first = mine + static_cast<size_t>(r) * rs;
            float M, L;
            merge_weights<true>(first, nranks, slab, wk, red, M, L);
            const int b = r / rows_per_b, h = r - b * rows_per_b;
            const int64_t ro = b * o_sb + static_cast<int64_t>(h) * o_sh;
            for (int d = threadIdx.x; d < D; d += blockDim.x) {
                const float O = merged_dim<true>(first, nranks, slab, wk, d);
                store_out(out, ro + d, L > 0.f ? O / L : 0.f, flags);
            }
            __syncthreads();  // wk is rewritten by the next row
        }
    }
}

}  // namespace
}  // namespace kvd

struct kvd_mgpu_p2p {
    int nranks, rank, batch, heads, head_dim, rows, ctas;
    int device;               // the rank's device
    size_t slab_floats, region_bytes;
    void* comm;               // the communicator given at creation (reset barriers); nullptr in a group
    void* region;             // this rank's gather buffer + flags (IPC-exported)
    unsigned int* epochs;     // local per-CTA epoch counters
    int* barrier_buf;         // [nranks + 1] ints for the reset's NCCL barriers
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
    // Co-resident bound of the persistent exchange grid (every CTA must be able
    // to run while the others wait).
    int per_sm = 0;
    cudaError_t e =
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, p2p_exchange_combine_kernel, kP2PThreads, 0);
    if (e != cudaSuccess) return e;
    const int64_t resident = static_cast<int64_t>(device_sm_count()) * (per_sm > 0 ? per_sm : 1);
    kvd_mgpu_p2p* c = new kvd_mgpu_p2p{};
    c->nranks = nranks; c->rank = rank; c->batch = batch; c->heads = num_q_heads; c->head_dim = head_dim;
    c->comm = comm;
    cudaGetDevice(&c->device);
    c->rows = batch * num_q_heads;
    const int64_t nblk = (c->rows + kP2PRows - 1) / kP2PRows;
    c->ctas = static_cast<int>(nblk < resident ? nblk : resident);
    c->slab_floats = static_cast<size_t>(c->rows) * (head_dim + 4);
    const size_t gather_bytes = align256(2 * static_cast<size_t>(nranks) * c->slab_floats * sizeof(float));
    const size_t flag_bytes = align256(static_cast<size_t>(nranks) * c->ctas * sizeof(unsigned int));
    c->region_bytes = gather_bytes + flag_bytes;
    e = cudaMalloc(&c->region, c->region_bytes);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&c->epochs), c->ctas * sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&c->barrier_buf), (nranks + 1) * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->region, 0, c->region_bytes);
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
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    cudaError_t first = cudaDeviceSynchronize();
    for (int p = 0; p < c->nranks; ++p)
        if (c->opened[p]) {
            const cudaError_t e = cudaIpcCloseMemHandle(c->opened[p]);
            if (first == cudaSuccess) first = e;
        }
    if (c->region) cudaFree(c->region);
    if (c->epochs) cudaFree(c->epochs);
    if (c->barrier_buf) cudaFree(c->barrier_buf);
    delete c;
    cudaSetDevice(prev);
    return first;
}

extern "C" cudaError_t kvd_mgpu_p2p_create_group(kvd_mgpu_p2p** ctxs, int nranks, const int* devices, int batch,
                                                 int num_q_heads, int head_dim) {
    using namespace kvd;
    if (!ctxs || !devices || batch < 1 || num_q_heads < 1 || head_dim < 1 || (head_dim & 3) != 0 || nranks < 1 ||
        nranks > kMaxRanks)
        return cudaErrorInvalidValue;
    for (int r = 0; r < nranks; ++r) ctxs[r] = nullptr;
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return e;
    const int rows = batch * num_q_heads;
    int64_t ctas = (rows + kP2PRows - 1) / kP2PRows;
    // every rank runs the same grid: the co-resident bound of the smallest device
    for (int r = 0; r < nranks && e == cudaSuccess; ++r) {
        e = cudaSetDevice(devices[r]);
        int per_sm = 0;
        if (e == cudaSuccess)
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, p2p_exchange_combine_kernel, kP2PThreads, 0);
        const int64_t resident = static_cast<int64_t>(device_sm_count()) * (per_sm > 0 ? per_sm : 1);
        if (resident < ctas) ctas = resident;
    }
    // direct peer access between the distinct devices of the group
    for (int r = 0; r < nranks && e == cudaSuccess; ++r)
        for (int q = 0; q < nranks && e == cudaSuccess; ++q) {
            if (devices[q] == devices[r]) continue;
            int can = 0;
            e = cudaDeviceCanAccessPeer(&can, devices[r], devices[q]);
            if (e == cudaSuccess && !can) e = cudaErrorPeerAccessUnsupported;
            if (e == cudaSuccess) e = cudaSetDevice(devices[r]);
            if (e == cudaSuccess) {
                e = cudaDeviceEnablePeerAccess(devices[q], 0);
                if (e == cudaErrorPeerAccessAlreadyEnabled) {
                    cudaGetLastError();  // already enabled (by the caller or an earlier group): fine
                    e = cudaSuccess;
                }
            }
        }
    const size_t slab = static_cast<size_t>(rows) * (head_dim + 4);
    const size_t gather_bytes = align256(2 * static_cast<size_t>(nranks) * slab * sizeof(float));
    const size_t flag_bytes = align256(static_cast<size_t>(nranks) * ctas * sizeof(unsigned int));
    for (int r = 0; r < nranks && e == cudaSuccess; ++r) {
        e = cudaSetDevice(devices[r]);
        if (e != cudaSuccess) break;
        kvd_mgpu_p2p* c = new kvd_mgpu_p2p{};
        ctxs[r] = c;
        c->nranks = nranks; c->rank = r; c->batch = batch; c->heads = num_q_heads; c->head_dim = head_dim;
        c->device = devices[r];
        c->comm = nullptr;
        c->rows = rows;
        c->ctas = static_cast<int>(ctas);
        c->slab_floats = slab;
        c->region_bytes = gather_bytes + flag_bytes;
        e = cudaMalloc(&c->region, c->region_bytes);
        if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&c->epochs), c->ctas * sizeof(unsigned int));
        if (e == cudaSuccess) e = cudaMemset(c->region, 0, c->region_bytes);
        if (e == cudaSuccess) e = cudaMemset(c->epochs, 0, c->ctas * sizeof(unsigned int));
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
    }
    for (int r = 0; r < nranks && e == cudaSuccess; ++r)
        for (int q = 0; q < nranks; ++q) {
            ctxs[r]->peers.gather[q] = static_cast<float*>(ctxs[q]->region);
            ctxs[r]->peers.flags[q] = reinterpret_cast<unsigned int*>(static_cast<char*>(ctxs[q]->region) + gather_bytes);
        }
    if (e != cudaSuccess) {
        for (int r = 0; r < nranks; ++r)
            if (ctxs[r]) {
                kvd_mgpu_p2p_destroy(ctxs[r]);
                ctxs[r] = nullptr;
            }
    }
    cudaSetDevice(prev);
    return e;
}

namespace {
// Every rank of the context's communicator reaches this point before any
// returns: an NCCL all-gather of one int, waited for on the host.
cudaError_t p2p_barrier(kvd_mgpu_p2p* c, cudaStream_t stream) {
    const kvd::NcclApi& api = kvd::nccl();
    if (!api.ok) return cudaErrorSharedObjectInitFailed;
    cudaError_t e = kvd::from_nccl(api.all_gather(c->barrier_buf + c->nranks, c->barrier_buf, 1, ncclInt32,
                                                  static_cast<ncclComm_t>(c->comm), stream));
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    return e;
}
}  // namespace

extern "C" cudaError_t kvd_mgpu_p2p_reset(kvd_mgpu_p2p* c, cudaStream_t stream) {
    if (!c) return cudaErrorInvalidValue;
    if (!c->comm) {  // a single-process group: the caller resets every rank with no decode in flight
        int prev = 0;
        cudaGetDevice(&prev);
        cudaError_t e = cudaSetDevice(c->device);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = cudaMemset(c->region, 0, c->region_bytes);
        if (e == cudaSuccess) e = cudaMemset(c->epochs, 0, c->ctas * sizeof(unsigned int));
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        cudaSetDevice(prev);
        return e;
    }
    // 1. none of this rank's exchanges is still running
    cudaError_t e = cudaDeviceSynchronize();
    // 2. none of any rank's (every rank is past step 1)
    if (e == cudaSuccess) e = p2p_barrier(c, stream);
    // 3. epochs, flags and gather buffers back to their state at creation
    if (e == cudaSuccess) e = cudaMemsetAsync(c->region, 0, c->region_bytes, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(c->epochs, 0, c->ctas * sizeof(unsigned int), stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    // 4. no rank pushes into a peer's buffers before that peer has cleared them
    if (e == cudaSuccess) e = p2p_barrier(c, stream);
    return e;
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
    if (!c || !desc || !out || !workspace || !Q || !K || !V || !k_scale || !v_scale) return cudaErrorInvalidValue;
    if (desc->batch != c->batch || desc->num_q_heads != c->heads || desc->head_dim != c->head_dim ||
        (desc->flags & KVD_FLAG_PARTIAL_OUT))
        return cudaErrorInvalidValue;
    const size_t need = kvd_mgpu_p2p_workspace_size(desc);
    if (need == 0 || workspace_bytes < need) return cudaErrorInvalidValue;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != c->device) return cudaErrorInvalidDevice;  // the rank's own GPU
    const kvd_decode_desc r = record_desc(*desc);
    const size_t rec = record_bytes(r);
    char* ws = static_cast<char*>(workspace);
    float* local = reinterpret_cast<float*>(ws);
    char* dws = ws + 2 * rec;
    const size_t dws_bytes = workspace_bytes - (dws - ws);
    // 1. this rank's token range -> records. A dense tensor-core decode leaves
    //    its split records in the workspace and the exchange kernel merges them,
    //    so no separate combine launch runs.
    SplitRecords splits{local, 1};
    cudaError_t e;
    int n = 0;
    if (!r.seq_lens && fast_path_ok(r, Q, K, V) && gqa_path_ok(r)) {
        e = launch_gqa_tc(r, Q, K, V, k_scale, v_scale, local, dws, dws_bytes, stream, &n, nullptr, nullptr,
                          &splits);
        if (splits.P == 1) splits.partials = local;
    } else {
        e = kvd_decode_launch(&r, Q, K, V, k_scale, v_scale, local, dws, dws_bytes, stream);
        n = *launches;
    }
    if (e != cudaSuccess) {
        *launches = n;
        return e;
    }
    // 2. merge, push, wait, merge: one kernel
    // Programmatic dependent launch: the exchange's CTAs may be scheduled while the
    // decode's last CTAs run and wait (griddepcontrol.wait) for its completion.
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(c->ctas), 1, 1);
    cfg.blockDim = dim3(kP2PThreads, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, p2p_exchange_combine_kernel, static_cast<const float*>(splits.partials), splits.P,
                           c->peers, c->epochs, c->nranks, c->rank, c->rows, c->head_dim, c->heads, out,
                           static_cast<int64_t>(desc->o_stride_b), static_cast<int64_t>(desc->o_stride_h),
                           static_cast<uint32_t>(desc->flags & (KVD_FLAG_OUT_BF16 | KVD_FLAG_OUT_F16)));
    if (e == cudaSuccess) ++n;
    *launches = n;
    return e;
}
