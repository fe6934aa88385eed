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
    r.flags = KVD_FLAG_PARTIAL_OUT | (d.flags & (KVD_FLAG_Q_BF16 | KVD_FLAG_Q_F16));
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
