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
// The sequence split without NCCL on the hot path: ONE kernel, launched as a
// programmatic dependent of the local decode, merges this rank's split records
// of each row, pushes the merged record straight into every rank's gather
// buffer over NVLink (peer stores through CUDA IPC mappings), waits (bounded)
// for every rank's record of its rows and merges them into output rows. NCCL
// is used at set-up (to swap the IPC handles) and by the collective reset only.
//
// Tagged words: records cross NVLink as 8-byte words {value bits, epoch << 32}.
// An aligned 8-byte store is single-copy atomic, so a reader that sees the
// current epoch in a word also sees the value stored with it: no fence and no
// flag has to follow a push. The tensor-core decode (dense batch, group <= 4)
// writes its split records in the same form, so the exchange CTAs, resident
// beside the decode's, merge and push each row as soon as its records are
// there, during the decode's last items. Otherwise the decode writes float
// records and the kernel first waits (griddepcontrol.wait) for the whole
// decode grid.
//
// Epochs: CTA c keeps its own call count epochs[c] in local device memory and
// uses e = epochs[c] + 1, storing e back when it ends. Every rank makes the
// same calls, so CTA c of every rank uses the same e. The tagged decode tags
// its records with epochs[0] + 1, read by each of its CTAs before it allows
// this kernel to launch, so before CTA 0 can move epochs[0] on. Gather buffers
// alternate by parity e & 1: a rank can be at most one call ahead of a peer
// (its call e + 1 needs the peer's records of call e, pushed after the peer
// finished call e - 1), so two parities never collide. A rank that misses a
// call breaks the agreement: the others time out, and kvd_mgpu_p2p_reset
// restores it.
//
// Persistent grid: at most as many CTAs as fit on an idle GPU, each looping
// over its rows (first merging and pushing all of them, then waiting for the
// peers'). A programmatic dependent starts only after every CTA of the decode
// has started, so the decode runs to its end whatever the exchange waits for;
// and every exchange CTA pushes all its rows before it waits for a peer.
namespace kvd {
namespace {

constexpr int kP2PThreads = 128;  // 4 warps
constexpr int kP2PWarps = kP2PThreads / 32;
constexpr int kMaxRanks = 8;
constexpr int kMaxMerge = 256;  // records merged per row (split count cap of the planner)
constexpr int kMaxDim = 256;    // head_dim bound of the exchange (merged in passes of 128 dimensions)
constexpr int kRecs = 4;        // records a thread holds at once (x 4 dimensions = 16 tagged words)

struct P2PPeers {
    unsigned long long* gather[kMaxRanks];  // rank p's gather buffer [2][nranks][rows][D+4] tagged words
};

__device__ __forceinline__ void st_tagged(unsigned long long* p, float v, unsigned int e) {
    const unsigned long long w = (static_cast<unsigned long long>(e) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Two consecutive tagged words (p 16-byte aligned); each is single-copy atomic.
__device__ __forceinline__ void ld_tagged2(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ bool tag_is(unsigned long long w, unsigned int e) {
    return static_cast<unsigned int>(w >> 32) == e;
}

// One more poll of a word that does not carry the epoch yet: sleeps ns
// (doubled up to 512 ns for the next poll). t0 is the start of the first wait
// (0 before); returns false past kWaitTimeoutNs.
__device__ __forceinline__ bool backoff(uint64_t& t0, unsigned int& ns) {
    const uint64_t now = globaltimer_ns();
    if (t0 == 0) {
        t0 = now;
    } else if (now - t0 > kWaitTimeoutNs) {
        return false;
    }
    __nanosleep(ns);
    if (ns < 512) ns *= 2;
    return true;
}

// Waits (bounded) until the tagged word w, loaded from p, carries epoch e.
__device__ __forceinline__ bool wait_word(const unsigned long long* p, unsigned int e, unsigned long long& w,
                                          uint64_t& t0) {
    unsigned int ns = 64;
    while (!tag_is(w, e)) {
        if (!backoff(t0, ns)) return false;
        w = ld_tagged(p);
    }
    return true;
}

// About 4 KB: a CTA must fit in the shared memory that two CTAs of the
// group-1 decode leave on an SM, so that it runs while they do.
struct MergeSmem {
    float ms[kMaxMerge];  // the records' maxima, then their weights
    float ls[kMaxMerge];
    float part[kP2PWarps][128];  // per-warp partial sums of one pass of 128 dimensions
    float red[kP2PWarps];
};

// Log-sum-exp weights of n records from their maxima sm.ms[k] and sums
// sm.ls[k]: M = max_k ms[k], w_k = 2^(ms[k] - M) written over sm.ms[k], and
// L = sum_k w_k ls[k], returned to every thread. Starts after a barrier that
// made ms and ls complete; ends with one that makes the weights visible.
__device__ __forceinline__ void lse_weights(int n, MergeSmem& sm, float& M, float& L) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    if (n <= 32) {  // few records: every thread reads them all
        M = -INFINITY;
        for (int k = 0; k < n; ++k) M = fmaxf(M, sm.ms[k]);
        L = 0.f;
        float mine = 0.f;
        for (int k = 0; k < n; ++k) {
            const float f = M == -INFINITY ? 0.f : exp2f(sm.ms[k] - M);
            if (k == t) mine = f;
            L = fmaf(f, sm.ls[k], L);
        }
        __syncthreads();  // every thread has read the maxima
        if (t < n) sm.ms[t] = mine;
        __syncthreads();
        return;
    }
    float m = -INFINITY;
    for (int k = t; k < n; k += blockDim.x) m = fmaxf(m, sm.ms[k]);
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) sm.red[warp] = m;
    __syncthreads();
    M = sm.red[0];
    for (int w = 1; w < kP2PWarps; ++w) M = fmaxf(M, sm.red[w]);
    float l = 0.f;
    for (int k = t; k < n; k += blockDim.x) {  // each thread its own records only
        const float f = M == -INFINITY ? 0.f : exp2f(sm.ms[k] - M);
        sm.ms[k] = f;
        l = fmaf(f, sm.ls[k], l);
    }
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    __syncthreads();  // every thread has read the maxima in red
    if (lane == 0) sm.red[warp] = l;
    __syncthreads();  // the sums are in red and the weights in ms
    L = 0.f;
    for (int w = 0; w < kP2PWarps; ++w) L += sm.red[w];
}

// One thread's share of a row of n tagged records (record k at first +
// k * stride: m, l, 2 unused, o[D]): with_ml, m and l of records t, t + 128,
// ... into sm.ms / sm.ls; and o[4g .. 4g+3] (g = dimension group) of the
// records k0 + warp + 4j (j < kRecs) into o[j]. All loads are issued before
// the first check. wait == false: returns whether every word carries epoch e.
// wait == true: a word that does not is polled alone until it does (bounded);
// false on timeout.
__device__ __forceinline__ bool load_share(const unsigned long long* first, int n, size_t stride, int g, int k0,
                                           bool with_ml, unsigned int e, MergeSmem& sm, float (&o)[kRecs][4],
                                           bool wait, uint64_t& t0) {
    const int t = threadIdx.x, warp = t >> 5;
    unsigned long long w[kRecs][4];
#pragma unroll
    for (int j = 0; j < kRecs; ++j) {
        const int k = k0 + warp + kP2PWarps * j;
        if (k < n) {
            const unsigned long long* q = first + k * stride + 4 + 4 * g;
            ld_tagged2(q, w[j][0], w[j][1]);
            ld_tagged2(q + 2, w[j][2], w[j][3]);
        }
    }
    bool all = true;
    if (with_ml)
        for (int k = t; k < n; k += blockDim.x) {
            unsigned long long m, l;
            ld_tagged2(first + k * stride, m, l);
            if (wait) {
                if (!wait_word(first + k * stride, e, m, t0) || !wait_word(first + k * stride + 1, e, l, t0))
                    return false;
            } else if (!tag_is(m, e) || !tag_is(l, e)) {
                all = false;
            }
            sm.ms[k] = __uint_as_float(static_cast<unsigned int>(m));
            sm.ls[k] = __uint_as_float(static_cast<unsigned int>(l));
        }
#pragma unroll
    for (int j = 0; j < kRecs; ++j) {
        const int k = k0 + warp + kP2PWarps * j;
        if (k < n) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (!tag_is(w[j][i], e)) {
                    if (!wait) {
                        all = false;
                        continue;
                    }
                    if (!wait_word(first + k * stride + 4 + 4 * g + i, e, w[j][i], t0)) return false;
                }
                o[j][i] = __uint_as_float(static_cast<unsigned int>(w[j][i]));
            }
        }
    }
    return all;
}

// Log-sum-exp merge of the n tagged records of one row (record k at first +
// k * stride, D+4 words; n <= kMaxMerge, D <= kMaxDim, D % 4 == 0) by the
// whole CTA, once every word it uses carries epoch e. Lane l of each warp
// takes dimensions 4l .. 4l+3 (and 128 higher, for D > 128); warp w takes
// records w, w + 4, ..., kRecs at a time, so up to 16 records cost one round
// of loads. emit(d, O, L) receives each dimension's unnormalised sum
// O = sum_k w_k o_k[d], w_k = 2^(m_k - M), with L = sum_k w_k l_k; M and L
// are also returned. When a first round finds words missing, one thread polls
// (with backoff) until the first word of every record carries e, and the CTA
// loads again, so a waiting CTA adds one poller, not one a thread. A thread
// reads a word again only after it has seen it tagged with e. Returns false
// (on every thread) when a wait ran out.
template <class Emit>
__device__ __forceinline__ bool merge_tagged(const unsigned long long* first, int n, size_t stride, int D,
                                             unsigned int e, MergeSmem& sm, float& M, float& L, Emit emit) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int groups = D >> 2;
    float o[kRecs][4];
    uint64_t t0 = 0;
    const int g0 = lane < groups ? lane : 0;  // this lane's first dimension group
    bool ok = load_share(first, n, stride, g0, 0, true, e, sm, o, false, t0);
    if (!__syncthreads_and(ok)) {
        ok = true;
        if (t == 0) {
            unsigned int ns = 64;
            for (int k = 0; k < n && ok; ++k)
                while (!tag_is(ld_tagged(first + k * stride), e))
                    if (!backoff(t0, ns)) {
                        ok = false;
                        break;
                    }
        }
        if (!__syncthreads_and(ok)) return false;
        ok = load_share(first, n, stride, g0, 0, true, e, sm, o, true, t0);
        if (!__syncthreads_and(ok)) return false;
    }
    lse_weights(n, sm, M, L);
    // per-warp partial sums over its records, in passes of 128 dimensions
    for (int base = 0; base < D; base += 128) {
        const int g = (base >> 2) + lane;  // this lane's dimension group in the pass
        if (g < groups) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            for (int k0 = 0; k0 < n && ok; k0 += kP2PWarps * kRecs) {
                // records not held from the first round: load again (waiting where a tag is not there yet)
                if ((base > 0 || k0 > 0) && !load_share(first, n, stride, g, k0, false, e, sm, o, true, t0)) {
                    ok = false;
                    break;
                }
#pragma unroll
                for (int j = 0; j < kRecs; ++j) {
                    const int k = k0 + warp + kP2PWarps * j;
                    if (k < n) {
                        const float f = sm.ms[k];
#pragma unroll
                        for (int i = 0; i < 4; ++i) acc[i] = fmaf(f, o[j][i], acc[i]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) sm.part[warp][4 * lane + i] = acc[i];
        }
        if (!__syncthreads_and(ok)) return false;
        if (base + t < D) {
            float O = 0.f;
#pragma unroll
            for (int w = 0; w < kP2PWarps; ++w) O += sm.part[w][t];
            emit(base + t, O, L);
        }
        __syncthreads();  // sm is rewritten by the next pass or row
    }
    return true;
}

// The same merge over n float records written by a decode grid that has
// completed (record k at first + k * stride).
template <class Emit>
__device__ __forceinline__ void merge_float(const float* first, int n, size_t stride, int D, MergeSmem& sm, float& M,
                                            float& L, Emit emit) {
    const int t = threadIdx.x;
    for (int k = t; k < n; k += blockDim.x) {
        sm.ms[k] = __ldcg(first + k * stride);
        sm.ls[k] = __ldcg(first + k * stride + 1);
    }
    __syncthreads();
    lse_weights(n, sm, M, L);
    for (int d = t; d < D; d += blockDim.x) {
        float O = 0.f;
#pragma unroll 8
        for (int k = 0; k < n; ++k) O = fmaf(sm.ms[k], __ldcg(first + k * stride + 4 + d), O);
        emit(d, O, L);
    }
    __syncthreads();  // sm is rewritten by the next row
}

// Records of this rank: tagged (P per row, from a tagged decode that may still
// be running) or float (src, P per row, from a completed decode grid).
// At most 144 registers a thread (launched with kP2PThreads threads) and
// about 4 KB of shared memory: a CTA then fits on an SM beside two CTAs of the
// group-1 decode (120 registers a thread after allocation rounding, 2 x 95 KB
// of shared memory) and runs while they do.
__global__ void __maxnreg__(144) p2p_exchange_combine_kernel(
    const float* __restrict__ src, const unsigned long long* tagged, int P, const __grid_constant__ P2PPeers peers,
    unsigned int* epochs, int nranks, int rank, int rows, int D, int rows_per_b, void* out, int64_t o_sb,
    int64_t o_sh, uint32_t flags) {
    const int c = blockIdx.x, ctas = gridDim.x, t = threadIdx.x;
    const int rs = D + 4;
    __shared__ MergeSmem sm;
    // The next call's tagged decode may launch now: it sets up beside this grid and
    // waits for its completion before it touches global memory.
    allow_dependents();
    if (!tagged) grid_dependency_wait();  // launched as a programmatic dependent: the float records are complete
    const unsigned int e = *reinterpret_cast<volatile unsigned int*>(epochs + c) + 1;
    const int par = static_cast<int>(e & 1u);
    const size_t slab = static_cast<size_t>(rows) * rs;  // one rank's records
    // 1. per row: merge this rank's split records and push the merged record
    //    into every rank's gather buffer
    for (int r = c; r < rows; r += ctas) {
        const size_t dst_off = (static_cast<size_t>(par) * nranks + rank) * slab + static_cast<size_t>(r) * rs;
        auto push = [&](int d, float O, float) {
            for (int p = 0; p < nranks; ++p) st_tagged(peers.gather[p] + dst_off + 4 + d, O, e);
        };
        float M, L;
        if (tagged) {
            if (!merge_tagged(tagged + static_cast<size_t>(r) * P * rs, P, rs, D, e, sm, M, L, push)) {
                if (t == 0) record_status(KVD_STATUS_WAIT_TIMEOUT);  // the decode did not finish this row
                return;
            }
        } else {
            merge_float(src + static_cast<size_t>(r) * P * rs, P, rs, D, sm, M, L, push);
        }
        if (t < nranks) {  // the row's M and L, one rank per thread
            st_tagged(peers.gather[t] + dst_off, M, e);
            st_tagged(peers.gather[t] + dst_off + 1, L, e);
        }
    }
    // 2. per row: every rank's record (bounded waits on the tags), merged into
    //    the output row
    const unsigned long long* mine = peers.gather[rank] + static_cast<size_t>(par) * nranks * slab;
    for (int r = c; r < rows; r += ctas) {
        const int b = r / rows_per_b, h = r - b * rows_per_b;
        const int64_t ro = b * o_sb + static_cast<int64_t>(h) * o_sh;
        float M, L;
        auto write = [&](int d, float O, float Lr) { store_out(out, ro + d, Lr > 0.f ? O / Lr : 0.f, flags); };
        if (!merge_tagged(mine + static_cast<size_t>(r) * rs, nranks, slab, D, e, sm, M, L, write)) {
            if (t == 0) record_status(KVD_STATUS_WAIT_TIMEOUT);  // a rank missed this call: rows stay unwritten
            return;
        }
    }
    if (t == 0) epochs[c] = e;  // this CTA's call is complete
}

}  // namespace
}  // namespace kvd

struct kvd_mgpu_p2p {
    int nranks, rank, batch, heads, head_dim, rows, ctas;
    int device;               // the rank's device
    size_t slab_floats, region_bytes;
    void* comm;               // the communicator given at creation (reset barriers); nullptr in a group
    void* region;             // this rank's gather buffer of tagged words (IPC-exported)
    unsigned int* epochs;     // [ctas] the exchange CTAs' call counts (local)
    int* barrier_buf;         // [nranks + 1] ints for the reset's NCCL barriers
    kvd::P2PPeers peers;
    void* opened[kvd::kMaxRanks];  // IPC mappings of the peers' regions
};

extern "C" cudaError_t kvd_mgpu_p2p_create(kvd_mgpu_p2p** out, int batch, int num_q_heads, int head_dim, void* comm,
                                           int nranks, int rank) {
    using namespace kvd;
    if (!out || !comm || batch < 1 || num_q_heads < 1 || head_dim < 1 || head_dim > kMaxDim || (head_dim & 3) != 0 || nranks < 1 ||
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
    c->ctas = static_cast<int>(c->rows < resident ? c->rows : resident);
    c->slab_floats = static_cast<size_t>(c->rows) * (head_dim + 4);
    c->region_bytes = align256(2 * static_cast<size_t>(nranks) * c->slab_floats * sizeof(unsigned long long));
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
        c->peers.gather[p] = static_cast<unsigned long long*>(base);
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
    if (!ctxs || !devices || batch < 1 || num_q_heads < 1 || head_dim < 1 || head_dim > kMaxDim || (head_dim & 3) != 0 || nranks < 1 ||
        nranks > kMaxRanks)
        return cudaErrorInvalidValue;
    for (int r = 0; r < nranks; ++r) ctxs[r] = nullptr;
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return e;
    const int rows = batch * num_q_heads;
    int64_t ctas = rows;
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
        c->region_bytes = align256(2 * static_cast<size_t>(nranks) * slab * sizeof(unsigned long long));
        e = cudaMalloc(&c->region, c->region_bytes);
        if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&c->epochs), c->ctas * sizeof(unsigned int));
        if (e == cudaSuccess) e = cudaMemset(c->region, 0, c->region_bytes);
        if (e == cudaSuccess) e = cudaMemset(c->epochs, 0, c->ctas * sizeof(unsigned int));
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
    }
    for (int r = 0; r < nranks && e == cudaSuccess; ++r)
        for (int q = 0; q < nranks; ++q) {
            ctxs[r]->peers.gather[q] = static_cast<unsigned long long*>(ctxs[q]->region);
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
    // 3. epochs and gather buffers back to their state at creation
    if (e == cudaSuccess) e = cudaMemsetAsync(c->region, 0, c->region_bytes, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(c->epochs, 0, c->ctas * sizeof(unsigned int), stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    // 4. no rank pushes into a peer's buffers before that peer has cleared them
    if (e == cudaSuccess) e = p2p_barrier(c, stream);
    return e;
}

namespace {
// Bytes of the tagged split records of a tensor-core decode of `r` (0 when
// the decode cannot write them).
size_t tagged_record_bytes(const kvd_decode_desc& r) {
    const int P = kvd::gqa_tagged_splits(r);
    return P > 0 ? kvd::align256(static_cast<size_t>(r.batch) * r.num_q_heads * P * (r.head_dim + 4) *
                                 sizeof(unsigned long long))
                 : 0;
}
}  // namespace

extern "C" size_t kvd_mgpu_p2p_workspace_size(const kvd_decode_desc* desc) {
    if (!desc) return 0;
    const size_t base = kvd_mgpu_seq_split_workspace_size(desc, 1);
    return base ? base + tagged_record_bytes(record_desc(*desc)) : 0;
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
    // workspace: float records [rec] | (unused) [rec] | decode workspace | tagged records
    const size_t base = kvd_mgpu_seq_split_workspace_size(desc, 1);
    char* ws = static_cast<char*>(workspace);
    float* local = reinterpret_cast<float*>(ws);
    char* dws = ws + 2 * rec;
    const size_t dws_bytes = base - 2 * rec;
    // 1. this rank's token range -> records. A dense tensor-core decode leaves
    //    its split records in the workspace (tagged where it can) and the
    //    exchange kernel merges them, so no separate combine launch runs.
    SplitRecords splits{local, 1, nullptr, 0, c->epochs, false};
    if (tagged_record_bytes(r) > 0) {
        splits.tagged = reinterpret_cast<unsigned long long*>(ws + base);
        splits.tagged_P = gqa_tagged_splits(r);
    }
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
    // 2. merge, push, wait, merge: one kernel, launched as a programmatic
    // dependent so that its CTAs are resident while the decode runs. With
    // tagged records they merge and push each row as soon as its records are
    // there; otherwise they wait (griddepcontrol.wait) for the decode grid.
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(c->ctas), 1, 1);
    cfg.blockDim = dim3(kP2PThreads, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, p2p_exchange_combine_kernel, static_cast<const float*>(splits.partials),
                           static_cast<const unsigned long long*>(splits.tagged_used ? splits.tagged : nullptr),
                           splits.P, c->peers, c->epochs, c->nranks, c->rank, c->rows, c->head_dim, c->heads, out,
                           static_cast<int64_t>(desc->o_stride_b), static_cast<int64_t>(desc->o_stride_h),
                           static_cast<uint32_t>(desc->flags & (KVD_FLAG_OUT_BF16 | KVD_FLAG_OUT_F16)));
    if (e == cudaSuccess) ++n;
    *launches = n;
    return e;
}
