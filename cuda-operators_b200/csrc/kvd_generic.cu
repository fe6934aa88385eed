// kvd_generic.cu -- split-KV decode for shapes the TMA kernel does not take:
// head_dim outside {64, 128} (up to 512), or pointers / strides that are not
// 16-byte aligned. Plain coalesced global loads, one block per (head, split),
// online softmax per 64-token chunk, partials combined by a second kernel.
// Same mathematics and output contract as kvd_splitkv.cu; it exists so that
// every shape the reference's solve() accepts (kv_cache/KV_int8_split_optimized.cu
// accepts any head_dim whose query fits in shared memory) still runs on the GPU.
#include "kvd_common.cuh"
#include "kvd_decode.cuh"

namespace kvd {

namespace {
constexpr int kGenThreads = 128;
constexpr int kGenChunk = 64;
constexpr int kGenMaxD = 512;
constexpr int kGenDPT = kGenMaxD / kGenThreads;  // dims per thread

struct GenParams {
    const void* Q;  // fp32, bf16 or fp16 (flags)
    const int8_t* K;
    const int8_t* V;
    const float* ks;
    const float* vs;
    void* out;        // normalised rows (fp32, bf16 or fp16) or fp32 records
    float* partials;  // [units][splits] records of D+4 floats, or nullptr when splits == 1
    const int32_t* seq_lens;
    int B, Hq, D, group, S, splits, span;
    int64_t kv_sb, kv_sh, sc_sb, sc_sh, q_sb, q_sh, o_sb, o_sh;
    float qscale;
    uint32_t flags;
    PagedView pv;  // pv.table == nullptr: dense cache
    // Causal prefill (Lq > 0): unit = (b, hq, query i); the queries are the last
    // q_lens[b] cached tokens and query i attends to tokens [0, its position].
    int Lq;
    const int32_t* q_lens;
    int64_t q_st, o_st;
};

// Code row offset and scale offset of token t of (b, kv head hk). A paged
// block id outside the pool reads block 0 with both scales forced to 0 (score
// 0, weight 0) and records KVD_STATUS_BAD_BLOCK.
__device__ __forceinline__ void token_offsets(const GenParams& p, int b, int hk, int t, int64_t& row, int64_t& sc,
                                              bool& ok) {
    ok = true;
    if (!p.pv.table) {
        row = b * p.kv_sb + static_cast<int64_t>(hk) * p.kv_sh + static_cast<int64_t>(t) * p.D;
        sc = b * p.sc_sb + static_cast<int64_t>(hk) * p.sc_sh + t;
        return;
    }
    const int j = t / p.pv.block_size, off = t - j * p.pv.block_size;
    int blk = p.pv.table[b * p.pv.bt_stride + j];
    if (blk < 0 || blk >= p.pv.num_blocks) {
        record_status(KVD_STATUS_BAD_BLOCK);
        blk = 0;
        ok = false;
    }
    row = blk * p.pv.kv_sblk + static_cast<int64_t>(hk) * p.kv_sh + static_cast<int64_t>(off) * p.pv.kv_st;
    sc = blk * p.pv.sc_sblk + static_cast<int64_t>(hk) * p.sc_sh + off;
}

__global__ void __launch_bounds__(kGenThreads) generic_decode_kernel(const GenParams p) {
    __shared__ float qs[kGenMaxD];
    __shared__ float sc[kGenChunk];
    __shared__ float wt[kGenChunk];
    __shared__ float pb[kGenChunk];
    __shared__ int64_t rowoff[kGenChunk];
    __shared__ float kscl[kGenChunk], vscl[kGenChunk];
    const int64_t u = blockIdx.x;
    const int split = blockIdx.y;
    const int64_t bh = p.Lq > 0 ? u / p.Lq : u;
    const int qi = p.Lq > 0 ? static_cast<int>(u - bh * p.Lq) : 0;
    const int b = static_cast<int>(bh / p.Hq), hq = static_cast<int>(bh % p.Hq);
    const int hk = hq / p.group;
    int len = p.seq_lens ? min(max(0, p.seq_lens[b]), p.S) : p.S;  // clamp to the capacity
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (p.Lq > 0) {  // prefill: this query's causal prefix
        const int ql = p.q_lens ? min(max(0, p.q_lens[b]), p.Lq) : p.Lq;
        const int64_t ro = b * p.o_sb + static_cast<int64_t>(hq) * p.o_sh + qi * p.o_st;
        if (qi >= ql) {  // no such query: zero row
            for (int d = tid; d < p.D; d += kGenThreads) store_out(p.out, ro + d, 0.f, p.flags);
            return;
        }
        len = max(0, min(len, len - ql + qi + 1));
    }
    const int t_lo = min(len, split * p.span), t_hi = min(len, (split + 1) * p.span);
    const int64_t q0 = b * p.q_sb + static_cast<int64_t>(hq) * p.q_sh + qi * p.q_st;
    for (int d = tid; d < p.D; d += kGenThreads) qs[d] = load_q(p.Q, q0 + d, p.flags) * p.qscale;
    float acc[kGenDPT];
#pragma unroll
    for (int j = 0; j < kGenDPT; ++j) acc[j] = 0.f;
    float m = -INFINITY, l = 0.f;
    for (int c0 = t_lo; c0 < t_hi; c0 += kGenChunk) {
        const int n = min(kGenChunk, t_hi - c0);
        if (tid < n) {
            int64_t row, so;
            bool ok;
            token_offsets(p, b, hk, c0 + tid, row, so, ok);
            rowoff[tid] = row;
            kscl[tid] = ok ? p.ks[so] : 0.f;
            vscl[tid] = ok ? p.vs[so] : 0.f;
        }
        __syncthreads();
        for (int t = warp; t < n; t += kGenThreads / 32) {
            const int8_t* kr = p.K + rowoff[t];
            float dot = 0.f;
            for (int d = lane; d < p.D; d += 32) dot = fmaf(qs[d], static_cast<float>(kr[d]), dot);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if (lane == 0) sc[t] = dot * kscl[t];
        }
        __syncthreads();
        float cm = -INFINITY;
        for (int t = 0; t < n; ++t) cm = fmaxf(cm, sc[t]);
        const float m_new = fmaxf(m, cm);
        const float alpha = exp2f(m - m_new);  // m == -inf -> 0
        if (tid < n) {  // into separate arrays: other threads may still be reading sc[] for the max
            const float pr = exp2f(sc[tid] - m_new);
            pb[tid] = pr;
            wt[tid] = pr * vscl[tid];
        }
        __syncthreads();
        float ps = 0.f;
        for (int t = 0; t < n; ++t) ps += pb[t];
        l = l * alpha + ps;
#pragma unroll
        for (int j = 0; j < kGenDPT; ++j) {
            const int d = tid + j * kGenThreads;
            if (d < p.D) {
                float a = acc[j] * alpha;
                for (int t = 0; t < n; ++t)
                    a = fmaf(wt[t], static_cast<float>(p.V[rowoff[t] + d]), a);
                acc[j] = a;
            }
        }
        m = m_new;
        __syncthreads();
    }
    const bool partial_out = (p.flags & KVD_FLAG_PARTIAL_OUT) != 0;
    float* rec;
    if (p.splits == 1) {
        const int64_t ro = b * p.o_sb + static_cast<int64_t>(hq) * p.o_sh + qi * p.o_st;
        if (!partial_out) {
#pragma unroll
            for (int j = 0; j < kGenDPT; ++j) {
                const int d = tid + j * kGenThreads;
                if (d < p.D) store_out(p.out, ro + d, l > 0.f ? acc[j] / l : 0.f, p.flags);
            }
            return;
        }
        rec = static_cast<float*>(p.out) + ro;
    } else {
        rec = p.partials + (u * p.splits + split) * static_cast<int64_t>(p.D + 4);
    }
    if (tid == 0) { rec[0] = m; rec[1] = l; }
#pragma unroll
    for (int j = 0; j < kGenDPT; ++j) {
        const int d = tid + j * kGenThreads;
        if (d < p.D) rec[4 + d] = acc[j];
    }
}

// Merges `nparts` records per row (record r of part k at base + k*part_stride
// + r*rec_stride) into normalised output rows or combined records.
__global__ void __launch_bounds__(128) combine_records_kernel(
    const float* base, int nparts, int64_t part_stride, int64_t rec_stride, int rows_per_b, int D,
    void* out, int64_t o_sb, int64_t o_sh, uint32_t flags) {
    grid_dependency_wait();  // when launched as a programmatic dependent of the decode that wrote the records
    const int64_t r = blockIdx.x;
    const float* first = base + r * rec_stride;
    float M = -INFINITY;
    for (int k = 0; k < nparts; ++k) M = fmaxf(M, first[k * part_stride]);
    const int b = static_cast<int>(r / rows_per_b), h = static_cast<int>(r % rows_per_b);
    const int64_t ro = b * o_sb + static_cast<int64_t>(h) * o_sh;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float O = 0.f, L = 0.f;
        if (M != -INFINITY) {
            for (int k = 0; k < nparts; ++k) {
                const float* rec = first + k * part_stride;
                const float f = exp2f(rec[0] - M);
                O = fmaf(f, rec[4 + d], O);
                L = fmaf(f, rec[1], L);
            }
        }
        if (flags & KVD_FLAG_PARTIAL_OUT) {
            float* row = static_cast<float*>(out) + ro;
            if (d == 0) { row[0] = M; row[1] = L; }
            row[4 + d] = O;
        } else {
            store_out(out, ro + d, L > 0.f ? O / L : 0.f, flags);
        }
    }
}

int generic_splits(const kvd_decode_desc& d, int sms) {
    const int64_t units = static_cast<int64_t>(d.batch) * d.num_q_heads;
    const int max_by_len = (d.max_seq_len + kGenChunk - 1) / kGenChunk;
    int64_t want = (4LL * sms + units - 1) / units;
    if (want < 1) want = 1;
    if (want > max_by_len) want = max_by_len;
    if (want > 65535) want = 65535;
    return static_cast<int>(want < 1 ? 1 : want);
}
}  // namespace

size_t generic_workspace_size(const kvd_decode_desc& d) {
    const int splits = generic_splits(d, device_sm_count());
    if (splits <= 1) return 0;
    return static_cast<size_t>(d.batch) * d.num_q_heads * splits * (d.head_dim + 4) * sizeof(float);
}

cudaError_t launch_generic(const kvd_decode_desc& d, const void* Q, const int8_t* K,
                           const int8_t* V, const float* ks, const float* vs, void* out,
                           void* ws, size_t ws_bytes, cudaStream_t st, int* launches, const PagedView* pv) {
    if (d.head_dim > kGenMaxD) return cudaErrorInvalidValue;
    const int64_t units = static_cast<int64_t>(d.batch) * d.num_q_heads;
    int splits = generic_splits(d, device_sm_count());
    const size_t rec_bytes = static_cast<size_t>(d.head_dim + 4) * sizeof(float);
    if (splits > 1 && (ws == nullptr || ws_bytes < rec_bytes * units * 2)) splits = 1;
    else if (splits > 1) {
        const int64_t fit = static_cast<int64_t>(ws_bytes / (rec_bytes * units));
        if (fit < splits) splits = static_cast<int>(fit);
    }
    const int max_len = d.max_seq_len > 0 ? d.max_seq_len : 1;
    GenParams p{};
    p.Q = Q; p.K = K; p.V = V; p.ks = ks; p.vs = vs; p.out = out;
    p.partials = splits > 1 ? static_cast<float*>(ws) : nullptr;
    p.seq_lens = d.seq_lens;
    p.B = d.batch; p.Hq = d.num_q_heads; p.D = d.head_dim;
    p.group = d.num_q_heads / d.num_kv_heads;
    p.S = d.max_seq_len;
    p.splits = splits;
    p.span = (max_len + splits - 1) / splits;
    p.kv_sb = d.kv_stride_b; p.kv_sh = d.kv_stride_h;
    p.sc_sb = d.sc_stride_b; p.sc_sh = d.sc_stride_h;
    p.q_sb = d.q_stride_b; p.q_sh = d.q_stride_h;
    p.o_sb = d.o_stride_b; p.o_sh = d.o_stride_h;
    const float scale = d.softmax_scale > 0.f ? d.softmax_scale : 1.0f / sqrtf(static_cast<float>(d.head_dim));
    p.qscale = scale * 1.4426950408889634f;
    p.flags = d.flags;
    p.pv = pv ? *pv : PagedView{};
    generic_decode_kernel<<<dim3(static_cast<unsigned>(units), splits), kGenThreads, 0, st>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ++*launches;
    if (splits > 1) {
        const int64_t rs = d.head_dim + 4;
        combine_records_kernel<<<static_cast<unsigned>(units), 128, 0, st>>>(
            static_cast<const float*>(ws), splits, rs, rs * splits, d.num_q_heads, d.head_dim, out,
            d.o_stride_b, d.o_stride_h, d.flags);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        ++*launches;
    }
    return cudaSuccess;
}

cudaError_t launch_generic_prefill(const kvd_prefill_desc& d, const void* Q, const int8_t* K, const int8_t* V,
                                   const float* ks, const float* vs, void* out, cudaStream_t st, int* launches) {
    if (d.head_dim > kGenMaxD) return cudaErrorInvalidValue;
    GenParams p{};
    p.Q = Q; p.K = K; p.V = V; p.ks = ks; p.vs = vs; p.out = out;
    p.partials = nullptr;
    p.seq_lens = d.seq_lens;
    p.B = d.batch; p.Hq = d.num_q_heads; p.D = d.head_dim;
    p.group = d.num_q_heads / d.num_kv_heads;
    p.S = d.max_seq_len;
    p.splits = 1;
    p.span = d.max_seq_len > 0 ? d.max_seq_len : 1;
    p.kv_sb = d.kv_stride_b; p.kv_sh = d.kv_stride_h;
    p.sc_sb = d.sc_stride_b; p.sc_sh = d.sc_stride_h;
    p.q_sb = d.q_stride_b; p.q_sh = d.q_stride_h;
    p.o_sb = d.o_stride_b; p.o_sh = d.o_stride_h;
    const float scale = d.softmax_scale > 0.f ? d.softmax_scale : 1.0f / sqrtf(static_cast<float>(d.head_dim));
    p.qscale = scale * 1.4426950408889634f;
    p.flags = d.flags;
    p.pv = PagedView{};
    p.Lq = d.max_queries; p.q_lens = d.q_lens; p.q_st = d.q_stride_t; p.o_st = d.o_stride_t;
    const int64_t units = static_cast<int64_t>(d.batch) * d.num_q_heads * d.max_queries;
    if (units > 0x7fffffffLL) return cudaErrorInvalidValue;
    generic_decode_kernel<<<dim3(static_cast<unsigned>(units), 1), kGenThreads, 0, st>>>(p);
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) ++*launches;
    return e;
}

cudaError_t launch_combine_records(const float* base, int nparts, int64_t part_stride, int64_t rec_stride,
                                   int64_t rows, int rows_per_b, int D, void* out, int64_t o_sb, int64_t o_sh,
                                   uint32_t flags, cudaStream_t st, int* launches) {
    // Programmatic dependent of the decode that wrote the records: its CTAs may be
    // scheduled as the decode's retire; each waits for the decode's completion first.
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(rows), 1, 1);
    cfg.blockDim = dim3(128, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, combine_records_kernel, base, nparts, part_stride, rec_stride,
                                             rows_per_b, D, out, o_sb, o_sh, flags);
    if (e == cudaSuccess) ++*launches;
    return e;
}

// Public combine for partials gathered from several GPUs: part k holds
// num_heads records at parts + k*part_stride.
cudaError_t launch_combine_parts(const float* parts, int num_parts, int64_t part_stride, int num_heads,
                                 int head_dim, void* out, int64_t out_stride, uint32_t flags,
                                 cudaStream_t st, int* launches) {
    combine_records_kernel<<<num_heads, 128, 0, st>>>(parts, num_parts, part_stride, head_dim + 4,
                                                      num_heads, head_dim, out, 0, out_stride, flags);
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) ++*launches;
    return e;
}

}  // namespace kvd
