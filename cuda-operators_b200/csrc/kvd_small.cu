// kvd_small.cu -- one-launch decode of small dense MHA problems (the north
// star's configuration 1: B=1, 8 heads, D=64, 1,024 tokens, 1.1 MB a step).
//
// Such a step moves too few bytes to fill the GPU, so its time is launch
// latency plus one HBM round trip plus whatever runs serially after it. The
// persistent split-KV kernel needs either whole-head CTAs (8 CTAs each
// streaming 8 tiles back to back) or a second launch for the combine. Here a
// thread-block cluster of up to 8 CTAs covers one query head: CTA r of the
// cluster loads its token range (at most 256 tokens) with ONE batch of bulk
// copies, computes its (m, l, o) record in shared memory, and cluster rank 0
// merges the records of all ranks through distributed shared memory and writes
// the output row. No workspace, no global counters, one launch.
//
// Mathematics as the reference's `cpu_reference`
// (kv_cache/KV_int8_split_optimized.cu:385-437): score = (q . code) * k_scale
// / sqrt(D), softmax over the head, value = code * v_scale; here in base 2
// (scores carry log2(e)) with an exact INT8 -> fp32 conversion.
#include <cooperative_groups.h>

#include "kvd_common.cuh"
#include "kvd_decode.cuh"

namespace cg = cooperative_groups;

namespace kvd {

template <int D>
struct SmCfg {
    static constexpr int SPAN = kSmallMaxSpan;          // tokens per CTA at most
    static constexpr int THREADS = 128;
    static constexpr int LPT = D / 16;                   // lanes per token in QK (16 dims each)
    static constexpr int TPI = (THREADS / 32) * (32 / LPT);  // tokens per QK iteration
    static constexpr int C4 = D / 4;                     // PV: column groups of 4 dims
    static constexpr int SUB = THREADS / C4;             // PV: token subsets
    static constexpr int OFF_K = 0;
    static constexpr int OFF_V = SPAN * D;
    static constexpr int OFF_KS = 2 * SPAN * D;          // 16-byte aligned superset window of the scales
    static constexpr int OFF_VS = OFF_KS + (SPAN + 4) * 4;
    static constexpr int OFF_Q = OFF_VS + (SPAN + 4) * 4;
    static constexpr int OFF_W = OFF_Q + D * 4;          // scores, then weights p * v_scale
    static constexpr int OFF_RED = OFF_W + SPAN * 4;     // 8 floats of warp partials
    static constexpr int OFF_PV = OFF_RED + 32;          // [SUB][D] partial PV sums
    static constexpr int OFF_REC = OFF_PV + SUB * D * 4; // record: m, l, -, -, o[D]
    static constexpr int OFF_BAR = OFF_REC + (D + 4) * 4;
    static constexpr int SMEM_BYTES = OFF_BAR + 8;
    static_assert(OFF_KS % 16 == 0 && OFF_Q % 16 == 0 && OFF_PV % 16 == 0 && OFF_REC % 16 == 0, "alignment");
    static_assert(SUB * C4 == THREADS && D <= THREADS, "thread mapping");
};

struct SmallParams {
    const float* Q;
    const int8_t* K;
    const int8_t* V;
    const float* ks;
    const float* vs;
    float* out;
    int Hq, S, span;
    int64_t kv_sb, kv_sh, sc_sb, sc_sh, q_sb, q_sh, o_sb, o_sh;
    float qscale;     // softmax_scale * log2(e)
    uint32_t flags;   // KVD_FLAG_PARTIAL_OUT or 0
};

// 1-D global -> shared bulk copy without an L2 hint (a small cache stays in L2
// between steps).
__device__ __forceinline__ void bulk_g2s_plain(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

template <int D>
__global__ void __launch_bounds__(SmCfg<D>::THREADS) small_decode_kernel(const SmallParams p) {
    using C = SmCfg<D>;
    extern __shared__ __align__(128) uint8_t smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int nrank = static_cast<int>(cluster.num_blocks());
    const int head = blockIdx.y;                       // b * Hq + hq
    const int b = head / p.Hq, hq = head - b * p.Hq;   // MHA: kv head = hq
    const int t0 = rank * p.span;
    const int n = max(0, min(p.span, p.S - t0));
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    float* W = reinterpret_cast<float*>(smem + C::OFF_W);
    float* red = reinterpret_cast<float*>(smem + C::OFF_RED);
    float* rec = reinterpret_cast<float*>(smem + C::OFF_REC);

    // Launched as a programmatic dependent of the kernel before it, and lets the
    // next one launch at once: the CTAs set up while the previous grid ends and
    // wait for it (griddepcontrol.wait) before touching global memory.
    allow_dependents();
    // ---- one batch of bulk copies: K rows, V rows, both scale windows, the query row
    int koff = 0, voff = 0;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    grid_dependency_wait();
    bool ok = true;
    if (n > 0) {
        const int64_t kv_off = b * p.kv_sb + hq * p.kv_sh + static_cast<int64_t>(t0) * D;
        const int64_t sc_off = b * p.sc_sb + hq * p.sc_sh + t0;
        const uintptr_t ka = reinterpret_cast<uintptr_t>(p.ks + sc_off);
        const uintptr_t va = reinterpret_cast<uintptr_t>(p.vs + sc_off);
        const uintptr_t ka0 = ka & ~uintptr_t(15), va0 = va & ~uintptr_t(15);
        koff = static_cast<int>((ka - ka0) >> 2);
        voff = static_cast<int>((va - va0) >> 2);
        if (tid == 0) {
            const uint32_t kwin = static_cast<uint32_t>(((ka + 4u * n + 15u) & ~uintptr_t(15)) - ka0);
            const uint32_t vwin = static_cast<uint32_t>(((va + 4u * n + 15u) & ~uintptr_t(15)) - va0);
            const uint32_t rows = static_cast<uint32_t>(n * D);
            mbar_arrive_expect_tx(bar, 2u * rows + kwin + vwin + 4u * D);
            bulk_g2s_plain(smem + C::OFF_K, p.K + kv_off, rows, bar);
            bulk_g2s_plain(smem + C::OFF_V, p.V + kv_off, rows, bar);
            bulk_g2s_plain(smem + C::OFF_KS, reinterpret_cast<const void*>(ka0), kwin, bar);
            bulk_g2s_plain(smem + C::OFF_VS, reinterpret_cast<const void*>(va0), vwin, bar);
            bulk_g2s_plain(smem + C::OFF_Q, p.Q + b * p.q_sb + static_cast<int64_t>(hq) * p.q_sh, 4u * D, bar);
        }
        // bounded: on expiry the status word is set and the whole CTA skips its work
        ok = __syncthreads_and(mbar_wait(bar, 0) ? 1 : 0) != 0;
    }
    float m = -INFINITY, l = 0.f;
    if (n > 0 && ok) {
        const float* ksm = reinterpret_cast<const float*>(smem + C::OFF_KS) + koff;
        const float* vsm = reinterpret_cast<const float*>(smem + C::OFF_VS) + voff;
        // ---- QK: a group of LPT lanes per token, 16 dims per lane
        const int grp = lane / C::LPT, li = lane % C::LPT;
        float2 q2[8];
        {
            const float4* qs = reinterpret_cast<const float4*>(smem + C::OFF_Q) + li * 4;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float4 v = qs[j];
                q2[2 * j] = make_float2(v.x * p.qscale, v.y * p.qscale);
                q2[2 * j + 1] = make_float2(v.z * p.qscale, v.w * p.qscale);
            }
        }
        for (int base = 0; base < n; base += C::TPI) {
            const int t = base + warp * (32 / C::LPT) + grp;
            float dot = 0.f;
            if (t < n) {
                const uint4 w4 = *reinterpret_cast<const uint4*>(smem + C::OFF_K + t * D + li * 16);
                float2 a = make_float2(0.f, 0.f), c = make_float2(0.f, 0.f), lo, hi;
                dequant4(w4.x, lo, hi); a = __ffma2_rn(q2[0], lo, a); c = __ffma2_rn(q2[1], hi, c);
                dequant4(w4.y, lo, hi); a = __ffma2_rn(q2[2], lo, a); c = __ffma2_rn(q2[3], hi, c);
                dequant4(w4.z, lo, hi); a = __ffma2_rn(q2[4], lo, a); c = __ffma2_rn(q2[5], hi, c);
                dequant4(w4.w, lo, hi); a = __ffma2_rn(q2[6], lo, a); c = __ffma2_rn(q2[7], hi, c);
                const float2 s2 = __fadd2_rn(a, c);
                dot = s2.x + s2.y;
            }
#pragma unroll
            for (int o = 1; o < C::LPT; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if (t < n && li == 0) W[t] = dot * ksm[t];
        }
        __syncthreads();
        // ---- max over the range
        float mx = -INFINITY;
        for (int t = tid; t < n; t += C::THREADS) mx = fmaxf(mx, W[t]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red[warp] = mx;
        __syncthreads();
        m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
        // ---- weights p * v_scale and their sum
        float ls = 0.f;
        for (int t = tid; t < n; t += C::THREADS) {
            const float pr = exp2f(W[t] - m);
            ls += pr;
            W[t] = pr * vsm[t];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
        if (lane == 0) red[4 + warp] = ls;
        __syncthreads();
        l = (red[4] + red[5]) + (red[6] + red[7]);
        // ---- PV: thread = (4-dim column group, token subset)
        const int cgp = tid % C::C4, sub = tid / C::C4;
        float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
        for (int t = sub; t < n; t += C::SUB) {
            const float w = W[t];
            const float2 w2 = make_float2(w, w);
            float2 lo, hi;
            dequant4(*reinterpret_cast<const uint32_t*>(smem + C::OFF_V + t * D + 4 * cgp), lo, hi);
            acc0 = __ffma2_rn(w2, lo, acc0);
            acc1 = __ffma2_rn(w2, hi, acc1);
        }
        reinterpret_cast<float4*>(smem + C::OFF_PV)[sub * C::C4 + cgp] = make_float4(acc0.x, acc0.y, acc1.x, acc1.y);
        __syncthreads();
        if (tid < D) {
            const float* pv = reinterpret_cast<const float*>(smem + C::OFF_PV);
            float o = 0.f;
#pragma unroll
            for (int s = 0; s < C::SUB; ++s) o += pv[s * D + tid];
            rec[4 + tid] = o;
        }
    } else if (tid < D) {
        rec[4 + tid] = 0.f;  // empty range or a timed-out copy: an empty record
    }
    if (tid == 0) { rec[0] = m; rec[1] = l; }

    float* row = p.out + b * p.o_sb + static_cast<int64_t>(hq) * p.o_sh;
    if (nrank == 1) {
        __syncthreads();
        if (tid < D) {
            if (p.flags & KVD_FLAG_PARTIAL_OUT) {
                if (tid == 0) { row[0] = rec[0]; row[1] = rec[1]; }
                row[4 + tid] = rec[4 + tid];
            } else {
                row[tid] = rec[1] > 0.f ? rec[4 + tid] / rec[1] : 0.f;
            }
        }
        return;
    }
    // ---- merge the cluster's records in rank 0 through distributed shared memory
    cluster.sync();  // every rank's record is written
    if (rank == 0 && tid < D) {
        float M = -INFINITY;
        for (int r = 0; r < nrank; ++r) M = fmaxf(M, cluster.map_shared_rank(rec, r)[0]);
        float O = 0.f, L = 0.f;
        if (M != -INFINITY) {
            for (int r = 0; r < nrank; ++r) {
                const float* rr = cluster.map_shared_rank(rec, r);
                const float f = exp2f(rr[0] - M);
                O = fmaf(f, rr[4 + tid], O);
                L = fmaf(f, rr[1], L);
            }
        }
        if (p.flags & KVD_FLAG_PARTIAL_OUT) {
            if (tid == 0) { row[0] = M; row[1] = L; }
            row[4 + tid] = O;
        } else {
            row[tid] = L > 0.f ? O / L : 0.f;
        }
    }
    cluster.sync();  // no rank exits while rank 0 may still read its record
}

namespace {
template <int D>
cudaError_t launch_small_d(const SmallParams& p, int cs, int heads, cudaStream_t st) {
    using C = SmCfg<D>;
    static PerDeviceOnce once;
    cudaError_t e = once.run([] {
        return cudaFuncSetAttribute(small_decode_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    C::SMEM_BYTES);
    });
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(cs), static_cast<unsigned>(heads), 1);
    cfg.blockDim = dim3(C::THREADS, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(cs);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, small_decode_kernel<D>, p);
}
}  // namespace

// Cluster size (CTAs per head) of a small dense decode, or 0 when the shape is
// not small: MHA, fp32, head_dim 64 or 128, 1..8*256 tokens, and few enough
// heads that every CTA runs in the first wave (one per SM).
int small_cluster_size(const kvd_decode_desc& d) {
    if (d.seq_lens || (d.flags & kDtypeFlags) || d.num_q_heads != d.num_kv_heads) return 0;
    if (d.head_dim != 64 && d.head_dim != 128) return 0;
    const int S = d.max_seq_len;
    if (S < 1 || S > kSmallMaxCluster * kSmallMaxSpan) return 0;
    const int cs = min(kSmallMaxCluster, (S + 127) / 128);
    const int64_t heads = static_cast<int64_t>(d.batch) * d.num_q_heads;
    if (heads * cs > device_sm_count() || heads > 65535) return 0;
    return cs;
}

cudaError_t launch_small(const kvd_decode_desc& d, const float* Q, const int8_t* K, const int8_t* V,
                         const float* ks, const float* vs, float* out, cudaStream_t st, int* launches) {
    const int cs = small_cluster_size(d);
    if (cs < 1) return cudaErrorInvalidValue;
    SmallParams p{};
    p.Q = Q; p.K = K; p.V = V; p.ks = ks; p.vs = vs; p.out = out;
    p.Hq = d.num_q_heads;
    p.S = d.max_seq_len;
    p.span = (d.max_seq_len + cs - 1) / cs;
    p.kv_sb = d.kv_stride_b; p.kv_sh = d.kv_stride_h;
    p.sc_sb = d.sc_stride_b; p.sc_sh = d.sc_stride_h;
    p.q_sb = d.q_stride_b; p.q_sh = d.q_stride_h;
    p.o_sb = d.o_stride_b; p.o_sh = d.o_stride_h;
    const float scale = d.softmax_scale > 0.f ? d.softmax_scale : 1.0f / sqrtf(static_cast<float>(d.head_dim));
    p.qscale = scale * 1.4426950408889634f;
    p.flags = d.flags & KVD_FLAG_PARTIAL_OUT;
    const int heads = d.batch * d.num_q_heads;
    const cudaError_t e = d.head_dim == 64 ? launch_small_d<64>(p, cs, heads, st) : launch_small_d<128>(p, cs, heads, st);
    if (e == cudaSuccess) ++*launches;
    return e;
}

}  // namespace kvd
