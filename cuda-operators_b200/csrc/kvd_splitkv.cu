// kvd_splitkv.cu -- persistent split-KV flash-decode kernel for MHA on the
// CUDA cores of sm_100a, plus the log-sum-exp combine of split heads.
//
// Replaces the per-head kernels of kv_cache/KV_int8.cu:49-274,
// kv_cache/KV_int8_single_buffer.cu:49-228 and the three-kernel split of
// kv_cache/KV_int8_split_optimized.cu:109-243 / kv_cache/new_kvint8.cu:5-80.
//
// Work decomposition. Every head (b, hq) is cut into tiles of TOK tokens; all
// tiles of all heads form one ordered list of N tiles. CTA c (one per SM)
// streams the contiguous range [c*N/G, (c+1)*N/G) -- equal work per SM for
// dense and ragged batches alike, no per-head waves. A run of tiles of one
// head inside a CTA is a "segment": a segment that covers the whole head
// writes the output row directly; at most two segments per CTA (its first and
// its last) are partial and go to workspace slots 2c / 2c+1, which the combine
// kernel merges.
//
// Inside a CTA: one producer warp issues 1-D bulk copies (TMA engine) of the K
// tile, V tile, the two scale windows and, at segment starts, the query row
// into a ring of NS stages guarded by full/empty mbarriers. CW consumer warps
// share each stage: a lane group of LPT = D/16 lanes owns 4 tokens of the tile
// and 16 dims each. Codes are dequantised exactly in registers, QK and PV use
// packed fp32x2 FMAs, each lane group keeps its own online-softmax state, and
// the states are merged (group -> warp by shuffles, warp -> CTA through shared
// memory) only at segment ends. Several CTAs share an SM so that one CTA's
// segment merge or barrier wait is covered by the others' streaming.
#include <cstdio>

#include "kvd_common.cuh"
#include "kvd_decode.cuh"

namespace kvd {

template <int D>
struct SkCfg {
    static constexpr int DPL = 16;                 // dims per lane
    static constexpr int LPT = D / DPL;            // lanes per token: 8 (D=128) or 4 (D=64)
    static constexpr int GPW = 32 / LPT;           // lane groups per warp
    static constexpr int CW = sk_consumer_warps(D);
    static constexpr int NS = D == 64 ? KVD_SK64_NS : KVD_SK128_NS;
    static constexpr int MINB = sk_ctas_per_sm(D);
    static constexpr int TPG = 4;                  // tokens per group per tile
    static constexpr int TOK = CW * GPW * TPG;     // tokens per tile
    static constexpr int THREADS = (CW + 1) * 32;  // + producer warp
    static constexpr int KV_BYTES = TOK * D;
    static constexpr int SC_FLOATS = TOK + 4;      // 16-byte aligned superset window
    static constexpr int OFF_K = 0;
    static constexpr int OFF_V = OFF_K + KV_BYTES;
    static constexpr int OFF_KS = OFF_V + KV_BYTES;
    static constexpr int OFF_VS = OFF_KS + SC_FLOATS * 4;
    static constexpr int OFF_Q = OFF_VS + SC_FLOATS * 4;
    static constexpr int STAGE_BYTES = OFF_Q + D * 4;
    static constexpr int ROW_STRIDE = CW * GPW * D;  // bytes between a group's consecutive tokens
    static constexpr int MERGE_FLOATS = CW * (D + 2);  // one (m, l, o[D]) state per consumer warp
    static constexpr int OFF_MERGE = NS * STAGE_BYTES;
    static constexpr int OFF_META = OFF_MERGE + ((MERGE_FLOATS * 4 + 15) & ~15);
    static constexpr int OFF_BAR = OFF_META + NS * 16;
    static constexpr int SMEM_BYTES = OFF_BAR + (2 * NS + 2) * 8;
    static_assert(TOK == tile_tokens(D), "tile size mismatch");
    static_assert(STAGE_BYTES % 16 == 0 && OFF_MERGE % 16 == 0 && OFF_BAR % 8 == 0, "alignment");
    static_assert(SMEM_BYTES * MINB <= 232448, "shared memory");
    static_assert(CW * 32 >= D, "the CTA merge gives one consumer thread per output dim");
};

struct TileLoc {
    int b, hq, i, nt, len;
};

// Maps a global tile index to (b, hq, tile i of nt, len).
template <int TOK>
__device__ __forceinline__ TileLoc locate_tile(const DecodeParams& p, int64_t g) {
    TileLoc L;
    if (p.tile_prefix == nullptr) {
        const int64_t u = g / p.tiles_per_head;
        L.i = static_cast<int>(g - u * p.tiles_per_head);
        L.b = static_cast<int>(u / p.Hq);
        L.hq = static_cast<int>(u - static_cast<int64_t>(L.b) * p.Hq);
        L.nt = p.tiles_per_head;
        L.len = p.S;
    } else {
        int lo = 0, hi = p.B;  // find b with prefix[b] <= g < prefix[b+1]
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (static_cast<int64_t>(__ldg(p.tile_prefix + mid)) <= g) lo = mid; else hi = mid;
        }
        L.b = lo;
        L.len = min(max(0, __ldg(p.seq_lens + lo)), p.S);  // lengths beyond the capacity are clamped
        L.nt = L.len > 0 ? (L.len + TOK - 1) / TOK : 1;
        const int64_t r = g - __ldg(p.tile_prefix + lo);
        L.hq = static_cast<int>(r / L.nt);
        L.i = static_cast<int>(r - static_cast<int64_t>(L.hq) * L.nt);
    }
    return L;
}

__device__ __forceinline__ int64_t tile_begin(int64_t n_tiles, int grid, int c) {
    return (static_cast<int64_t>(c) * n_tiles) / grid;
}

// Stage metadata written by the producer before its arrive.
struct __align__(16) StageMeta {
    int32_t u;      // b*Hq + hq
    int32_t n;      // valid tokens in the tile
    int32_t flags;  // bit0 first tile of head, bit1 last tile of head
    int32_t offs;   // k window offset | v window offset << 8 (in floats)
};

// ------------------------------------------------------------------ producer
template <int D>
__device__ __forceinline__ void splitkv_producer(const DecodeParams& p, uint8_t* smem,
                                                 int64_t g_begin, int64_t g_end) {
    using C = SkCfg<D>;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* empty = full + C::NS;
    StageMeta* meta = reinterpret_cast<StageMeta*>(smem + C::OFF_META);
    const uint64_t pol = policy_evict_first();
    int s = 0;
    uint32_t round_par = 0;  // parity of (tile index / NS)
    bool wrapped = false;
    int64_t issued = 0;
    for (int64_t g = g_begin; g < g_end; ++g) {
        if (wrapped && !mbar_wait(&empty[s], round_par ^ 1u)) break;
        const TileLoc L = locate_tile<C::TOK>(p, g);
        const int hk = L.hq / p.group;
        const int t0 = L.i * C::TOK;
        const int n = max(0, min(C::TOK, L.len - t0));
        const bool seg_start = (L.i == 0) || (g == g_begin);
        uint8_t* st = smem + s * C::STAGE_BYTES;
        uint32_t bytes = 0, kwin = 0, vwin = 0;
        int koff = 0, voff = 0;
        const int8_t* kp = nullptr;
        const int8_t* vp = nullptr;
        const char* ksw = nullptr;
        const char* vsw = nullptr;
        if (n > 0) {
            const int64_t kv_off = L.b * p.kv_sb + hk * p.kv_sh + static_cast<int64_t>(t0) * D;
            kp = p.K + kv_off;
            vp = p.V + kv_off;
            const int64_t sc_off = L.b * p.sc_sb + hk * p.sc_sh + t0;
            // Scale windows: the 16-byte aligned superset of [t0, t0+n). Every
            // 16-byte block read holds at least one in-range scale, so the read
            // never leaves the pages the scales live on.
            const uintptr_t ka = reinterpret_cast<uintptr_t>(p.ks + sc_off);
            const uintptr_t va = reinterpret_cast<uintptr_t>(p.vs + sc_off);
            const uintptr_t ka0 = ka & ~uintptr_t(15), va0 = va & ~uintptr_t(15);
            koff = static_cast<int>((ka - ka0) >> 2);
            voff = static_cast<int>((va - va0) >> 2);
            kwin = static_cast<uint32_t>(((ka + 4u * n + 15u) & ~uintptr_t(15)) - ka0);
            vwin = static_cast<uint32_t>(((va + 4u * n + 15u) & ~uintptr_t(15)) - va0);
            ksw = reinterpret_cast<const char*>(ka0);
            vsw = reinterpret_cast<const char*>(va0);
            bytes = 2u * static_cast<uint32_t>(n * D) + kwin + vwin;
        }
        const uint32_t qbytes = seg_start ? 4u * D : 0u;
        StageMeta mt;
        mt.u = L.b * p.Hq + L.hq;
        mt.n = n;
        mt.flags = (L.i == 0 ? 1 : 0) | (L.i == L.nt - 1 ? 2 : 0);
        mt.offs = koff | (voff << 8);
        meta[s] = mt;
        mbar_arrive_expect_tx(&full[s], bytes + qbytes);
        if (n > 0) {
            bulk_g2s(st + C::OFF_K, kp, static_cast<uint32_t>(n * D), &full[s], pol);
            bulk_g2s(st + C::OFF_V, vp, static_cast<uint32_t>(n * D), &full[s], pol);
            bulk_g2s(st + C::OFF_KS, ksw, kwin, &full[s], pol);
            bulk_g2s(st + C::OFF_VS, vsw, vwin, &full[s], pol);
        }
        if (seg_start) {
            const float* qp = p.Q + L.b * p.q_sb + static_cast<int64_t>(L.hq) * p.q_sh;
            bulk_g2s(st + C::OFF_Q, qp, qbytes, &full[s], pol);
        }
        ++issued;
        if (++s == C::NS) {
            s = 0;
            round_par ^= 1u;
            wrapped = true;
        }
    }
    // Never leave copies in flight into this CTA's shared memory: wait (bounded)
    // for the last stages issued.
    for (int64_t j = issued > C::NS ? issued - C::NS : 0; j < issued; ++j)
        mbar_wait(&full[j % C::NS], static_cast<uint32_t>((j / C::NS) & 1));
}

// ----------------------------------------------------------------- consumers
// Lane roles (per consumer warp): lane group grp = lane / LPT owns tokens
// row(t) = (t*CW + warp)*GPW + grp, t = 0..3, of every tile; lane li = lane % LPT
// of the group owns dims [16*li, 16*li + 16). For QK a lane walks its four
// tokens in the order t ^ r, r = the lane's token after the reduction, so the
// transpose-reduce below needs no selects.
template <int D>
__device__ __forceinline__ void splitkv_consumer(const DecodeParams& p, uint8_t* smem,
                                                 int64_t g_begin, int64_t g_end) {
    using C = SkCfg<D>;
    constexpr int LPT = C::LPT, GPW = C::GPW, CW = C::CW;
    constexpr int TB0 = LPT == 8 ? 2 : 1;  // lowest lane bit that selects the token after the reduce
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* empty = full + C::NS;
    uint64_t* mbar = empty + C::NS;
    const StageMeta* meta = reinterpret_cast<const StageMeta*>(smem + C::OFF_META);
    float* mrg_acc = reinterpret_cast<float*>(smem + C::OFF_MERGE);
    float* mrg_ml = mrg_acc + CW * D;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = lane / LPT, li = lane % LPT;
    const int r = (li / TB0) & 3;                              // token this lane scores
    const int base = (warp * GPW + grp) * D + li * 16;        // byte offset of token 0's slice
    const int my_row = (r * CW + warp) * GPW + grp;
    int koff[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) koff[t] = C::OFF_K + base + (t ^ r) * C::ROW_STRIDE;

    float2 q2[8], acc[8];
    float m = -INFINITY, l = 0.f;
    bool seg_has_cta_first = true, seg_from_head_start = false;
    uint32_t merge_par = 0, ph = 0;
    int s = 0;

    for (int64_t g = g_begin; g < g_end; ++g) {
        if (!mbar_wait(&full[s], ph)) return;
        const StageMeta mt = meta[s];
        const uint8_t* st = smem + s * C::STAGE_BYTES;
        if ((mt.flags & 1) || g == g_begin) {
            const float4* qs = reinterpret_cast<const float4*>(st + C::OFF_Q) + li * 4;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float4 v = qs[j];
                q2[2 * j] = make_float2(v.x * p.qscale, v.y * p.qscale);
                q2[2 * j + 1] = make_float2(v.z * p.qscale, v.w * p.qscale);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = make_float2(0.f, 0.f);
            m = -INFINITY;
            l = 0.f;
            seg_has_cta_first = (g == g_begin);
            seg_from_head_start = (mt.flags & 1) != 0;
        }

        // ---- QK partial dots over this lane's 16 dims, tokens in order t ^ r.
        float dk[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint4 w4 = *reinterpret_cast<const uint4*>(st + koff[t]);
            float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f), lo, hi;
            dequant4(w4.x, lo, hi); a = __ffma2_rn(q2[0], lo, a); b = __ffma2_rn(q2[1], hi, b);
            dequant4(w4.y, lo, hi); a = __ffma2_rn(q2[2], lo, a); b = __ffma2_rn(q2[3], hi, b);
            dequant4(w4.z, lo, hi); a = __ffma2_rn(q2[4], lo, a); b = __ffma2_rn(q2[5], hi, b);
            dequant4(w4.w, lo, hi); a = __ffma2_rn(q2[6], lo, a); b = __ffma2_rn(q2[7], hi, b);
            const float2 c = __fadd2_rn(a, b);
            dk[t] = c.x + c.y;
        }
        // Transpose-reduce across the LPT lanes of the group; afterwards the
        // lane holds the full dot of token r.
        constexpr int X1 = LPT / 2, X2 = LPT / 4;
        const float e0 = dk[0] + __shfl_xor_sync(0xffffffffu, dk[2], X1);
        const float e1 = dk[1] + __shfl_xor_sync(0xffffffffu, dk[3], X1);
        float dot = e0 + __shfl_xor_sync(0xffffffffu, e1, X2);
        if constexpr (LPT == 8) dot += __shfl_xor_sync(0xffffffffu, dot, 1);

        const float* ksm = reinterpret_cast<const float*>(st + C::OFF_KS);
        const float* vsm = reinterpret_cast<const float*>(st + C::OFF_VS);
        const bool valid = my_row < mt.n;
        const float sc = valid ? dot * ksm[(mt.offs & 0xff) + my_row] : -INFINITY;

        // ---- online softmax (base 2), lazily rescaled: m may trail the true
        // max by up to 8, so every weight stays below 2^8.
        float tmax = sc;
#pragma unroll
        for (int o = TB0; o < LPT; o <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
        if (tmax > m + 8.f) {
            const float alpha = exp2f(m - tmax);
            l *= alpha;
            const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = __fmul2_rn(acc[j], a2);
            m = tmax;
        }
        const float pr = valid ? exp2f(sc - m) : 0.f;
        l += pr;
        const float wv = valid ? pr * vsm[(mt.offs >> 8) + my_row] : 0.f;

        // ---- PV
        const uint8_t* vrow = st + C::OFF_V + base;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float w = __shfl_sync(0xffffffffu, wv, grp * LPT + t * TB0);
            const float2 w2 = make_float2(w, w);
            const uint4 x4 = *reinterpret_cast<const uint4*>(vrow + t * C::ROW_STRIDE);
            float2 lo, hi;
            dequant4(x4.x, lo, hi); acc[0] = __ffma2_rn(w2, lo, acc[0]); acc[1] = __ffma2_rn(w2, hi, acc[1]);
            dequant4(x4.y, lo, hi); acc[2] = __ffma2_rn(w2, lo, acc[2]); acc[3] = __ffma2_rn(w2, hi, acc[3]);
            dequant4(x4.z, lo, hi); acc[4] = __ffma2_rn(w2, lo, acc[4]); acc[5] = __ffma2_rn(w2, hi, acc[5]);
            dequant4(x4.w, lo, hi); acc[6] = __ffma2_rn(w2, lo, acc[6]); acc[7] = __ffma2_rn(w2, hi, acc[7]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == C::NS) {
            s = 0;
            ph ^= 1u;
        }

        if (!((mt.flags & 2) || g == g_end - 1)) continue;

        // ---- segment end. 1) lane group: sum l over its lanes.
        float lg = l;
#pragma unroll
        for (int o = 1; o < LPT; o <<= 1) lg += __shfl_xor_sync(0xffffffffu, lg, o);
        if (LPT == 8) lg *= 0.5f;  // each token was counted by two lanes
        // 2) warp: rescale the groups to the warp max and add them up.
        float mw = m;
#pragma unroll
        for (int o = LPT; o < 32; o <<= 1) mw = fmaxf(mw, __shfl_xor_sync(0xffffffffu, mw, o));
        const float f = m == -INFINITY ? 0.f : exp2f(m - mw);
        lg *= f;
        const float2 f2 = make_float2(f, f);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = __fmul2_rn(acc[j], f2);
#pragma unroll
        for (int o = LPT; o < 32; o <<= 1) {
            lg += __shfl_xor_sync(0xffffffffu, lg, o);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                acc[j].x += __shfl_xor_sync(0xffffffffu, acc[j].x, o);
                acc[j].y += __shfl_xor_sync(0xffffffffu, acc[j].y, o);
            }
        }
        if (grp == 0) {
            float4* ag = reinterpret_cast<float4*>(mrg_acc + warp * D + li * 16);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                ag[j] = make_float4(acc[2 * j].x, acc[2 * j].y, acc[2 * j + 1].x, acc[2 * j + 1].y);
            if (li == 0) {
                mrg_ml[2 * warp] = mw;
                mrg_ml[2 * warp + 1] = lg;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&mbar[0]);
        if (!mbar_wait(&mbar[0], merge_par)) return;
        // 3) CTA: merge the CW warp states; thread d owns output dim d.
        const int ct = threadIdx.x;
        if (ct < D) {
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < CW; ++w) M = fmaxf(M, mrg_ml[2 * w]);
            float O = 0.f, Lsum = 0.f;
            if (M != -INFINITY) {
#pragma unroll
                for (int w = 0; w < CW; ++w) {
                    const float fw = exp2f(mrg_ml[2 * w] - M);
                    O = fmaf(fw, mrg_acc[w * D + ct], O);
                    Lsum = fmaf(fw, mrg_ml[2 * w + 1], Lsum);
                }
            }
            const int b = mt.u / p.Hq, hq = mt.u - b * p.Hq;
            if (seg_from_head_start && (mt.flags & 2)) {
                float* row = p.out + b * p.o_sb + static_cast<int64_t>(hq) * p.o_sh;
                if (p.flags & KVD_FLAG_PARTIAL_OUT) {
                    if (ct == 0) { row[0] = M; row[1] = Lsum; }
                    row[4 + ct] = O;
                } else {
                    row[ct] = Lsum > 0.f ? O / Lsum : 0.f;
                }
            } else {
                const int slot = 2 * blockIdx.x + (seg_has_cta_first ? 0 : 1);
                float* rec = p.partials + static_cast<int64_t>(slot) * (D + 4);
                if (ct == 0) { rec[0] = M; rec[1] = Lsum; }
                rec[4 + ct] = O;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&mbar[1]);
        if (!mbar_wait(&mbar[1], merge_par)) return;
        merge_par ^= 1u;
    }
}

template <int D>
__global__ void __launch_bounds__(SkCfg<D>::THREADS, SkCfg<D>::MINB) splitkv_kernel(const DecodeParams p) {
    using C = SkCfg<D>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* empty = full + C::NS;
    uint64_t* mbar = empty + C::NS;
    const int64_t N = p.tile_prefix ? static_cast<int64_t>(__ldg(p.tile_prefix + p.B)) : p.n_tiles;
    const int64_t g_begin = tile_begin(N, p.grid, blockIdx.x);
    const int64_t g_end = tile_begin(N, p.grid, blockIdx.x + 1);
    if (g_begin >= g_end) return;
    if (threadIdx.x == 0) {
#pragma unroll
        for (int s = 0; s < C::NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], C::CW);
        }
        mbar_init(&mbar[0], C::CW);
        mbar_init(&mbar[1], C::CW);
        fence_mbar_init();
    }
    __syncthreads();
    if ((threadIdx.x >> 5) == C::CW) {
        if ((threadIdx.x & 31) == 0) splitkv_producer<D>(p, smem, g_begin, g_end);
        return;
    }
    splitkv_consumer<D>(p, smem, g_begin, g_end);
}

// --------------------------------------------------------------- LSE combine
// One block per CTA boundary c (1..grid-1). The head containing tile
// tile_begin(c) is merged by the block of the first boundary strictly inside
// it; its segments are CTA c-1's last segment and the first segment of every
// later non-empty CTA that starts inside the head.
template <int TOK>
__global__ void __launch_bounds__(128) splitkv_combine_kernel(const DecodeParams p) {
    const int c = blockIdx.x + 1;
    const int64_t N = p.tile_prefix ? static_cast<int64_t>(__ldg(p.tile_prefix + p.B)) : p.n_tiles;
    const int64_t tb = tile_begin(N, p.grid, c);
    if (tb >= N) return;
    const TileLoc L = locate_tile<TOK>(p, tb);
    if (L.i == 0) return;
    const int64_t g0 = tb - L.i, g1 = g0 + L.nt;
    const int64_t tbp = tile_begin(N, p.grid, c - 1);
    if (tbp > g0) return;
    const int D = p.D, R = D + 4;
    const float* first = p.partials + static_cast<int64_t>(2 * (c - 1) + (tbp == g0 ? 0 : 1)) * R;

    float M = first[0];
    for (int cc = c; cc < p.grid; ++cc) {
        const int64_t a = tile_begin(N, p.grid, cc);
        if (a >= g1) break;
        if (tile_begin(N, p.grid, cc + 1) > a) M = fmaxf(M, p.partials[static_cast<int64_t>(2 * cc) * R]);
    }
    float* row = p.out + L.b * p.o_sb + static_cast<int64_t>(L.hq) * p.o_sh;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float O = 0.f, Ls = 0.f;
        if (M != -INFINITY) {
            float f = exp2f(first[0] - M);
            O = f * first[4 + d];
            Ls = f * first[1];
            for (int cc = c; cc < p.grid; ++cc) {
                const int64_t a = tile_begin(N, p.grid, cc);
                if (a >= g1) break;
                if (tile_begin(N, p.grid, cc + 1) <= a) continue;
                const float* r = p.partials + static_cast<int64_t>(2 * cc) * R;
                f = exp2f(r[0] - M);
                O = fmaf(f, r[4 + d], O);
                Ls = fmaf(f, r[1], Ls);
            }
        }
        if (p.flags & KVD_FLAG_PARTIAL_OUT) {
            if (d == 0) { row[0] = M; row[1] = Ls; }
            row[4 + d] = O;
        } else {
            row[d] = Ls > 0.f ? O / Ls : 0.f;
        }
    }
}

// -------------------------------------------------------------- ragged plan
// prefix[0] = 0, prefix[b+1] = sum_{b' <= b} Hq * max(1, ceil(len_b'/tok)).
__global__ void __launch_bounds__(1024) plan_kernel(const int32_t* seq_lens, int B, int Hq, int tok,
                                                    int cap, int32_t* prefix) {
    __shared__ int32_t warp_tot[32];
    __shared__ int32_t carry;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) { carry = 0; prefix[0] = 0; }
    __syncthreads();
    for (int base = 0; base < B; base += blockDim.x) {
        const int b = base + tid;
        int v = 0;
        if (b < B) {
            const int len = min(max(0, seq_lens[b]), cap);
            v = Hq * (len > 0 ? (len + tok - 1) / tok : 1);
        }
        int incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        if (lane == 31) warp_tot[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            int w = lane < (int)(blockDim.x >> 5) ? warp_tot[lane] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += y;
            }
            warp_tot[lane] = w;
        }
        __syncthreads();
        const int before = (warp > 0 ? warp_tot[warp - 1] : 0) + carry;
        if (b < B) prefix[b + 1] = before + incl;
        __syncthreads();
        if (tid == blockDim.x - 1) carry = before + incl;
        __syncthreads();
    }
}

// ------------------------------------------------------------------ launch
namespace {
template <int D>
cudaError_t launch_sk(const DecodeParams& p, cudaStream_t st, int* launches) {
    using C = SkCfg<D>;
    static PerDeviceOnce once;
    cudaError_t e = once.run([] {
        return cudaFuncSetAttribute(splitkv_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    });
    if (e != cudaSuccess) return e;
    splitkv_kernel<D><<<p.grid, C::THREADS, C::SMEM_BYTES, st>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ++*launches;
    // Dense batches whose CTA ranges all start at a head boundary split no head.
    const bool whole_heads = p.tile_prefix == nullptr && p.n_tiles % p.grid == 0 &&
                             (p.n_tiles / p.grid) % p.tiles_per_head == 0;
    if (p.grid > 1 && !whole_heads) {
        splitkv_combine_kernel<C::TOK><<<p.grid - 1, 128, 0, st>>>(p);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        ++*launches;
    }
    return cudaSuccess;
}
}  // namespace

cudaError_t launch_splitkv(const DecodeParams& p, cudaStream_t st, int* launches) {
    if (p.D == 128) return launch_sk<128>(p, st, launches);
    if (p.D == 64) return launch_sk<64>(p, st, launches);
    return cudaErrorInvalidValue;
}

cudaError_t launch_plan(const int32_t* seq_lens, int B, int Hq, int tok, int cap, int32_t* prefix,
                        cudaStream_t st, int* launches) {
    plan_kernel<<<1, 1024, 0, st>>>(seq_lens, B, Hq, tok, cap, prefix);
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) ++*launches;
    return e;
}

}  // namespace kvd
