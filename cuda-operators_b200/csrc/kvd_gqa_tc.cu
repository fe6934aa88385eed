// kvd_gqa_tc.cu -- grouped-query INT8 decode on the 5th-generation tensor cores
// (tcgen05, sm_100a). One CTA processes whole (batch, kv head) work items: the
// G query heads of a group share every K/V tile, which is read from HBM once.
//
// No reference counterpart (the reference has no GQA mapping,
// kv_cache/new_kvint8.cu:83-84); the mathematics is the reference's score
// (q . k_code) * k_scale / sqrt(D) and value code * v_scale, per query head.
//
// Exactness. Both products run as integer MMAs (kind::i8, int32 accumulate),
// which are exact:
//  * QK: the fp32 query row of each head, scaled by softmax_scale*log2(e), is
//    turned into a 31-bit fixed point number Qi = round(q * 2^E) with one
//    exponent per (item, head), split into four signed bytes
//    Qi = sum_j L_j 2^(8j). B operand = [4G limb rows x 128 dims], A operand =
//    the K code tile as loaded (128 tokens x 128 dims, 128-byte swizzle).
//    score = (sum_j acc_j 2^(8j)) * 2^-E * k_scale.
//  * PV: weights w = 2^(s - m) * v_scale (m = running max, lazily updated so
//    w stays below 2^8 * max v_scale) are scaled per (tile, head) to a 32-bit
//    unsigned fixed point W = round(w * 2^F) whose four bytes are the limbs;
//    A operand = the V code tile read MN-major (dims contiguous), B operand =
//    [128 tokens x 4G limbs]. o += (sum_j acc_j 2^(8j)) * 2^-F.
// The only roundings are fp32 ones after the exact integer sums, and the
// fixed-point steps, whose absolute error is 2^-31 of the head's largest
// query element and 2^-32 of the tile's largest weight.
//
// Roles (192 threads): warps 0-3 epilogue (TMEM lane quarter = warp), warp 4
// TMA producer, warp 5 MMA issuer (also owns the TMEM allocation). Every wait
// is bounded; on expiry the kernel records KVD_STATUS_WAIT_TIMEOUT and unwinds.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>

#include "kvd_common.cuh"
#include "kvd_decode.cuh"

namespace kvd {

struct GqaParams {
    const float* Q;
    const float* ks;
    const float* vs;
    float* out;
    float* partials;           // [B*Hq][P] records of D+4 floats when P > 1
    const int32_t* seq_lens;   // device [B] or nullptr
    int B, Hq, Hkv, S, P, span, n_items, grid;
    int64_t sc_sb, sc_sh, q_sb, q_sh, o_sb, o_sh;
    float qscale;
    uint32_t flags;
};

template <int G, int NS_>
struct GqaCfg {
    static constexpr int D = 128;
    static constexpr int TOK = 128;
    static constexpr int NS = NS_;
    static constexpr int NP = (4 * G < 16) ? 16 : 4 * G;        // MMA N: limbs x heads, padded
    static constexpr int TMEM_COLS = (4 * NP <= 32) ? 32 : (4 * NP <= 64 ? 64 : (4 * NP <= 128 ? 128 : 256));
    static constexpr int THREADS = 192;
    static constexpr int SC_FLOATS = TOK + 4;
    // stage: K tile | V tile | ks window | vs window, K/V 1024-byte aligned
    static constexpr int OFF_K = 0;
    static constexpr int OFF_V = 16384;
    static constexpr int OFF_KS = 32768;
    static constexpr int OFF_VS = OFF_KS + SC_FLOATS * 4;
    static constexpr int STAGE_BYTES = ((OFF_VS + SC_FLOATS * 4) + 1023) & ~1023;
    static constexpr int QB_BYTES = NP * 128;                    // K-major, 128-byte swizzle
    static constexpr int WB_BYTES = TOK * NP;                    // MN-major, no swizzle
    static constexpr int OFF_QB = NS * STAGE_BYTES;              // 2 buffers
    static constexpr int OFF_WB = OFF_QB + 2 * QB_BYTES;         // 2 buffers
    static constexpr int OFF_RED = OFF_WB + 2 * WB_BYTES;        // [2][4][32] floats
    static constexpr int OFF_META = OFF_RED + 2 * 4 * 32 * 4;    // [NS] x 16 bytes
    static constexpr int OFF_BAR = OFF_META + NS * 16;
    // barriers: full[NS], empty[NS], then at 2*NS: s_full[2], s_free[2], w_full[2], o_full[2],
    // o_free[2], q_full[2], red, done, drain
    static constexpr int NBAR = 2 * NS + 15;
    static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
    static constexpr int SMEM_USED = OFF_TMEM + 16;
    static constexpr int SMEM_BYTES = SMEM_USED + 1024;          // slack to align the base to 1024
    static_assert(G >= 1 && G <= 16, "group size");
    static_assert(STAGE_BYTES % 1024 == 0 && OFF_QB % 1024 == 0 && QB_BYTES % 1024 == 0, "swizzle atoms");
    static_assert(SMEM_BYTES <= 232448, "shared memory");
};

// ---------------------------------------------------------- PTX wrappers
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cta.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;"
        ::"r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] x B[smem desc], int8 x int8 -> int32.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate ? 1u : 0u)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

// 32 consecutive TMEM columns of this warp's lane quarter -> 32 registers.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05): start, leading/stride byte
// offsets (16-byte units), version 1, base offset 0, layout type.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1u) << 46;  // version
    d |= static_cast<uint64_t>(layout & 7u) << 61;
    return d;
}
constexpr uint32_t kLayoutNone = 0, kLayoutSw128 = 2;

// Instruction descriptor, kind::i8: int32 accumulator, A/B signedness and
// majorness, N and M.
__host__ __device__ constexpr uint32_t idesc_i8(bool a_signed, bool b_signed, bool a_mn, bool b_mn, int N, int M) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) | ((a_mn ? 1u : 0u) << 15) |
           ((b_mn ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// Exact int32 -> fp32 for |v| < 2^22: 0x4B400000 + v is the float 1.5*2^23 + v.
__device__ __forceinline__ float small_int_to_float(uint32_t v) {
    return __uint_as_float(0x4B400000u + v) - 12582912.0f;
}

// Four exact limb sums -> fp32 value of sum_j acc_j 2^(8j).
__device__ __forceinline__ float combine_limbs(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3) {
    float f = small_int_to_float(a3) * 16777216.0f;
    f = fmaf(small_int_to_float(a2), 65536.0f, f);
    f = fmaf(small_int_to_float(a1), 256.0f, f);
    return f + small_int_to_float(a0);
}

__device__ __forceinline__ float pow2i(int e) {  // 2^e for e in [-126, 127]
    return __int_as_float((e + 127) << 23);
}

}  // namespace kvd

namespace kvd {

struct GItem {
    int b, hk, split, t_lo, t_hi, ntiles;
};

__device__ __forceinline__ GItem gqa_item(const GqaParams& p, int it) {
    GItem I;
    const int u = it / p.P;
    I.split = it - u * p.P;
    I.b = u / p.Hkv;
    I.hk = u - I.b * p.Hkv;
    const int len = p.seq_lens ? min(max(0, __ldg(p.seq_lens + I.b)), p.S) : p.S;
    I.t_lo = I.split * p.span;
    I.t_hi = min(len, I.t_lo + p.span);
    const int n = I.t_hi - I.t_lo;
    I.ntiles = n > 0 ? (n + 127) / 128 : 1;
    return I;
}

struct __align__(16) GMeta {
    int32_t it, n, flags, offs;  // flags: bit0 first tile of item, bit1 last tile of item
};

// ------------------------------------------------------------------ producer
template <int G, int NS>
__device__ __forceinline__ void gqa_producer(const CUtensorMap* kmap, const CUtensorMap* vmap, const GqaParams& p,
                                             uint8_t* smem) {
    using C = GqaCfg<G, NS>;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* empty = full + NS;
    GMeta* meta = reinterpret_cast<GMeta*>(smem + C::OFF_META);
    const uint64_t pol = policy_evict_first();
    int s = 0;
    uint32_t round_par = 0;
    bool wrapped = false, ok = true;
    int64_t issued = 0;
    for (int it = blockIdx.x; it < p.n_items && ok; it += p.grid) {
        const GItem I = gqa_item(p, it);
        for (int tt = 0; tt < I.ntiles; ++tt) {
            if (wrapped && !mbar_wait(&empty[s], round_par ^ 1u)) { ok = false; break; }
            const int t0 = I.t_lo + tt * C::TOK;
            const int n = max(0, min(C::TOK, I.t_hi - t0));
            uint8_t* st = smem + s * C::STAGE_BYTES;
            uint32_t bytes = 0, kwin = 0, vwin = 0;
            int koff = 0, voff = 0;
            uintptr_t ka0 = 0, va0 = 0;
            if (n > 0) {
                const int64_t sc_off = I.b * p.sc_sb + I.hk * p.sc_sh + t0;
                const uintptr_t ka = reinterpret_cast<uintptr_t>(p.ks + sc_off);
                const uintptr_t va = reinterpret_cast<uintptr_t>(p.vs + sc_off);
                ka0 = ka & ~uintptr_t(15);
                va0 = va & ~uintptr_t(15);
                koff = static_cast<int>((ka - ka0) >> 2);
                voff = static_cast<int>((va - va0) >> 2);
                kwin = static_cast<uint32_t>(((ka + 4u * n + 15u) & ~uintptr_t(15)) - ka0);
                vwin = static_cast<uint32_t>(((va + 4u * n + 15u) & ~uintptr_t(15)) - va0);
                bytes = 2u * 16384u + kwin + vwin;  // tensor boxes always deliver the whole box
            }
            GMeta mt;
            mt.it = it;
            mt.n = n;
            mt.flags = (tt == 0 ? 1 : 0) | (tt == I.ntiles - 1 ? 2 : 0);
            mt.offs = koff | (voff << 8);
            meta[s] = mt;
            mbar_arrive_expect_tx(&full[s], bytes);
            if (n > 0) {
                tma_load_4d(st + C::OFF_K, kmap, 0, t0, I.hk, I.b, &full[s], pol);
                tma_load_4d(st + C::OFF_V, vmap, 0, t0, I.hk, I.b, &full[s], pol);
                bulk_g2s(st + C::OFF_KS, reinterpret_cast<const void*>(ka0), kwin, &full[s], pol);
                bulk_g2s(st + C::OFF_VS, reinterpret_cast<const void*>(va0), vwin, &full[s], pol);
            }
            ++issued;
            if (++s == NS) { s = 0; round_par ^= 1u; wrapped = true; }
        }
    }
    for (int64_t j = issued > NS ? issued - NS : 0; j < issued; ++j)
        mbar_wait(&full[j % NS], static_cast<uint32_t>((j / NS) & 1));
}

// ------------------------------------------------------------------ MMA issuer
template <int G, int NS>
__device__ __forceinline__ bool gqa_mma_pv(uint8_t* smem, uint32_t tmem, int64_t j, int sj) {
    using C = GqaCfg<G, NS>;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* empty = bars + NS;
    uint64_t* w_full = bars + 2 * NS + 4;
    uint64_t* o_full = bars + 2 * NS + 6;
    uint64_t* o_free = bars + 2 * NS + 8;
    const int bj = static_cast<int>(j & 1);
    if (!mbar_wait(&w_full[bj], static_cast<uint32_t>((j >> 1) & 1))) return false;
    if (j >= 2 && !mbar_wait(&o_free[bj], static_cast<uint32_t>(((j >> 1) - 1) & 1))) return false;
    tc_fence_after();
    constexpr uint32_t idesc = idesc_i8(true, false, true, true, C::NP, 128);
    const uint32_t vbase = smem_u32(smem + sj * C::STAGE_BYTES + C::OFF_V);
    const uint32_t wbase = smem_u32(smem + C::OFF_WB + bj * C::WB_BYTES);
    const uint32_t dcol = tmem + 2 * C::NP + bj * C::NP;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
        const uint64_t ad = smem_desc(vbase + 4096u * kk, 16u, 1024u, kLayoutSw128);
        const uint64_t bd = smem_desc(wbase + 512u * kk, 128u, 2048u, kLayoutNone);
        mma_i8(dcol, ad, bd, idesc, kk > 0);
    }
    mma_commit(&o_full[bj]);
    mma_commit(&empty[sj]);
    return true;
}

template <int G, int NS>
__device__ __forceinline__ void gqa_mma(const GqaParams& p, uint8_t* smem, uint32_t tmem) {
    using C = GqaCfg<G, NS>;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* full = bars;
    uint64_t* s_full = bars + 2 * NS;
    uint64_t* s_free = bars + 2 * NS + 2;
    uint64_t* q_full = bars + 2 * NS + 10;
    constexpr uint32_t idesc_qk = idesc_i8(true, true, false, false, C::NP, 128);
    int64_t i = 0;
    int s = 0;
    uint32_t ph = 0;
    int64_t prev_i = -1;
    int prev_s = 0;
    int kq = 0;
    for (int it = blockIdx.x; it < p.n_items; it += p.grid, ++kq) {
        const GItem I = gqa_item(p, it);
        for (int tt = 0; tt < I.ntiles; ++tt, ++i) {
            if (!mbar_wait(&full[s], ph)) return;
            if (tt == 0 && !mbar_wait(&q_full[kq & 1], static_cast<uint32_t>((kq >> 1) & 1))) return;
            const int bi = static_cast<int>(i & 1);
            if (i >= 2 && !mbar_wait(&s_free[bi], static_cast<uint32_t>(((i >> 1) - 1) & 1))) return;
            tc_fence_after();
            const uint32_t kbase = smem_u32(smem + s * C::STAGE_BYTES + C::OFF_K);
            const uint32_t qbase = smem_u32(smem + C::OFF_QB + (kq & 1) * C::QB_BYTES);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint64_t ad = smem_desc(kbase + 32u * kk, 16u, 1024u, kLayoutSw128);
                const uint64_t bd = smem_desc(qbase + 32u * kk, 16u, 1024u, kLayoutSw128);
                mma_i8(tmem + bi * C::NP, ad, bd, idesc_qk, kk > 0);
            }
            mma_commit(&s_full[bi]);
            if (prev_i >= 0 && !gqa_mma_pv<G, NS>(smem, tmem, prev_i, prev_s)) return;
            prev_i = i;
            prev_s = s;
            if (++s == NS) { s = 0; ph ^= 1u; }
        }
    }
    if (prev_i >= 0) gqa_mma_pv<G, NS>(smem, tmem, prev_i, prev_s);
}

}  // namespace kvd

namespace kvd {

// NP consecutive TMEM columns of this warp's lane quarter.
template <int NP>
__device__ __forceinline__ void tmem_ld_np(uint32_t taddr, uint32_t (&r)[NP]) {
    if constexpr (NP == 16) {
        tmem_ld16(taddr, r);
    } else if constexpr (NP == 32) {
        tmem_ld32(taddr, r);
    } else {
        static_assert(NP == 64, "NP");
        uint32_t (&lo)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[0]);
        uint32_t (&hi)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[32]);
        tmem_ld32(taddr, lo);
        tmem_ld32(taddr + 32, hi);
    }
}

// CTA-wide (4 epilogue warps) max or sum of K values per thread, bounded.
template <int K, bool MAX>
__device__ __forceinline__ bool epi_reduce(float (&v)[K], float* red, uint64_t* bar, uint32_t& use) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        float x = v[k];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float y = __shfl_xor_sync(0xffffffffu, x, o);
            x = MAX ? fmaxf(x, y) : x + y;
        }
        v[k] = x;
    }
    float* rb = red + (use & 1u) * 128;
    if (lane == 0) {
#pragma unroll
        for (int k = 0; k < K; ++k) rb[warp * 32 + k] = v[k];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
    const bool ok = mbar_wait(bar, use & 1u);
    ++use;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const float a = rb[k], b = rb[32 + k], c = rb[64 + k], d = rb[96 + k];
        v[k] = MAX ? fmaxf(fmaxf(a, b), fmaxf(c, d)) : (a + b) + (c + d);
    }
    return ok;
}

// Query limbs of item `it` into buffer `buf`: thread r owns dim r of all G
// heads. Qi = round(q * qscale * 2^E_h), |Qi| < 2^31, split into four signed
// bytes written into the K-major 128-byte-swizzled B operand (row 4h + j).
// Every thread ends with the same reduced maxima, so each one also keeps the
// per-head scales 2^-E_h (sEn) in registers for the item's scores.
template <int G, int NS>
__device__ __forceinline__ bool gqa_qlimbs(const GqaParams& p, uint8_t* smem, int it, int buf, uint32_t& use,
                                           float (&sEn)[G]) {
    using C = GqaCfg<G, NS>;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* q_full = bars + 2 * NS + 10;
    uint64_t* red_bar = bars + 2 * NS + 12;
    float* red = reinterpret_cast<float*>(smem + C::OFF_RED);
    const int r = threadIdx.x, lane = threadIdx.x & 31;
    const GItem I = gqa_item(p, it);
    const float* q = p.Q + I.b * p.q_sb + static_cast<int64_t>(I.hk) * G * p.q_sh + r;
    float qv[G], am[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        qv[h] = __ldg(q + h * p.q_sh) * p.qscale;
        am[h] = fabsf(qv[h]);
    }
    if (!epi_reduce<G, true>(am, red, red_bar, use)) return false;
    uint8_t* qb = smem + C::OFF_QB + buf * C::QB_BYTES;
#pragma unroll
    for (int h = 0; h < G; ++h) {
        int E = 0;
        if (am[h] > 0.f) {
            int ex;
            frexpf(am[h], &ex);  // am < 2^ex
            E = min(126, max(-126, 30 - ex));
        }
        int qi = __float2int_rn(qv[h] * pow2i(E));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int L = static_cast<int>(static_cast<int8_t>(qi & 0xFF));
            qi = (qi - L) >> 8;
            const int n = 4 * h + j;
            qb[(n >> 3) * 1024 + (n & 7) * 128 + ((((r >> 4) ^ (n & 7)) << 4) | (r & 15))] =
                static_cast<uint8_t>(L);
        }
        sEn[h] = pow2i(-E);
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&q_full[buf]);
    return true;
}

struct PvSnap {
    int64_t i;
    int it, flags;
};

template <int G, int NS>
__device__ __forceinline__ bool gqa_pv_epi(const GqaParams& p, uint8_t* smem, uint32_t tmem, const PvSnap& A,
                                           const float (&mA)[G], const int (&FA)[G], const float (&LA)[G],
                                           float (&o)[G], float (&mpv)[G]) {
    using C = GqaCfg<G, NS>;
    constexpr int NP = C::NP;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* o_full = bars + 2 * NS + 6;
    uint64_t* o_free = bars + 2 * NS + 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = threadIdx.x;
    const int bj = static_cast<int>(A.i & 1);
    if (!mbar_wait(&o_full[bj], static_cast<uint32_t>((A.i >> 1) & 1))) return false;
    tc_fence_after();
    uint32_t orr[NP];
    tmem_ld_np<NP>(tmem + (static_cast<uint32_t>(warp * 32) << 16) + 2 * NP + bj * NP, orr);
    tmem_wait_ld();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&o_free[bj]);
    if (A.flags & 1) {
#pragma unroll
        for (int h = 0; h < G; ++h) { o[h] = 0.f; mpv[h] = mA[h]; }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
        const float f = combine_limbs(orr[4 * h], orr[4 * h + 1], orr[4 * h + 2], orr[4 * h + 3]);
        const float al = (mpv[h] == mA[h]) ? 1.f : exp2f(mpv[h] - mA[h]);
        o[h] = fmaf(f, pow2i(-FA[h]), o[h] * al);
        mpv[h] = mA[h];
    }
    if (A.flags & 2) {
        const GItem I = gqa_item(p, A.it);
        const bool records = p.P > 1 || (p.flags & KVD_FLAG_PARTIAL_OUT);
#pragma unroll
        for (int h = 0; h < G; ++h) {
            const int hq = I.hk * G + h;
            float* row = p.out + I.b * p.o_sb + static_cast<int64_t>(hq) * p.o_sh;
            if (!records) {
                row[r] = LA[h] > 0.f ? o[h] / LA[h] : 0.f;
            } else {
                float* rec = p.P > 1
                    ? p.partials + ((static_cast<int64_t>(I.b) * p.Hq + hq) * p.P + I.split) * (C::D + 4)
                    : row;
                if (r == 0) { rec[0] = mA[h]; rec[1] = LA[h]; }
                rec[4 + r] = o[h];
            }
        }
    }
    return true;
}

template <int G, int NS>
__device__ __forceinline__ void gqa_epilogue(const GqaParams& p, uint8_t* smem, uint32_t tmem) {
    using C = GqaCfg<G, NS>;
    constexpr int NP = C::NP;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* full = bars;
    uint64_t* empty = bars + NS;
    uint64_t* s_full = bars + 2 * NS;
    uint64_t* s_free = bars + 2 * NS + 2;
    uint64_t* w_full = bars + 2 * NS + 4;
    uint64_t* red_bar = bars + 2 * NS + 12;
    const GMeta* meta = reinterpret_cast<const GMeta*>(smem + C::OFF_META);
    float* red = reinterpret_cast<float*>(smem + C::OFF_RED);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = threadIdx.x;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    uint32_t use = 0;

    // Zero both query-limb buffers (pad rows must stay zero), then item 0's limbs.
    for (int x = r; x < 2 * C::QB_BYTES / 16; x += 128)
        reinterpret_cast<uint4*>(smem + C::OFF_QB)[x] = make_uint4(0u, 0u, 0u, 0u);
    float sEn[G];
    if (!gqa_qlimbs<G, NS>(p, smem, blockIdx.x, 0, use, sEn)) return;

    float m[G], l[G], sE[G], o[G], mpv[G], mA[G], LA[G];
    int FA[G];
#pragma unroll
    for (int h = 0; h < G; ++h) { m[h] = -INFINITY; l[h] = 0.f; sE[h] = 1.f; o[h] = 0.f; mpv[h] = -INFINITY;
                                  mA[h] = -INFINITY; LA[h] = 0.f; FA[h] = 0; }
    PvSnap A{-1, 0, 0};
    int64_t i = 0;
    int s = 0;
    uint32_t ph = 0;
    int kq = 0;
    for (int it = blockIdx.x; it < p.n_items; it += p.grid, ++kq) {
        const GItem I = gqa_item(p, it);
        for (int tt = 0; tt < I.ntiles; ++tt, ++i) {
            const int bi = static_cast<int>(i & 1);
            // ---- scores of tile i (thread r = token r of the tile)
            if (!mbar_wait(&s_full[bi], static_cast<uint32_t>((i >> 1) & 1))) return;
            tc_fence_after();
            uint32_t sr[NP];
            tmem_ld_np<NP>(lane_base + bi * NP, sr);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[bi]);
            if (!mbar_wait(&full[s], ph)) return;
            const GMeta mt = meta[s];
            if (tt == 0) {
#pragma unroll
                for (int h = 0; h < G; ++h) { m[h] = -INFINITY; l[h] = 0.f; sE[h] = sEn[h]; }
            }
            const bool valid = r < mt.n;
            const float* ksm = reinterpret_cast<const float*>(smem + s * C::STAGE_BYTES + C::OFF_KS);
            const float* vsm = reinterpret_cast<const float*>(smem + s * C::STAGE_BYTES + C::OFF_VS);
            const float ksv = valid ? ksm[(mt.offs & 0xff) + r] : 0.f;
            const float vsv = valid ? vsm[(mt.offs >> 8) + r] : 0.f;
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == NS) { s = 0; ph ^= 1u; }
            float sc[G], rv[G + 1];
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float dot = combine_limbs(sr[4 * h], sr[4 * h + 1], sr[4 * h + 2], sr[4 * h + 3]);
                sc[h] = valid ? dot * sE[h] * ksv : -INFINITY;
                rv[h] = sc[h];
            }
            rv[G] = vsv;
            if (!epi_reduce<G + 1, true>(rv, red, red_bar, use)) return;
            const float vsmax = rv[G];
            // ---- online softmax (base 2, lazy max) and the weight limbs
            uint32_t W[NP / 4];
#pragma unroll
            for (int x = 0; x < NP / 4; ++x) W[x] = 0u;
            int FB[G];
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float tmax = rv[h];
                const float mnew = (tmax > m[h] + 8.f) ? tmax : m[h];
                const float alpha = (mnew == -INFINITY) ? 1.f : exp2f(m[h] - mnew);
                l[h] *= alpha;
                m[h] = mnew;
                const float pr = valid ? exp2f(sc[h] - m[h]) : 0.f;
                l[h] += pr;
                const float bound = (tmax == -INFINITY) ? 0.f : exp2f(tmax - m[h]) * vsmax;
                int F = 0;
                if (bound > 0.f) {
                    int ex;
                    frexpf(bound, &ex);  // bound < 2^ex, so w * 2^(31-ex) < 2^31
                    F = min(126, max(-126, 31 - ex));
                }
                FB[h] = F;
                W[h] = valid ? __float2uint_rn(pr * vsv * pow2i(F)) : 0u;
            }
            uint8_t* wb = smem + C::OFF_WB + bi * C::WB_BYTES;
#pragma unroll
            for (int g = 0; g < NP / 16; ++g)
                *reinterpret_cast<uint4*>(wb + g * 2048 + r * 16) = make_uint4(W[4 * g], W[4 * g + 1], W[4 * g + 2], W[4 * g + 3]);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&w_full[bi]);
            float LB[G];
            if (tt == I.ntiles - 1) {
#pragma unroll
                for (int h = 0; h < G; ++h) LB[h] = l[h];
                if (!epi_reduce<G, false>(LB, red, red_bar, use)) return;
            } else {
#pragma unroll
                for (int h = 0; h < G; ++h) LB[h] = 0.f;
            }
            if (tt == 0 && it + p.grid < p.n_items) {
                if (!gqa_qlimbs<G, NS>(p, smem, it + p.grid, (kq + 1) & 1, use, sEn)) return;
            }
            // ---- PV epilogue of the previous tile (thread r = output dim r)
            if (A.i >= 0 && !gqa_pv_epi<G, NS>(p, smem, tmem, A, mA, FA, LA, o, mpv)) return;
#pragma unroll
            for (int h = 0; h < G; ++h) { mA[h] = m[h]; FA[h] = FB[h]; LA[h] = LB[h]; }
            A.i = i;
            A.it = it;
            A.flags = mt.flags;
        }
    }
    if (A.i >= 0) gqa_pv_epi<G, NS>(p, smem, tmem, A, mA, FA, LA, o, mpv);
}

template <int G, int NS, int MINB>
__global__ void __launch_bounds__(192, MINB) gqa_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                                                          const __grid_constant__ CUtensorMap vmap,
                                                          const GqaParams p) {
    using C = GqaCfg<G, NS>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    if (static_cast<int>(blockIdx.x) >= p.n_items) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* done = bars + 2 * NS + 13;
    uint64_t* drain = bars + 2 * NS + 14;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&bars[s], 1);          // full
            mbar_init(&bars[NS + s], 5);     // empty: MMA commit + 4 epilogue warps
        }
        const int b0 = 2 * NS;
        mbar_init(&bars[b0 + 0], 1);  mbar_init(&bars[b0 + 1], 1);   // s_full
        mbar_init(&bars[b0 + 2], 4);  mbar_init(&bars[b0 + 3], 4);   // s_free
        mbar_init(&bars[b0 + 4], 4);  mbar_init(&bars[b0 + 5], 4);   // w_full
        mbar_init(&bars[b0 + 6], 1);  mbar_init(&bars[b0 + 7], 1);   // o_full
        mbar_init(&bars[b0 + 8], 4);  mbar_init(&bars[b0 + 9], 4);   // o_free
        mbar_init(&bars[b0 + 10], 4); mbar_init(&bars[b0 + 11], 4);  // q_full
        mbar_init(&bars[b0 + 12], 4);                                // red
        mbar_init(done, 4);
        mbar_init(drain, 1);
        fence_mbar_init();
    }
    if (warp == 5) tmem_alloc(reinterpret_cast<uint32_t*>(smem + C::OFF_TMEM), C::TMEM_COLS);
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + C::OFF_TMEM);
    if (warp == 4) {
        if (lane == 0) gqa_producer<G, NS>(&kmap, &vmap, p, smem);
        return;
    }
    if (warp == 5) {
        if (lane == 0) {
            gqa_mma<G, NS>(p, smem, tmem);
            mma_commit(drain);  // arrives once every MMA issued above has completed
            mbar_wait(drain, 0);
            mbar_wait(done, 0);  // epilogue warps have finished reading TMEM
        }
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
        return;
    }
    gqa_epilogue<G, NS>(p, smem, tmem);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(done);
}

}  // namespace kvd

// ------------------------------------------------------------------ host side
namespace kvd {
namespace {

constexpr int kGqaNS = KVD_GQA_NS;
constexpr int kGqaCtas = KVD_GQA_CTAS;

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// 4-D view {D bytes, tokens, kv heads, batch} of a K or V cache, box of
// 128 bytes x 128 tokens, 128-byte swizzle (the canonical K-major operand
// layout for K, and the MN-major one for V).
bool make_kv_map(CUtensorMap* m, const int8_t* base, int B, int Hkv, int cap, int64_t kv_sb, int64_t kv_sh) {
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    const int64_t sh = kv_sh > 0 ? kv_sh : static_cast<int64_t>(cap) * 128;
    const int64_t sb = kv_sb > 0 ? kv_sb : sh * Hkv;
    cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(cap), static_cast<cuuint64_t>(Hkv), static_cast<cuuint64_t>(B)};
    cuuint64_t strides[3] = {128, static_cast<cuuint64_t>(sh), static_cast<cuuint64_t>(sb)};
    cuuint32_t box[4] = {128, 128, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int gqa_split_count(const kvd_decode_desc& d) {
    const int64_t units = static_cast<int64_t>(d.batch) * d.num_kv_heads;
    const int64_t grid_max = static_cast<int64_t>(device_sm_count()) * kGqaCtas;
    if (units >= grid_max) return 1;
    const int max_by_len = d.max_seq_len > 0 ? (d.max_seq_len + 127) / 128 : 1;
    int64_t P = (grid_max + units - 1) / units;
    if (P > max_by_len) P = max_by_len;
    return static_cast<int>(P < 1 ? 1 : P);
}

template <int G>
cudaError_t launch_gqa_g(const CUtensorMap& km, const CUtensorMap& vm, const GqaParams& p, cudaStream_t st) {
    using C = GqaCfg<G, kGqaNS>;
    static bool configured[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    auto kern = gqa_tc_kernel<G, kGqaNS, kGqaCtas>;
    if (dev < 64 && !configured[dev]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    kern<<<p.grid, C::THREADS, C::SMEM_BYTES, st>>>(km, vm, p);
    return cudaGetLastError();
}

}  // namespace

bool gqa_path_ok(const kvd_decode_desc& d) {
    const int G = d.num_q_heads / d.num_kv_heads;
    if (d.head_dim != 128 || d.max_seq_len < 1) return false;
    if (G != 2 && G != 4 && G != 8 && G != 16) return false;
    return tensor_map_encoder() != nullptr;
}

size_t gqa_workspace_size(const kvd_decode_desc& d) {
    const int P = gqa_split_count(d);
    if (P <= 1) return 0;
    return static_cast<size_t>(d.batch) * d.num_q_heads * P * (d.head_dim + 4) * sizeof(float);
}

cudaError_t launch_gqa_tc(const kvd_decode_desc& d, const float* Q, const int8_t* K, const int8_t* V,
                          const float* ks, const float* vs, float* out, void* ws, size_t ws_bytes,
                          cudaStream_t st, int* launches) {
    const int G = d.num_q_heads / d.num_kv_heads;
    const int64_t rec_row_bytes = static_cast<int64_t>(d.batch) * d.num_q_heads * (d.head_dim + 4) * 4;
    int P = gqa_split_count(d);
    if (P > 1) {
        const int64_t fit = ws ? static_cast<int64_t>(ws_bytes) / rec_row_bytes : 0;
        if (fit < P) P = static_cast<int>(fit);
        if (P < 2) P = 1;
    }
    const int S = d.max_seq_len;
    const int span = ((((S + P - 1) / P) + 127) / 128) * 128;
    P = (S + span - 1) / span;
    if (P < 1) P = 1;
    CUtensorMap km, vm;
    if (!make_kv_map(&km, K, d.batch, d.num_kv_heads, S, d.kv_stride_b, d.kv_stride_h) ||
        !make_kv_map(&vm, V, d.batch, d.num_kv_heads, S, d.kv_stride_b, d.kv_stride_h))
        return cudaErrorInvalidValue;
    GqaParams p{};
    p.Q = Q; p.ks = ks; p.vs = vs; p.out = out;
    p.partials = P > 1 ? static_cast<float*>(ws) : nullptr;
    p.seq_lens = d.seq_lens;
    p.B = d.batch; p.Hq = d.num_q_heads; p.Hkv = d.num_kv_heads; p.S = S; p.P = P; p.span = span;
    p.n_items = d.batch * d.num_kv_heads * P;
    const int64_t grid_max = static_cast<int64_t>(device_sm_count()) * kGqaCtas;
    p.grid = static_cast<int>(grid_max < p.n_items ? grid_max : p.n_items);
    p.sc_sb = d.sc_stride_b; p.sc_sh = d.sc_stride_h;
    p.q_sb = d.q_stride_b; p.q_sh = d.q_stride_h;
    p.o_sb = d.o_stride_b; p.o_sh = d.o_stride_h;
    const float scale = d.softmax_scale > 0.f ? d.softmax_scale : 1.0f / sqrtf(static_cast<float>(d.head_dim));
    p.qscale = scale * 1.4426950408889634f;
    p.flags = d.flags;
    cudaError_t e;
    switch (G) {
        case 2: e = launch_gqa_g<2>(km, vm, p, st); break;
        case 4: e = launch_gqa_g<4>(km, vm, p, st); break;
        case 8: e = launch_gqa_g<8>(km, vm, p, st); break;
        case 16: e = launch_gqa_g<16>(km, vm, p, st); break;
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    ++*launches;
    if (P > 1) {
        const int64_t rs = d.head_dim + 4;
        e = launch_combine_records(static_cast<const float*>(ws), P, rs, rs * P,
                                   static_cast<int64_t>(d.batch) * d.num_q_heads, d.num_q_heads, d.head_dim, out,
                                   d.o_stride_b, d.o_stride_h, d.flags, st, launches);
    }
    return e;
}

}  // namespace kvd
