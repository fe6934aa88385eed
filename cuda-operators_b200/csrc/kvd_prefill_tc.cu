// kvd_prefill_tc.cu -- causal prefill over the INT8 cache on the tcgen05
// tensor cores (no reference counterpart: the reference's prefill attention,
// attention/, is fp32 with no KV cache).
//
// Work item = (batch b, kv head hk, block of 128 query rows); row r is query
// qb*QPB + r/G of query head hk*G + r%G (QPB = 128/G), so the G heads of a
// group share every K/V tile. The item walks 64-token tiles of its causal
// prefix:
//   * a producer warp loads the INT8 K and V tiles (TMA, 128-byte swizzle) and
//     both scale windows into a 3-deep ring;
//   * a converter warpgroup turns each tile into bf16 MMA operands (codes are
//     exact in bf16): K as the K-major B operand of S = Q K^T, V transposed as
//     the K-major B operand of O += P V; it also writes each item's queries,
//     scaled by softmax_scale*log2(e), as two bf16 terms (hi + lo, about 16
//     significant bits) into the A operand;
//   * one thread issues the MMAs (kind::f16, M = 128, fp32 accumulators in
//     tensor memory): S = Qhi K^T + Qlo K^T (N = 64), then O += Phi V + Plo V
//     (N = 128) one tile behind;
//   * a softmax warpgroup owns one query row per thread: scores (times the
//     token's k_scale), causal mask, a lazily rescaled online softmax in base 2
//     (the running max may trail by up to 8; when it moves the thread rescales
//     its O row in tensor memory), and weights p * v_scale split into bf16
//     hi + lo for the PV MMA. At the end of the item it divides O by l and
//     stores the output rows.
// Every wait is bounded; on expiry the kernel records KVD_STATUS_WAIT_TIMEOUT
// and unwinds.
#include <cuda.h>

#include <cstdio>

#include "kvd_common.cuh"
#include "kvd_decode.cuh"
#include "kvd_tc.cuh"

namespace kvd {
namespace {

constexpr int PD = 128;        // head_dim
constexpr int PM = 128;        // query rows per item (MMA M)
constexpr int PT = 64;         // tokens per tile (S columns, PV K)
constexpr int PNS = 3;         // INT8 tile ring depth
constexpr int P_THREADS = 320; // softmax warps 0-3, converter warps 4-7, producer 8, MMA 9

// Shared memory (bytes from a 1024-aligned base).
constexpr int OFF_QH = 0;                        // Q hi: 2 swizzle atoms of 128 rows x 128 B
constexpr int OFF_QL = OFF_QH + 32768;           // Q lo
constexpr int OFF_K8 = OFF_QL + 32768;           // [PNS] INT8 K tiles, 64 rows x 128 B, as TMA wrote them
constexpr int OFF_V8 = OFF_K8 + PNS * 8192;      // [PNS] INT8 V tiles
constexpr int OFF_SC = OFF_V8 + PNS * 8192;      // [PNS] k_scale[64], v_scale[64]
constexpr int OFF_KB = ((OFF_SC + PNS * 512) + 1023) & ~1023;  // [2] bf16 K: 2 atoms of 64 rows x 128 B
constexpr int OFF_VT = OFF_KB + 2 * 16384;       // [2] bf16 V^T: 1 atom of 128 rows x 128 B
constexpr int OFF_PH = OFF_VT + 2 * 16384;       // P hi: 128 rows x 64 tokens
constexpr int OFF_PL = OFF_PH + 16384;           // P lo
constexpr int OFF_BAR = OFF_PL + 16384;
// barriers
constexpr int B_K8FULL = 0, B_K8EMPTY = PNS, B_KBFULL = 2 * PNS, B_KBEMPTY = B_KBFULL + 2, B_VTFULL = B_KBEMPTY + 2,
              B_VTEMPTY = B_VTFULL + 2, B_QFULL = B_VTEMPTY + 2, B_QEMPTY = B_QFULL + 1, B_SFULL = B_QEMPTY + 1,
              B_SFREE = B_SFULL + 2, B_PFULL = B_SFREE + 2, B_ODONE = B_PFULL + 1, B_OREAD = B_ODONE + 1,
              B_DONE = B_OREAD + 1, B_DRAIN = B_DONE + 1, P_NBAR = B_DRAIN + 1;
constexpr int OFF_TMEM = OFF_BAR + P_NBAR * 8;
constexpr int P_SMEM_BYTES = OFF_TMEM + 16 + 1024;  // slack to align the base to 1024
constexpr uint32_t P_TMEM_COLS = 256;               // S: 2 x 64 columns, O: 128 columns
constexpr uint32_t COL_O = 128;
static_assert(OFF_KB % 1024 == 0 && OFF_VT % 1024 == 0 && OFF_PH % 1024 == 0 && OFF_PL % 1024 == 0, "atoms");
static_assert(P_SMEM_BYTES <= 232448, "shared memory");

struct PfParams {
    const void* Q;
    const float* ks;
    const float* vs;
    void* out;
    const int32_t* seq_lens;
    const int32_t* q_lens;
    int B, Hq, Hkv, G, S, Lq, QPB, QB, n_items, grid;
    int64_t sc_sb, sc_sh, q_sb, q_sh, q_st, o_sb, o_sh, o_st;
    float qscale;
    uint32_t flags;
};

struct PfItem {
    int b, hk, qb, L, ql, ntiles;
};

// Items are numbered query block first, last block (the longest prefixes)
// first, then (b, kv head); dealt round robin to the persistent CTAs.
__device__ __forceinline__ PfItem pf_item(const PfParams& p, int it) {
    PfItem I;
    const int per = p.B * p.Hkv;
    I.qb = p.QB - 1 - it / per;
    const int rem = it % per;
    I.b = rem / p.Hkv;
    I.hk = rem - I.b * p.Hkv;
    I.L = p.seq_lens ? min(max(0, __ldg(p.seq_lens + I.b)), p.S) : p.S;
    I.ql = p.q_lens ? min(max(0, __ldg(p.q_lens + I.b)), p.Lq) : p.Lq;
    I.ql = min(I.ql, I.L);
    const int q0 = I.qb * p.QPB;
    if (q0 >= I.ql) {
        I.ntiles = 0;
    } else {
        const int ntok = I.L - I.ql + min(I.ql, q0 + p.QPB);  // tokens up to the block's last query
        I.ntiles = (ntok + PT - 1) / PT;
    }
    return I;
}

__device__ __forceinline__ int pf_next(const PfParams& p, int it) {
    while (it < p.n_items && pf_item(p, it).ntiles == 0) it += p.grid;
    return it;
}

// ------------------------------------------------------------------ producer
// Lane 0 of warp 8: INT8 K and V tiles (box 128 B x 64 tokens) and the two
// scale windows of every tile into the ring. Tokens past the capacity are
// zero-filled by TMA; the scale copies stop at the capacity (the softmax
// masks those tokens without reading their scales).
__device__ __forceinline__ void pf_producer(const CUtensorMap* kmap, const CUtensorMap* vmap, const PfParams& p,
                                            uint8_t* smem) {
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    const uint64_t pol = policy_evict_last();  // every query block of (b, kv head) reads the same tiles
    int64_t j = 0;
    bool ok = true;
    for (int it = pf_next(p, blockIdx.x); it < p.n_items && ok; it = pf_next(p, it + p.grid)) {
        const PfItem I = pf_item(p, it);
        for (int tt = 0; tt < I.ntiles; ++tt, ++j) {
            const int s = static_cast<int>(j % PNS);
            if (j >= PNS && !mbar_wait(&bars[B_K8EMPTY + s], static_cast<uint32_t>(((j / PNS) - 1) & 1))) {
                ok = false;
                break;
            }
            const int t0 = tt * PT;
            const int nsc = min(PT, p.S - t0);
            const uint32_t seg = static_cast<uint32_t>(4 * nsc + 15) & ~15u;
            const int64_t so = I.b * p.sc_sb + I.hk * p.sc_sh + t0;
            uint64_t* full = &bars[B_K8FULL + s];
            mbar_arrive_expect_tx(full, 2u * 8192u + 2u * seg);
            tma_load_4d(smem + OFF_K8 + s * 8192, kmap, 0, t0, I.hk, I.b, full, pol);
            tma_load_4d(smem + OFF_V8 + s * 8192, vmap, 0, t0, I.hk, I.b, full, pol);
            bulk_g2s(smem + OFF_SC + s * 512, p.ks + so, seg, full, pol);
            bulk_g2s(smem + OFF_SC + s * 512 + 256, p.vs + so, seg, full, pol);
        }
    }
    for (int64_t x = j > PNS ? j - PNS : 0; x < j; ++x)  // no copy in flight at exit
        mbar_wait(&bars[B_K8FULL + x % PNS], static_cast<uint32_t>((x / PNS) & 1));
}

// ------------------------------------------------------------------ converters
__device__ __forceinline__ uint32_t bf16x2(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ float code(uint32_t w, int k) {
    return static_cast<float>(static_cast<int8_t>((w >> (8 * k)) & 0xFFu));
}

// Row r of the item's queries, scaled by softmax_scale*log2(e), as bf16
// hi + lo in the K-major 128-byte-swizzled A operand (2 atoms of 64 dims).
__device__ __forceinline__ void pf_load_q(const PfParams& p, const PfItem& I, uint8_t* smem, int r) {
    const int i = I.qb * p.QPB + r / p.G, g = r % p.G;
    const bool valid = i < I.ql;
    const int64_t q0 = I.b * p.q_sb + static_cast<int64_t>(I.hk * p.G + g) * p.q_sh + static_cast<int64_t>(i) * p.q_st;
#pragma unroll 2
    for (int c = 0; c < PD / 8; ++c) {  // 8 dims = one 16-byte chunk of bf16
        float x[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = valid ? load_q(p.Q, q0 + 8 * c + k, p.flags) * p.qscale : 0.f;
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * k], x[2 * k + 1]);
            hi[k] = *reinterpret_cast<const uint32_t*>(&h);
            lo[k] = bf16x2(x[2 * k] - __low2float(h), x[2 * k + 1] - __high2float(h));
        }
        const int atom = c >> 3, chunk = c & 7;
        const int off = atom * 16384 + (r >> 3) * 1024 + (r & 7) * 128 + ((chunk ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(smem + OFF_QH + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(smem + OFF_QL + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
}

// INT8 tile slot s -> bf16 K (K-major, rows = tokens, 2 atoms of 64 dims) and
// bf16 V^T (K-major, rows = dims, 64 tokens per row) in buffer jb. The INT8
// tiles are in the TMA 128-byte swizzle: byte (t, d) at
// t*128 + ((d/16 ^ t%8) * 16) + d%16.
__device__ __forceinline__ void pf_convert_tile(uint8_t* smem, int s, int jb, int ct) {
    const uint8_t* k8 = smem + OFF_K8 + s * 8192;
    const uint8_t* v8 = smem + OFF_V8 + s * 8192;
    uint8_t* kb = smem + OFF_KB + jb * 16384;
    uint8_t* vt = smem + OFF_VT + jb * 16384;
#pragma unroll
    for (int u = 0; u < 4; ++u) {  // K: 64 tokens x 8 chunks of 16 codes
        const int task = ct + 128 * u, t = task >> 3, c8 = task & 7;
        const uint4 w = *reinterpret_cast<const uint4*>(k8 + t * 128 + ((c8 ^ (t & 7)) << 4));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            uint32_t o[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t src = ww[2 * half + k / 2];
                o[k] = bf16x2(code(src, 2 * (k & 1)), code(src, 2 * (k & 1) + 1));
            }
            const int atom = c8 >> 2, chunk = (c8 & 3) * 2 + half;
            *reinterpret_cast<uint4*>(kb + atom * 8192 + (t >> 3) * 1024 + (t & 7) * 128 + ((chunk ^ (t & 7)) << 4)) =
                make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {  // V^T: 32 token pairs x 8 chunks of 16 dims
        const int task = ct + 128 * u, t = 2 * (task >> 3), c8 = task & 7;
        const uint4 a = *reinterpret_cast<const uint4*>(v8 + t * 128 + ((c8 ^ (t & 7)) << 4));
        const uint4 b = *reinterpret_cast<const uint4*>(v8 + (t + 1) * 128 + ((c8 ^ ((t + 1) & 7)) << 4));
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int x = 0; x < 16; ++x) {
            const int d = 16 * c8 + x;
            *reinterpret_cast<uint32_t*>(vt + (d >> 3) * 1024 + (d & 7) * 128 + (((t >> 3) ^ (d & 7)) << 4) +
                                         (t & 7) * 2) = bf16x2(code(aw[x >> 2], x & 3), code(bw[x >> 2], x & 3));
        }
    }
}

// Warps 4-7: each item's queries, then every tile's bf16 operands.
__device__ __forceinline__ void pf_converters(const PfParams& p, uint8_t* smem) {
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    const int ct = threadIdx.x - 128, lane = threadIdx.x & 31;
    int64_t j = 0;
    int ni = 0;
    for (int it = pf_next(p, blockIdx.x); it < p.n_items; it = pf_next(p, it + p.grid), ++ni) {
        const PfItem I = pf_item(p, it);
        if (ni > 0 && !mbar_wait(&bars[B_QEMPTY], static_cast<uint32_t>((ni - 1) & 1))) return;
        pf_load_q(p, I, smem, ct);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_QFULL]);
        for (int tt = 0; tt < I.ntiles; ++tt, ++j) {
            const int s = static_cast<int>(j % PNS), jb = static_cast<int>(j & 1);
            if (!mbar_wait(&bars[B_K8FULL + s], static_cast<uint32_t>((j / PNS) & 1))) return;
            if (j >= 2) {
                const uint32_t par = static_cast<uint32_t>(((j >> 1) - 1) & 1);
                if (!mbar_wait(&bars[B_KBEMPTY + jb], par) || !mbar_wait(&bars[B_VTEMPTY + jb], par)) return;
            }
            pf_convert_tile(smem, s, jb, ct);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars[B_KBFULL + jb]);
                mbar_arrive(&bars[B_VTFULL + jb]);
                mbar_arrive(&bars[B_K8EMPTY + s]);
            }
        }
    }
}

// ------------------------------------------------------------------ MMA issuer
// Lane 0 of warp 9: per tile S = Qhi K^T + Qlo K^T into S buffer j&1, then the
// PV of the previous tile, O += Phi V + Plo V (overwriting O at an item's
// first tile, after the softmax has read the previous item's O).
__device__ __forceinline__ void pf_mma(const PfParams& p, uint8_t* smem, uint32_t tmem) {
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    constexpr uint32_t id_s = idesc_bf16(PT, PM);
    constexpr uint32_t id_o = idesc_bf16(PD, PM);
    const uint32_t qh = smem_u32(smem + OFF_QH), ql = smem_u32(smem + OFF_QL);
    const uint32_t ph = smem_u32(smem + OFF_PH), pl = smem_u32(smem + OFF_PL);
    auto pv = [&](int64_t jj, bool first, int nii) -> bool {
        const int jb = static_cast<int>(jj & 1);
        if (!mbar_wait(&bars[B_PFULL], static_cast<uint32_t>(jj & 1))) return false;
        if (!mbar_wait(&bars[B_VTFULL + jb], static_cast<uint32_t>((jj >> 1) & 1))) return false;
        if (first && nii > 0 && !mbar_wait(&bars[B_OREAD], static_cast<uint32_t>((nii - 1) & 1))) return false;
        tc_fence_after();
        const uint32_t vt = smem_u32(smem + OFF_VT + jb * 16384);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int kk = 0; kk < PT / 16; ++kk) {
                const uint64_t ad = smem_desc((half ? pl : ph) + 32u * kk, 16u, 1024u, kLayoutSw128);
                const uint64_t bd = smem_desc(vt + 32u * kk, 16u, 1024u, kLayoutSw128);
                mma_f16(tmem + COL_O, ad, bd, id_o, !(first && half == 0 && kk == 0));
            }
        }
        mma_commit(&bars[B_ODONE]);
        mma_commit(&bars[B_VTEMPTY + jb]);
        return true;
    };
    int64_t j = 0, pj = -1;
    bool pfirst = false;
    int ni = 0, pni = 0;
    for (int it = pf_next(p, blockIdx.x); it < p.n_items; it = pf_next(p, it + p.grid), ++ni) {
        const PfItem I = pf_item(p, it);
        for (int tt = 0; tt < I.ntiles; ++tt, ++j) {
            const int jb = static_cast<int>(j & 1);
            if (!mbar_wait(&bars[B_KBFULL + jb], static_cast<uint32_t>((j >> 1) & 1))) return;
            if (tt == 0 && !mbar_wait(&bars[B_QFULL], static_cast<uint32_t>(ni & 1))) return;
            if (j >= 2 && !mbar_wait(&bars[B_SFREE + jb], static_cast<uint32_t>(((j >> 1) - 1) & 1))) return;
            tc_fence_after();
            const uint32_t kb = smem_u32(smem + OFF_KB + jb * 16384);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
#pragma unroll
                for (int kk = 0; kk < PD / 16; ++kk) {
                    const uint32_t koff = (kk >> 2) * 16384u + (kk & 3) * 32u;
                    const uint64_t ad = smem_desc((half ? ql : qh) + koff, 16u, 1024u, kLayoutSw128);
                    const uint64_t bd = smem_desc(kb + (kk >> 2) * 8192u + (kk & 3) * 32u, 16u, 1024u, kLayoutSw128);
                    mma_f16(tmem + jb * PT, ad, bd, id_s, half > 0 || kk > 0);
                }
            }
            mma_commit(&bars[B_SFULL + jb]);
            mma_commit(&bars[B_KBEMPTY + jb]);
            if (tt == I.ntiles - 1) mma_commit(&bars[B_QEMPTY]);
            if (pj >= 0 && !pv(pj, pfirst, pni)) return;
            pj = j;
            pfirst = tt == 0;
            pni = ni;
        }
    }
    if (pj >= 0) pv(pj, pfirst, pni);
}

// ------------------------------------------------------------------ softmax
// Warps 0-3, thread r = query row r = TMEM lane r. Walks every item of the
// CTA (items without tiles only zero their rows).
__device__ __forceinline__ void pf_store_row(const PfParams& p, const PfItem& I, int r, const float* o, float inv,
                                             int d0, int n) {
    const int i = I.qb * p.QPB + r / p.G, g = r % p.G;
    if (i >= p.Lq) return;
    const int64_t ro = I.b * p.o_sb + static_cast<int64_t>(I.hk * p.G + g) * p.o_sh + static_cast<int64_t>(i) * p.o_st;
    for (int d = 0; d < n; ++d) store_out(p.out, ro + d0 + d, o ? o[d] * inv : 0.f, p.flags);
}

__device__ __forceinline__ void pf_softmax(const PfParams& p, uint8_t* smem, uint32_t tmem) {
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    const int r = threadIdx.x, wq = r >> 5, lane = r & 31;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(wq * 32) << 16);
    int64_t j = 0;
    for (int it = blockIdx.x; it < p.n_items; it += p.grid) {
        const PfItem I = pf_item(p, it);
        const int i = I.qb * p.QPB + r / p.G;
        if (I.ntiles == 0) {  // no query of this block exists: zero rows
            pf_store_row(p, I, r, nullptr, 0.f, 0, PD);
            continue;
        }
        const bool valid = i < I.ql;
        const int pos = I.L - I.ql + i;  // this query's own position
        float m = -INFINITY, l = 0.f;
        for (int tt = 0; tt < I.ntiles; ++tt, ++j) {
            const int s = static_cast<int>(j % PNS), sb = static_cast<int>(j & 1);
            const int t0 = tt * PT;
            // ---- scores of tile j
            if (!mbar_wait(&bars[B_SFULL + sb], static_cast<uint32_t>((j >> 1) & 1))) return;
            tc_fence_after();
            uint32_t sr[PT];
            tmem_ld32(lane_base + sb * PT, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
            tmem_ld32(lane_base + sb * PT + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[B_SFREE + sb]);
            if (!mbar_wait(&bars[B_K8FULL + s], static_cast<uint32_t>((j / PNS) & 1))) return;  // scales
            const float* ksm = reinterpret_cast<const float*>(smem + OFF_SC + s * 512);
            const float* vsm = ksm + 64;
            float tmax = -INFINITY;
#pragma unroll
            for (int c = 0; c < PT; ++c) {
                const bool ok = valid && t0 + c <= pos;
                const float v = ok ? __uint_as_float(sr[c]) * ksm[c] : -INFINITY;
                sr[c] = __float_as_uint(v);
                tmax = fmaxf(tmax, v);
            }
            // ---- PV of the previous tile must be done before P or O change
            if (j >= 1 && !mbar_wait(&bars[B_ODONE], static_cast<uint32_t>((j - 1) & 1))) return;
            tc_fence_after();
            const bool need = m != -INFINITY && tmax > m + 8.f;  // lazy: the max may trail by up to 8
            if (__any_sync(0xffffffffu, need)) {
                const float f = need ? ex2_fast(m - tmax) : 1.f;
#pragma unroll 1
                for (int c = 0; c < PD / 32; ++c) {
                    uint32_t o[32];
                    tmem_ld32(lane_base + COL_O + 32 * c, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int x = 0; x < 32; ++x) o[x] = __float_as_uint(__uint_as_float(o[x]) * f);
                    tmem_st32(lane_base + COL_O + 32 * c, o);
                }
                tmem_wait_st();
                l *= f;
            }
            if (need || (m == -INFINITY && tmax != -INFINITY)) m = tmax;
            // ---- weights w = 2^(s - m) * v_scale as bf16 hi + lo, rows K-major
#pragma unroll
            for (int ch = 0; ch < PT / 8; ++ch) {
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    float w2[2];
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int c = 8 * ch + 2 * k + e;
                        const float v = __uint_as_float(sr[c]);
                        const float pr = v == -INFINITY ? 0.f : ex2_fast(v - m);
                        l += pr;
                        w2[e] = v == -INFINITY ? 0.f : pr * vsm[c];
                    }
                    const __nv_bfloat162 h = __floats2bfloat162_rn(w2[0], w2[1]);
                    hi[k] = *reinterpret_cast<const uint32_t*>(&h);
                    lo[k] = bf16x2(w2[0] - __low2float(h), w2[1] - __high2float(h));
                }
                const int off = (r >> 3) * 1024 + (r & 7) * 128 + ((ch ^ (r & 7)) << 4);
                *reinterpret_cast<uint4*>(smem + OFF_PH + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(smem + OFF_PL + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
            fence_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars[B_PFULL]);
                mbar_arrive(&bars[B_K8EMPTY + s]);
            }
            // ---- end of the item: O / l to the output rows
            if (tt == I.ntiles - 1) {
                if (!mbar_wait(&bars[B_ODONE], static_cast<uint32_t>(j & 1))) return;
                tc_fence_after();
                const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
                for (int c = 0; c < PD / 32; ++c) {
                    uint32_t o[32];
                    tmem_ld32(lane_base + COL_O + 32 * c, o);
                    tmem_wait_ld();
                    float of[32];
#pragma unroll
                    for (int x = 0; x < 32; ++x) of[x] = __uint_as_float(o[x]);
                    pf_store_row(p, I, r, valid ? of : nullptr, inv, 32 * c, 32);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars[B_OREAD]);
            }
        }
    }
}

__global__ void __launch_bounds__(P_THREADS, 1) prefill_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                  const __grid_constant__ CUtensorMap vmap,
                                                                  const PfParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    if (threadIdx.x == 0) {
        for (int s = 0; s < PNS; ++s) {
            mbar_init(&bars[B_K8FULL + s], 1);   // producer arrive + transaction bytes
            mbar_init(&bars[B_K8EMPTY + s], 8);  // 4 converter warps + 4 softmax warps
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars[B_KBFULL + b], 4);
            mbar_init(&bars[B_KBEMPTY + b], 1);
            mbar_init(&bars[B_VTFULL + b], 4);
            mbar_init(&bars[B_VTEMPTY + b], 1);
            mbar_init(&bars[B_SFULL + b], 1);
            mbar_init(&bars[B_SFREE + b], 4);
        }
        mbar_init(&bars[B_QFULL], 4);
        mbar_init(&bars[B_QEMPTY], 1);
        mbar_init(&bars[B_PFULL], 4);
        mbar_init(&bars[B_ODONE], 1);
        mbar_init(&bars[B_OREAD], 4);
        mbar_init(&bars[B_DONE], 4);
        mbar_init(&bars[B_DRAIN], 1);
        fence_mbar_init();
    }
    if (warp == 9) tmem_alloc(reinterpret_cast<uint32_t*>(smem + OFF_TMEM), P_TMEM_COLS);
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + OFF_TMEM);
    if (warp < 4) {
        pf_softmax(p, smem, tmem);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_DONE]);
    } else if (warp < 8) {
        pf_converters(p, smem);
    } else if (warp == 8) {
        if (lane == 0) pf_producer(&kmap, &vmap, p, smem);
    } else {
        if (lane == 0) {
            pf_mma(p, smem, tmem);
            mma_commit(&bars[B_DRAIN]);  // arrives once every MMA issued above has completed
            mbar_wait(&bars[B_DRAIN], 0);
            mbar_wait(&bars[B_DONE], 0);  // the softmax warps have finished with tensor memory
        }
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, P_TMEM_COLS);
    }
}

}  // namespace

bool prefill_tc_ok(const kvd_prefill_desc& d, const int8_t* K, const int8_t* V, const float* ks, const float* vs) {
    const int G = d.num_q_heads / d.num_kv_heads;
    if (d.head_dim != PD || (G != 1 && G != 2 && G != 4 && G != 8 && G != 16)) return false;
    const uintptr_t a = reinterpret_cast<uintptr_t>(K) | reinterpret_cast<uintptr_t>(V) |
                        reinterpret_cast<uintptr_t>(ks) | reinterpret_cast<uintptr_t>(vs);
    if ((a & 15) != 0 || ((d.kv_stride_b | d.kv_stride_h) & 15) != 0 || ((d.sc_stride_b | d.sc_stride_h) & 3) != 0)
        return false;
    return d.kv_stride_b > 0 && d.kv_stride_h > 0;
}

cudaError_t launch_prefill_tc(const kvd_prefill_desc& d, const void* Q, const int8_t* K, const int8_t* V,
                              const float* ks, const float* vs, void* out, cudaStream_t st, int* launches) {
    CUtensorMap km, vm;
    if (!make_kv_map_rows(&km, K, d.batch, d.num_kv_heads, d.max_seq_len, d.kv_stride_b, d.kv_stride_h, PT) ||
        !make_kv_map_rows(&vm, V, d.batch, d.num_kv_heads, d.max_seq_len, d.kv_stride_b, d.kv_stride_h, PT))
        return cudaErrorNotSupported;
    PfParams p{};
    p.Q = Q; p.ks = ks; p.vs = vs; p.out = out;
    p.seq_lens = d.seq_lens; p.q_lens = d.q_lens;
    p.B = d.batch; p.Hq = d.num_q_heads; p.Hkv = d.num_kv_heads; p.G = d.num_q_heads / d.num_kv_heads;
    p.S = d.max_seq_len; p.Lq = d.max_queries;
    p.QPB = PM / p.G;
    p.QB = (p.Lq + p.QPB - 1) / p.QPB;
    const int64_t items = static_cast<int64_t>(p.QB) * p.B * p.Hkv;
    if (items > 0x7fffffffLL) return cudaErrorInvalidValue;
    p.n_items = static_cast<int>(items);
    p.grid = p.n_items < device_sm_count() ? p.n_items : device_sm_count();
    p.sc_sb = d.sc_stride_b; p.sc_sh = d.sc_stride_h;
    p.q_sb = d.q_stride_b; p.q_sh = d.q_stride_h; p.q_st = d.q_stride_t;
    p.o_sb = d.o_stride_b; p.o_sh = d.o_stride_h; p.o_st = d.o_stride_t;
    const float scale = d.softmax_scale > 0.f ? d.softmax_scale : 1.0f / sqrtf(static_cast<float>(d.head_dim));
    p.qscale = scale * 1.4426950408889634f;
    p.flags = d.flags;
    static bool configured[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && !configured[dev]) {
        e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    prefill_tc_kernel<<<p.grid, P_THREADS, P_SMEM_BYTES, st>>>(km, vm, p);
    e = cudaGetLastError();
    if (e == cudaSuccess) ++*launches;
    return e;
}

}  // namespace kvd
