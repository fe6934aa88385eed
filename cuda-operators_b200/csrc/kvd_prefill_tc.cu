// kvd_prefill_tc.cu -- causal prefill over the INT8 cache on the tcgen05
// tensor cores (no reference counterpart: the reference's prefill attention,
// attention/, is fp32 with no KV cache).
//
// Work item = (batch b, kv head hk, block of 128 query rows); row r is query
// qb*QPB + r/G of query head hk*G + r%G (QPB = 128/G), so the G heads of a
// group share every K/V tile. The item walks 64-token tiles of its causal
// prefix:
//   * a producer thread loads the INT8 K and V tiles (TMA, 128-byte swizzle)
//     into a 6-deep ring and both scale windows into an 8-deep ring of their
//     own;
//   * a converter warpgroup widens each INT8 tile to bf16 (codes are exact in
//     bf16) in one row-per-token, 128-byte-swizzled layout that is the K-major
//     B operand of S = Q K^T for K and the MN-major B operand of O += P V for
//     V (no transposition); the widening uses no conversion instruction: a
//     sign flip, a byte permute that builds the float 2^23 + 128 + code, one
//     packed add and a byte permute of the upper halves. It also writes each
//     item's queries, scaled by softmax_scale*log2(e), as two bf16 terms
//     (hi + lo, about 16 significant bits) into tensor memory (the A operand
//     of S);
//   * one elected lane of the MMA warp issues the MMAs (kind::f16, M = 128,
//     fp32 accumulators in tensor memory, A operands read from tensor memory):
//     S(j) = Qhi K^T + Qlo K^T (N = 64) into one of two S buffers, two tiles
//     ahead of O += Phi V + Plo V (N = 128);
//   * a softmax warpgroup owns one query row per thread (= TMEM lane): scores
//     times the token's k_scale, the causal mask (only on the tiles that
//     reach the block's first query), a lazily rescaled online softmax in base
//     2 (the running max may trail by up to 8; when it moves the thread
//     rescales its O row in tensor memory), and weights p * v_scale split into
//     bf16 hi + lo, stored with tcgen05.st into one of two P buffers in tensor
//     memory, so the softmax of tile j+1 overlaps the PV MMAs of tile j. At the
//     end of the item it divides O by l and stores the output rows.
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
constexpr int PNS = 6;         // INT8 tile ring depth
constexpr int PSC = 8;         // scale ring depth
constexpr int P_THREADS = 320; // softmax warps 0-3, converter warps 4-7, producer 8, MMA 9

// Shared memory (bytes from a 1024-aligned base).
constexpr int OFF_K8 = 0;                        // [PNS] INT8 K tiles, 64 rows x 128 B, as TMA wrote them
constexpr int OFF_V8 = OFF_K8 + PNS * 8192;      // [PNS] INT8 V tiles
constexpr int OFF_KB = OFF_V8 + PNS * 8192;      // [2] bf16 K: 2 atoms of 64 token rows x 128 B
constexpr int OFF_VB = OFF_KB + 2 * 16384;       // [2] bf16 V, same layout
constexpr int OFF_SC = OFF_VB + 2 * 16384;       // [PSC] k_scale[64], v_scale[64]
constexpr int OFF_BAR = OFF_SC + PSC * 512;
// Barriers. Per buffer b of the double-buffered stages, the k-th completion
// belongs to tile j = 2k+b: SREADY (S(j) may be issued: bf16 K(j) written by
// the 4 converter warps and S(j-2) read by the 4 softmax warps, which arrive
// once up front for j < 2), SDONE (S(j) computed: the softmax may read it, the
// bf16 K buffer is free), PVREADY (PV(j) may be issued: P(j) written by the
// softmax warps and bf16 V(j) by the converter warps), PVDONE (PV(j) done: P
// buffer and bf16 V buffer free, O updated).
constexpr int B_K8FULL = 0, B_K8EMPTY = B_K8FULL + PNS, B_SCFULL = B_K8EMPTY + PNS, B_SCEMPTY = B_SCFULL + PSC,
              B_SREADY = B_SCEMPTY + PSC, B_SDONE = B_SREADY + 2, B_PVREADY = B_SDONE + 2, B_PVDONE = B_PVREADY + 2,
              B_QFULL = B_PVDONE + 2, B_QEMPTY = B_QFULL + 1, B_OREAD = B_QEMPTY + 1,
              B_DONE = B_OREAD + 1, B_DRAIN = B_DONE + 1, P_NBAR = B_DRAIN + 1;
constexpr int OFF_TMEM = OFF_BAR + P_NBAR * 8;
constexpr int P_SMEM_BYTES = OFF_TMEM + 16 + 1024;  // slack to align the base to 1024
// Tensor memory (all 512 columns): S buffers at columns 0 and 64 (fp32), P
// buffers at 128 and 192 (bf16 pairs: hi in the first 32 columns, lo in the
// next 32), O at 256 (fp32), the item's queries at 384 (bf16 pairs: hi in
// 384-447, lo in 448-511). S and P V read their A operand from tensor memory,
// so shared memory only feeds the B operands.
constexpr uint32_t P_TMEM_COLS = 512;
constexpr uint32_t COL_P = 128, COL_O = 256, COL_Q = 384;
static_assert(OFF_K8 % 1024 == 0 && OFF_KB % 1024 == 0 && OFF_VB % 1024 == 0, "swizzle atoms");
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
    int vec_out;  // fp32 output rows 16-byte aligned: float4 stores
    int vec_q;    // query rows 16-byte aligned: 16-byte loads and L2 prefetch
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
    // query i sits at position L - ql + i; with more queries than tokens the first rows
    // would sit before position 0 and are written as zeros
    I.ql = p.q_lens ? min(max(0, __ldg(p.q_lens + I.b)), p.Lq) : p.Lq;
    const int q0 = I.qb * p.QPB;
    const int ntok = I.L - I.ql + min(I.ql, q0 + p.QPB);  // tokens up to the block's last query
    I.ntiles = q0 < I.ql && ntok > 0 ? (ntok + PT - 1) / PT : 0;
    return I;
}

__device__ __forceinline__ int pf_next(const PfParams& p, int it) {
    while (it < p.n_items && pf_item(p, it).ntiles == 0) it += p.grid;
    return it;
}

// ------------------------------------------------------------------ producer
// Lane 0 of warp 8: INT8 K and V tiles (box 128 B x 64 tokens) into the tile
// ring and the two scale windows of every tile into the scale ring. Tokens
// past the capacity are zero-filled by TMA; the scale copies stop at the
// capacity (the softmax masks those tokens without using their scales).
__device__ __forceinline__ void pf_producer(const CUtensorMap* kmap, const CUtensorMap* vmap, const PfParams& p,
                                            uint8_t* smem) {
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    const uint64_t pol = policy_evict_last();  // every query block of (b, kv head) reads the same tiles
    int64_t j = 0;
    bool ok = true;
    for (int it = pf_next(p, blockIdx.x); it < p.n_items && ok; it = pf_next(p, it + p.grid)) {
        const PfItem I = pf_item(p, it);
        for (int tt = 0; tt < I.ntiles; ++tt, ++j) {
            const int s = static_cast<int>(j % PNS), c = static_cast<int>(j % PSC);
            if ((j >= PNS && !mbar_wait(&bars[B_K8EMPTY + s], static_cast<uint32_t>(((j / PNS) - 1) & 1))) ||
                (j >= PSC && !mbar_wait(&bars[B_SCEMPTY + c], static_cast<uint32_t>(((j / PSC) - 1) & 1)))) {
                ok = false;
                break;
            }
            const int t0 = tt * PT;
            uint64_t* full = &bars[B_K8FULL + s];
            mbar_arrive_expect_tx(full, 2u * 8192u);
            tma_load_4d(smem + OFF_K8 + s * 8192, kmap, 0, t0, I.hk, I.b, full, pol);
            tma_load_4d(smem + OFF_V8 + s * 8192, vmap, 0, t0, I.hk, I.b, full, pol);
            const int nsc = min(PT, p.S - t0);
            const uint32_t seg = static_cast<uint32_t>(4 * nsc + 15) & ~15u;
            const int64_t so = I.b * p.sc_sb + I.hk * p.sc_sh + t0;
            uint64_t* scfull = &bars[B_SCFULL + c];
            mbar_arrive_expect_tx(scfull, 2u * seg);
            bulk_g2s(smem + OFF_SC + c * 512, p.ks + so, seg, scfull, pol);
            bulk_g2s(smem + OFF_SC + c * 512 + 256, p.vs + so, seg, scfull, pol);
        }
    }
    for (int64_t x = j > PNS ? j - PNS : 0; x < j; ++x)  // no copy in flight at exit
        mbar_wait(&bars[B_K8FULL + x % PNS], static_cast<uint32_t>((x / PNS) & 1));
    for (int64_t x = j > PSC ? j - PSC : 0; x < j; ++x)
        mbar_wait(&bars[B_SCFULL + x % PSC], static_cast<uint32_t>((x / PSC) & 1));
}

// ------------------------------------------------------------------ converters
__device__ __forceinline__ uint32_t bf16x2(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// Four INT8 codes -> two bf16 pairs, exactly: dequant4 returns each code as a
// float whose low 16 bits are zero (at most 8 significant bits), so its upper
// half is the bf16 of the code.
__device__ __forceinline__ void widen4(uint32_t w, uint32_t& lo, uint32_t& hi) {
    float2 a, b;
    dequant4(w, a, b);
    lo = __byte_perm(__float_as_uint(a.x), __float_as_uint(a.y), 0x7632);
    hi = __byte_perm(__float_as_uint(b.x), __float_as_uint(b.y), 0x7632);
}

// Element offset of query row r of an item (query qb*QPB + r/G of head
// hk*G + r%G); valid = the query exists (i < q_len).
__device__ __forceinline__ int64_t pf_q_row(const PfParams& p, const PfItem& I, int r, bool& valid) {
    const int i = I.qb * p.QPB + r / p.G, g = r % p.G;
    valid = i < I.ql;
    return I.b * p.q_sb + static_cast<int64_t>(I.hk * p.G + g) * p.q_sh + static_cast<int64_t>(i) * p.q_st;
}

// 32 scaled query elements (dims 32*qd ..) as bf16 hi + lo pairs into this
// thread's TMEM lane: hi at column COL_Q + 16*qd, lo 64 columns further.
__device__ __forceinline__ void pf_store_q32(uint32_t lane_base, int qd, const float (&x)[32]) {
    uint32_t hi[16], lo[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * k], x[2 * k + 1]);
        hi[k] = *reinterpret_cast<const uint32_t*>(&h);
        lo[k] = bf16x2(x[2 * k] - __low2float(h), x[2 * k + 1] - __high2float(h));
    }
    tmem_st16(lane_base + COL_Q + 16u * qd, hi);
    tmem_st16(lane_base + COL_Q + 64u + 16u * qd, lo);
}

// Row r of the item's queries, scaled by softmax_scale*log2(e), into TMEM
// lane r (the A operand of S). Rows that are 16-byte aligned are read 16
// bytes at a time, a half row (64 dims) in flight at once; others element by
// element.
__device__ __forceinline__ void pf_load_q(const PfParams& p, const PfItem& I, uint32_t lane_base, int r) {
    bool valid;
    const int64_t q0 = pf_q_row(p, I, r, valid);
    if (p.vec_q) {
        const bool f32 = (p.flags & (KVD_FLAG_Q_BF16 | KVD_FLAG_Q_F16)) == 0;
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
            uint4 raw[16];
            const int n16 = f32 ? 16 : 8;  // 16-byte loads per 64 dims
            const uint4* src = f32 ? reinterpret_cast<const uint4*>(static_cast<const float*>(p.Q) + q0 + 64 * half)
                                   : reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.Q) + q0 + 64 * half);
#pragma unroll
            for (int k = 0; k < 16; ++k)
                raw[k] = (valid && k < n16) ? __ldg(src + k) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int qq = 0; qq < 2; ++qq) {  // 32 dims at a time
                float x[32];
                if (f32) {
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const uint4 a = raw[8 * qq + k];
                        x[4 * k] = __uint_as_float(a.x) * p.qscale;
                        x[4 * k + 1] = __uint_as_float(a.y) * p.qscale;
                        x[4 * k + 2] = __uint_as_float(a.z) * p.qscale;
                        x[4 * k + 3] = __uint_as_float(a.w) * p.qscale;
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint4 a = raw[4 * qq + k];
                        const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            float2 f;
                            if (p.flags & KVD_FLAG_Q_BF16) {
                                f = make_float2(__uint_as_float(w[e] << 16), __uint_as_float(w[e] & 0xFFFF0000u));
                            } else {
                                f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
                            }
                            x[8 * k + 2 * e] = f.x * p.qscale;
                            x[8 * k + 2 * e + 1] = f.y * p.qscale;
                        }
                    }
                }
                pf_store_q32(lane_base, 2 * half + qq, x);
            }
        }
        return;
    }
#pragma unroll 1
    for (int qd = 0; qd < PD / 32; ++qd) {
        float x[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) x[k] = valid ? load_q(p.Q, q0 + 32 * qd + k, p.flags) * p.qscale : 0.f;
        pf_store_q32(lane_base, qd, x);
    }
}

// Start moving row r of item `it`'s queries into L2 (aligned rows only), so
// that the item's Q load after the current item hits L2.
__device__ __forceinline__ void pf_prefetch_q(const PfParams& p, int it, int r) {
    if (!p.vec_q || it >= p.n_items) return;
    const PfItem I = pf_item(p, it);
    bool valid;
    const int64_t q0 = pf_q_row(p, I, r, valid);
    if (!valid) return;
    const bool f32 = (p.flags & (KVD_FLAG_Q_BF16 | KVD_FLAG_Q_F16)) == 0;
    const void* a = f32 ? static_cast<const void*>(static_cast<const float*>(p.Q) + q0)
                        : static_cast<const void*>(static_cast<const uint16_t*>(p.Q) + q0);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(f32 ? 512u : 256u) : "memory");
}

// INT8 tile (TMA 128-byte swizzle: code (t, d) at t*128 + ((d/16 ^ t%8) * 16)
// + d%16) -> bf16 tile with rows = tokens, 2 atoms of 64 dims: element (t, d)
// at (d/64)*8192 + (t/8)*1024 + (t%8)*128 + (((d%64)/8 ^ t%8) * 16) + (d%8)*2.
// Thread ct of the warpgroup widens 4 of the 512 16-code chunks; each group of
// 8 lanes takes 4 chunks of an even token and the other 4 chunk columns of the
// next token, so its 16-byte loads and stores hit 8 distinct bank groups.
__device__ __forceinline__ void pf_widen_tile(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int ct) {
    uint4 w[4];
    int t[4], c8[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {  // every load first: the stores cannot alias them
        const int task = ct + 128 * u, e = task & 3, hb = (task >> 2) & 1, grp = (task >> 3) & 1;
        t[u] = 2 * (task >> 4) + hb;
        c8[u] = e + 4 * (hb ^ grp);
        w[u] = *reinterpret_cast<const uint4*>(src + t[u] * 128 + ((c8[u] ^ (t[u] & 7)) << 4));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        uint4 a, b;
        widen4(w[u].x, a.x, a.y);
        widen4(w[u].y, a.z, a.w);
        widen4(w[u].z, b.x, b.y);
        widen4(w[u].w, b.z, b.w);
        const int ch = (c8[u] & 3) * 2, t7 = t[u] & 7;
        uint8_t* row = dst + (c8[u] >> 2) * 8192 + (t[u] >> 3) * 1024 + t7 * 128;
        *reinterpret_cast<uint4*>(row + ((ch ^ t7) << 4)) = a;
        *reinterpret_cast<uint4*>(row + (((ch + 1) ^ t7) << 4)) = b;
    }
}

// Warps 4-7, per item: the queries, then the bf16 K of the first two tiles,
// then per tile t the K of tile t+2 and the V of tile t: the order in which
// the MMA thread consumes them (S runs two tiles ahead of PV).
__device__ __forceinline__ bool pf_convert(uint8_t* smem, uint64_t* bars, int64_t j, bool v_side, int ct, int lane) {
    const int s = static_cast<int>(j % PNS), jb = static_cast<int>(j & 1);
    if (!v_side && !mbar_wait(&bars[B_K8FULL + s], static_cast<uint32_t>((j / PNS) & 1))) return false;
    // the buffer is free once S(j-2) (K) or PV(j-2) (V) has completed
    if (j >= 2 && !mbar_wait(&bars[(v_side ? B_PVDONE : B_SDONE) + jb], static_cast<uint32_t>(((j >> 1) - 1) & 1)))
        return false;
    pf_widen_tile(smem + (v_side ? OFF_V8 : OFF_K8) + s * 8192, smem + (v_side ? OFF_VB : OFF_KB) + jb * 16384, ct);
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
        mbar_arrive(&bars[(v_side ? B_PVREADY : B_SREADY) + jb]);
        if (v_side) mbar_arrive(&bars[B_K8EMPTY + s]);  // both halves of the INT8 slot are widened
    }
    return true;
}

__device__ __forceinline__ void pf_converters(const PfParams& p, uint8_t* smem, uint32_t tmem) {
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    const int ct = threadIdx.x - 128, lane = threadIdx.x & 31;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(ct & ~31) << 16);  // warp 4+q: TMEM lanes 32q..32q+31
    int64_t j0 = 0;
    int ni = 0;
    for (int it = pf_next(p, blockIdx.x); it < p.n_items; it = pf_next(p, it + p.grid), ++ni) {
        const PfItem I = pf_item(p, it);
        if (ni > 0 && !mbar_wait(&bars[B_QEMPTY], static_cast<uint32_t>((ni - 1) & 1))) return;
        tc_fence_after();  // the previous item's S MMAs have finished reading the queries
        pf_load_q(p, I, lane_base, ct);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_QFULL]);
        pf_prefetch_q(p, pf_next(p, it + p.grid), ct);
        for (int t = 0; t < min(2, I.ntiles); ++t)
            if (!pf_convert(smem, bars, j0 + t, false, ct, lane)) return;
        for (int t = 0; t < I.ntiles; ++t) {
            if (t + 2 < I.ntiles && !pf_convert(smem, bars, j0 + t + 2, false, ct, lane)) return;
            if (!pf_convert(smem, bars, j0 + t, true, ct, lane)) return;
        }
        j0 += I.ntiles;
    }
}

// ------------------------------------------------------------------ MMA issuer
// A bounded wait whose result is the same in every lane of the warp.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

// Warp 9 (one elected lane issues), per item: S of the first two tiles, then per tile t the PV
// of tile t (once P(t) is written) and the S of tile t+2 (its buffer was read by
// the softmax at tile t). S(j) = Qhi K^T + Qlo K^T into S buffer j&1
// with Q from tensor memory; PV(j): O += Phi V + Plo V with P from P buffer
// j&1 (overwriting O at an item's first tile, after the softmax has read the
// previous item's O). An item's PVs all precede the next item's first S, which
// waits for the next item's queries.
__device__ __forceinline__ void pf_mma(const PfParams& p, uint8_t* smem, uint32_t tmem) {
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    constexpr uint32_t id_s = idesc_bf16(PT, PM);
    constexpr uint32_t id_o = idesc_bf16(PD, PM, true);  // V is the MN-major B operand
    auto s_mma = [&](int64_t j) -> bool {
        const int jb = static_cast<int>(j & 1);
        if (!mbar_wait_warp(&bars[B_SREADY + jb], static_cast<uint32_t>((j >> 1) & 1))) return false;
        tc_fence_after();
        const uint64_t kd = smem_desc(smem_u32(smem + OFF_KB + jb * 16384), 16u, 1024u, kLayoutSw128);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int kk = 0; kk < PD / 16; ++kk)  // 16 dims: 32 bytes within a row, 64-dim atoms 8 KB apart
                mma_f16_ts_warp(tmem + jb * PT, tmem + COL_Q + 64u * half + 8u * kk,
                           kd + (((kk >> 2) * 8192u + (kk & 3) * 32u) >> 4), id_s, half > 0 || kk > 0);
        }
        mma_commit_warp(&bars[B_SDONE + jb]);
        return true;
    };
    auto pv_mma = [&](int64_t j, bool first, int ni) -> bool {
        const int jb = static_cast<int>(j & 1);
        const uint32_t par = static_cast<uint32_t>((j >> 1) & 1);
        if (!mbar_wait_warp(&bars[B_PVREADY + jb], par)) return false;
        if (first && ni > 0 && !mbar_wait_warp(&bars[B_OREAD], static_cast<uint32_t>((ni - 1) & 1))) return false;
        tc_fence_after();
        // 16 tokens = 2 groups of 8 token rows (SBO 1024); dims 64-127 one atom on (LBO 8192)
        const uint64_t vd = smem_desc(smem_u32(smem + OFF_VB + jb * 16384), 8192u, 1024u, kLayoutSw128);
        const uint32_t pa = tmem + COL_P + static_cast<uint32_t>(jb) * 64u;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int kk = 0; kk < PT / 16; ++kk)
                mma_f16_ts_warp(tmem + COL_O, pa + 32u * half + 8u * kk, vd + (2048u * kk >> 4), id_o,
                           !(first && half == 0 && kk == 0));
        }
        mma_commit_warp(&bars[B_PVDONE + jb]);
        return true;
    };
    int64_t j0 = 0;
    int ni = 0;
    for (int it = pf_next(p, blockIdx.x); it < p.n_items; it = pf_next(p, it + p.grid), ++ni) {
        const PfItem I = pf_item(p, it);
        const int nt = I.ntiles;
        if (!mbar_wait_warp(&bars[B_QFULL], static_cast<uint32_t>(ni & 1))) return;
        for (int t = 0; t < min(2, nt); ++t)
            if (!s_mma(j0 + t)) return;
        if (nt <= 2) mma_commit_warp(&bars[B_QEMPTY]);
        for (int t = 0; t < nt; ++t) {
            if (!pv_mma(j0 + t, t == 0, ni)) return;
            // S(t+2) after PV(t): its completion (SDONE) then also means that PV(t) has read P
            // buffer t&1, which the softmax rewrites at tile t+2
            if (t + 2 < nt) {
                if (!s_mma(j0 + t + 2)) return;
                if (t + 3 == nt) mma_commit_warp(&bars[B_QEMPTY]);  // the item's last S: the queries may be replaced
            }
        }
        j0 += nt;
    }
}

// ------------------------------------------------------------------ softmax
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// Output columns d0..d0+31 of row r of an item: raw fp32 accumulators times
// inv, or zeros. Rows past max_queries do not exist.
__device__ __forceinline__ void pf_store_row(const PfParams& p, const PfItem& I, int r, const uint32_t (&o)[32],
                                             float inv, bool zero, int d0) {
    const int i = I.qb * p.QPB + r / p.G, g = r % p.G;
    if (i >= p.Lq) return;
    const int64_t ro = I.b * p.o_sb + static_cast<int64_t>(I.hk * p.G + g) * p.o_sh +
                       static_cast<int64_t>(i) * p.o_st + d0;
    if (p.vec_out) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + ro);
#pragma unroll
        for (int x = 0; x < 8; ++x)
            dst[x] = zero ? make_float4(0.f, 0.f, 0.f, 0.f)
                          : make_float4(__uint_as_float(o[4 * x]) * inv, __uint_as_float(o[4 * x + 1]) * inv,
                                        __uint_as_float(o[4 * x + 2]) * inv, __uint_as_float(o[4 * x + 3]) * inv);
    } else {
#pragma unroll
        for (int d = 0; d < 32; ++d) store_out(p.out, ro + d, zero ? 0.f : __uint_as_float(o[d]) * inv, p.flags);
    }
}

// Warps 0-3, thread r = query row r = TMEM lane r. Walks every item of the
// CTA (items without tiles only zero their rows).
__device__ __forceinline__ void pf_softmax(const PfParams& p, uint8_t* smem, uint32_t tmem) {
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    const int r = threadIdx.x, wq = r >> 5, lane = r & 31;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(wq * 32) << 16);
    if (lane == 0) {  // S(0) and S(1) overwrite nothing the softmax still needs
        mbar_arrive(&bars[B_SREADY]);
        mbar_arrive(&bars[B_SREADY + 1]);
    }
    int64_t j = 0;
    for (int it = blockIdx.x; it < p.n_items; it += p.grid) {
        const PfItem I = pf_item(p, it);
        if (I.ntiles == 0) {  // no query of this block exists: zero rows
            const uint32_t none[32] = {};
#pragma unroll 1
            for (int d0 = 0; d0 < PD; d0 += 32) pf_store_row(p, I, r, none, 0.f, true, d0);
            continue;
        }
        const int i = I.qb * p.QPB + r / p.G;
        const int pos = I.L - I.ql + i;                // this query's own position
        const bool valid = i < I.ql && pos >= 0;
        const int pos_lo = I.L - I.ql + I.qb * p.QPB;  // the block's first query
        float m = -INFINITY;
        float2 lp[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};  // row sum, 4 independent chains
        for (int tt = 0; tt < I.ntiles; ++tt, ++j) {
            const int sb = static_cast<int>(j & 1), c = static_cast<int>(j % PSC), t0 = tt * PT;
            // ---- scores of tile j
            if (!mbar_wait(&bars[B_SDONE + sb], static_cast<uint32_t>((j >> 1) & 1))) return;
            tc_fence_after();
            uint32_t sr[PT];
            tmem_ld32(lane_base + sb * PT, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
            tmem_ld32(lane_base + sb * PT + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[B_SREADY + sb]);  // S(j+2) may overwrite the buffer
            if (!mbar_wait(&bars[B_SCFULL + c], static_cast<uint32_t>((j / PSC) & 1))) return;
            const float4* ks4 = reinterpret_cast<const float4*>(smem + OFF_SC + c * 512);
            const float4* vs4 = ks4 + 16;
            // the causal mask only matters on tiles that reach past the block's first query; masked
            // scores become -inf (the weights loop below has no branch: 2^-inf = 0)
            float tm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // 4 independent chains
            if (t0 + PT - 1 > pos_lo) {
                const int lim = valid ? pos - t0 : -1;  // tokens c <= lim are visible to this row
#pragma unroll
                for (int k = 0; k < PT / 4; ++k) {
                    const float4 kq = ks4[k];
                    const float2 va = __fmul2_rn(make_float2(__uint_as_float(sr[4 * k]), __uint_as_float(sr[4 * k + 1])),
                                                 make_float2(kq.x, kq.y));
                    const float2 vb = __fmul2_rn(make_float2(__uint_as_float(sr[4 * k + 2]), __uint_as_float(sr[4 * k + 3])),
                                                 make_float2(kq.z, kq.w));
                    const float v0 = 4 * k <= lim ? va.x : -INFINITY, v1 = 4 * k + 1 <= lim ? va.y : -INFINITY;
                    const float v2 = 4 * k + 2 <= lim ? vb.x : -INFINITY, v3 = 4 * k + 3 <= lim ? vb.y : -INFINITY;
                    sr[4 * k] = __float_as_uint(v0);
                    sr[4 * k + 1] = __float_as_uint(v1);
                    sr[4 * k + 2] = __float_as_uint(v2);
                    sr[4 * k + 3] = __float_as_uint(v3);
                    tm[k & 3] = fmax3(fmax3(tm[k & 3], v0, v1), v2, v3);
                }
            } else {
#pragma unroll
                for (int k = 0; k < PT / 4; ++k) {
                    const float4 kq = ks4[k];
                    const float2 va = __fmul2_rn(make_float2(__uint_as_float(sr[4 * k]), __uint_as_float(sr[4 * k + 1])),
                                                 make_float2(kq.x, kq.y));
                    const float2 vb = __fmul2_rn(make_float2(__uint_as_float(sr[4 * k + 2]), __uint_as_float(sr[4 * k + 3])),
                                                 make_float2(kq.z, kq.w));
                    sr[4 * k] = __float_as_uint(va.x);
                    sr[4 * k + 1] = __float_as_uint(va.y);
                    sr[4 * k + 2] = __float_as_uint(vb.x);
                    sr[4 * k + 3] = __float_as_uint(vb.y);
                    tm[k & 3] = fmax3(fmax3(tm[k & 3], va.x, va.y), vb.x, vb.y);
                }
            }
            const float tmax = fmaxf(fmaxf(tm[0], tm[1]), fmaxf(tm[2], tm[3]));
            // ---- lazy rescale: the running max may trail by up to 8
            const bool need = m != -INFINITY && tmax > m + 8.f;
            if (__any_sync(0xffffffffu, need)) {
                // m is finite, so tt >= 1: PV(j-1) of this item must be complete before O changes
                if (!mbar_wait(&bars[B_PVDONE + ((j - 1) & 1)], static_cast<uint32_t>(((j - 1) >> 1) & 1))) return;
                tc_fence_after();
                const float f = need ? ex2_fast(m - tmax) : 1.f;
#pragma unroll 1
                for (int cc = 0; cc < PD / 32; ++cc) {
                    uint32_t o[32];
                    tmem_ld32(lane_base + COL_O + 32 * cc, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int x = 0; x < 32; ++x) o[x] = __float_as_uint(__uint_as_float(o[x]) * f);
                    tmem_st32(lane_base + COL_O + 32 * cc, o);
                }
                tmem_wait_st();
                lp[0] = __fmul2_rn(lp[0], make_float2(f, f));
                lp[1] = __fmul2_rn(lp[1], make_float2(f, f));
            }
            if (need || (m == -INFINITY && tmax != -INFINITY)) m = tmax;
            // (P buffer sb is free: PV(j-2) was issued before S(j), whose completion was awaited above)
            // ---- weights w = 2^(s - m) * v_scale as bf16 hi + lo, 32 tokens at a time
            const uint32_t pcol = lane_base + COL_P + static_cast<uint32_t>(sb) * 64u;
            const float me = m == -INFINITY ? 0.f : m;  // a row with every score masked so far: all weights 0
            const float2 nm = make_float2(-me, -me);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const int cp = 16 * q + k;  // token pair
                    const float2 d = __fadd2_rn(make_float2(__uint_as_float(sr[2 * cp]), __uint_as_float(sr[2 * cp + 1])), nm);
                    const float2 pp = make_float2(ex2_fast(d.x), ex2_fast(d.y));
                    lp[k & 1] = __fadd2_rn(lp[k & 1], pp);
                    const float4 vq = vs4[cp >> 1];  // scales in the ring are always finite
                    const float2 w = __fmul2_rn(pp, (cp & 1) ? make_float2(vq.z, vq.w) : make_float2(vq.x, vq.y));
                    const uint32_t h = bf16x2(w.x, w.y);
                    hi[k] = h;
                    const float2 res =
                        __fadd2_rn(w, make_float2(-__uint_as_float(h << 16), -__uint_as_float(h & 0xFFFF0000u)));
                    lo[k] = bf16x2(res.x, res.y);
                }
                tmem_st16(pcol + 16u * q, hi);
                tmem_st16(pcol + 32u + 16u * q, lo);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars[B_PVREADY + sb]);
                mbar_arrive(&bars[B_SCEMPTY + c]);
            }
            // ---- end of the item: O / l to the output rows once PV(j) has completed
            if (tt == I.ntiles - 1) {
                if (!mbar_wait(&bars[B_PVDONE + sb], static_cast<uint32_t>((j >> 1) & 1))) return;
                tc_fence_after();
                const float l = (lp[0].x + lp[0].y) + (lp[1].x + lp[1].y);
                const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
                for (int cc = 0; cc < PD / 32; ++cc) {
                    uint32_t o[32];
                    tmem_ld32(lane_base + COL_O + 32 * cc, o);
                    tmem_wait_ld();
                    pf_store_row(p, I, r, o, inv, !valid, 32 * cc);  // rows without a query get zeros
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
            mbar_init(&bars[B_K8EMPTY + s], 4);  // converter warps
        }
        for (int c = 0; c < PSC; ++c) {
            mbar_init(&bars[B_SCFULL + c], 1);
            mbar_init(&bars[B_SCEMPTY + c], 4);  // softmax warps
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars[B_SREADY + b], 8);   // converter warps + softmax warps
            mbar_init(&bars[B_SDONE + b], 1);
            mbar_init(&bars[B_PVREADY + b], 8);  // converter warps + softmax warps
            mbar_init(&bars[B_PVDONE + b], 1);
        }
        mbar_init(&bars[B_QFULL], 4);
        mbar_init(&bars[B_QEMPTY], 1);
        mbar_init(&bars[B_OREAD], 4);
        mbar_init(&bars[B_DONE], 4);
        mbar_init(&bars[B_DRAIN], 1);
        fence_mbar_init();
    }
    // the scale ring starts as zeros, so a masked token past the capacity (whose scales are
    // never copied) multiplies a weight of 0 by a finite number
    for (int x = threadIdx.x; x < PSC * 512 / 16; x += P_THREADS)
        reinterpret_cast<uint4*>(smem + OFF_SC)[x] = make_uint4(0u, 0u, 0u, 0u);
    fence_async_smem();  // before any bulk copy into the ring
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
        pf_converters(p, smem, tmem);
    } else if (warp == 8) {
        if (lane == 0) pf_producer(&kmap, &vmap, p, smem);
    } else {
        pf_mma(p, smem, tmem);
        mma_commit_warp(&bars[B_DRAIN]);  // arrives once every MMA issued above has completed
        mbar_wait(&bars[B_DRAIN], 0);
        mbar_wait(&bars[B_DONE], 0);  // the softmax warps have finished with tensor memory
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
    p.vec_out = (d.flags & (KVD_FLAG_OUT_BF16 | KVD_FLAG_OUT_F16)) == 0 &&
                (reinterpret_cast<uintptr_t>(out) & 15) == 0 && ((d.o_stride_b | d.o_stride_h | d.o_stride_t) & 3) == 0;
    const int qe = (d.flags & (KVD_FLAG_Q_BF16 | KVD_FLAG_Q_F16)) ? 8 : 4;  // elements per 16 bytes
    p.vec_q = (reinterpret_cast<uintptr_t>(Q) & 15) == 0 && d.q_stride_b % qe == 0 && d.q_stride_h % qe == 0 &&
              d.q_stride_t % qe == 0;
    static PerDeviceOnce once;
    cudaError_t e = once.run([] {
        return cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES);
    });
    if (e != cudaSuccess) return e;
    prefill_tc_kernel<<<p.grid, P_THREADS, P_SMEM_BYTES, st>>>(km, vm, p);
    e = cudaGetLastError();
    if (e == cudaSuccess) ++*launches;
    return e;
}

}  // namespace kvd
