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
// Roles: NWG epilogue warpgroups (warp w reads TMEM lane quarter w % 4; for
// groups of 8 or 16 the heads are split between two warpgroups, which halves
// the per-tile epilogue latency), then one TMA producer warp and one MMA
// issuer warp (which also owns the TMEM allocation). Every wait is bounded; on
// expiry the kernel records KVD_STATUS_WAIT_TIMEOUT and unwinds.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>

#include "kvd_common.cuh"
#include "kvd_decode.cuh"
#include "kvd_quant.cuh"
#include "kvd_tc.cuh"

namespace kvd {

struct GqaParams {
    const void* Q;                // fp32, bf16 or fp16 (flags)
    const float* ks;
    const float* vs;
    void* out;                 // normalised rows (fp32, bf16 or fp16) or fp32 records
    float* partials;           // [B*Hq][P] records of D+4 floats when P > 1
    const int32_t* seq_lens;   // device [B] or nullptr
    const int32_t* order;      // ragged: sequences sorted by length, longest first; else nullptr
    int B, Hq, Hkv, S, P, span, n_items, grid;
    int64_t sc_sb, sc_sh, q_sb, q_sh, o_sb, o_sh;
    float qscale;
    uint32_t flags;
    // Paged cache (table != nullptr): the maps view the pools as
    // {D, block_size, Hkv, num_blocks}; lbs = log2(block_size) >= 3.
    const int32_t* table;
    int64_t bt_stride, sc_sblk;
    int lbs, nblk;
    // Fused quantise-on-append (k_new != nullptr, dense cache): token
    // seq_lens[b] of every (b, kv head) is quantised from k_new / v_new into
    // the cache before the tile that holds it is loaded, every length reads as
    // seq_lens[b] + 1 (clamped to S), and the last CTA to finish writes the new
    // lengths back (done_ctas is zeroed by the order kernel).
    const float* k_new;
    const float* v_new;
    int64_t new_sb, new_sh, kv_sb, kv_sh;
    int8_t* Kw;
    int8_t* Vw;
    float* ksw;
    float* vsw;
    int32_t* lens_rw;
    unsigned int* done_ctas;
    int len_add;
    // Tagged split records for a consumer that runs beside this grid (the
    // multi-GPU exchange), dense batches only: record (row, split) of D+4 words
    // at tagged + ((b * Hq + hq) * P + split) * (D + 4), each word {value bits,
    // tag << 32} written with one 8-byte store, so a reader that sees the tag
    // sees the value and no fence or count is needed. tag = *tag_src + 1, read
    // by every CTA before it allows its programmatic dependents to launch. The
    // grid is itself launched as a programmatic dependent of the previous
    // exchange: its CTAs set up while that kernel ends and wait for it
    // (griddepcontrol.wait) before any global memory access.
    // Compiled for groups up to kTagMaxGroup only (the larger groups' kernels
    // are at their register limit). nullptr: float records.
    unsigned long long* tagged;
    const unsigned int* tag_src;
};
constexpr int kTagMaxGroup = 4;

template <int G, int NK_, int NV_, int QM_>
struct GqaCfg {
    static constexpr int D = 128;
    static constexpr int TOK = 128;
    static constexpr int NK = NK_;                                // K tile ring depth
    static constexpr int NV = NV_;                                // V tile (+ scales) ring depth
    static constexpr int NP = (4 * G < 16) ? 16 : 4 * G;        // MMA N: limbs x heads, padded
    static constexpr int TMEM_COLS = (4 * NP <= 32) ? 32 : (4 * NP <= 64 ? 64 : (4 * NP <= 128 ? 128 : 256));
    static constexpr int NWG = G >= 8 ? 2 : 1;                  // epilogue warpgroups, heads split between them
    static constexpr int HPW = G / NWG;                           // heads per warpgroup
    static constexpr int CPW = NP / NWG;                          // MMA columns per warpgroup
    // Query mode: QM = 0 splits each query row into four exact byte limbs (QK
    // N = NP, four accumulator columns per head); QM = 1 (KVD_FLAG_QK_INT8)
    // quantises it to one int8 row per head, so QK has N = 16 and one column
    // per head: head h of warpgroup w is B row / accumulator column w*QPW + h.
    static constexpr bool QI8 = QM_ != 0;
    static constexpr int NQ = QI8 ? 16 : NP;                      // QK MMA N (<= NP)
    static constexpr int QPW = NQ / NWG;                          // QK rows / columns per warpgroup
    static constexpr int SW = QI8 ? HPW : CPW;                    // score columns an epilogue thread loads
    static constexpr int THREADS = 32 * (4 * NWG + 2);
    static constexpr int SC_FLOATS = TOK + 4;
    static constexpr int TILE_BYTES = TOK * D;                    // one K or V tile, 128-byte swizzle
    static constexpr int SC_BYTES = 2 * SC_FLOATS * 4;            // ks and vs windows of one tile
    static constexpr int OFF_KR = 0;                              // [NK] K tiles
    static constexpr int OFF_VR = OFF_KR + NK * TILE_BYTES;       // [NV] V tiles
    static constexpr int OFF_SC = OFF_VR + NV * TILE_BYTES;       // [NV] scale windows
    static constexpr int QB_BYTES = NP * 128;                     // K-major, 128-byte swizzle
    static constexpr int WB_BYTES = TOK * NP;                     // MN-major, no swizzle
    static constexpr int OFF_QB = (OFF_SC + NV * SC_BYTES + 1023) & ~1023;  // 2 buffers
    static constexpr int OFF_WB = OFF_QB + 2 * QB_BYTES;          // 2 buffers
    static constexpr int OFF_RED = OFF_WB + 2 * WB_BYTES;         // [NWG][2][4][32] floats
    static constexpr int OFF_META = OFF_RED + NWG * 2 * 4 * 32 * 4;  // [NV] x 16 bytes
    static constexpr int OFF_BAR = OFF_META + NV * 16;
    // barriers: kfull[NK], kempty[NK], vfull[NV], vempty[NV], s_full[2], s_free[2], w_full[2],
    // o_full[2], o_free[2], q_full[2], red[NWG], done, drain, append
    static constexpr int B_KFULL = 0, B_KEMPTY = NK, B_VFULL = 2 * NK, B_VEMPTY = 2 * NK + NV;
    static constexpr int B_SFULL = 2 * NK + 2 * NV, B_SFREE = B_SFULL + 2, B_WFULL = B_SFREE + 2,
                         B_OFULL = B_WFULL + 2, B_OFREE = B_OFULL + 2, B_QFULL = B_OFREE + 2, B_RED = B_QFULL + 2,
                         B_DONE = B_RED + NWG, B_DRAIN = B_DONE + 1, B_APPEND = B_DRAIN + 1;
    static constexpr int NBAR = B_APPEND + 1;
    static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;  // TMEM address, then the fused-append list count
    static constexpr int OFF_APPENDED = OFF_TMEM + 8;
    static constexpr int OFF_TAG = OFF_TMEM + 12;  // tagged records: the call's tag
    static constexpr int SMEM_USED = OFF_TMEM + 16;
    static constexpr int SMEM_BYTES = SMEM_USED + 1024;           // slack to align the base to 1024
    static_assert(G >= 1 && G <= 16 && G % NWG == 0 && CPW % 16 == 0, "group size");
    static_assert(OFF_VR % 1024 == 0 && OFF_QB % 1024 == 0 && QB_BYTES % 1024 == 0, "swizzle atoms");
    static_assert(SMEM_BYTES <= 232448, "shared memory");
};

// Exact int32 -> fp32 for |v| < 2^22: 0x4B400000 + v is the float 1.5*2^23 + v.
__device__ __forceinline__ float small_int_to_float(uint32_t v) {
    return __uint_as_float(0x4B400000u + v) - 12582912.0f;
}

// Four exact limb sums (|acc_j| < 2^22) -> fp32 value of sum_j acc_j 2^(8j).
// Pairs are joined exactly in int32 (|hi|, |lo| < 2^30), then converted.
__device__ __forceinline__ float combine_limbs(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3) {
    const int hi = static_cast<int>(a3) * 256 + static_cast<int>(a2);
    const int lo = static_cast<int>(a1) * 256 + static_cast<int>(a0);
    return fmaf(__int2float_rn(hi), 65536.0f, __int2float_rn(lo));
}

__device__ __forceinline__ float pow2i(int e) {  // 2^e for e in [-126, 127]
    return __int_as_float((e + 127) << 23);
}


// Smallest e with x < 2^e, for x >= 0 finite (subnormals and 0 give -126).
__device__ __forceinline__ int exp_above(float x) {
    return static_cast<int>((__float_as_uint(x) >> 23) & 0xFFu) - 126;
}

}  // namespace kvd

namespace kvd {

struct GItem {
    int b, hk, split, t_lo, t_hi, ntiles;
};

// Items are numbered split-major: item = (split * B + k) * Hkv + hk, where k
// walks the sequences longest first for ragged batches. Dealt round-robin to
// the CTAs, long items therefore go out first (longest-processing-time
// order). A split past the end of its sequence is empty (no tiles) and is
// skipped by every role, except split 0 of an empty sequence, which still
// writes its zero output.
__device__ __forceinline__ int seq_len_of(const GqaParams& p, int b) {
    return p.seq_lens ? min(max(0, __ldg(p.seq_lens + b)) + p.len_add, p.S) : p.S;
}

// Fused append: the cache position of sequence b's new token, or -1 when the
// cache is full (no append).
__device__ __forceinline__ int append_pos(const GqaParams& p, int b) {
    const int len = max(0, __ldg(p.seq_lens + b));
    return len < p.S ? len : -1;
}

__device__ __forceinline__ int split_count(const GqaParams& p, int len) {
    return len > 0 ? (len + p.span - 1) / p.span : 1;
}

__device__ __forceinline__ GItem gqa_item(const GqaParams& p, int it) {
    GItem I;
    const int per_split = p.B * p.Hkv;
    I.split = it / per_split;
    const int rem = it - I.split * per_split;
    const int k = rem / p.Hkv;
    I.hk = rem - k * p.Hkv;
    I.b = p.order ? __ldg(p.order + k) : k;
    const int len = seq_len_of(p, I.b);
    I.t_lo = I.split * p.span;
    I.t_hi = min(len, I.t_lo + p.span);
    const int n = I.t_hi - I.t_lo;
    I.ntiles = n > 0 ? (n + 127) / 128 : (I.split == 0 ? 1 : 0);
    return I;
}

// First non-empty item of this CTA at or after `it` (stepping by the grid).
__device__ __forceinline__ int next_item(const GqaParams& p, int it) {
    while (it < p.n_items && gqa_item(p, it).ntiles == 0) it += p.grid;
    return it;
}

__device__ __forceinline__ void st_tagged_gpu(unsigned long long* p, float v, unsigned int tag) {
    const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

struct __align__(16) GMeta {
    int32_t it, n, flags, offs;  // flags: bit0 first tile of item, bit1 last tile of item
};

// ------------------------------------------------------------------ producer
// Paged cache: the whole producer warp issues the copies of a tile, one box
// of min(block_size, 128) token rows per block (a tile never straddles a
// block when block_size >= 128; at most 16 boxes per tile, block_size >= 8),
// so a tile of small blocks costs one warp-wide issue instead of many serial
// ones. Lane j < 16 owns box j (its K box and V box). Scales: for blocks of
// 128 tokens or more, two bulk copies per tile (lanes 0 and 16); for smaller
// blocks, which would need two tiny copies per block, lane l loads the scales
// of tokens 4l..4l+3 with one 16-byte load per pool and stores them into the
// slot. Table reads run two tiles ahead and scale loads one tile ahead, so
// neither latency stalls the issue. Each ring slot is armed once with the
// sum of the bytes its lanes copy. K runs one tile ahead of V here.
// A block id outside the pool is not read: its scales are zeroed (score 0,
// weight 0) and the status word records it.
struct PTile {
    int it, tt, t0, n;
    GItem I;
};

// First tile of this CTA; it = n_items when there is none.
__device__ __forceinline__ PTile ptile_first(const GqaParams& p) {
    PTile T;
    T.it = next_item(p, blockIdx.x);
    T.tt = 0;
    T.t0 = 0;
    T.n = 0;
    T.I = GItem{0, 0, 0, 0, 0, 0};
    if (T.it < p.n_items) {
        T.I = gqa_item(p, T.it);
        T.t0 = T.I.t_lo;
        T.n = max(0, min(128, T.I.t_hi - T.t0));
    }
    return T;
}

__device__ __forceinline__ PTile ptile_next(const GqaParams& p, const PTile& A) {
    PTile T = A;
    if (T.it >= p.n_items) return T;
    if (++T.tt >= T.I.ntiles) {
        T.tt = 0;
        T.it = next_item(p, T.it + p.grid);
        if (T.it >= p.n_items) return T;
        T.I = gqa_item(p, T.it);
    }
    T.t0 = T.I.t_lo + T.tt * 128;
    T.n = max(0, min(128, T.I.t_hi - T.t0));
    return T;
}

// Block id of this lane's box (lane & 15) of tile T, -1 past the tile.
__device__ __forceinline__ int ptile_block(const GqaParams& p, const PTile& T, int rows, int lane) {
    const int tok = (lane & 15) * rows;
    if (T.it >= p.n_items || tok >= T.n) return -1;
    return __ldg(p.table + T.I.b * p.bt_stride + ((T.t0 + tok) >> p.lbs));
}

// Scales of tokens 4*lane .. 4*lane+3 of tile T (blocks of 8..64 tokens);
// zero past the tile or in a block outside the pool.
__device__ __forceinline__ void ptile_scales(const GqaParams& p, const PTile& T, int blk, int lane, float4& kq,
                                             float4& vq) {
    const int tl = 4 * lane;
    const int sblk = __shfl_sync(0xffffffffu, blk, (tl >> p.lbs) & 15);
    kq = make_float4(0.f, 0.f, 0.f, 0.f);
    vq = kq;
    if (T.it < p.n_items && tl < T.n && sblk >= 0 && sblk < p.nblk) {
        const int64_t so = sblk * p.sc_sblk + T.I.hk * p.sc_sh + ((T.t0 + tl) & ((1 << p.lbs) - 1));
        kq = __ldcs(reinterpret_cast<const float4*>(p.ks + so));
        vq = __ldcs(reinterpret_cast<const float4*>(p.vs + so));
    }
}

template <int G, int NK, int NV, int QM>
__device__ __forceinline__ void gqa_producer_paged(const CUtensorMap* kmap, const CUtensorMap* vmap,
                                                   const GqaParams& p, uint8_t* smem) {
    using C = GqaCfg<G, NK, NV, QM>;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    GMeta* meta = reinterpret_cast<GMeta*>(smem + C::OFF_META);
    const uint64_t pol = policy_evict_first();
    const int lane = threadIdx.x & 31, j = lane & 15;
    const int bs = 1 << p.lbs;
    const int rows = bs < C::TOK ? bs : C::TOK;
    const bool small = rows < C::TOK;
    const uint32_t box = static_cast<uint32_t>(rows) * C::D;
    int64_t ik = 0, iv = 0;  // tiles issued on each ring
    // K boxes of tile T (this lane's box): wait for the slot, arm it, issue.
    auto issue_k = [&](const PTile& T, int blk) -> bool {
        const int tok = j * rows;
        const bool good = tok < T.n && blk >= 0 && blk < p.nblk;
        const int sk = static_cast<int>(ik % NK);
        if (ik >= NK && !mbar_wait(&bars[C::B_KEMPTY + sk], static_cast<uint32_t>(((ik / NK) - 1) & 1)))
            return false;
        const uint32_t bytes = __reduce_add_sync(0xffffffffu, (lane < 16 && good) ? box : 0u);
        if (lane == 0) mbar_arrive_expect_tx(&bars[C::B_KFULL + sk], bytes);
        __syncwarp();
        if (lane < 16 && good)
            tma_load_4d(smem + C::OFF_KR + sk * C::TILE_BYTES + tok * C::D, kmap, 0, (T.t0 + tok) & (bs - 1), T.I.hk,
                        blk, &bars[C::B_KFULL + sk], pol);
        ++ik;
        return true;
    };
    PTile T0 = ptile_first(p);
    PTile T1 = ptile_next(p, T0);
    int b0 = ptile_block(p, T0, rows, lane), b1 = ptile_block(p, T1, rows, lane);
    float4 kq0, vq0;
    if (small) ptile_scales(p, T0, b0, lane, kq0, vq0);
    // K runs one tile ahead of V: K(T0) now, then each step issues K(T1) before V(T0).
    bool ok = T0.it >= p.n_items || issue_k(T0, b0);
    while (ok && T0.it < p.n_items) {
        const PTile T2 = ptile_next(p, T1);
        const int b2 = ptile_block(p, T2, rows, lane);  // two tiles ahead
        float4 kq1, vq1;
        if (small) ptile_scales(p, T1, b1, lane, kq1, vq1);  // one tile ahead
        if (T1.it < p.n_items && !issue_k(T1, b1)) break;
        const int tok = j * rows;
        const bool act = tok < T0.n;
        const bool good = act && b0 >= 0 && b0 < p.nblk;
        if (act && !good && lane < 16) record_status(KVD_STATUS_BAD_BLOCK);
        const int off = (T0.t0 + tok) & (bs - 1);
        // ---- V slot: V boxes, scales, metadata
        const int sv = static_cast<int>(iv % NV);
        if (iv >= NV && !mbar_wait(&bars[C::B_VEMPTY + sv], static_cast<uint32_t>(((iv / NV) - 1) & 1))) break;
        float* sck = reinterpret_cast<float*>(smem + C::OFF_SC + sv * C::SC_BYTES);
        const int cnt = act ? min(rows, T0.n - tok) : 0;
        const uint32_t seg = static_cast<uint32_t>(4 * cnt + 15) & ~15u;  // bulk scale copy (rows == 128)
        float* dst = lane < 16 ? sck : sck + C::SC_FLOATS;
        if (small) {
            reinterpret_cast<float4*>(sck)[lane] = kq0;
            reinterpret_cast<float4*>(sck + C::SC_FLOATS)[lane] = vq0;
        } else if (act && !good && (lane & 15) == 0) {
            for (int x = 0; x < cnt; ++x) dst[x] = 0.f;
            fence_async_smem();  // order these writes before later bulk copies into the slot
        }
        if (lane == 0)
            meta[sv] = GMeta{T0.it, T0.n, (T0.tt == 0 ? 1 : 0) | (T0.tt == T0.I.ntiles - 1 ? 2 : 0), 0};
        const uint32_t mine = !good ? 0u : small ? (lane < 16 ? box : 0u) : (lane < 16 ? box + seg : lane == 16 ? seg : 0u);
        const uint32_t bytes = __reduce_add_sync(0xffffffffu, mine);
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(&bars[C::B_VFULL + sv], bytes);
        __syncwarp();
        if (good) {
            const int64_t so = b0 * p.sc_sblk + T0.I.hk * p.sc_sh + off;
            if (lane < 16)
                tma_load_4d(smem + C::OFF_VR + sv * C::TILE_BYTES + tok * C::D, vmap, 0, off, T0.I.hk, b0,
                            &bars[C::B_VFULL + sv], pol);
            if (!small && lane == 0) bulk_g2s(dst, p.ks + so, seg, &bars[C::B_VFULL + sv], pol);
            if (!small && lane == 16) bulk_g2s(dst, p.vs + so, seg, &bars[C::B_VFULL + sv], pol);
        }
        ++iv;
        T0 = T1;
        T1 = T2;
        b0 = b1;
        b1 = b2;
        if (small) { kq0 = kq1; vq0 = vq1; }
    }
    // no copy may be in flight when the CTA exits
    for (int64_t x = ik > NK ? ik - NK : 0; x < ik; ++x)
        mbar_wait(&bars[C::B_KFULL + x % NK], static_cast<uint32_t>((x / NK) & 1));
    for (int64_t x = iv > NV ? iv - NV : 0; x < iv; ++x)
        mbar_wait(&bars[C::B_VFULL + x % NV], static_cast<uint32_t>((x / NV) & 1));
}

// Lane 0 streams K tiles, lane 1 streams V tiles with both scale windows and
// the tile metadata; the two rings are released independently (K as soon as
// QK has read it, V after PV and the softmax), so K loads run ahead of V.
template <int G, int NK, int NV, int QM>
__device__ __forceinline__ void gqa_producer(const CUtensorMap* kmap, const CUtensorMap* vmap, const GqaParams& p,
                                             uint8_t* smem, bool v_side) {
    using C = GqaCfg<G, NK, NV, QM>;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    const int R = v_side ? NV : NK;
    uint64_t* full = bars + (v_side ? C::B_VFULL : C::B_KFULL);
    uint64_t* empty = bars + (v_side ? C::B_VEMPTY : C::B_KEMPTY);
    GMeta* meta = reinterpret_cast<GMeta*>(smem + C::OFF_META);
    const uint64_t pol = policy_evict_first();
    int s = 0;
    uint32_t round_par = 0;
    bool wrapped = false, ok = true;
    int64_t issued = 0;
    bool appended = p.k_new == nullptr;  // fused append finished (or none)
    for (int it = next_item(p, blockIdx.x); it < p.n_items && ok; it = next_item(p, it + p.grid)) {
        const GItem I = gqa_item(p, it);
        const int apos = appended ? -1 : append_pos(p, I.b);
        for (int tt = 0; tt < I.ntiles; ++tt) {
            if (wrapped && !mbar_wait(&empty[s], round_par ^ 1u)) { ok = false; break; }
            const int t0 = I.t_lo + tt * C::TOK;
            const int n = max(0, min(C::TOK, I.t_hi - t0));
            // the first tile holding a new token waits for the epilogue warps to have written them all
            if (!appended && apos >= t0 && apos < t0 + n) {
                if (!mbar_wait(&bars[C::B_APPEND], 0)) { ok = false; break; }
                appended = true;
            }
            if (!v_side) {
                mbar_arrive_expect_tx(&full[s], n > 0 ? static_cast<uint32_t>(C::TILE_BYTES) : 0u);
                if (n > 0) tma_load_4d(smem + C::OFF_KR + s * C::TILE_BYTES, kmap, 0, t0, I.hk, I.b, &full[s], pol);
            } else {
                uint32_t kwin = 0, vwin = 0;
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
                }
                GMeta mt;
                mt.it = it;
                mt.n = n;
                mt.flags = (tt == 0 ? 1 : 0) | (tt == I.ntiles - 1 ? 2 : 0);
                mt.offs = koff | (voff << 8);
                meta[s] = mt;
                mbar_arrive_expect_tx(&full[s], n > 0 ? static_cast<uint32_t>(C::TILE_BYTES) + kwin + vwin : 0u);
                if (n > 0) {
                    uint8_t* sc = smem + C::OFF_SC + s * C::SC_BYTES;
                    tma_load_4d(smem + C::OFF_VR + s * C::TILE_BYTES, vmap, 0, t0, I.hk, I.b, &full[s], pol);
                    bulk_g2s(sc, reinterpret_cast<const void*>(ka0), kwin, &full[s], pol);
                    bulk_g2s(sc + C::SC_FLOATS * 4, reinterpret_cast<const void*>(va0), vwin, &full[s], pol);
                }
            }
            ++issued;
            if (++s == R) { s = 0; round_par ^= 1u; wrapped = true; }
        }
    }
    for (int64_t j = issued > R ? issued - R : 0; j < issued; ++j)
        mbar_wait(&full[j % R], static_cast<uint32_t>((j / R) & 1));
}

// ------------------------------------------------------------------ MMA issuer
template <int G, int NK, int NV, int QM>
__device__ __forceinline__ bool gqa_mma_pv(uint8_t* smem, uint32_t tmem, int64_t j) {
    using C = GqaCfg<G, NK, NV, QM>;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    const int bj = static_cast<int>(j & 1);
    const int sv = static_cast<int>(j % NV);
    if (!mbar_wait(&bars[C::B_VFULL + sv], static_cast<uint32_t>((j / NV) & 1))) return false;
    if (!mbar_wait(&bars[C::B_WFULL + bj], static_cast<uint32_t>((j >> 1) & 1))) return false;
    if (j >= 2 && !mbar_wait(&bars[C::B_OFREE + bj], static_cast<uint32_t>(((j >> 1) - 1) & 1))) return false;
    tc_fence_after();
    constexpr uint32_t idesc = idesc_i8(true, false, true, true, C::NP, 128);
    const uint32_t vbase = smem_u32(smem + C::OFF_VR + sv * C::TILE_BYTES);
    const uint32_t wbase = smem_u32(smem + C::OFF_WB + bj * C::WB_BYTES);
    const uint32_t dcol = tmem + 2 * C::NP + bj * C::NP;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
        const uint64_t ad = smem_desc(vbase + 4096u * kk, 16u, 1024u, kLayoutSw128);
        const uint64_t bd = smem_desc(wbase + 512u * kk, 128u, 2048u, kLayoutNone);
        mma_i8(dcol, ad, bd, idesc, kk > 0);
    }
    mma_commit(&bars[C::B_OFULL + bj]);
    mma_commit(&bars[C::B_VEMPTY + sv]);
    return true;
}

template <int G, int NK, int NV, int QM>
__device__ __forceinline__ void gqa_mma(const GqaParams& p, uint8_t* smem, uint32_t tmem) {
    using C = GqaCfg<G, NK, NV, QM>;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    constexpr uint32_t idesc_qk = idesc_i8(true, true, false, false, C::NQ, 128);
    int64_t i = 0;
    int kq = 0;
    for (int it = next_item(p, blockIdx.x); it < p.n_items; it = next_item(p, it + p.grid), ++kq) {
        const GItem I = gqa_item(p, it);
        for (int tt = 0; tt < I.ntiles; ++tt, ++i) {
            const int sk = static_cast<int>(i % NK);
            if (!mbar_wait(&bars[C::B_KFULL + sk], static_cast<uint32_t>((i / NK) & 1))) return;
            if (tt == 0 && !mbar_wait(&bars[C::B_QFULL + (kq & 1)], static_cast<uint32_t>((kq >> 1) & 1))) return;
            const int bi = static_cast<int>(i & 1);
            if (i >= 2 && !mbar_wait(&bars[C::B_SFREE + bi], static_cast<uint32_t>(((i >> 1) - 1) & 1))) return;
            tc_fence_after();
            const uint32_t kbase = smem_u32(smem + C::OFF_KR + sk * C::TILE_BYTES);
            const uint32_t qbase = smem_u32(smem + C::OFF_QB + (kq & 1) * C::QB_BYTES);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint64_t ad = smem_desc(kbase + 32u * kk, 16u, 1024u, kLayoutSw128);
                const uint64_t bd = smem_desc(qbase + 32u * kk, 16u, 1024u, kLayoutSw128);
                mma_i8(tmem + bi * C::NP, ad, bd, idesc_qk, kk > 0);
            }
            mma_commit(&bars[C::B_SFULL + bi]);
            mma_commit(&bars[C::B_KEMPTY + sk]);
            if (i >= 1 && !gqa_mma_pv<G, NK, NV, QM>(smem, tmem, i - 1)) return;
        }
    }
    if (i >= 1) gqa_mma_pv<G, NK, NV, QM>(smem, tmem, i - 1);
}

}  // namespace kvd

namespace kvd {

// NP consecutive TMEM columns of this warp's lane quarter.
template <int NP>
__device__ __forceinline__ void tmem_ld_np(uint32_t taddr, uint32_t (&r)[NP]) {
    if constexpr (NP == 1) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r[0]) : "r"(taddr));
    } else if constexpr (NP == 2) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(taddr));
    } else if constexpr (NP == 4) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(taddr));
    } else if constexpr (NP == 8) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                       "=r"(r[7])
                     : "r"(taddr));
    } else if constexpr (NP == 16) {
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

// Warp-wide float max in one instruction (a NaN operand is ignored).
__device__ __forceinline__ float warp_max(float x) {
    float y;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(y) : "f"(x));
    return y;
}

// Max or sum of K values per thread over the 128 threads of one epilogue
// warpgroup (4 warps), through shared memory and a bounded mbarrier wait.
// Split in two so that independent work can run between posting the warp's
// values and collecting the warpgroup result.
template <int K, bool MAX>
__device__ __forceinline__ void epi_reduce_post(float (&v)[K], float* red, uint64_t* bar, uint32_t use) {
    static_assert(K <= 16, "one 16-float row per warp");
    const int wq = (threadIdx.x >> 5) & 3, lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        if constexpr (MAX) {
            v[k] = warp_max(v[k]);
        } else {
            float x = v[k];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
            v[k] = x;
        }
    }
    float* row = red + (use & 1u) * 128 + wq * 16;  // this warp's row of the exchange buffer
    if (lane == 0) {
#pragma unroll
        for (int k = 0; k + 4 <= K; k += 4) *reinterpret_cast<float4*>(row + k) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
#pragma unroll
        for (int k = K & ~3; k < K; ++k) row[k] = v[k];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
}

template <int K, bool MAX>
__device__ __forceinline__ bool epi_reduce_finish(float (&v)[K], float* red, uint64_t* bar, uint32_t& use) {
    const bool ok = mbar_wait(bar, use & 1u);
    const float* rb = red + (use & 1u) * 128;
    ++use;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        float t[K];
#pragma unroll
        for (int k = 0; k + 4 <= K; k += 4) {
            const float4 q = *reinterpret_cast<const float4*>(rb + w * 16 + k);
            t[k] = q.x; t[k + 1] = q.y; t[k + 2] = q.z; t[k + 3] = q.w;
        }
#pragma unroll
        for (int k = K & ~3; k < K; ++k) t[k] = rb[w * 16 + k];
#pragma unroll
        for (int k = 0; k < K; ++k) v[k] = w == 0 ? t[k] : (MAX ? fmaxf(v[k], t[k]) : v[k] + t[k]);
    }
    return ok;
}

template <int K, bool MAX>
__device__ __forceinline__ bool epi_reduce(float (&v)[K], float* red, uint64_t* bar, uint32_t& use) {
    epi_reduce_post<K, MAX>(v, red, bar, use);
    return epi_reduce_finish<K, MAX>(v, red, bar, use);
}

// Query limbs of item `it` into buffer `buf` for this warpgroup's heads:
// thread r owns dim r. Qi = round(q * qscale * 2^E_h), |Qi| < 2^31, split into
// four signed bytes written into the K-major 128-byte-swizzled B operand
// (row 4h + j). Every thread of the warpgroup ends with the same reduced
// maxima, so each keeps the per-head scales 2^-E_h (sEn) in registers.
template <int G, int NK, int NV, int QM>
__device__ __forceinline__ bool gqa_qlimbs(const GqaParams& p, uint8_t* smem, int it, int buf, uint32_t& use,
                                           float (&sEn)[GqaCfg<G, NK, NV, QM>::HPW]) {
    using C = GqaCfg<G, NK, NV, QM>;
    constexpr int HPW = C::HPW;
    const int wg = threadIdx.x >> 7, r = threadIdx.x & 127, lane = threadIdx.x & 31;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* q_full = bars + C::B_QFULL;
    uint64_t* red_bar = bars + C::B_RED + wg;
    float* red = reinterpret_cast<float*>(smem + C::OFF_RED) + wg * 256;
    const GItem I = gqa_item(p, it);
    const int h0 = wg * HPW;
    const int64_t q0 = I.b * p.q_sb + static_cast<int64_t>(I.hk * G + h0) * p.q_sh + r;
    float qv[HPW], am[HPW];
#pragma unroll
    for (int h = 0; h < HPW; ++h) {
        const float x = load_q(p.Q, q0 + h * p.q_sh, p.flags);
        qv[h] = C::QI8 ? x : x * p.qscale;  // the int8 query is the raw row, quantised like a cache row
        am[h] = fabsf(qv[h]);
    }
    if (!epi_reduce<HPW, true>(am, red, red_bar, use)) return false;
    uint8_t* qb = smem + C::OFF_QB + buf * C::QB_BYTES;
#pragma unroll
    for (int h = 0; h < HPW; ++h) {
        if constexpr (C::QI8) {
            // The cache's quantiser rule (kvd_quant.cuh): scale = max|q| / 127 and
            // code = clamp(rint(q / scale), -127, 127), both IEEE; a zero row gives
            // scale 0 and codes 0. One B row per head: row wg*QPW + h.
            float sq = 0.f, c = 0.f;
            if (am[h] != 0.f) {
                sq = am[h] / 127.0f;
                c = fminf(fmaxf(rintf(qv[h] / sq), -127.0f), 127.0f);
            }
            const int n = wg * C::QPW + h;
            qb[(n >> 3) * 1024 + (n & 7) * 128 + ((((r >> 4) ^ (n & 7)) << 4) | (r & 15))] =
                static_cast<uint8_t>(static_cast<int8_t>(c));
            sEn[h] = sq * p.qscale;
            continue;
        }
        const int E = am[h] > 0.f ? min(126, max(-126, 30 - exp_above(am[h]))) : 0;  // |q| * 2^E < 2^30
        int qi = __float2int_rn(qv[h] * pow2i(E));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int L = static_cast<int>(static_cast<int8_t>(qi & 0xFF));
            qi = (qi - L) >> 8;
            const int n = 4 * (h0 + h) + j;
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

// Fused append, done by the epilogue warps before their first tile: the
// CTA's candidate items (blockIdx.x + j * grid) are tested in parallel, one
// per epilogue thread, and those whose range holds sequence b's new token are
// listed as (b * Hkv + kv head, position) in shared memory (the reduction
// buffer, free at this point); each warp then quantises the K and V rows of
// every EW-th listed item, four at a time with their loads in flight together
// (one float4 per lane, the rule and bits of quantize_row_warp), makes the
// writes visible to the TMA engine and arrives on the append barrier, which
// the producer waits on before the first tile holding a new token.
template <int G, int NK, int NV, int QM>
__device__ __forceinline__ void fused_append_rows(const GqaParams& p, uint8_t* smem) {
    using C = GqaCfg<G, NK, NV, QM>;
    constexpr int ET = 128 * C::NWG;  // epilogue threads
    constexpr int EW = ET / 32;
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
    int* count = reinterpret_cast<int*>(smem + C::OFF_APPENDED);
    int* list = reinterpret_cast<int*>(smem + C::OFF_RED);  // NWG * 256 ints = 2 per epilogue thread
    const int per_cta = (p.n_items - static_cast<int>(blockIdx.x) + p.grid - 1) / p.grid;
    for (int base = 0; base < per_cta; base += ET) {
        if (t == 0) *count = 0;
        named_bar_sync(1, ET);
        if (base + t < per_cta) {
            const int it = static_cast<int>(blockIdx.x) + (base + t) * p.grid;
            const GItem I = gqa_item(p, it);
            const int apos = append_pos(p, I.b);
            if (apos >= I.t_lo && apos < I.t_hi) {
                const int e = atomicAdd(count, 1);
                list[2 * e] = I.b * p.Hkv + I.hk;
                list[2 * e + 1] = apos;
            }
        }
        named_bar_sync(1, ET);
        const int n = *count;
        // up to four rows per round with all their loads in flight together
        for (int e0 = w; e0 < n; e0 += 4 * EW) {
            float4 xk[4], xv[4];
            int64_t crow[4], srow[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int e = e0 + j * EW;
                if (e < n) {
                    const int bh = list[2 * e], apos = list[2 * e + 1];
                    const int b = bh / p.Hkv, hk = bh - b * p.Hkv;
                    const int64_t nrow = b * p.new_sb + hk * p.new_sh + 4 * lane;
                    xk[j] = __ldg(reinterpret_cast<const float4*>(p.k_new + nrow));
                    xv[j] = __ldg(reinterpret_cast<const float4*>(p.v_new + nrow));
                    crow[j] = b * p.kv_sb + hk * p.kv_sh + static_cast<int64_t>(apos) * C::D;
                    srow[j] = b * p.sc_sb + hk * p.sc_sh + apos;
                }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (e0 + j * EW < n) {
                    quantize_row128_regs(xk[j], p.Kw + crow[j], p.ksw + srow[j], lane);
                    quantize_row128_regs(xv[j], p.Vw + crow[j], p.vsw + srow[j], lane);
                }
            }
        }
        named_bar_sync(1, ET);  // the list is rewritten by the next chunk
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(reinterpret_cast<uint64_t*>(smem + C::OFF_BAR) + C::B_APPEND);
}

struct PvSnap {
    int64_t i;
    int it, flags;
};

// PV epilogue of tile A.i for this warpgroup's heads (thread r = output dim r).
template <int G, int NK, int NV, int QM>
__device__ __forceinline__ bool gqa_pv_epi(const GqaParams& p, uint8_t* smem, uint32_t tmem, const PvSnap& A,
                                           const float (&mA)[GqaCfg<G, NK, NV, QM>::HPW],
                                           const int (&FA)[GqaCfg<G, NK, NV, QM>::HPW],
                                           const float (&LA)[GqaCfg<G, NK, NV, QM>::HPW],
                                           float (&o)[GqaCfg<G, NK, NV, QM>::HPW], float (&mpv)[GqaCfg<G, NK, NV, QM>::HPW],
                                           unsigned int tag) {
    using C = GqaCfg<G, NK, NV, QM>;
    constexpr int NP = C::NP, HPW = C::HPW, CPW = C::CPW;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* o_full = bars + C::B_OFULL;
    uint64_t* o_free = bars + C::B_OFREE;
    const int wq = (threadIdx.x >> 5) & 3, wg = threadIdx.x >> 7, lane = threadIdx.x & 31, r = threadIdx.x & 127;
    const int bj = static_cast<int>(A.i & 1);
    if (!mbar_wait(&o_full[bj], static_cast<uint32_t>((A.i >> 1) & 1))) return false;
    tc_fence_after();
    uint32_t orr[CPW];
    tmem_ld_np<CPW>(tmem + (static_cast<uint32_t>(wq * 32) << 16) + 2 * NP + bj * NP + wg * CPW, orr);
    tmem_wait_ld();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&o_free[bj]);
    if (A.flags & 1) {
#pragma unroll
        for (int h = 0; h < HPW; ++h) { o[h] = 0.f; mpv[h] = mA[h]; }
    }
#pragma unroll
    for (int h = 0; h < HPW; ++h) {
        const float f = combine_limbs(orr[4 * h], orr[4 * h + 1], orr[4 * h + 2], orr[4 * h + 3]);
        if (mpv[h] != mA[h]) {  // the running max moved (rare): rescale the accumulated output
            o[h] *= ex2_fast(mpv[h] - mA[h]);
            mpv[h] = mA[h];
        }
        o[h] = fmaf(f, __int_as_float(1065353216 - FA[h] * 8388608), o[h]);
    }
    if (A.flags & 2) {
        const GItem I = gqa_item(p, A.it);
        const bool split_row = p.P > 1 && split_count(p, seq_len_of(p, I.b)) > 1;
        const bool records = split_row || (p.flags & KVD_FLAG_PARTIAL_OUT);
#pragma unroll
        for (int h = 0; h < HPW; ++h) {
            const int hq = I.hk * G + wg * HPW + h;
            const int64_t ro = I.b * p.o_sb + static_cast<int64_t>(hq) * p.o_sh;
            if constexpr (G <= kTagMaxGroup) {
                if (p.tagged) {  // every row of a dense batch, P >= 1 records
                    unsigned long long* rec =
                        p.tagged + ((static_cast<int64_t>(I.b) * p.Hq + hq) * p.P + I.split) * (C::D + 4);
                    if (r == 0) {
                        st_tagged_gpu(rec, mA[h], tag);
                        st_tagged_gpu(rec + 1, LA[h], tag);
                    }
                    st_tagged_gpu(rec + 4 + r, o[h], tag);
                    continue;
                }
            }
            if (!records) {
                store_out(p.out, ro + r, LA[h] > 0.f ? o[h] / LA[h] : 0.f, p.flags);
            } else {
                float* rec = split_row
                    ? p.partials + ((static_cast<int64_t>(I.b) * p.Hq + hq) * p.P + I.split) * (C::D + 4)
                    : static_cast<float*>(p.out) + ro;
                if (r == 0) { rec[0] = mA[h]; rec[1] = LA[h]; }
                rec[4 + r] = o[h];
            }
        }
    }
    return true;
}

// One epilogue warpgroup: scores, online softmax and weight limbs of every
// tile for heads [wg*HPW, (wg+1)*HPW), then the PV epilogue one tile behind.
template <int G, int NK, int NV, int QM>
__device__ __forceinline__ void gqa_epilogue(const GqaParams& p, uint8_t* smem, uint32_t tmem) {
    using C = GqaCfg<G, NK, NV, QM>;
    constexpr int NP = C::NP, HPW = C::HPW, CPW = C::CPW;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* vfull = bars + C::B_VFULL;
    uint64_t* vempty = bars + C::B_VEMPTY;
    uint64_t* s_full = bars + C::B_SFULL;
    uint64_t* s_free = bars + C::B_SFREE;
    uint64_t* w_full = bars + C::B_WFULL;
    const int wq = (threadIdx.x >> 5) & 3, wg = threadIdx.x >> 7, lane = threadIdx.x & 31, r = threadIdx.x & 127;
    uint64_t* red_bar = bars + C::B_RED + wg;
    float* red = reinterpret_cast<float*>(smem + C::OFF_RED) + wg * 256;
    const GMeta* meta = reinterpret_cast<const GMeta*>(smem + C::OFF_META);
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(wq * 32) << 16) + wg * C::QPW;  // this warpgroup's scores
    uint32_t use = 0;

    if (p.k_new) fused_append_rows<G, NK, NV, QM>(p, smem);
    const unsigned int tag = *reinterpret_cast<const unsigned int*>(smem + C::OFF_TAG);  // tagged records

    // Zero this warpgroup's rows of both query-limb buffers (pad rows stay
    // zero), then item 0's limbs (its reduction orders the zeroing first).
    {
        const int rows = C::NQ / C::NWG;
        for (int x = r; x < 2 * rows * 8; x += 128) {
            const int buf = x / (rows * 8), rem = x % (rows * 8);
            const int n = wg * rows + rem / 8, chunk = rem % 8;
            *reinterpret_cast<uint4*>(smem + C::OFF_QB + buf * C::QB_BYTES + (n >> 3) * 1024 + (n & 7) * 128 +
                                      chunk * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    float sEn[HPW];
    if (!gqa_qlimbs<G, NK, NV, QM>(p, smem, next_item(p, blockIdx.x), 0, use, sEn)) return;

    float m[HPW], l[HPW], sE[HPW], o[HPW], mpv[HPW], mA[HPW], LA[HPW];
    int FA[HPW];
#pragma unroll
    for (int h = 0; h < HPW; ++h) { m[h] = -INFINITY; l[h] = 0.f; sE[h] = 1.f; o[h] = 0.f; mpv[h] = -INFINITY;
                                    mA[h] = -INFINITY; LA[h] = 0.f; FA[h] = 0; }
    PvSnap A{-1, 0, 0};
    int64_t i = 0;
    int s = 0;
    uint32_t ph = 0;
    int kq = 0;
    for (int it = next_item(p, blockIdx.x); it < p.n_items; it = next_item(p, it + p.grid), ++kq) {
        const GItem I = gqa_item(p, it);
        for (int tt = 0; tt < I.ntiles; ++tt, ++i) {
            const int bi = static_cast<int>(i & 1);
            // ---- scores of tile i (thread r = token r of the tile)
            if (!mbar_wait(&s_full[bi], static_cast<uint32_t>((i >> 1) & 1))) return;
            tc_fence_after();
            uint32_t sr[C::SW];
            tmem_ld_np<C::SW>(lane_base + bi * NP, sr);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[bi]);
            if (!mbar_wait(&vfull[s], ph)) return;  // metadata and scale windows of tile i
            const GMeta mt = meta[s];
            if (tt == 0) {
#pragma unroll
                for (int h = 0; h < HPW; ++h) { m[h] = -INFINITY; l[h] = 0.f; sE[h] = sEn[h]; }
            }
            const bool valid = r < mt.n;
            const float* ksm = reinterpret_cast<const float*>(smem + C::OFF_SC + s * C::SC_BYTES);
            const float* vsm = ksm + C::SC_FLOATS;
            const float ksv = valid ? ksm[(mt.offs & 0xff) + r] : 0.f;
            const float vsv = valid ? vsm[(mt.offs >> 8) + r] : 0.f;
            __syncwarp();
            if (lane == 0) mbar_arrive(&vempty[s]);
            if (++s == NV) { s = 0; ph ^= 1u; }
            float sc[HPW], rv[HPW + 1];
#pragma unroll
            for (int h = 0; h < HPW; ++h) {
                // int8 query: one exact int32 column (|acc| <= 128*127*127 < 2^24) per head
                float dot;
                if constexpr (C::QI8) dot = __int2float_rn(static_cast<int>(sr[h]));
                else dot = combine_limbs(sr[4 * h], sr[4 * h + 1], sr[4 * h + 2], sr[4 * h + 3]);
                sc[h] = valid ? dot * sE[h] * ksv : -INFINITY;
                rv[h] = sc[h];
            }
            rv[HPW] = vsv;
            // Post this tile's maxima, run the previous tile's PV epilogue
            // (thread r = output dim r) while the other warps catch up, then
            // collect the warpgroup maxima.
            epi_reduce_post<HPW + 1, true>(rv, red, red_bar, use);
            if (A.i >= 0 && !gqa_pv_epi<G, NK, NV, QM>(p, smem, tmem, A, mA, FA, LA, o, mpv, tag)) return;
            if (!epi_reduce_finish<HPW + 1, true>(rv, red, red_bar, use)) return;
            const float vsmax = rv[HPW];
            // ---- online softmax (base 2, lazy max) and the weight limbs
            uint32_t W[CPW / 4];
#pragma unroll
            for (int x = 0; x < CPW / 4; ++x) W[x] = 0u;
            int FB[HPW];
            const int ea = 30 - exp_above(vsmax);
#pragma unroll
            for (int h = 0; h < HPW; ++h) {
                const float tmax = rv[h];  // same in every thread of the warpgroup
                if (tmax > m[h] + 8.f) {
                    l[h] *= ex2_fast(m[h] - tmax);  // 0 while m is still -inf
                    m[h] = tmax;
                }
                const float pr = valid ? ex2_fast(sc[h] - m[h]) : 0.f;
                l[h] += pr;
                // Weight exponent: p <= 2^(tmax - m) <= 2^ceil(tmax - m) and v_scale < 2^exp_above(vsmax),
                // so w * 2^F < 2^30 with F = 30 - ceil(tmax - m) - exp_above(vsmax). A tile without
                // valid tokens (tmax = -inf, NaN difference) gets ceil = -126 and weights 0.
                const int ep = __float2int_ru(fmaxf(tmax - m[h], -126.f));
                const int F = min(126, max(-126, ea - ep));
                FB[h] = F;
                // pr = 0 and v_scale = 0 for invalid tokens, so W = 0 there without a select.
                W[h] = __float2uint_rn(pr * (vsv * __int_as_float(F * 8388608 + 1065353216)));
            }
            uint8_t* wb = smem + C::OFF_WB + bi * C::WB_BYTES;
#pragma unroll
            for (int g = 0; g < CPW / 16; ++g)
                *reinterpret_cast<uint4*>(wb + (wg * (CPW / 16) + g) * 2048 + r * 16) =
                    make_uint4(W[4 * g], W[4 * g + 1], W[4 * g + 2], W[4 * g + 3]);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&w_full[bi]);
            float LB[HPW];
            if (tt == I.ntiles - 1) {
#pragma unroll
                for (int h = 0; h < HPW; ++h) LB[h] = l[h];
                if (!epi_reduce<HPW, false>(LB, red, red_bar, use)) return;
            } else {
#pragma unroll
                for (int h = 0; h < HPW; ++h) LB[h] = 0.f;
            }
            if (tt == 0) {
                const int nxt = next_item(p, it + p.grid);
                if (nxt < p.n_items && !gqa_qlimbs<G, NK, NV, QM>(p, smem, nxt, (kq + 1) & 1, use, sEn)) return;
            }
#pragma unroll
            for (int h = 0; h < HPW; ++h) { mA[h] = m[h]; FA[h] = FB[h]; LA[h] = LB[h]; }
            A.i = i;
            A.it = it;
            A.flags = mt.flags;
        }
    }
    if (A.i >= 0) gqa_pv_epi<G, NK, NV, QM>(p, smem, tmem, A, mA, FA, LA, o, mpv, tag);
}

// Fused append, end of a CTA: once every thread of the CTA is past its last
// length read, count the CTA; the last CTA of the grid writes the new lengths
// (seq_lens[b] + 1, or KVD_STATUS_CACHE_FULL when the cache was full).
__device__ __forceinline__ void fused_append_finish(const GqaParams& p) {
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(p.done_ctas, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last) {
        __threadfence();
        for (int b = threadIdx.x; b < p.B; b += blockDim.x) {
            const int len = max(0, p.lens_rw[b]);
            if (len < p.S) p.lens_rw[b] = len + 1;
            else record_status(KVD_STATUS_CACHE_FULL);
        }
    }
}

template <int G, int NK, int NV, int QM, int MINB>
__global__ void __launch_bounds__(GqaCfg<G, NK, NV, QM>::THREADS, MINB) gqa_tc_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, const GqaParams p) {
    using C = GqaCfg<G, NK, NV, QM>;
    constexpr int EW = 4 * C::NWG;  // epilogue warps; then the producer warp, then the MMA warp
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    // A follow-up kernel launched as a programmatic dependent (the split combine,
    // the multi-GPU record exchange) may be scheduled onto SMs as this grid's
    // CTAs retire; it waits for this grid's completion before reading its
    // output. With tagged records the dependent (the exchange) reads them while
    // this grid runs and moves the tag word on when it ends: every CTA reads
    // the tag first and allows the dependents to launch only after that. (A
    // dense batch: the item loop below reads no global memory before that.)
    bool tagged = false;
    if constexpr (G <= kTagMaxGroup) tagged = p.tagged != nullptr;
    if (!tagged) {
        // launched as a programmatic dependent of the kernel before it: wait for
        // it (and its memory) before the first global access
        grid_dependency_wait();
        allow_dependents();
    }
    if (next_item(p, blockIdx.x) >= p.n_items) {  // no (non-empty) item for this CTA (exiting allows the dependents)
        if (p.k_new) fused_append_finish(p);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* done = bars + C::B_DONE;
    uint64_t* drain = bars + C::B_DRAIN;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NK; ++s) {
            mbar_init(&bars[C::B_KFULL + s], 1);       // producer arrive + transaction bytes
            mbar_init(&bars[C::B_KEMPTY + s], 1);      // QK commit
        }
        for (int s = 0; s < NV; ++s) {
            mbar_init(&bars[C::B_VFULL + s], 1);       // producer arrive + transaction bytes
            mbar_init(&bars[C::B_VEMPTY + s], 1 + EW); // PV commit + every epilogue warp
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars[C::B_SFULL + b], 1);
            mbar_init(&bars[C::B_SFREE + b], EW);
            mbar_init(&bars[C::B_WFULL + b], EW);
            mbar_init(&bars[C::B_OFULL + b], 1);
            mbar_init(&bars[C::B_OFREE + b], EW);
            mbar_init(&bars[C::B_QFULL + b], EW);
        }
        for (int wg = 0; wg < C::NWG; ++wg) mbar_init(&bars[C::B_RED + wg], 4);
        mbar_init(done, EW);
        mbar_init(drain, 1);
        *reinterpret_cast<int*>(smem + C::OFF_APPENDED) = 0;
        mbar_init(&bars[C::B_APPEND], EW);  // every epilogue warp, after its share of the fused append
        fence_mbar_init();
    }
    if (warp == EW + 1) tmem_alloc(reinterpret_cast<uint32_t*>(smem + C::OFF_TMEM), C::TMEM_COLS);
    __syncthreads();
    if (tagged) {
        // launched as a programmatic dependent of the previous exchange: wait for it (and its
        // memory), read the tag it left, then let this call's exchange launch
        grid_dependency_wait();
        if (threadIdx.x == 0) {
            unsigned int tag;
            asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(tag) : "l"(p.tag_src) : "memory");
            *reinterpret_cast<unsigned int*>(smem + C::OFF_TAG) = tag + 1;
        }
        __syncthreads();
        allow_dependents();  // every CTA of this grid has read the tag
    }
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + C::OFF_TMEM);
    if (warp == EW) {
        if (p.table) gqa_producer_paged<G, NK, NV, QM>(&kmap, &vmap, p, smem);
        else if (lane < 2) gqa_producer<G, NK, NV, QM>(&kmap, &vmap, p, smem, lane == 1);
    } else if (warp == EW + 1) {
        if (lane == 0) {
            gqa_mma<G, NK, NV, QM>(p, smem, tmem);
            mma_commit(drain);  // arrives once every MMA issued above has completed
            mbar_wait(drain, 0);
            mbar_wait(done, 0);  // epilogue warps have finished reading TMEM
        }
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    } else {
        gqa_epilogue<G, NK, NV, QM>(p, smem, tmem);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(done);
    }
    if (p.k_new) fused_append_finish(p);
}

}  // namespace kvd

// Ragged batches: sequences sorted by length, longest first (one block,
// bitonic sort of (length, index) keys; B <= 4096).
__global__ void __launch_bounds__(1024) seq_order_kernel(const int32_t* seq_lens, int B, int S, int32_t* order,
                                                        int len_add, unsigned int* done_ctas) {
    __shared__ unsigned long long keys[4096];
    if (threadIdx.x == 0 && done_ctas) *done_ctas = 0u;
    int n2 = 1;
    while (n2 < B) n2 <<= 1;
    for (int i = threadIdx.x; i < n2; i += blockDim.x) {
        unsigned long long k = ~0ull;
        if (i < B) {
            const int len = min(max(0, seq_lens[i]) + len_add, S);
            k = (static_cast<unsigned long long>(0x7FFFFFFF - len) << 32) | static_cast<unsigned>(i);
        }
        keys[i] = k;
    }
    __syncthreads();
    for (int k = 2; k <= n2; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n2; i += blockDim.x) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const bool asc = (i & k) == 0;
                    const unsigned long long a = keys[i], b = keys[ixj];
                    if ((a > b) == asc) { keys[i] = b; keys[ixj] = a; }
                }
            }
            __syncthreads();
        }
    }
    for (int i = threadIdx.x; i < B; i += blockDim.x) order[i] = static_cast<int32_t>(keys[i] & 0xffffffffu);
}

// Ragged batches: merge the split records of rows whose sequence had more
// than one split (single-split rows were written by the decode kernel).
__global__ void __launch_bounds__(128) gqa_ragged_combine_kernel(const float* partials, const int32_t* seq_lens,
                                                                 int Hq, int P, int span, int S, int D, void* out,
                                                                 int64_t o_sb, int64_t o_sh, uint32_t flags) {
    const int64_t r = blockIdx.x;
    const int b = static_cast<int>(r / Hq), hq = static_cast<int>(r - static_cast<int64_t>(b) * Hq);
    const int len = min(max(0, seq_lens[b]), S);
    const int ns = len > 0 ? (len + span - 1) / span : 1;
    if (ns <= 1) return;
    const float* first = partials + r * P * static_cast<int64_t>(D + 4);
    float M = -INFINITY;
    for (int k = 0; k < ns; ++k) M = fmaxf(M, first[k * (D + 4)]);
    const int64_t ro = b * o_sb + static_cast<int64_t>(hq) * o_sh;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float O = 0.f, L = 0.f;
        if (M != -INFINITY) {
            for (int k = 0; k < ns; ++k) {
                const float* rec = first + k * (D + 4);
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
            kvd::store_out(out, ro + d, L > 0.f ? O / L : 0.f, flags);
        }
    }
}

// ------------------------------------------------------------------ host side
namespace kvd {
namespace {

constexpr int kGqaNK = KVD_GQA_NK;
constexpr int kGqaNV = KVD_GQA_NV;
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
    return make_kv_map_rows(m, base, B, Hkv, cap, kv_sb, kv_sh, 128);
}

}  // namespace

// As make_kv_map with a box of `rows` tokens (<= 256).
bool make_kv_map_rows(void* map, const int8_t* base, int B, int Hkv, int cap, int64_t kv_sb, int64_t kv_sh,
                      int rows) {
    CUtensorMap* m = static_cast<CUtensorMap*>(map);
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    const int64_t sh = kv_sh > 0 ? kv_sh : static_cast<int64_t>(cap) * 128;
    const int64_t sb = kv_sb > 0 ? kv_sb : sh * Hkv;
    cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(cap), static_cast<cuuint64_t>(Hkv), static_cast<cuuint64_t>(B)};
    cuuint64_t strides[3] = {128, static_cast<cuuint64_t>(sh), static_cast<cuuint64_t>(sb)};
    cuuint32_t box[4] = {128, static_cast<cuuint32_t>(rows), 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

namespace {

// 4-D view {D bytes, block_size tokens, kv heads, blocks} of a paged K or V
// pool, box of 128 bytes x min(block_size, 128) tokens, 128-byte swizzle. The
// boxes of one tile land at multiples of 1024 bytes (block_size >= 8), so the
// tile has the same swizzled layout as a dense 128-token box.
bool make_paged_map(CUtensorMap* m, const int8_t* base, int Hkv, const PagedView& pv, int64_t kv_sh) {
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(pv.block_size), static_cast<cuuint64_t>(Hkv),
                          static_cast<cuuint64_t>(pv.num_blocks)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(pv.kv_st), static_cast<cuuint64_t>(kv_sh),
                             static_cast<cuuint64_t>(pv.kv_sblk)};
    cuuint32_t box[4] = {128, static_cast<cuuint32_t>(pv.block_size < 128 ? pv.block_size : 128), 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Splits per (batch, kv head) item. Items are dealt round-robin to the
// persistent CTAs, so pick the split count P that minimises
// rounds(P) * (tiles per item + 1), the +1 standing for the per-item cost
// (query limbs, output write); P > 1 also costs a record-combine launch.
int gqa_split_count(const kvd_decode_desc& d) {
    const int64_t units = static_cast<int64_t>(d.batch) * d.num_kv_heads;
    const int64_t grid = static_cast<int64_t>(device_sm_count()) * kGqaCtas;
    const int S = d.max_seq_len > 0 ? d.max_seq_len : 1;
    const int max_tiles = (S + 127) / 128;
    int best_p = 1;
    double best = -1.0;
    for (int P = 1; P <= max_tiles && P <= 256; ++P) {
        const int span = ((((S + P - 1) / P) + 127) / 128) * 128;
        const int pe = (S + span - 1) / span;
        if (pe != P) continue;
        const int64_t items = units * P;
        const double rounds = static_cast<double>((items + grid - 1) / grid);
        const double cost = rounds * (span / 128 + 1) + (P > 1 ? 2.0 : 0.0);
        if (best < 0 || cost < best) { best = cost; best_p = P; }
        if (items >= 64 * grid) break;
    }
    return best_p;
}

template <int G, int QM>
cudaError_t launch_gqa_g(const CUtensorMap& km, const CUtensorMap& vm, const GqaParams& p, cudaStream_t st) {
    using C = GqaCfg<G, kGqaNK, kGqaNV, QM>;
    auto kern = gqa_tc_kernel<G, kGqaNK, kGqaNV, QM, kGqaCtas>;
    static PerDeviceOnce once;
    const cudaError_t e = once.run([kern] {
        return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    });
    if (e != cudaSuccess) return e;
    {  // a programmatic dependent of the kernel before it (see gqa_tc_kernel)
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(static_cast<unsigned>(p.grid), 1, 1);
        cfg.blockDim = dim3(C::THREADS, 1, 1);
        cfg.dynamicSmemBytes = C::SMEM_BYTES;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, kern, km, vm, p);
    }
}

}  // namespace

bool gqa_path_ok(const kvd_decode_desc& d) {
    const int G = d.num_q_heads / d.num_kv_heads;
    if (d.head_dim != 128 || d.max_seq_len < 1) return false;
    if (G != 1 && G != 2 && G != 4 && G != 8 && G != 16) return false;
    return tensor_map_encoder() != nullptr;
}

namespace {
// Work plan of one launch: token span per item, splits per sequence, and the
// workspace it needs (ragged order array, split records).
struct GqaPlan {
    int P, span;
    size_t order_bytes, rec_bytes;
};

GqaPlan plan_gqa(const kvd_decode_desc& d, size_t ws_limit) {
    GqaPlan g{};
    const int S = d.max_seq_len > 0 ? d.max_seq_len : 1;
    const int64_t units = static_cast<int64_t>(d.batch) * d.num_kv_heads;
    const int64_t grid = static_cast<int64_t>(device_sm_count()) * kGqaCtas;
    const int s_tiles = (S + 127) / 128;
    // order array + one counter word (fused append)
    g.order_bytes = (d.seq_lens && d.batch <= 4096) ? ((static_cast<size_t>(d.batch) * 4 + 4 + 255) & ~size_t(255)) : 0;
    int span_tiles;
    if (d.seq_lens) {
        // Ragged: split long sequences into items of at most 16 tiles (fewer if
        // that leaves too few items to balance), longest items dealt first.
        span_tiles = 16;
        while (span_tiles > 1 && units * ((s_tiles + span_tiles - 1) / span_tiles) < 4 * grid) span_tiles /= 2;
        if (span_tiles > s_tiles) span_tiles = s_tiles;
    } else {
        const int P0 = gqa_split_count(d);
        span_tiles = (s_tiles + P0 - 1) / P0;
    }
    g.span = 128 * span_tiles;
    g.P = (S + g.span - 1) / g.span;
    g.rec_bytes = g.P > 1 ? static_cast<size_t>(d.batch) * d.num_q_heads * g.P * (d.head_dim + 4) * sizeof(float) : 0;
    if (g.order_bytes + g.rec_bytes > ws_limit) {  // no room for split records: whole sequences per item
        g.span = 128 * s_tiles;
        g.P = 1;
        g.rec_bytes = 0;
        if (g.order_bytes > ws_limit) g.order_bytes = 0;
    }
    return g;
}
}  // namespace

int gqa_tagged_splits(const kvd_decode_desc& d) {
    if (!gqa_path_ok(d) || d.seq_lens || d.num_q_heads / d.num_kv_heads > kTagMaxGroup) return 0;
    return plan_gqa(d, ~size_t(0)).P;
}

bool gqa_fused_append_ok(const kvd_decode_desc& d, size_t ws_bytes) {
    return gqa_path_ok(d) && d.seq_lens && plan_gqa(d, ws_bytes).order_bytes > 0;
}

size_t gqa_workspace_size(const kvd_decode_desc& d) {
    const GqaPlan g = plan_gqa(d, ~size_t(0));
    return g.order_bytes + g.rec_bytes;
}

cudaError_t launch_gqa_tc(const kvd_decode_desc& d, const void* Q, const int8_t* K, const int8_t* V,
                          const float* ks, const float* vs, void* out, void* ws, size_t ws_bytes,
                          cudaStream_t st, int* launches, const PagedView* pv, const AppendView* av,
                          SplitRecords* keep_splits) {
    const int G = d.num_q_heads / d.num_kv_heads;
    const GqaPlan g = plan_gqa(d, ws ? ws_bytes : 0);
    const int S = d.max_seq_len;
    if (av && (pv || !g.order_bytes || !d.seq_lens)) return cudaErrorNotSupported;
    CUtensorMap km, vm;
    if (pv) {
        if (!make_paged_map(&km, K, d.num_kv_heads, *pv, d.kv_stride_h) ||
            !make_paged_map(&vm, V, d.num_kv_heads, *pv, d.kv_stride_h))
            return cudaErrorInvalidValue;
    } else if (!make_kv_map(&km, K, d.batch, d.num_kv_heads, S, d.kv_stride_b, d.kv_stride_h) ||
               !make_kv_map(&vm, V, d.batch, d.num_kv_heads, S, d.kv_stride_b, d.kv_stride_h)) {
        return cudaErrorInvalidValue;
    }
    GqaParams p{};
    if (pv) {
        p.table = pv->table;
        p.bt_stride = pv->bt_stride;
        p.sc_sblk = pv->sc_sblk;
        p.nblk = pv->num_blocks;
        int lbs = 0;
        while ((1 << lbs) < pv->block_size) ++lbs;
        p.lbs = lbs;
    }
    p.Q = Q; p.ks = ks; p.vs = vs; p.out = out;
    p.order = g.order_bytes ? static_cast<const int32_t*>(ws) : nullptr;
    p.partials = g.rec_bytes ? reinterpret_cast<float*>(static_cast<char*>(ws) + g.order_bytes) : nullptr;
    p.seq_lens = d.seq_lens;
    p.B = d.batch; p.Hq = d.num_q_heads; p.Hkv = d.num_kv_heads; p.S = S; p.P = g.P; p.span = g.span;
    p.n_items = d.batch * d.num_kv_heads * g.P;
    const int64_t grid_max = static_cast<int64_t>(device_sm_count()) * kGqaCtas;
    p.grid = static_cast<int>(grid_max < p.n_items ? grid_max : p.n_items);
    p.sc_sb = d.sc_stride_b; p.sc_sh = d.sc_stride_h;
    p.q_sb = d.q_stride_b; p.q_sh = d.q_stride_h;
    p.o_sb = d.o_stride_b; p.o_sh = d.o_stride_h;
    const float scale = d.softmax_scale > 0.f ? d.softmax_scale : 1.0f / sqrtf(static_cast<float>(d.head_dim));
    p.qscale = scale * 1.4426950408889634f;
    p.flags = d.flags;
    // Tagged records: dense batches only, where every item is non-empty
    // (max_seq_len >= 1) and every row gets exactly P records.
    if (keep_splits && keep_splits->tagged && keep_splits->tagged_P == g.P && !d.seq_lens && !pv && !av &&
        G <= kTagMaxGroup) {
        p.tagged = keep_splits->tagged;
        p.tag_src = keep_splits->tag_src;
    }
    unsigned int* done_ctas = nullptr;
    if (av) {
        p.k_new = av->k_new; p.v_new = av->v_new; p.new_sb = av->new_sb; p.new_sh = av->new_sh;
        p.kv_sh = d.kv_stride_h > 0 ? d.kv_stride_h : static_cast<int64_t>(S) * 128;
        p.kv_sb = d.kv_stride_b > 0 ? d.kv_stride_b : p.kv_sh * d.num_kv_heads;
        p.Kw = const_cast<int8_t*>(K); p.Vw = const_cast<int8_t*>(V);
        p.ksw = const_cast<float*>(ks); p.vsw = const_cast<float*>(vs);
        p.lens_rw = av->seq_lens;
        done_ctas = reinterpret_cast<unsigned int*>(static_cast<char*>(ws) + static_cast<size_t>(d.batch) * 4);
        p.done_ctas = done_ctas;
        p.len_add = 1;
    }
    cudaError_t e;
    if (p.order) {
        seq_order_kernel<<<1, 1024, 0, st>>>(d.seq_lens, d.batch, S, static_cast<int32_t*>(ws), p.len_add,
                                             done_ctas);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        ++*launches;
    }
    const bool qi8 = (d.flags & KVD_FLAG_QK_INT8) != 0;
    switch (G) {
        case 1: e = qi8 ? launch_gqa_g<1, 1>(km, vm, p, st) : launch_gqa_g<1, 0>(km, vm, p, st); break;
        case 2: e = qi8 ? launch_gqa_g<2, 1>(km, vm, p, st) : launch_gqa_g<2, 0>(km, vm, p, st); break;
        case 4: e = qi8 ? launch_gqa_g<4, 1>(km, vm, p, st) : launch_gqa_g<4, 0>(km, vm, p, st); break;
        case 8: e = qi8 ? launch_gqa_g<8, 1>(km, vm, p, st) : launch_gqa_g<8, 0>(km, vm, p, st); break;
        case 16: e = qi8 ? launch_gqa_g<16, 1>(km, vm, p, st) : launch_gqa_g<16, 0>(km, vm, p, st); break;
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    ++*launches;
    if (keep_splits) {  // the caller merges the split records itself (dense batches only)
        keep_splits->partials = g.P > 1 && !d.seq_lens ? p.partials : nullptr;
        keep_splits->P = g.P > 1 && !d.seq_lens ? g.P : 1;
        keep_splits->tagged_used = p.tagged != nullptr;
        if (g.P == 1 || !d.seq_lens) return cudaSuccess;
    }
    if (g.P > 1) {
        const int64_t rows = static_cast<int64_t>(d.batch) * d.num_q_heads;
        if (d.seq_lens) {
            gqa_ragged_combine_kernel<<<static_cast<unsigned>(rows), 128, 0, st>>>(
                p.partials, d.seq_lens, d.num_q_heads, g.P, g.span, S, d.head_dim, out, d.o_stride_b, d.o_stride_h,
                d.flags);
            e = cudaGetLastError();
            if (e == cudaSuccess) ++*launches;
        } else {
            const int64_t rs = d.head_dim + 4;
            e = launch_combine_records(p.partials, g.P, rs, rs * g.P, rows, d.num_q_heads, d.head_dim, out,
                                       d.o_stride_b, d.o_stride_h, d.flags, st, launches);
        }
    }
    return e;
}

}  // namespace kvd
