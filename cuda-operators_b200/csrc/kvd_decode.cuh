// kvd_decode.cuh -- launch-side declarations shared by the decode translation
// units (split-KV flash decode on CUDA cores, combine, generic fallback).
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <cuda_runtime.h>

#include "kvdecode.h"

namespace kvd {

// Device ordinals the library keeps per-device state for (kernel attributes,
// cached SM counts); calls on higher ordinals return cudaErrorInvalidDevice.
constexpr int kMaxDevices = 64;

// Unique id of the calling thread's current CUDA context (ids are never reused
// within a process), or 0 when none is current yet.
unsigned long long current_context_id();

// Runs a set-up step (a kernel attribute) once per device and CUDA context,
// for the device current on the calling thread: a new context of the device
// (after cudaDeviceReset) runs it again. Thread-safe: concurrent first calls
// wait for one another; a failed step is retried by the next call.
class PerDeviceOnce {
public:
    template <class F>
    cudaError_t run(F&& fn) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
        const unsigned long long ctx = current_context_id();
        if (ctx != 0 && done_[dev].load(std::memory_order_acquire) == ctx) return cudaSuccess;
        std::lock_guard<std::mutex> lock(mu_);
        if (ctx != 0 && done_[dev].load(std::memory_order_relaxed) == ctx) return cudaSuccess;
        e = fn();  // binds the device's primary context if none was current
        if (e == cudaSuccess) done_[dev].store(current_context_id(), std::memory_order_release);
        return e;
    }

private:
    std::mutex mu_;
    std::atomic<unsigned long long> done_[kMaxDevices] = {};  // context id the step last ran in
};

// One-launch small-problem decode (kvd_small.cu): at most kSmallMaxCluster
// CTAs (a thread-block cluster) per head, kSmallMaxSpan tokens per CTA.
constexpr int kSmallMaxCluster = 8;
constexpr int kSmallMaxSpan = 256;

// Everything a decode kernel needs, passed by value.
struct DecodeParams {
    const float* Q;
    const int8_t* K;
    const int8_t* V;
    const float* ks;
    const float* vs;
    float* out;
    int B, Hq, Hkv, D, group;
    int S;                       // dense length (seq_lens == nullptr)
    const int32_t* seq_lens;     // device [B] or nullptr
    const int32_t* tile_prefix;  // ragged: device [B+1] cumulative tiles (x Hq); else nullptr
    int64_t kv_sb, kv_sh, sc_sb, sc_sh, q_sb, q_sh, o_sb, o_sh;
    float qscale;                // softmax_scale * log2(e)
    uint32_t flags;
    int64_t n_tiles;             // dense: total tiles; ragged: read from tile_prefix[B]
    int tiles_per_head;          // dense only
    int grid;                    // persistent CTAs
    float* partials;             // 2*grid records of D+4 floats (nullptr when grid == 1)
};

// Shape of the CUDA-core split-KV kernel per head dimension: consumer warps
// per CTA, ring stages, resident CTAs per SM. A lane group of D/16 lanes owns
// 4 tokens of a tile, so a tile holds CW * (32 / (D/16)) * 4 tokens.
#ifndef KVD_SK128_CW
#define KVD_SK128_CW 8
#endif
#ifndef KVD_SK128_NS
#define KVD_SK128_NS 3
#endif
#ifndef KVD_SK128_CTAS
#define KVD_SK128_CTAS 2
#endif
#ifndef KVD_SK64_CW
#define KVD_SK64_CW 4
#endif
#ifndef KVD_SK64_NS
#define KVD_SK64_NS 3
#endif
#ifndef KVD_SK64_CTAS
#define KVD_SK64_CTAS 2
#endif

// Element-type flags of Q and of the output rows.
constexpr uint32_t kDtypeFlags = KVD_FLAG_Q_BF16 | KVD_FLAG_Q_F16 | KVD_FLAG_OUT_BF16 | KVD_FLAG_OUT_F16;

// Route MHA with head_dim 128 to the tensor-core kernel: 1 = dense batches,
// 2 = dense and ragged batches, 0 = never (CUDA-core split-KV kernel).
#ifndef KVD_MHA_TENSOR_CORES
#define KVD_MHA_TENSOR_CORES 2
#endif

// K ring stages, V ring stages and resident CTAs per SM of the tcgen05 GQA kernel.
// A K slot is free again as soon as QK has read it, a V slot only after PV and
// the softmax (which reads the slot's scales) are done, so the V ring is the
// deeper one: 2 + 3 gave config 5 -4.5 % and config 4 -3 % against 3 + 2.
#ifndef KVD_GQA_NK
#define KVD_GQA_NK 2
#endif
#ifndef KVD_GQA_NV
#define KVD_GQA_NV 3
#endif
#ifndef KVD_GQA_CTAS
#define KVD_GQA_CTAS 2
#endif

constexpr int sk_consumer_warps(int D) { return D == 64 ? KVD_SK64_CW : KVD_SK128_CW; }
constexpr int sk_ctas_per_sm(int D) { return D == 64 ? KVD_SK64_CTAS : KVD_SK128_CTAS; }
// Tokens per tile of the CUDA-core kernel for a head dimension.
constexpr int tile_tokens(int D) { return sk_consumer_warps(D) * (32 / (D / 16)) * 4; }

// Paged-cache addressing handed to the launchers next to a descriptor whose
// max_seq_len is the table's capacity (max_blocks_per_seq * block_size).
// Token t of sequence b, kv head h: block table[b*bt_stride + t/block_size],
// codes at blk*kv_sblk + h*kv_sh + (t%block_size)*kv_st, scales at
// blk*sc_sblk + h*sc_sh + t%block_size.
struct PagedView {
    const int32_t* table;
    int64_t bt_stride;
    int block_size, num_blocks;
    int64_t kv_sblk, kv_st, sc_sblk;
};

// Fused quantise-on-append for launch_gqa_tc: the new token's fp32 K/V rows
// and the lengths, which the launch reads as seq_lens[b] + 1 and then updates.
struct AppendView {
    const float* k_new;
    const float* v_new;
    int64_t new_sb, new_sh;
    int32_t* seq_lens;
};

bool fast_path_ok(const kvd_decode_desc& d, const void* Q, const int8_t* K, const int8_t* V);

// Launch count of the current host thread's last entry-point call (kvd_last_launch_count).
int* launch_counter();

// Per-device cached properties.
int device_sm_count();

// Launchers (return the launch status; add their launch count to *launches).
cudaError_t launch_plan(const int32_t* seq_lens, int B, int Hq, int tok, int cap, int32_t* prefix,
                        cudaStream_t st, int* launches);
cudaError_t launch_splitkv(const DecodeParams& p, cudaStream_t st, int* launches);
int small_cluster_size(const kvd_decode_desc& d);
cudaError_t launch_small(const kvd_decode_desc& d, const float* Q, const int8_t* K, const int8_t* V,
                         const float* ks, const float* vs, float* out, cudaStream_t st, int* launches);
cudaError_t launch_generic(const kvd_decode_desc& d, const void* Q, const int8_t* K,
                           const int8_t* V, const float* ks, const float* vs, void* out,
                           void* ws, size_t ws_bytes, cudaStream_t st, int* launches,
                           const PagedView* pv = nullptr);
size_t generic_workspace_size(const kvd_decode_desc& d);
cudaError_t launch_combine_records(const float* base, int nparts, int64_t part_stride, int64_t rec_stride,
                                   int64_t rows, int rows_per_b, int D, void* out, int64_t o_sb, int64_t o_sh,
                                   uint32_t flags, cudaStream_t st, int* launches);
bool gqa_path_ok(const kvd_decode_desc& d);
size_t gqa_workspace_size(const kvd_decode_desc& d);
// Split records a dense tensor-core decode left in its workspace when the
// caller asked it to skip the combine: row r's P records of D+4 floats start
// at partials + r*P*(D+4). P == 1: the rows were written to `out` directly.
struct SplitRecords {
    const float* partials;
    int P;
    // in: room for tagged records of tagged_P splits per row (gqa_tagged_splits)
    // and the device word w: the records are tagged *w + 1; tagged == nullptr: none
    unsigned long long* tagged;
    int tagged_P;
    const unsigned int* tag_src;
    bool tagged_used;  // out: the decode wrote tagged records
};
// Split count per row of the tensor-core decode when it may write tagged
// records for `d` (dense batch, group <= 4, head_dim 128), else 0.
int gqa_tagged_splits(const kvd_decode_desc& d);
cudaError_t launch_gqa_tc(const kvd_decode_desc& d, const void* Q, const int8_t* K, const int8_t* V,
                          const float* ks, const float* vs, void* out, void* ws, size_t ws_bytes,
                          cudaStream_t st, int* launches, const PagedView* pv = nullptr,
                          const AppendView* av = nullptr, SplitRecords* keep_splits = nullptr);
bool gqa_fused_append_ok(const kvd_decode_desc& d, size_t ws_bytes);
// 4-D TMA view {D bytes, tokens, kv heads, batch} of a dense K or V cache with
// a box of 128 bytes x `rows` tokens, 128-byte swizzle (CUtensorMap* as void*).
bool make_kv_map_rows(void* map, const int8_t* base, int B, int Hkv, int cap, int64_t kv_sb, int64_t kv_sh,
                      int rows);
bool prefill_tc_ok(const kvd_prefill_desc& d, const int8_t* K, const int8_t* V, const float* ks, const float* vs);
cudaError_t launch_prefill_tc(const kvd_prefill_desc& d, const void* Q, const int8_t* K, const int8_t* V,
                              const float* ks, const float* vs, void* out, cudaStream_t st, int* launches);
cudaError_t launch_generic_prefill(const kvd_prefill_desc& d, const void* Q, const int8_t* K, const int8_t* V,
                                   const float* ks, const float* vs, void* out, cudaStream_t st, int* launches);
cudaError_t launch_paged_append(const kvd_paged_desc& d, const float* k_new, const float* v_new, int64_t new_sb,
                                int64_t new_sh, int8_t* K, int8_t* V, float* ks, float* vs, int32_t* seq_lens,
                                cudaStream_t st);
cudaError_t launch_combine_parts(const float* parts, int num_parts, int64_t part_stride, int num_heads,
                                 int head_dim, void* out, int64_t out_stride, uint32_t flags,
                                 cudaStream_t st, int* launches);

}  // namespace kvd
