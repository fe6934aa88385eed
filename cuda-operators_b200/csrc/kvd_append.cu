// kvd_append.cu -- quantise-on-append and row quantisation kernels.
//
// The reference only consumes INT8 codes and scales (kv_cache/new_kvint8.cu:83-84:
// "No ... quantization"); the quantiser here follows the symmetric per-token
// rule of the north-star spec and is bit-exact with the host function
// kvo_quantize_row of the test oracle:
//   amax  = max_d |x_d|                         (fp32, exact)
//   scale = amax / 127                          (IEEE fp32 division, round to nearest even)
//   code  = clamp(rint(x_d / scale), -127, 127)  (IEEE division, ties to even)
//   amax == 0 -> scale = 0, codes = 0.
// NaN inputs follow fmaxf/fminf semantics (a NaN operand is ignored), which
// the host function mirrors. This file must not be built with fast-math.
#include "kvd_common.cuh"
#include "kvd_decode.cuh"
#include "kvd_quant.cuh"

namespace kvd {

// One block per sequence b: every (kv head, K|V) row of the new token is
// quantised into slot seq_lens[b]; then the length is bumped once.
__global__ void __launch_bounds__(256) append_kernel(kvd_append_desc d, const float* k_new,
                                                     const float* v_new, int8_t* K, int8_t* V,
                                                     float* ks, float* vs, int32_t* seq_lens) {
    const int b = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int len = max(0, seq_lens[b]);
    const bool full = len >= d.capacity;
    if (!full) {
        for (int r = warp; r < 2 * d.num_kv_heads; r += blockDim.x >> 5) {
            const int h = r >> 1;
            const bool is_v = (r & 1) != 0;
            const float* x = (is_v ? v_new : k_new) + b * d.new_stride_b + static_cast<int64_t>(h) * d.new_stride_h;
            int8_t* cache = (is_v ? V : K) + b * d.kv_stride_b + static_cast<int64_t>(h) * d.kv_stride_h +
                            static_cast<int64_t>(len) * d.head_dim;
            float* sc = (is_v ? vs : ks) + b * d.sc_stride_b + static_cast<int64_t>(h) * d.sc_stride_h + len;
            quantize_row_warp(x, d.head_dim, cache, sc, lane);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (full) record_status(KVD_STATUS_CACHE_FULL);
        else seq_lens[b] = len + 1;
    }
}

// Paged cache: as append_kernel, with slot seq_lens[b] in the block the
// table names for it.
__global__ void __launch_bounds__(256) paged_append_kernel(kvd_paged_desc d, const float* k_new,
                                                           const float* v_new, int64_t new_sb, int64_t new_sh,
                                                           int8_t* K, int8_t* V, float* ks, float* vs,
                                                           int32_t* seq_lens) {
    const int b = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int len = max(0, seq_lens[b]);
    const int64_t cap = static_cast<int64_t>(d.max_blocks_per_seq) * d.block_size;
    const bool full = len >= cap;
    int blk = -1;
    if (!full) blk = d.block_table[b * d.block_table_stride + len / d.block_size];
    const bool bad = !full && (blk < 0 || blk >= d.num_blocks);
    if (!full && !bad) {
        const int off = len % d.block_size;
        for (int r = warp; r < 2 * d.num_kv_heads; r += blockDim.x >> 5) {
            const int h = r >> 1;
            const bool is_v = (r & 1) != 0;
            const float* x = (is_v ? v_new : k_new) + b * new_sb + static_cast<int64_t>(h) * new_sh;
            int8_t* cache = (is_v ? V : K) + blk * d.kv_stride_block + static_cast<int64_t>(h) * d.kv_stride_h +
                            static_cast<int64_t>(off) * d.kv_stride_t;
            float* sc = (is_v ? vs : ks) + blk * d.sc_stride_block + static_cast<int64_t>(h) * d.sc_stride_h + off;
            quantize_row_warp(x, d.head_dim, cache, sc, lane);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (full) record_status(KVD_STATUS_CACHE_FULL);
        else if (bad) record_status(KVD_STATUS_BAD_BLOCK);
        else seq_lens[b] = len + 1;
    }
}

__global__ void __launch_bounds__(256) quantize_rows_kernel(const float* x, int64_t rows, int dim,
                                                            int64_t x_stride, int8_t* codes,
                                                            int64_t code_stride, float* scales) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
         r += warps)
        quantize_row_warp(x + r * x_stride, dim, codes + r * code_stride, scales + r, lane);
}

cudaError_t launch_append(const kvd_append_desc& d, const float* k_new, const float* v_new, int8_t* K,
                          int8_t* V, float* ks, float* vs, int32_t* seq_lens, cudaStream_t st) {
    append_kernel<<<d.batch, 256, 0, st>>>(d, k_new, v_new, K, V, ks, vs, seq_lens);
    return cudaGetLastError();
}

cudaError_t launch_paged_append(const kvd_paged_desc& d, const float* k_new, const float* v_new, int64_t new_sb,
                                int64_t new_sh, int8_t* K, int8_t* V, float* ks, float* vs, int32_t* seq_lens,
                                cudaStream_t st) {
    paged_append_kernel<<<d.batch, 256, 0, st>>>(d, k_new, v_new, new_sb, new_sh, K, V, ks, vs, seq_lens);
    return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const float* x, int64_t rows, int dim, int64_t x_stride, int8_t* codes,
                                 int64_t code_stride, float* scales, int sms, cudaStream_t st) {
    int64_t blocks = (rows + 7) / 8;
    const int64_t cap = static_cast<int64_t>(sms) * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    quantize_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(x, rows, dim, x_stride, codes,
                                                                       code_stride, scales);
    return cudaGetLastError();
}

}  // namespace kvd
