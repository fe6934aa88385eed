// kvd_abi.cu -- the extern "C" boundary of libkvdecode_b200.so: argument
// checks, path selection, workspace planning and the reference-compatible
// entry points (see include/kvdecode.h for the contract of each symbol).
#include <cuda.h>

#include <cstdio>
#include <cstdint>
#include <mutex>

#include "kvd_common.cuh"
#include "kvd_decode.cuh"
#include "kvd_workspace.h"

namespace kvd {

__device__ int32_t g_status = 0;

cudaError_t launch_append(const kvd_append_desc& d, const float* k_new, const float* v_new, int8_t* K,
                          int8_t* V, float* ks, float* vs, int32_t* seq_lens, cudaStream_t st);
cudaError_t launch_quantize_rows(const float* x, int64_t rows, int dim, int64_t x_stride, int8_t* codes,
                                 int64_t code_stride, float* scales, int sms, cudaStream_t st);

unsigned long long current_context_id() {
    using Fn = CUresult (*)(CUcontext, unsigned long long*);
    static Fn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {  // through the runtime, so the library does not link the driver library
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetId", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<Fn>(ptr);
    });
    unsigned long long id = 0;
    if (!fn || fn(nullptr, &id) != CUDA_SUCCESS) return 0;
    return id;
}

int device_sm_count() {
    static std::atomic<int> cache[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 1;
    const bool cached = dev >= 0 && dev < kMaxDevices;
    if (cached) {
        const int n = cache[dev].load(std::memory_order_relaxed);
        if (n > 0) return n;
    }
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 1;
    if (cached) cache[dev].store(n, std::memory_order_relaxed);
    return n;
}

namespace {
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
thread_local int tl_launches = 0;

// Known flags; one Q type, one output type, and typed output only for
// normalised rows (records are fp32).
bool flags_ok(uint32_t f) {
    if ((f & ~(KVD_FLAG_PARTIAL_OUT | KVD_FLAG_QK_INT8 | kDtypeFlags)) != 0) return false;
    if ((f & KVD_FLAG_Q_BF16) && (f & KVD_FLAG_Q_F16)) return false;
    if ((f & KVD_FLAG_OUT_BF16) && (f & KVD_FLAG_OUT_F16)) return false;
    if ((f & KVD_FLAG_PARTIAL_OUT) && (f & (KVD_FLAG_OUT_BF16 | KVD_FLAG_OUT_F16))) return false;
    return true;
}

cudaError_t check_desc(const kvd_decode_desc* d) {
    if (d == nullptr) return cudaErrorInvalidValue;
    if (d->batch < 1 || d->num_q_heads < 1 || d->num_kv_heads < 1 || d->head_dim < 1) return cudaErrorInvalidValue;
    if (d->num_q_heads % d->num_kv_heads != 0) return cudaErrorInvalidValue;
    if (d->max_seq_len < 0) return cudaErrorInvalidValue;
    if (!flags_ok(d->flags)) return cudaErrorInvalidValue;
    return cudaSuccess;
}

size_t fast_prefix_bytes(const kvd_decode_desc& d) {
    return d.seq_lens ? align256(static_cast<size_t>(d.batch + 1) * sizeof(int32_t)) : 0;
}
}  // namespace

int* launch_counter() { return &tl_launches; }

bool fast_path_ok(const kvd_decode_desc& d, const void* Q, const int8_t* K, const int8_t* V) {
    if (d.head_dim != 64 && d.head_dim != 128) return false;
    if (!aligned16(Q) || !aligned16(K) || !aligned16(V)) return false;
    if (((d.kv_stride_b | d.kv_stride_h) & 15) != 0) return false;
    if (((d.q_stride_b | d.q_stride_h) & 3) != 0) return false;
    return true;
}

}  // namespace kvd

using namespace kvd;

extern "C" int kvd_abi_version(void) { return KVD_ABI_VERSION; }

extern "C" int kvd_last_launch_count(void) { return tl_launches; }

extern "C" const char* kvd_error_string(int error) { return cudaGetErrorString(static_cast<cudaError_t>(error)); }

extern "C" size_t kvd_workspace_size(const kvd_decode_desc* desc) {
    if (check_desc(desc) != cudaSuccess) return 0;
    const kvd_decode_desc& d = *desc;
    size_t fast = 0;
    if (d.head_dim == 64 || d.head_dim == 128)
        fast = fast_prefix_bytes(d) +
               static_cast<size_t>(2) * device_sm_count() * sk_ctas_per_sm(d.head_dim) * (d.head_dim + 4) *
                   sizeof(float);
    const size_t gen = generic_workspace_size(d);
    const size_t gqa = gqa_path_ok(d) ? gqa_workspace_size(d) : 0;
    size_t need = fast > gen ? fast : gen;
    return need > gqa ? need : gqa;
}

extern "C" cudaError_t kvd_decode_launch(const kvd_decode_desc* desc, const void* Q, const int8_t* K,
                                         const int8_t* V, const float* k_scale, const float* v_scale,
                                         void* out, void* workspace, size_t workspace_bytes,
                                         cudaStream_t stream) {
    tl_launches = 0;
    cudaError_t e = check_desc(desc);
    if (e != cudaSuccess) return e;
    if (!Q || !K || !V || !k_scale || !v_scale || !out) return cudaErrorInvalidValue;
    const kvd_decode_desc& d = *desc;
    if ((d.flags & KVD_FLAG_PARTIAL_OUT) && d.num_q_heads > 1 && d.o_stride_h < d.head_dim + 4)
        return cudaErrorInvalidValue;
    if (!workspace) workspace_bytes = 0;

    if (d.flags & KVD_FLAG_QK_INT8) {  // the int8 query mode exists on the tensor-core kernel only
        if (fast_path_ok(d, Q, K, V) && gqa_path_ok(d))
            return launch_gqa_tc(d, Q, K, V, k_scale, v_scale, out, workspace, workspace_bytes, stream,
                                 &tl_launches);
        return cudaErrorNotSupported;
    }
    if (!fast_path_ok(d, Q, K, V))
        return launch_generic(d, Q, K, V, k_scale, v_scale, out, workspace, workspace_bytes, stream,
                              &tl_launches);

    // Small dense MHA problems (too few bytes to fill the GPU): one launch, a
    // cluster of CTAs per head merging through distributed shared memory.
    if (small_cluster_size(d) > 0)
        return launch_small(d, static_cast<const float*>(Q), K, V, k_scale, v_scale, static_cast<float*>(out),
                            stream, &tl_launches);

    // Grouped-query heads share every K/V tile: tensor-core kernel. MHA with
    // D=128 takes it too: the tensor cores do QK and PV, so the SMs spend far
    // fewer instructions (and watts) per byte than the CUDA-core kernel.
    const bool mha_tc = KVD_MHA_TENSOR_CORES >= 2 || (KVD_MHA_TENSOR_CORES == 1 && !d.seq_lens);
    if ((d.num_q_heads > d.num_kv_heads || mha_tc || (d.flags & kDtypeFlags)) && gqa_path_ok(d))
        return launch_gqa_tc(d, Q, K, V, k_scale, v_scale, out, workspace, workspace_bytes, stream, &tl_launches);
    if (d.flags & kDtypeFlags)  // the CUDA-core split-KV kernel reads and writes fp32 only
        return launch_generic(d, Q, K, V, k_scale, v_scale, out, workspace, workspace_bytes, stream,
                              &tl_launches);

    const int tok = tile_tokens(d.head_dim);
    const size_t pre = fast_prefix_bytes(d);
    if (d.seq_lens && workspace_bytes < pre)  // ragged batches need room for the tile plan
        return launch_generic(d, Q, K, V, k_scale, v_scale, out, workspace, workspace_bytes, stream,
                              &tl_launches);

    DecodeParams p{};
    p.Q = static_cast<const float*>(Q); p.K = K; p.V = V; p.ks = k_scale; p.vs = v_scale;
    p.out = static_cast<float*>(out);
    p.B = d.batch; p.Hq = d.num_q_heads; p.Hkv = d.num_kv_heads; p.D = d.head_dim;
    p.group = d.num_q_heads / d.num_kv_heads;
    p.S = d.max_seq_len;
    p.seq_lens = d.seq_lens;
    p.kv_sb = d.kv_stride_b; p.kv_sh = d.kv_stride_h;
    p.sc_sb = d.sc_stride_b; p.sc_sh = d.sc_stride_h;
    p.q_sb = d.q_stride_b; p.q_sh = d.q_stride_h;
    p.o_sb = d.o_stride_b; p.o_sh = d.o_stride_h;
    const float scale = d.softmax_scale > 0.f ? d.softmax_scale : 1.0f / sqrtf(static_cast<float>(d.head_dim));
    p.qscale = scale * 1.4426950408889634f;  // scores in base-2 exponent units
    p.flags = d.flags;

    int64_t grid = static_cast<int64_t>(device_sm_count()) * sk_ctas_per_sm(d.head_dim);  // persistent CTAs
    if (!d.seq_lens) {
        p.tiles_per_head = d.max_seq_len > 0 ? (d.max_seq_len + tok - 1) / tok : 1;
        const int64_t heads = static_cast<int64_t>(d.batch) * d.num_q_heads;
        p.n_tiles = heads * p.tiles_per_head;
        if (grid > p.n_tiles) grid = p.n_tiles;
        // Small problems: one CTA per whole head needs no combine launch; take it
        // when its tile count does not exceed the split's rounds plus the combine
        // (about 8 tiles of work).
        const int64_t split_rounds = (p.n_tiles + grid - 1) / grid;
        if (heads <= grid && p.tiles_per_head <= split_rounds + 8) grid = heads;
    } else {
        p.tile_prefix = static_cast<const int32_t*>(workspace);
    }
    const size_t rec_bytes = static_cast<size_t>(d.head_dim + 4) * sizeof(float);
    const int64_t fit = static_cast<int64_t>((workspace_bytes - pre) / (2 * rec_bytes));
    if (grid > fit) grid = fit;
    if (grid < 1) grid = 1;  // one CTA finishes every head itself: no partials
    p.grid = static_cast<int>(grid);
    p.partials = grid > 1 ? reinterpret_cast<float*>(static_cast<char*>(workspace) + pre) : nullptr;

    if (d.seq_lens) {
        e = launch_plan(d.seq_lens, d.batch, d.num_q_heads, tok, d.max_seq_len, static_cast<int32_t*>(workspace), stream,
                        &tl_launches);
        if (e != cudaSuccess) return e;
    }
    return launch_splitkv(p, stream, &tl_launches);
}

namespace {
cudaError_t check_paged(const kvd_paged_desc* d) {
    if (d == nullptr || !d->seq_lens || !d->block_table) return cudaErrorInvalidValue;
    if (d->batch < 1 || d->num_q_heads < 1 || d->num_kv_heads < 1 || d->head_dim < 1) return cudaErrorInvalidValue;
    if (d->num_q_heads % d->num_kv_heads != 0) return cudaErrorInvalidValue;
    if (d->block_size < 1 || d->num_blocks < 1 || d->max_blocks_per_seq < 1) return cudaErrorInvalidValue;
    if (d->block_table_stride < d->max_blocks_per_seq) return cudaErrorInvalidValue;
    if (static_cast<int64_t>(d->max_blocks_per_seq) * d->block_size > 0x7fffffffLL) return cudaErrorInvalidValue;
    if (!flags_ok(d->flags)) return cudaErrorInvalidValue;
    return cudaSuccess;
}

// The dense descriptor the planners see: ragged lengths over a capacity of
// max_blocks_per_seq * block_size tokens; the pool addressing rides in a PagedView.
kvd_decode_desc paged_as_dense(const kvd_paged_desc& p, PagedView* pv) {
    kvd_decode_desc d{};
    d.batch = p.batch; d.num_q_heads = p.num_q_heads; d.num_kv_heads = p.num_kv_heads; d.head_dim = p.head_dim;
    d.max_seq_len = p.max_blocks_per_seq * p.block_size;
    d.flags = p.flags;
    d.seq_lens = p.seq_lens;
    d.kv_stride_b = 0; d.kv_stride_h = p.kv_stride_h;
    d.sc_stride_b = 0; d.sc_stride_h = p.sc_stride_h;
    d.q_stride_b = p.q_stride_b; d.q_stride_h = p.q_stride_h;
    d.o_stride_b = p.o_stride_b; d.o_stride_h = p.o_stride_h;
    d.softmax_scale = p.softmax_scale;
    pv->table = p.block_table;
    pv->bt_stride = p.block_table_stride;
    pv->block_size = p.block_size;
    pv->num_blocks = p.num_blocks;
    pv->kv_sblk = p.kv_stride_block;
    pv->kv_st = p.kv_stride_t;
    pv->sc_sblk = p.sc_stride_block;
    return d;
}

bool paged_tc_shape(const kvd_paged_desc& p, const kvd_decode_desc& d) {
    const int bs = p.block_size;
    return bs >= 8 && (bs & (bs - 1)) == 0 && gqa_path_ok(d);
}

bool paged_tc_ok(const kvd_paged_desc& p, const kvd_decode_desc& d, const void* Q, const int8_t* K,
                 const int8_t* V, const float* ks, const float* vs) {
    if (!paged_tc_shape(p, d)) return false;
    if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(ks) || !aligned16(vs)) return false;
    if (((p.kv_stride_block | p.kv_stride_h | p.kv_stride_t) & 15) != 0) return false;
    if (p.kv_stride_block <= 0 || p.kv_stride_h <= 0 || p.kv_stride_t <= 0) return false;
    if (((p.sc_stride_block | p.sc_stride_h) & 3) != 0) return false;
    if (((p.q_stride_b | p.q_stride_h) & 3) != 0) return false;
    return true;
}
}  // namespace

extern "C" size_t kvd_paged_workspace_size(const kvd_paged_desc* desc) {
    if (check_paged(desc) != cudaSuccess) return 0;
    PagedView pv;
    const kvd_decode_desc d = paged_as_dense(*desc, &pv);
    const size_t gen = generic_workspace_size(d);
    const size_t gqa = paged_tc_shape(*desc, d) ? gqa_workspace_size(d) : 0;
    return gen > gqa ? gen : gqa;
}

extern "C" cudaError_t kvd_paged_decode_launch(const kvd_paged_desc* desc, const void* Q, const int8_t* K_pool,
                                               const int8_t* V_pool, const float* k_scale_pool,
                                               const float* v_scale_pool, void* out, void* workspace,
                                               size_t workspace_bytes, cudaStream_t stream) {
    tl_launches = 0;
    cudaError_t e = check_paged(desc);
    if (e != cudaSuccess) return e;
    if (!Q || !K_pool || !V_pool || !k_scale_pool || !v_scale_pool || !out) return cudaErrorInvalidValue;
    if ((desc->flags & KVD_FLAG_PARTIAL_OUT) && desc->num_q_heads > 1 && desc->o_stride_h < desc->head_dim + 4)
        return cudaErrorInvalidValue;
    if (!workspace) workspace_bytes = 0;
    PagedView pv;
    const kvd_decode_desc d = paged_as_dense(*desc, &pv);
    if (paged_tc_ok(*desc, d, Q, K_pool, V_pool, k_scale_pool, v_scale_pool))
        return launch_gqa_tc(d, Q, K_pool, V_pool, k_scale_pool, v_scale_pool, out, workspace, workspace_bytes,
                             stream, &tl_launches, &pv);
    if (desc->flags & KVD_FLAG_QK_INT8) return cudaErrorNotSupported;
    return launch_generic(d, Q, K_pool, V_pool, k_scale_pool, v_scale_pool, out, workspace, workspace_bytes, stream,
                          &tl_launches, &pv);
}

extern "C" cudaError_t kvd_paged_append_int8_launch(const kvd_paged_desc* desc, const float* k_new,
                                                    const float* v_new, int64_t new_stride_b, int64_t new_stride_h,
                                                    int8_t* K_pool, int8_t* V_pool, float* k_scale_pool,
                                                    float* v_scale_pool, int32_t* seq_lens, cudaStream_t stream) {
    tl_launches = 0;
    if (!desc || !desc->block_table || !k_new || !v_new || !K_pool || !V_pool || !k_scale_pool || !v_scale_pool ||
        !seq_lens)
        return cudaErrorInvalidValue;
    if (desc->batch < 1 || desc->num_kv_heads < 1 || desc->head_dim < 1 || desc->block_size < 1 ||
        desc->num_blocks < 1 || desc->max_blocks_per_seq < 1 || desc->block_table_stride < desc->max_blocks_per_seq)
        return cudaErrorInvalidValue;
    const cudaError_t e = launch_paged_append(*desc, k_new, v_new, new_stride_b, new_stride_h, K_pool, V_pool,
                                              k_scale_pool, v_scale_pool, seq_lens, stream);
    if (e == cudaSuccess) tl_launches = 1;
    return e;
}

extern "C" cudaError_t kvd_combine_launch(const float* parts, int num_parts, int64_t part_stride, int num_heads,
                                          int head_dim, void* out, int64_t out_stride, uint32_t flags,
                                          cudaStream_t stream) {
    tl_launches = 0;
    if (!parts || !out || num_parts < 1 || num_heads < 1 || head_dim < 1) return cudaErrorInvalidValue;
    if (!flags_ok(flags) || (flags & (KVD_FLAG_Q_BF16 | KVD_FLAG_Q_F16 | KVD_FLAG_QK_INT8))) return cudaErrorInvalidValue;
    if (part_stride < static_cast<int64_t>(num_heads) * (head_dim + 4) && num_parts > 1) return cudaErrorInvalidValue;
    return launch_combine_parts(parts, num_parts, part_stride, num_heads, head_dim, out, out_stride, flags, stream,
                                &tl_launches);
}

extern "C" cudaError_t kvd_append_int8_launch(const kvd_append_desc* desc, const float* k_new, const float* v_new,
                                              int8_t* K, int8_t* V, float* k_scale, float* v_scale,
                                              int32_t* seq_lens, cudaStream_t stream) {
    tl_launches = 0;
    if (!desc || !k_new || !v_new || !K || !V || !k_scale || !v_scale || !seq_lens) return cudaErrorInvalidValue;
    if (desc->batch < 1 || desc->num_kv_heads < 1 || desc->head_dim < 1 || desc->capacity < 1)
        return cudaErrorInvalidValue;
    const cudaError_t e = launch_append(*desc, k_new, v_new, K, V, k_scale, v_scale, seq_lens, stream);
    if (e == cudaSuccess) tl_launches = 1;
    return e;
}

extern "C" cudaError_t kvd_append_decode_launch(const kvd_decode_desc* desc, const float* k_new,
                                                const float* v_new, int64_t new_stride_b, int64_t new_stride_h,
                                                const void* Q, int8_t* K, int8_t* V, float* k_scale, float* v_scale,
                                                void* out, void* workspace, size_t workspace_bytes,
                                                cudaStream_t stream) {
    tl_launches = 0;
    cudaError_t e = check_desc(desc);
    if (e != cudaSuccess) return e;
    const kvd_decode_desc& d = *desc;
    if (!d.seq_lens || !k_new || !v_new || !Q || !K || !V || !k_scale || !v_scale || !out) return cudaErrorInvalidValue;
    if (d.max_seq_len < 1) return cudaErrorInvalidValue;
    if ((d.flags & KVD_FLAG_PARTIAL_OUT) && d.num_q_heads > 1 && d.o_stride_h < d.head_dim + 4)
        return cudaErrorInvalidValue;
    if (!workspace) workspace_bytes = 0;
    int32_t* lens = const_cast<int32_t*>(d.seq_lens);
    const bool rows16 = ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) & 15) == 0 &&
                        ((new_stride_b | new_stride_h) & 3) == 0;  // one 16-byte load per lane
    if (rows16 && fast_path_ok(d, Q, K, V) && gqa_fused_append_ok(d, workspace_bytes)) {
        const AppendView av{k_new, v_new, new_stride_b, new_stride_h, lens};
        return launch_gqa_tc(d, Q, K, V, k_scale, v_scale, out, workspace, workspace_bytes, stream, &tl_launches,
                             nullptr, &av);
    }
    // Two launches: the append kernel, then the decode of the grown cache.
    kvd_append_desc a{};
    a.batch = d.batch; a.num_kv_heads = d.num_kv_heads; a.head_dim = d.head_dim; a.capacity = d.max_seq_len;
    a.kv_stride_b = d.kv_stride_b; a.kv_stride_h = d.kv_stride_h;
    a.sc_stride_b = d.sc_stride_b; a.sc_stride_h = d.sc_stride_h;
    a.new_stride_b = new_stride_b; a.new_stride_h = new_stride_h;
    e = launch_append(a, k_new, v_new, K, V, k_scale, v_scale, lens, stream);
    if (e != cudaSuccess) return e;
    e = kvd_decode_launch(desc, Q, K, V, k_scale, v_scale, out, workspace, workspace_bytes, stream);
    tl_launches += 1;
    return e;
}

namespace {
cudaError_t check_prefill(const kvd_prefill_desc* d) {
    if (!d) return cudaErrorInvalidValue;
    if (d->batch < 1 || d->num_q_heads < 1 || d->num_kv_heads < 1 || d->head_dim < 1) return cudaErrorInvalidValue;
    if (d->num_q_heads % d->num_kv_heads != 0 || d->max_seq_len < 1 || d->max_queries < 1)
        return cudaErrorInvalidValue;
    if (!flags_ok(d->flags) || (d->flags & (KVD_FLAG_PARTIAL_OUT | KVD_FLAG_QK_INT8))) return cudaErrorInvalidValue;
    return cudaSuccess;
}
}  // namespace

extern "C" size_t kvd_prefill_workspace_size(const kvd_prefill_desc* desc) {
    (void)desc;
    return 0;
}

extern "C" cudaError_t kvd_prefill_launch(const kvd_prefill_desc* desc, const void* Q, const int8_t* K,
                                          const int8_t* V, const float* k_scale, const float* v_scale, void* out,
                                          void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    tl_launches = 0;
    cudaError_t e = check_prefill(desc);
    if (e != cudaSuccess) return e;
    if (!Q || !K || !V || !k_scale || !v_scale || !out) return cudaErrorInvalidValue;
    (void)workspace;
    (void)workspace_bytes;
    if (prefill_tc_ok(*desc, K, V, k_scale, v_scale)) {  // head_dim 128: tensor-core kernel
        e = launch_prefill_tc(*desc, Q, K, V, k_scale, v_scale, out, stream, &tl_launches);
        if (e != cudaErrorNotSupported) return e;
    }
    return launch_generic_prefill(*desc, Q, K, V, k_scale, v_scale, out, stream, &tl_launches);
}

extern "C" cudaError_t kvd_quantize_rows_launch(const float* x, int64_t rows, int dim, int64_t x_stride,
                                                int8_t* codes, int64_t code_stride, float* scales,
                                                cudaStream_t stream) {
    tl_launches = 0;
    if (!x || !codes || !scales || rows < 0 || dim < 1) return cudaErrorInvalidValue;
    if (rows == 0) return cudaSuccess;
    const cudaError_t e =
        launch_quantize_rows(x, rows, dim, x_stride, codes, code_stride, scales, device_sm_count(), stream);
    if (e == cudaSuccess) tl_launches = 1;
    return e;
}

extern "C" cudaError_t kvd_device_status(int32_t* status) {
    if (!status) return cudaErrorInvalidValue;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return e;
    int32_t v = 0;
    e = cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
    if (e != cudaSuccess) return e;
    const int32_t zero = 0;
    e = cudaMemcpyToSymbol(g_status, &zero, sizeof(zero));
    *status = v;
    return e;
}

// ------------------------------------------------ reference-compatible ABI
namespace {
kvd_decode_desc reference_desc(int num_heads, int seq_len, int head_dim) {
    kvd_decode_desc d{};
    d.batch = 1;
    d.num_q_heads = num_heads;
    d.num_kv_heads = num_heads;
    d.head_dim = head_dim;
    d.max_seq_len = seq_len;
    d.flags = 0;
    d.seq_lens = nullptr;
    d.kv_stride_b = 0;
    d.kv_stride_h = static_cast<int64_t>(seq_len) * head_dim;
    d.sc_stride_b = 0;
    d.sc_stride_h = seq_len;
    d.q_stride_b = 0;
    d.q_stride_h = head_dim;
    d.o_stride_b = 0;
    d.o_stride_h = head_dim;
    d.softmax_scale = 0.f;
    return d;
}

cudaError_t reference_launch(const float* Q, const int8_t* K, const int8_t* V, const float* ks, const float* vs,
                             float* out, int num_heads, int seq_len, int head_dim, float* S, cudaStream_t st) {
    if (!Q || !K || !V || !ks || !vs || !out || !S || num_heads <= 0 || seq_len <= 0 || head_dim <= 0)
        return cudaErrorInvalidValue;
    const kvd_decode_desc d = reference_desc(num_heads, seq_len, head_dim);
    const size_t s_bytes = static_cast<size_t>(num_heads) * static_cast<size_t>(seq_len) * sizeof(float);
    return kvd_decode_launch(&d, Q, K, V, ks, vs, out, S, s_bytes, st);
}
}  // namespace

extern "C" cudaError_t kv_int8_split_launch(const float* Q, const int8_t* K_int8, const int8_t* V_int8,
                                            const float* k_scale, const float* v_scale, float* output,
                                            int num_heads, int seq_len, int head_dim, float* S,
                                            cudaStream_t stream) {
    return reference_launch(Q, K_int8, V_int8, k_scale, v_scale, output, num_heads, seq_len, head_dim, S, stream);
}

extern "C" cudaError_t kv_int8_simple_launch(const float* Q, const int8_t* K_int8, const int8_t* V_int8,
                                             const float* k_scale, const float* v_scale, float* output,
                                             int num_heads, int seq_len, int head_dim, float* S,
                                             cudaStream_t stream) {
    return reference_launch(Q, K_int8, V_int8, k_scale, v_scale, output, num_heads, seq_len, head_dim, S, stream);
}

extern "C" void solve(const float* Q, const int8_t* K_int8, const int8_t* V_int8, const float* k_scale,
                      const float* v_scale, float* output, int num_heads, int seq_len, int head_dim) {
    if (!Q || !K_int8 || !V_int8 || !k_scale || !v_scale || !output) {
        std::fprintf(stderr,
                     "[kvdecode] null pointer input: Q=%p K_int8=%p V_int8=%p k_scale=%p v_scale=%p output=%p\n",
                     static_cast<const void*>(Q), static_cast<const void*>(K_int8),
                     static_cast<const void*>(V_int8), static_cast<const void*>(k_scale),
                     static_cast<const void*>(v_scale), static_cast<void*>(output));
        return;
    }
    if (num_heads <= 0 || seq_len <= 0 || head_dim <= 0) {
        std::fprintf(stderr, "[kvdecode] invalid shape: num_heads=%d, seq_len=%d, head_dim=%d\n", num_heads,
                     seq_len, head_dim);
        return;
    }
    const kvd_decode_desc d = reference_desc(num_heads, seq_len, head_dim);
    OrderedWorkspace ws(kvd_workspace_size(&d), cudaStreamLegacy);
    if (ws.status() != cudaSuccess) {
        std::fprintf(stderr, "[kvdecode] workspace allocation failed: %s\n", cudaGetErrorString(ws.status()));
        return;
    }
    const cudaError_t e =
        kvd_decode_launch(&d, Q, K_int8, V_int8, k_scale, v_scale, output, ws.data(), ws.bytes(), cudaStreamLegacy);
    if (e != cudaSuccess)
        std::fprintf(stderr, "[kvdecode] launch failed: %s (%s)\n", cudaGetErrorName(e), cudaGetErrorString(e));
    const int launches = tl_launches;
    ws.close();
    tl_launches = launches;
}
