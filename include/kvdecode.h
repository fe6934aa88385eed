/*
 * kvdecode.h -- C ABI of libkvdecode_b200.so, a B200 (sm_100a) INT8 KV-cache
 * decode-attention library.
 *
 * Drop-in for the extern "C" entry points of Murmurwkk/cuda-operators'
 * kv_cache/ kernels. Plain pointers and sizes only; every pointer argument is
 * a DEVICE pointer unless stated otherwise. Layout of the reference entry
 * points (unchanged): Q [H][D] fp32, K/V [H][S][D] int8 codes, k_scale/v_scale
 * [H][S] fp32 (one scale per token), output [H][D] fp32, where H folds batch
 * and heads. Attention is out[h] = softmax_t((q_h . K[h,t]) * ks[h,t] / sqrt(D))
 * applied to V[h,t] * vs[h,t].
 *
 * All launches are asynchronous on the given stream (the default stream for
 * `solve`); the caller synchronises before reading results. Calls are
 * thread-safe (per-device one-time set-up is guarded); devices with an ordinal
 * of 64 or more are not supported (cudaErrorInvalidDevice).
 *
 * Programmatic dependent launch: the head_dim-128 decode kernel lets dependent
 * grids launch early (griddepcontrol.launch_dependents), and the library
 * launches its own follow-up kernels (split combine, record exchange) with the
 * programmatic stream-serialization attribute; they wait (griddepcontrol.wait)
 * before reading the decode's output. A caller's kernel launched after a
 * decode WITHOUT that attribute is ordered as usual; one launched WITH it must
 * itself wait (griddepcontrol.wait / cudaGridDependencySynchronize) before
 * reading the decode's output. The head_dim-128 and small-problem decode
 * kernels are themselves launched with the attribute: their CTAs may launch
 * while the kernel before them on the stream ends, and wait
 * (griddepcontrol.wait) before any global memory access, so they see
 * everything that kernel wrote. The record exchange of
 * kvd_mgpu_p2p_seq_split_decode lets the next kernel launch early too: a
 * caller's kernel that follows it with the attribute must wait in the same way.
 */
#ifndef KVDECODE_H
#define KVDECODE_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVD_ABI_VERSION 1

/* ------------------------------------------------------------------------ */
/* Reference-compatible entry points                                         */
/* ------------------------------------------------------------------------ */

/* Replaces `solve` of kv_cache/KV_int8.cu:306-316,
 * kv_cache/KV_int8_single_buffer.cu:260-270,
 * kv_cache/KV_int8_split_optimized.cu:294-304 and kv_cache/new_kvint8.cu:102-104
 * (identical signatures). Launches on the default stream and returns without
 * synchronising. Null pointers or non-positive sizes print one line to stderr
 * and return, as KV_int8_split_optimized.cu:306-324 does. Scratch for split
 * partials is allocated stream-ordered (cudaMallocAsync/cudaFreeAsync on the
 * default stream) instead of the reference's cudaMalloc/cudaFree per call. */
void solve(const float* Q, const int8_t* K_int8, const int8_t* V_int8,
           const float* k_scale, const float* v_scale, float* output,
           int num_heads, int seq_len, int head_dim);

/* Replaces kv_int8_split_launch, kv_cache/KV_int8_split_optimized.cu:268-292.
 * S is caller-owned scratch of at least num_heads*seq_len floats (the
 * reference's score buffer). This implementation keeps no score matrix; it
 * uses S for split-KV partials and picks the split count so that they fit.
 * Returns cudaErrorInvalidValue on a null pointer or a non-positive size
 * (KV_int8_split_optimized.cu:272-273), else the launch status. */
cudaError_t kv_int8_split_launch(const float* Q, const int8_t* K_int8, const int8_t* V_int8,
                                 const float* k_scale, const float* v_scale, float* output,
                                 int num_heads, int seq_len, int head_dim,
                                 float* S, cudaStream_t stream);

/* Replaces kv_int8_simple_launch, kv_cache/new_kvint8.cu:85-100. Same contract
 * as kv_int8_split_launch (same kernels). */
cudaError_t kv_int8_simple_launch(const float* Q, const int8_t* K_int8, const int8_t* V_int8,
                                  const float* k_scale, const float* v_scale, float* output,
                                  int num_heads, int seq_len, int head_dim,
                                  float* S, cudaStream_t stream);

/* ------------------------------------------------------------------------ */
/* Extended API (no reference counterpart: batch, GQA, ragged, strides)      */
/* ------------------------------------------------------------------------ */

/* Decode flags. */
#define KVD_FLAG_PARTIAL_OUT 1u  /* write (m, l, o) records instead of normalised output */
/* Element type of Q (default fp32; strides stay in elements). */
#define KVD_FLAG_Q_BF16 2u
#define KVD_FLAG_Q_F16 4u
/* Element type of the normalised output rows (default fp32; rounded to
 * nearest even). Not combinable with KVD_FLAG_PARTIAL_OUT: records are fp32. */
#define KVD_FLAG_OUT_BF16 8u
#define KVD_FLAG_OUT_F16 16u
/* INT8 Q.K fast mode (no reference counterpart; the reference computes Q.K in
 * fp32 over dequantised codes, kv_cache/KV_int8_split_optimized.cu:136-143).
 * Each query row (b, hq) is first quantised with the cache's own rule
 * (scale_q = max|q|/127, code = clamp(rint(q/scale_q), -127, 127), IEEE fp32)
 * and Q.K runs as one exact int8 tensor-core product per head:
 * score = (sum_d code_q * code_k) * scale_q * k_scale * softmax_scale. The
 * result equals the exact decode of the rounded query q^ = code_q * scale_q
 * within the usual tolerance (2e-5 + 1e-4 |ref|); against the unrounded query
 * it carries the rounding's effect, to first order at most
 * 2 * max_t |ds_t| * max_t |v_t| per output element, where ds_t is the score
 * change (q^ - q) . k_t * softmax_scale (the looser, stated tolerance of this
 * mode). Tensor-core kernel only: head_dim 128, groups 1/2/4/8/16, 16-byte
 * aligned Q/K/V; other shapes return cudaErrorNotSupported. */
#define KVD_FLAG_QK_INT8 32u

/* A partial record (KVD_FLAG_PARTIAL_OUT output and kvd_combine_launch input)
 * is KVD_PARTIAL_STRIDE(D) floats: [0] = m, a reference point in base-2
 * exponent units (scores times log2(e)); it is at most the max and at least
 * the max minus 8, because rescaling is lazy; [1] = l = sum_t 2^(s_t - m);
 * [2],[3] unused; [4 .. 4+D) = o = sum_t 2^(s_t - m) * v_t (not divided by l).
 * m + log2(l) is the base-2 log-sum-exp of the scores. An empty record has
 * m = -inf, l = 0, o = 0. */
#define KVD_PARTIAL_STRIDE(D) ((D) + 4)

typedef struct kvd_decode_desc {
    int32_t batch;          /* B >= 1 */
    int32_t num_q_heads;    /* Hq >= 1 */
    int32_t num_kv_heads;   /* Hkv >= 1, Hq % Hkv == 0; query head hq reads kv head hq/(Hq/Hkv) */
    int32_t head_dim;       /* D >= 1 */
    int32_t max_seq_len;    /* length of every sequence when seq_lens == NULL, else an upper bound */
    uint32_t flags;         /* KVD_FLAG_* */
    const int32_t* seq_lens;/* device [B] current lengths (0 allowed), or NULL */
    /* Strides in elements. Tokens of one head are contiguous: token stride is
     * D codes for K/V and 1 float for the scales. */
    int64_t kv_stride_b, kv_stride_h;   /* K and V share strides */
    int64_t sc_stride_b, sc_stride_h;   /* k_scale and v_scale share strides */
    int64_t q_stride_b, q_stride_h;     /* Q [B][Hq][D] by default */
    int64_t o_stride_b, o_stride_h;     /* output rows (or partial records) */
    float softmax_scale;    /* <= 0 selects 1/sqrt(D) */
} kvd_decode_desc;

/* Bytes of workspace kvd_decode_launch needs for this descriptor on the
 * current device (0 is possible). */
size_t kvd_workspace_size(const kvd_decode_desc* desc);

/* Split-KV flash decode. `workspace` may be smaller than kvd_workspace_size
 * (fewer splits are used) or NULL with workspace_bytes == 0. Concurrent calls
 * need separate workspaces. Q and out are fp32 unless desc->flags selects
 * bf16 or fp16 (KVD_FLAG_Q_*, KVD_FLAG_OUT_*). */
cudaError_t kvd_decode_launch(const kvd_decode_desc* desc,
                              const void* Q, const int8_t* K, const int8_t* V,
                              const float* k_scale, const float* v_scale, void* out,
                              void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* No counterpart in the reference. The same decode as kvd_decode_launch for
 * callers that cannot allocate device memory when they decode (a framework that
 * owns all device memory and gives a plugin only its inputs and outputs, or a
 * serving loop that bans allocation on its hot path): its scratch lives in a
 * fixed KVD_NOALLOC_SCRATCH_BYTES array inside the library, held by every GPU
 * that loads the library until exit. Descriptors whose kvd_workspace_size()
 * exceeds the array are rejected with cudaErrorInvalidValue (long contexts do:
 * 4 x 32 heads x 131,072 tokens needs 2.5 MB of split records). The first call
 * in each CUDA context of a device (the first call, and the first after a
 * cudaDeviceReset) resolves the array's address: make it outside any stream
 * capture. All calls share the array: calls that overlap on the GPU race.
 * Allocates nothing. */
#define KVD_NOALLOC_SCRATCH_BYTES (512u * 1024u)
cudaError_t kvd_decode_launch_noalloc(const kvd_decode_desc* desc,
                                      const void* Q, const int8_t* K, const int8_t* V,
                                      const float* k_scale, const float* v_scale, void* out,
                                      cudaStream_t stream);

/* ------------------------------------------------------------------------ */
/* Paged cache (no reference counterpart: the reference's caches are dense   */
/* [H][S][D] arrays, kv_cache/new_kvint8.cu:83-84)                            */
/* ------------------------------------------------------------------------ */

/* K and V codes and their scales live in pools of fixed-size blocks of
 * `block_size` tokens. Token t of sequence b, kv head h is at
 *   K_pool[blk * kv_stride_block + h * kv_stride_h + (t % block_size) * kv_stride_t + d]
 *   k_scale_pool[blk * sc_stride_block + h * sc_stride_h + (t % block_size)]
 * with blk = block_table[b * block_table_stride + t / block_size] (V alike).
 * Both common pool layouts are strides of this form: [blocks][Hkv][bs][D]
 * (kv_stride_t = D) and [blocks][bs][Hkv][D] (kv_stride_t = Hkv*D). A block id
 * outside [0, num_blocks) is not read: its tokens count as score 0 with a zero
 * value and the device status word records KVD_STATUS_BAD_BLOCK. The decode
 * uses the tensor-core kernel when head_dim is 128, the group size is 1, 2, 4,
 * 8 or 16, block_size is a power of two >= 8, pools and strides are 16-byte
 * aligned and scale strides are multiples of 4 floats; other shapes run on
 * the generic kernel (any block_size >= 1). */
#define KVD_STATUS_BAD_BLOCK 4
typedef struct kvd_paged_desc {
    int32_t batch, num_q_heads, num_kv_heads, head_dim;
    int32_t block_size;          /* tokens per block, >= 1 */
    int32_t num_blocks;          /* blocks in each pool */
    int32_t max_blocks_per_seq;  /* table entries per sequence; lengths are clamped to this x block_size */
    uint32_t flags;              /* KVD_FLAG_* */
    const int32_t* seq_lens;     /* device [B] current lengths (required) */
    const int32_t* block_table;  /* device [B][block_table_stride] pool block ids */
    int64_t block_table_stride;  /* >= max_blocks_per_seq */
    int64_t kv_stride_block, kv_stride_h, kv_stride_t;  /* K and V pools (elements) */
    int64_t sc_stride_block, sc_stride_h;               /* scale pools (floats); token stride 1 */
    int64_t q_stride_b, q_stride_h;
    int64_t o_stride_b, o_stride_h;
    float softmax_scale;         /* <= 0 selects 1/sqrt(D) */
} kvd_paged_desc;

size_t kvd_paged_workspace_size(const kvd_paged_desc* desc);

/* Decode over a paged cache; workspace rules as for kvd_decode_launch. */
cudaError_t kvd_paged_decode_launch(const kvd_paged_desc* desc,
                                    const void* Q, const int8_t* K_pool, const int8_t* V_pool,
                                    const float* k_scale_pool, const float* v_scale_pool, void* out,
                                    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Quantise-on-append into a paged cache: the rule and the seq_lens update of
 * kvd_append_int8_launch; token seq_lens[b] goes to the block the table names
 * for it. A sequence already holding max_blocks_per_seq*block_size tokens is
 * left unchanged (KVD_STATUS_CACHE_FULL); an out-of-range block id writes
 * nothing and leaves the length unchanged (KVD_STATUS_BAD_BLOCK). Reads the
 * batch/head/block/stride fields of `desc`; q/o strides and flags are unused. */
cudaError_t kvd_paged_append_int8_launch(const kvd_paged_desc* desc,
                                         const float* k_new, const float* v_new,
                                         int64_t new_stride_b, int64_t new_stride_h,
                                         int8_t* K_pool, int8_t* V_pool,
                                         float* k_scale_pool, float* v_scale_pool,
                                         int32_t* seq_lens, cudaStream_t stream);

/* Log-sum-exp combine of `num_parts` partial-record arrays, each [num_heads]
 * records of KVD_PARTIAL_STRIDE(head_dim) floats, part p starting at
 * parts + p*part_stride. Writes normalised rows out[h*out_stride + d] (fp32,
 * or bf16/fp16 with KVD_FLAG_OUT_*), or combined records when flags has
 * KVD_FLAG_PARTIAL_OUT. Used after gathering per-GPU partials of a sequence
 * split across GPUs. */
cudaError_t kvd_combine_launch(const float* parts, int num_parts, int64_t part_stride,
                               int num_heads, int head_dim, void* out, int64_t out_stride,
                               uint32_t flags, cudaStream_t stream);

/* Quantise-on-append: for every (b, h), quantise the new fp32 K and V rows
 * (k_new/v_new + b*new_stride_b + h*new_stride_h, D floats each) with the
 * symmetric per-token INT8 rule (scale = max|x|/127 in IEEE fp32,
 * code = clamp(round-half-even(x/scale), -127, 127); all-zero row -> scale 0,
 * codes 0), write codes at token seq_lens[b] of the cache and its scale, then
 * increment seq_lens[b]. A sequence already at `capacity` is left unchanged
 * and the device status word records KVD_STATUS_CACHE_FULL. */
typedef struct kvd_append_desc {
    int32_t batch, num_kv_heads, head_dim, capacity;
    int64_t kv_stride_b, kv_stride_h;   /* cache strides (elements) */
    int64_t sc_stride_b, sc_stride_h;
    int64_t new_stride_b, new_stride_h; /* k_new / v_new strides (floats) */
} kvd_append_desc;

cudaError_t kvd_append_int8_launch(const kvd_append_desc* desc,
                                   const float* k_new, const float* v_new,
                                   int8_t* K, int8_t* V, float* k_scale, float* v_scale,
                                   int32_t* seq_lens, cudaStream_t stream);

/* No counterpart in the reference. kvd_append_int8_launch followed by
 * kvd_decode_launch in one decode launch: the new token of every (b, kv head)
 * (k_new/v_new + b*new_stride_b + h*new_stride_h, D floats each) is quantised
 * with the same rule into position desc->seq_lens[b] of the cache, the decode
 * attends over seq_lens[b] + 1 tokens including it, and seq_lens is then
 * incremented (a sequence already at max_seq_len is left unchanged and
 * records KVD_STATUS_CACHE_FULL). desc->seq_lens is required and is written.
 * Results, cache contents and lengths are identical to the two separate calls.
 * The fusion runs on the tensor-core kernel (head_dim 128, groups 1/2/4/8/16,
 * B <= 4096, a workspace of at least kvd_workspace_size(desc)); other shapes
 * run the two steps as two launches. */
cudaError_t kvd_append_decode_launch(const kvd_decode_desc* desc,
                                     const float* k_new, const float* v_new,
                                     int64_t new_stride_b, int64_t new_stride_h,
                                     const void* Q, int8_t* K, int8_t* V, float* k_scale, float* v_scale,
                                     void* out, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* ------------------------------------------------------------------------ */
/* Causal prefill over the INT8 cache (no reference counterpart: the         */
/* reference's prefill attention, attention/, is fp32 with no KV cache)      */
/* ------------------------------------------------------------------------ */

/* The prompt's K/V are already in the cache (quantised by the append or row
 * kernels): sequence b holds seq_lens[b] tokens and its queries are the last
 * q_lens[b] of them (q_lens[b] <= seq_lens[b]). Query i sits at position
 * seq_lens[b] - q_lens[b] + i and attends to tokens [0, position]:
 *   out[b][h][i] = softmax_t((q . K[t]) * ks[t] * scale) . (V[t] * vs[t]), t <= position.
 * Query rows i >= q_lens[b], and rows whose position would be negative (more
 * queries than tokens), are written as 0. */
typedef struct kvd_prefill_desc {
    int32_t batch, num_q_heads, num_kv_heads, head_dim;
    int32_t max_seq_len;      /* cache capacity per sequence */
    int32_t max_queries;      /* query rows per (b, head) in Q and out */
    uint32_t flags;           /* KVD_FLAG_Q_*, KVD_FLAG_OUT_* */
    const int32_t* seq_lens;  /* device [B] or NULL (max_seq_len each) */
    const int32_t* q_lens;    /* device [B] or NULL (max_queries each) */
    int64_t kv_stride_b, kv_stride_h;          /* token stride D */
    int64_t sc_stride_b, sc_stride_h;          /* token stride 1 */
    int64_t q_stride_b, q_stride_h, q_stride_t;
    int64_t o_stride_b, o_stride_h, o_stride_t;
    float softmax_scale;      /* <= 0 selects 1/sqrt(D) */
} kvd_prefill_desc;

size_t kvd_prefill_workspace_size(const kvd_prefill_desc* desc);
cudaError_t kvd_prefill_launch(const kvd_prefill_desc* desc, const void* Q, const int8_t* K, const int8_t* V,
                               const float* k_scale, const float* v_scale, void* out,
                               void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Quantise `rows` contiguous fp32 rows of `dim` values (row stride x_stride
 * floats) to codes (row stride code_stride bytes) and one scale per row, with
 * the same rule as kvd_append_int8_launch. */
cudaError_t kvd_quantize_rows_launch(const float* x, int64_t rows, int dim, int64_t x_stride,
                                     int8_t* codes, int64_t code_stride, float* scales,
                                     cudaStream_t stream);

/* ------------------------------------------------------------------------ */
/* Multi-GPU sequence split (no reference counterpart: the reference is      */
/* single-GPU). One process or host thread per GPU.                           */
/* ------------------------------------------------------------------------ */

/* NCCL communicator helpers. NCCL is loaded at run time (the copy already in
 * the process if there is one, else libnccl.so.2); a caller may also pass a
 * communicator of its own (an ncclComm_t) to the decode below. The id is the
 * 128-byte ncclUniqueId; rank 0 makes it and the caller broadcasts it. Return
 * values are ncclResult_t codes (0 = success). */
int kvd_mgpu_get_unique_id(unsigned char* id /* [128] */);
int kvd_mgpu_comm_init(void** comm, int nranks, int rank, const unsigned char* id /* [128] */);
int kvd_mgpu_comm_destroy(void* comm);

/* Sequence split over NCCL: this rank's K/V/scales hold its own token range of
 * every sequence (a cache whose capacity is the range length; desc->seq_lens
 * counts this rank's tokens, or NULL for max_seq_len each). The rank decodes
 * its range into partial records, all-gathers the records of all `nranks`
 * ranks over `comm` and merges them into normalised rows `out` (the same on
 * every rank; typed per KVD_FLAG_OUT_*). Every rank must call it with the same
 * batch, heads and head_dim, in the same order. NCCL errors return
 * cudaErrorUnknown; a missing NCCL returns cudaErrorSharedObjectInitFailed. */
size_t kvd_mgpu_seq_split_workspace_size(const kvd_decode_desc* desc, int nranks);
cudaError_t kvd_mgpu_seq_split_decode(const kvd_decode_desc* desc,
                                      const void* Q, const int8_t* K, const int8_t* V,
                                      const float* k_scale, const float* v_scale, void* out,
                                      void* workspace, size_t workspace_bytes,
                                      void* comm, int nranks, cudaStream_t stream);

/* The same sequence split with the record exchange done by the library's own
 * kernel over NVLink instead of NCCL: one kernel merges this rank's split
 * records of each row, stores the merged record straight into every rank's
 * gather buffer (CUDA IPC mappings of peer memory) as 8-byte words that carry
 * the call's epoch (so no fence or flag follows the stores), waits for every
 * rank's record of its rows (bounded: a rank that never arrives turns into
 * KVD_STATUS_WAIT_TIMEOUT after 2 s) and merges them into output rows. For a
 * dense batch with up to 4 query heads per KV head and head_dim 128 the
 * decode writes its split records in the same tagged form and the exchange
 * kernel runs beside it, merging each row as soon as its records are there;
 * otherwise it starts when the decode has completed. The exchange kernel
 * never runs more CTAs than fit on the GPU at once, so any batch size
 * completes. kvd_mgpu_p2p_create is collective (every rank calls it with the
 * same sizes): it allocates the exchange buffers (cudaMalloc) and swaps IPC
 * handles once over `comm`, which must outlive the context. Up to 8 ranks,
 * head_dim a multiple of 4 and at most 256. Every rank must make the same
 * sequence of decode calls.
 *
 * After a call that recorded KVD_STATUS_WAIT_TIMEOUT (a rank missed a call or
 * stalled), the rows of the timed-out CTAs are not written and the ranks' call
 * counts no longer agree: every later call would pair records of different
 * steps. Call kvd_mgpu_p2p_reset on every rank (collective over `comm`; it
 * synchronises the device, clears the exchange state between two barriers)
 * before the next decode, or destroy and recreate the context. */
typedef struct kvd_mgpu_p2p kvd_mgpu_p2p;
cudaError_t kvd_mgpu_p2p_create(kvd_mgpu_p2p** ctx, int batch, int num_q_heads, int head_dim,
                                void* comm, int nranks, int rank);
cudaError_t kvd_mgpu_p2p_destroy(kvd_mgpu_p2p* ctx);
cudaError_t kvd_mgpu_p2p_reset(kvd_mgpu_p2p* ctx, cudaStream_t stream);

/* The same exchange for ONE process (or host thread) driving several GPUs: the
 * contexts of all `nranks` ranks are made at once, rank r's on device
 * devices[r], and linked by direct peer pointers (peer access is enabled
 * between distinct devices; no IPC, no NCCL). ctxs[r] is used with
 * kvd_mgpu_p2p_seq_split_decode while devices[r] is the current device (any
 * other current device returns cudaErrorInvalidDevice); the
 * ranks' calls must run concurrently (e.g. one stream per GPU, launched from
 * one thread), since each waits for the others' records (bounded, as above).
 * kvd_mgpu_p2p_reset on a group context needs no communicator: the caller
 * resets every rank's context with no decode in flight. Destroy each context. */
cudaError_t kvd_mgpu_p2p_create_group(kvd_mgpu_p2p** ctxs, int nranks, const int* devices, int batch,
                                      int num_q_heads, int head_dim);
size_t kvd_mgpu_p2p_workspace_size(const kvd_decode_desc* desc);
cudaError_t kvd_mgpu_p2p_seq_split_decode(kvd_mgpu_p2p* ctx, const kvd_decode_desc* desc,
                                          const void* Q, const int8_t* K, const int8_t* V,
                                          const float* k_scale, const float* v_scale, void* out,
                                          void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Device status word: kernels record bounded-wait timeouts, cache overflow
 * and bad block ids (KVD_STATUS_BAD_BLOCK, above) here instead of trapping. kvd_device_status synchronises the current device,
 * reads the word, clears it and returns it through *status. */
#define KVD_STATUS_OK 0
#define KVD_STATUS_WAIT_TIMEOUT 1
#define KVD_STATUS_CACHE_FULL 2
cudaError_t kvd_device_status(int32_t* status);

/* Number of kernel launches issued by the most recent kvd_decode_launch /
 * kv_int8_*_launch / solve call on this host thread (for launch accounting). */
int kvd_last_launch_count(void);

int kvd_abi_version(void);

/* cudaGetErrorString of the CUDA runtime linked into this library. */
const char* kvd_error_string(int error);

#ifdef __cplusplus
}
#endif
#endif /* KVDECODE_H */
