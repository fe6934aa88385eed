/*
 * kvd_oracle.h -- CPU oracle for the INT8 KV-cache decode-attention path.
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py may load this library, and only as
 * the checker or as the timed CPU baseline. The product library
 * (libkvdecode_b200.so) never links, loads or calls it.
 *
 * What it restates (reference = Murmurwkk/cuda-operators):
 *   - kvo_cpu_reference_f32: the fp32 host loop `cpu_reference` of
 *     kv_cache/KV_int8_split_optimized.cu:385-437, same operation order
 *     (fmaf over d, score = dot*k_scale*inv_sqrt_dim, expf(score-max),
 *     prob = score/denom inside the PV loop), parallelised over heads with
 *     OpenMP. This is the CPU baseline ("port").
 *   - kvo_decode_f64: the same mathematics in double precision over the same
 *     INT8 codes and fp32 scales, generalised to batch, grouped-query heads,
 *     ragged lengths and strided caches. This is the correctness oracle.
 *   - kvo_quantize_row: the symmetric per-token INT8 quantiser of the
 *     north-star spec (the reference ships no quantiser, new_kvint8.cu:83-84):
 *     amax = max|x| (fp32), scale = amax/127 (IEEE fp32 division),
 *     code = clamp(rint(x/scale), -127, 127) (round half to even),
 *     amax == 0 -> scale 0 and all codes 0.
 *   - kvo_partials_f64 / kvo_combine_f64: the split-KV (m, l, o) partial and its
 *     log-sum-exp combine, used to check sequence splitting on the host.
 *   - kvo_fill_reference_pattern: the deterministic inputs of the reference's
 *     only KV test, KV_int8_split_optimized.cu:473-486.
 */
#ifndef KVD_ORACLE_H
#define KVD_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Strided cache layout, host pointers. Token stride inside a head is head_dim
 * elements for K/V and 1 for scales. Strides are in elements. */
typedef struct kvo_layout {
    int32_t batch;
    int32_t num_q_heads;
    int32_t num_kv_heads;
    int32_t head_dim;
    int32_t max_seq_len;          /* length used when seq_lens == NULL */
    const int32_t* seq_lens;      /* host array [batch] or NULL */
    int64_t kv_stride_b, kv_stride_h;
    int64_t sc_stride_b, sc_stride_h;
    int64_t q_stride_b, q_stride_h;
    int64_t o_stride_b, o_stride_h;
    double softmax_scale;         /* <= 0 means 1/sqrt(head_dim) */
} kvo_layout;

/* Quantiser spec (one row of `dim` values). */
void kvo_quantize_row(const float* x, int dim, int8_t* codes, float* scale);
/* rows x dim, rows contiguous; OpenMP over rows. */
void kvo_quantize_rows(const float* x, int64_t rows, int dim, int8_t* codes, float* scales);

/* fp32 restatement of the reference cpu_reference (dense [H,S,D]). */
void kvo_cpu_reference_f32(const float* Q, const int8_t* K, const int8_t* V,
                           const float* k_scale, const float* v_scale, float* out,
                           int num_heads, int seq_len, int head_dim, int num_threads);

/* FP64 oracle; out is double [batch][num_q_heads][head_dim] (dense). */
void kvo_decode_f64(const kvo_layout* L, const float* Q, const int8_t* K, const int8_t* V,
                    const float* k_scale, const float* v_scale, double* out, int num_threads);

/* FP64 causal prefill (no reference counterpart): q [B][Hq][Lq][D] fp32 dense,
 * K/V [B][Hkv][cap][D], scales [B][Hkv][cap]. seq_lens[b] (or cap) tokens are in
 * the cache; the queries are its last q_lens[b] (or Lq) tokens, so query i sits
 * at position seq_lens[b] - q_lens[b] + i and attends to tokens [0, position].
 * Rows i >= q_lens[b] are 0. out double [B][Hq][Lq][D]. */
void kvo_prefill_f64(int B, int Hq, int Hkv, int Lq, int cap, int D, const int32_t* seq_lens,
                     const int32_t* q_lens, const float* Q, const int8_t* K, const int8_t* V,
                     const float* k_scale, const float* v_scale, double softmax_scale, double* out);

/* FP64 split partial over tokens [t_begin, t_end) of every head (clipped to the
 * head's length). Record per (b, hq): m (natural-log domain max of scores),
 * l = sum exp(s - m), o[d] = sum exp(s - m) v[d] (unnormalised).
 * part is double [batch*num_q_heads][2 + head_dim]. Empty range -> m=-inf, l=0, o=0. */
void kvo_partials_f64(const kvo_layout* L, const float* Q, const int8_t* K, const int8_t* V,
                      const float* k_scale, const float* v_scale,
                      int32_t t_begin, int32_t t_end, double* part);

/* Combine `nparts` partial arrays (each [heads][2+dim], contiguous, parts back to
 * back) into a normalised output double [heads][dim]. */
void kvo_combine_f64(const double* parts, int nparts, int heads, int dim, double* out);

/* |a - r| <= atol + rtol*|r|; NaN/Inf in either fails. Returns the number of bad
 * entries; writes the max absolute error and max normalised error. */
int64_t kvo_check(const float* actual, const double* ref, int64_t n, double atol, double rtol,
                  double* max_abs, double* max_norm);

/* Deterministic inputs of KV_int8_split_optimized.cu:473-486. */
void kvo_fill_reference_pattern(float* Q, int8_t* K, int8_t* V, float* k_scale, float* v_scale,
                                int num_heads, int seq_len, int head_dim);

#ifdef __cplusplus
}
#endif
#endif /* KVD_ORACLE_H */
