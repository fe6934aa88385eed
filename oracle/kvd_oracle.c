/*
 * kvd_oracle.c -- CPU oracle for the INT8 KV-cache decode-attention path.
 *
 * TEST INFRASTRUCTURE ONLY (see kvd_oracle.h): the product never links it.
 * Compile without -ffast-math and with -ffp-contract=off so every fp32 step is
 * the IEEE operation written here (the quantiser must be bit-exact and the
 * fp32 port must reproduce the reference host loop's rounding).
 */
#include "kvd_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Quantiser spec; the reference has no quantiser (kv_cache/new_kvint8.cu:83-84),
 * so this follows the north-star formula: scale = max|x| / 127,
 * code = clamp(round-half-even(x / scale), -127, 127). The NaN behaviour falls
 * out of fmaxf/fminf (a NaN operand is ignored) and is mirrored on the device. */
void kvo_quantize_row(const float* x, int dim, int8_t* codes, float* scale) {
    float amax = 0.0f;
    for (int d = 0; d < dim; ++d) amax = fmaxf(amax, fabsf(x[d]));
    if (amax == 0.0f) {
        *scale = 0.0f;
        memset(codes, 0, (size_t)dim);
        return;
    }
    const float s = amax / 127.0f;
    for (int d = 0; d < dim; ++d) {
        float r = rintf(x[d] / s);
        r = fminf(fmaxf(r, -127.0f), 127.0f);
        codes[d] = (int8_t)r;
    }
    *scale = s;
}

void kvo_quantize_rows(const float* x, int64_t rows, int dim, int8_t* codes, float* scales) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
        kvo_quantize_row(x + r * dim, dim, codes + r * dim, scales + r);
}

/* Restatement of cpu_reference, kv_cache/KV_int8_split_optimized.cu:385-437.
 * Same order of fp32 operations per head; heads are independent, so running
 * them on several threads does not change any result. */
static void cpu_reference_head(const float* Q, const int8_t* K, const int8_t* V,
                               const float* k_scale, const float* v_scale, float* out,
                               int h, int seq_len, int head_dim, float* scores) {
    const float inv_sqrt_dim = 1.0f / sqrtf((float)head_dim);
    float max_score = -FLT_MAX;
    for (int t = 0; t < seq_len; ++t) {
        float dot = 0.0f;
        for (int d = 0; d < head_dim; ++d) {
            const int64_t q_idx = (int64_t)h * head_dim + d;
            const int64_t kv_idx = ((int64_t)h * seq_len + t) * head_dim + d;
            dot = fmaf(Q[q_idx], (float)K[kv_idx], dot);
        }
        const float score = dot * k_scale[(int64_t)h * seq_len + t] * inv_sqrt_dim;
        scores[t] = score;
        max_score = fmaxf(max_score, score);
    }
    float denom = 0.0f;
    for (int t = 0; t < seq_len; ++t) {
        scores[t] = expf(scores[t] - max_score);
        denom += scores[t];
    }
    for (int d = 0; d < head_dim; ++d) {
        float sum = 0.0f;
        for (int t = 0; t < seq_len; ++t) {
            const int64_t kv_idx = ((int64_t)h * seq_len + t) * head_dim + d;
            const float prob = scores[t] / denom;
            const float v = (float)V[kv_idx] * v_scale[(int64_t)h * seq_len + t];
            sum = fmaf(prob, v, sum);
        }
        out[(int64_t)h * head_dim + d] = sum;
    }
}

void kvo_cpu_reference_f32(const float* Q, const int8_t* K, const int8_t* V,
                           const float* k_scale, const float* v_scale, float* out,
                           int num_heads, int seq_len, int head_dim, int num_threads) {
#ifdef _OPENMP
    if (num_threads <= 0) num_threads = omp_get_max_threads();
#else
    (void)num_threads;
#endif
#pragma omp parallel num_threads(num_threads)
    {
        float* scores = (float*)malloc(sizeof(float) * (size_t)(seq_len > 0 ? seq_len : 1));
#pragma omp for schedule(dynamic, 1)
        for (int h = 0; h < num_heads; ++h)
            cpu_reference_head(Q, K, V, k_scale, v_scale, out, h, seq_len, head_dim, scores);
        free(scores);
    }
}

static int layout_len(const kvo_layout* L, int b) {
    return L->seq_lens ? L->seq_lens[b] : L->max_seq_len;
}

static double layout_scale(const kvo_layout* L) {
    return L->softmax_scale > 0.0 ? L->softmax_scale : 1.0 / sqrt((double)L->head_dim);
}

/* Scores of one (b, hq) over tokens [t0, t1) in double: s_t = (q . k_t) * ks_t * scale. */
static void head_scores_f64(const kvo_layout* L, const float* Q, const int8_t* K,
                            const float* k_scale, int b, int hq, int t0, int t1, double* s) {
    const int group = L->num_q_heads / L->num_kv_heads;
    const int hk = hq / group;
    const int D = L->head_dim;
    const double scale = layout_scale(L);
    const float* q = Q + (int64_t)b * L->q_stride_b + (int64_t)hq * L->q_stride_h;
    const int8_t* kh = K + (int64_t)b * L->kv_stride_b + (int64_t)hk * L->kv_stride_h;
    const float* ksh = k_scale + (int64_t)b * L->sc_stride_b + (int64_t)hk * L->sc_stride_h;
    for (int t = t0; t < t1; ++t) {
        const int8_t* kr = kh + (int64_t)t * D;
        double dot = 0.0;
        for (int d = 0; d < D; ++d) dot += (double)q[d] * (double)kr[d];
        s[t - t0] = dot * (double)ksh[t] * scale;
    }
}

/* Unnormalised (m, l, o) of one (b, hq) over [t0, t1). */
static void head_partial_f64(const kvo_layout* L, const float* Q, const int8_t* K,
                             const int8_t* V, const float* k_scale, const float* v_scale,
                             int b, int hq, int t0, int t1, double* rec, double* s) {
    const int group = L->num_q_heads / L->num_kv_heads;
    const int hk = hq / group;
    const int D = L->head_dim;
    double* o = rec + 2;
    for (int d = 0; d < D; ++d) o[d] = 0.0;
    if (t1 <= t0) {
        rec[0] = -INFINITY;
        rec[1] = 0.0;
        return;
    }
    head_scores_f64(L, Q, K, k_scale, b, hq, t0, t1, s);
    double m = -INFINITY;
    for (int t = 0; t < t1 - t0; ++t) m = s[t] > m ? s[t] : m;
    const int8_t* vh = V + (int64_t)b * L->kv_stride_b + (int64_t)hk * L->kv_stride_h;
    const float* vsh = v_scale + (int64_t)b * L->sc_stride_b + (int64_t)hk * L->sc_stride_h;
    double l = 0.0;
    for (int t = t0; t < t1; ++t) {
        const double p = exp(s[t - t0] - m);
        l += p;
        const int8_t* vr = vh + (int64_t)t * D;
        const double w = p * (double)vsh[t];
        for (int d = 0; d < D; ++d) o[d] += w * (double)vr[d];
    }
    rec[0] = m;
    rec[1] = l;
}

void kvo_decode_f64(const kvo_layout* L, const float* Q, const int8_t* K, const int8_t* V,
                    const float* k_scale, const float* v_scale, double* out, int num_threads) {
#ifdef _OPENMP
    if (num_threads <= 0) num_threads = omp_get_max_threads();
#else
    (void)num_threads;
#endif
    const int B = L->batch, Hq = L->num_q_heads, D = L->head_dim;
    int max_len = 1;
    for (int b = 0; b < B; ++b) max_len = layout_len(L, b) > max_len ? layout_len(L, b) : max_len;
#pragma omp parallel num_threads(num_threads)
    {
        double* s = (double*)malloc(sizeof(double) * (size_t)max_len);
        double* rec = (double*)malloc(sizeof(double) * (size_t)(D + 2));
#pragma omp for schedule(dynamic, 1)
        for (int64_t u = 0; u < (int64_t)B * Hq; ++u) {
            const int b = (int)(u / Hq), hq = (int)(u % Hq);
            head_partial_f64(L, Q, K, V, k_scale, v_scale, b, hq, 0, layout_len(L, b), rec, s);
            double* o = out + u * D;
            const double l = rec[1];
            for (int d = 0; d < D; ++d) o[d] = l > 0.0 ? rec[2 + d] / l : 0.0;
        }
        free(rec);
        free(s);
    }
}

void kvo_prefill_f64(int B, int Hq, int Hkv, int Lq, int cap, int D, const int32_t* seq_lens,
                     const int32_t* q_lens, const float* Q, const int8_t* K, const int8_t* V,
                     const float* k_scale, const float* v_scale, double softmax_scale, double* out) {
    kvo_layout L;
    memset(&L, 0, sizeof(L));
    L.batch = B; L.num_q_heads = Hq; L.num_kv_heads = Hkv; L.head_dim = D; L.max_seq_len = cap;
    L.kv_stride_b = (int64_t)Hkv * cap * D; L.kv_stride_h = (int64_t)cap * D;
    L.sc_stride_b = (int64_t)Hkv * cap; L.sc_stride_h = cap;
    L.q_stride_b = (int64_t)Hq * Lq * D; L.q_stride_h = (int64_t)Lq * D;
    L.softmax_scale = softmax_scale;
#pragma omp parallel
    {
        double* s = (double*)malloc(sizeof(double) * (size_t)(cap > 0 ? cap : 1));
        double* rec = (double*)malloc(sizeof(double) * (size_t)(D + 2));
#pragma omp for schedule(dynamic, 1)
        for (int64_t u = 0; u < (int64_t)B * Hq * Lq; ++u) {
            const int i = (int)(u % Lq), hq = (int)((u / Lq) % Hq), b = (int)(u / ((int64_t)Lq * Hq));
            double* o = out + u * D;
            const int ql = q_lens ? q_lens[b] : Lq;
            int len = seq_lens ? seq_lens[b] : cap;
            if (len > cap) len = cap;
            const int pos = len - ql + i;  /* the query's own position */
            if (i >= ql || pos < 0) {
                for (int d = 0; d < D; ++d) o[d] = 0.0;
                continue;
            }
            head_partial_f64(&L, Q + (int64_t)i * D, K, V, k_scale, v_scale, b, hq, 0, pos + 1, rec, s);
            const double l = rec[1];
            for (int d = 0; d < D; ++d) o[d] = l > 0.0 ? rec[2 + d] / l : 0.0;
        }
        free(rec);
        free(s);
    }
}

void kvo_partials_f64(const kvo_layout* L, const float* Q, const int8_t* K, const int8_t* V,
                      const float* k_scale, const float* v_scale,
                      int32_t t_begin, int32_t t_end, double* part) {
    const int B = L->batch, Hq = L->num_q_heads, D = L->head_dim;
    const int span = t_end > t_begin ? t_end - t_begin : 1;
#pragma omp parallel
    {
        double* s = (double*)malloc(sizeof(double) * (size_t)span);
#pragma omp for schedule(dynamic, 1)
        for (int64_t u = 0; u < (int64_t)B * Hq; ++u) {
            const int b = (int)(u / Hq), hq = (int)(u % Hq);
            const int len = layout_len(L, b);
            const int t0 = t_begin < len ? t_begin : len;
            const int t1 = t_end < len ? t_end : len;
            head_partial_f64(L, Q, K, V, k_scale, v_scale, b, hq, t0, t1, part + u * (D + 2), s);
        }
        free(s);
    }
}

void kvo_combine_f64(const double* parts, int nparts, int heads, int dim, double* out) {
    const int64_t rec = dim + 2;
    for (int h = 0; h < heads; ++h) {
        double m = -INFINITY;
        for (int p = 0; p < nparts; ++p) {
            const double mp = parts[((int64_t)p * heads + h) * rec];
            m = mp > m ? mp : m;
        }
        double l = 0.0;
        for (int d = 0; d < dim; ++d) out[(int64_t)h * dim + d] = 0.0;
        if (m == -INFINITY) continue;
        for (int p = 0; p < nparts; ++p) {
            const double* r = parts + ((int64_t)p * heads + h) * rec;
            if (r[0] == -INFINITY) continue;
            const double f = exp(r[0] - m);
            l += r[1] * f;
            for (int d = 0; d < dim; ++d) out[(int64_t)h * dim + d] += r[2 + d] * f;
        }
        for (int d = 0; d < dim; ++d) out[(int64_t)h * dim + d] = l > 0.0 ? out[(int64_t)h * dim + d] / l : 0.0;
    }
}

int64_t kvo_check(const float* actual, const double* ref, int64_t n, double atol, double rtol,
                  double* max_abs, double* max_norm) {
    int64_t bad = 0;
    double ma = 0.0, mn = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        const double a = (double)actual[i], r = ref[i];
        if (!isfinite(a) || !isfinite(r)) {
            ++bad;
            continue;
        }
        const double delta = fabs(a - r);
        const double bound = atol + rtol * fabs(r);
        if (delta > ma) ma = delta;
        if (delta / bound > mn) mn = delta / bound;
        if (delta > bound) ++bad;
    }
    if (max_abs) *max_abs = ma;
    if (max_norm) *max_norm = mn;
    return bad;
}

/* KV_int8_split_optimized.cu:473-486. */
void kvo_fill_reference_pattern(float* Q, int8_t* K, int8_t* V, float* k_scale, float* v_scale,
                                int num_heads, int seq_len, int head_dim) {
    const size_t q_count = (size_t)num_heads * (size_t)head_dim;
    const size_t kv_count = (size_t)num_heads * (size_t)seq_len * (size_t)head_dim;
    const size_t scale_count = (size_t)num_heads * (size_t)seq_len;
    for (size_t i = 0; i < q_count; ++i) Q[i] = (float)((int)(i % 17) - 8) * 0.125f;
    for (size_t i = 0; i < kv_count; ++i) {
        K[i] = (int8_t)((int)(i % 23) - 11);
        V[i] = (int8_t)((int)((i * 3) % 29) - 14);
    }
    for (size_t i = 0; i < scale_count; ++i) {
        k_scale[i] = 0.015625f + (float)(i % 5) * 0.001f;
        v_scale[i] = 0.03125f + (float)(i % 7) * 0.001f;
    }
}
