/* A plain C11 host program using libkvdecode_b200.so the way the reference's
 * callers use the entry points of its kv_cache/ files: include the header, link the
 * library, call `solve` and `kv_int8_split_launch` with device pointers.
 * Built with gcc (not nvcc) by tests/test_c_host.py, so it also shows that
 * include/kvdecode.h is valid C.
 *
 *   c_host_example args          no GPU needed: argument errors and ABI version
 *   c_host_example run H S D     the reference's self-test inputs
 *                                (kv_cache/KV_int8_split_optimized.cu:473-486)
 *                                through solve and kv_int8_split_launch, checked
 *                                against a double-precision host loop with the
 *                                reference's tolerance, max abs err <= 1e-4
 *                                (KV_int8_split_optimized.cu:535)
 * Exit status 0 on success. */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "kvdecode.h"

static int check_args(void) {
    int fails = 0;
    float* dummy = (float*)(uintptr_t)256;
    /* KV_int8_split_optimized.cu:272-273: a null pointer or a non-positive size */
    if (kv_int8_split_launch(NULL, (const int8_t*)dummy, (const int8_t*)dummy, dummy, dummy, dummy, 4, 128, 64,
                             dummy, 0) != cudaErrorInvalidValue)
        ++fails;
    if (kv_int8_simple_launch(dummy, (const int8_t*)dummy, (const int8_t*)dummy, dummy, dummy, dummy, 0, 128, 64,
                              dummy, 0) != cudaErrorInvalidValue)
        ++fails;
    if (kvd_abi_version() != KVD_ABI_VERSION) ++fails;
    printf("args: %s\n", fails ? "FAILED" : "ok");
    return fails;
}

/* out[h][d] = sum_t softmax_t(q_h . K[h,t] * ks[h,t] / sqrt(D)) * V[h,t,d] * vs[h,t] */
static void host_attention(const float* q, const int8_t* k, const int8_t* v, const float* ks, const float* vs,
                           double* out, int H, int S, int D) {
    double* s = (double*)malloc(sizeof(double) * (size_t)S);
    for (int h = 0; h < H; ++h) {
        double mx = -INFINITY, l = 0.0;
        for (int t = 0; t < S; ++t) {
            double dot = 0.0;
            for (int d = 0; d < D; ++d) dot += (double)q[h * D + d] * (double)k[((size_t)h * S + t) * D + d];
            s[t] = dot * ks[h * S + t] / sqrt((double)D);
            if (s[t] > mx) mx = s[t];
        }
        for (int t = 0; t < S; ++t) {
            s[t] = exp(s[t] - mx);
            l += s[t];
        }
        for (int d = 0; d < D; ++d) {
            double o = 0.0;
            for (int t = 0; t < S; ++t) o += s[t] * (double)v[((size_t)h * S + t) * D + d] * vs[h * S + t];
            out[h * D + d] = o / l;
        }
    }
    free(s);
}

#define CK(x)                                                                              \
    do {                                                                                   \
        cudaError_t e_ = (x);                                                              \
        if (e_ != cudaSuccess) {                                                           \
            fprintf(stderr, "%s failed: %s\n", #x, cudaGetErrorString(e_));                \
            return 2;                                                                      \
        }                                                                                  \
    } while (0)

static int run(int H, int S, int D) {
    const size_t nq = (size_t)H * D, nkv = (size_t)H * S * D, ns = (size_t)H * S;
    float* q = (float*)malloc(nq * 4);
    int8_t* k = (int8_t*)malloc(nkv);
    int8_t* v = (int8_t*)malloc(nkv);
    float* ks = (float*)malloc(ns * 4);
    float* vs = (float*)malloc(ns * 4);
    float* out = (float*)malloc(nq * 4);
    double* ref = (double*)malloc(nq * 8);
    /* the reference's deterministic self-test pattern */
    for (size_t i = 0; i < nq; ++i) q[i] = (float)((int)(i % 17) - 8) * 0.125f;
    for (size_t i = 0; i < nkv; ++i) {
        k[i] = (int8_t)((int)(i % 23) - 11);
        v[i] = (int8_t)((int)((i * 3) % 29) - 14);
    }
    for (size_t i = 0; i < ns; ++i) {
        ks[i] = 0.015625f + (float)(i % 5) * 0.001f;
        vs[i] = 0.03125f + (float)(i % 7) * 0.001f;
    }
    host_attention(q, k, v, ks, vs, ref, H, S, D);
    float *dq, *dks, *dvs, *dout, *dS;
    int8_t *dk, *dv;
    CK(cudaMalloc((void**)&dq, nq * 4));
    CK(cudaMalloc((void**)&dk, nkv));
    CK(cudaMalloc((void**)&dv, nkv));
    CK(cudaMalloc((void**)&dks, ns * 4));
    CK(cudaMalloc((void**)&dvs, ns * 4));
    CK(cudaMalloc((void**)&dout, nq * 4));
    CK(cudaMalloc((void**)&dS, ns * 4));
    CK(cudaMemcpy(dq, q, nq * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dk, k, nkv, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dv, v, nkv, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dks, ks, ns * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dvs, vs, ns * 4, cudaMemcpyHostToDevice));
    int fails = 0;
    for (int entry = 0; entry < 2; ++entry) {
        CK(cudaMemset(dout, 0xFF, nq * 4));
        if (entry == 0) {
            solve(dq, dk, dv, dks, dvs, dout, H, S, D);
        } else {
            cudaStream_t st;
            CK(cudaStreamCreate(&st));
            CK(kv_int8_split_launch(dq, dk, dv, dks, dvs, dout, H, S, D, dS, st));
            CK(cudaStreamSynchronize(st));
            CK(cudaStreamDestroy(st));
        }
        CK(cudaDeviceSynchronize());
        CK(cudaMemcpy(out, dout, nq * 4, cudaMemcpyDeviceToHost));
        double worst = 0.0;
        for (size_t i = 0; i < nq; ++i) {
            const double err = fabs((double)out[i] - ref[i]);
            if (!(err <= worst)) worst = isnan(err) ? INFINITY : err;
        }
        printf("%s H=%d S=%d D=%d: max abs err %.3g\n", entry == 0 ? "solve" : "kv_int8_split_launch", H, S, D,
               worst);
        if (!(worst <= 1e-4)) ++fails;
    }
    cudaFree(dq); cudaFree(dk); cudaFree(dv); cudaFree(dks); cudaFree(dvs); cudaFree(dout); cudaFree(dS);
    free(q); free(k); free(v); free(ks); free(vs); free(out); free(ref);
    return fails;
}

int main(int argc, char** argv) {
    if (argc >= 2 && strcmp(argv[1], "args") == 0) return check_args() ? 1 : 0;
    if (argc >= 5 && strcmp(argv[1], "run") == 0) return run(atoi(argv[2]), atoi(argv[3]), atoi(argv[4])) ? 1 : 0;
    fprintf(stderr, "usage: %s args | run H S D\n", argv[0]);
    return 2;
}
