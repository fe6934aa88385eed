// Test support: kvd_decode_launch_noalloc across a cudaDeviceReset, in a
// process of its own (the reset destroys every allocation of the process's
// primary context, so it must not run inside the test runner).
//
// Round r = 0, 1: allocate and fill a decode's inputs, decode once through
// kvd_decode_launch (a workspace from cudaMalloc) and twice through
// kvd_decode_launch_noalloc, compare; then cudaDeviceReset. Round 1 runs in a
// new primary context: the library must look the scratch array's address up
// again instead of reusing round 0's. Prints the largest difference per round
// and exits 0 only if every output matches the workspace entry's within
// 2e-5 + 1e-4 |ref|.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include <cuda_runtime.h>

#include "kvdecode.h"

#define CHECK(x)                                                                                 \
    do {                                                                                         \
        cudaError_t e_ = (x);                                                                    \
        if (e_ != cudaSuccess) {                                                                 \
            std::fprintf(stderr, "%s:%d %s: %s\n", __FILE__, __LINE__, #x, cudaGetErrorString(e_)); \
            return 2;                                                                            \
        }                                                                                        \
    } while (0)

int main() {
    const int B = 2, H = 8, S = 3000, D = 128;  // dense MHA on the tensor-core kernel, split records in scratch
    const size_t nq = size_t(B) * H * D, nkv = size_t(B) * H * S * D, ns = size_t(B) * H * S;
    std::vector<float> q(nq), ks(ns), vs(ns);
    std::vector<signed char> k(nkv), v(nkv);
    unsigned s = 12345u;
    auto rnd = [&s]() { s = s * 1664525u + 1013904223u; return static_cast<int>(s >> 8); };
    for (auto& x : q) x = static_cast<float>(rnd() % 2001 - 1000) / 1000.0f;
    for (auto& x : k) x = static_cast<signed char>(rnd() % 255 - 127);
    for (auto& x : v) x = static_cast<signed char>(rnd() % 255 - 127);
    for (auto& x : ks) x = 0.005f + 0.02f * static_cast<float>(rnd() % 1000) / 1000.0f;
    for (auto& x : vs) x = 0.005f + 0.02f * static_cast<float>(rnd() % 1000) / 1000.0f;
    kvd_decode_desc d{};
    d.batch = B; d.num_q_heads = H; d.num_kv_heads = H; d.head_dim = D; d.max_seq_len = S;
    d.kv_stride_b = int64_t(H) * S * D; d.kv_stride_h = int64_t(S) * D;
    d.sc_stride_b = int64_t(H) * S; d.sc_stride_h = S;
    d.q_stride_b = H * D; d.q_stride_h = D; d.o_stride_b = H * D; d.o_stride_h = D;
    int failures = 0;
    for (int round = 0; round < 2; ++round) {
        float *dq, *dks, *dvs, *dref, *dout;
        int8_t *dk, *dv;
        void* ws;
        CHECK(cudaMalloc(&dq, nq * 4));
        CHECK(cudaMalloc(&dk, nkv));
        CHECK(cudaMalloc(&dv, nkv));
        CHECK(cudaMalloc(&dks, ns * 4));
        CHECK(cudaMalloc(&dvs, ns * 4));
        CHECK(cudaMalloc(&dref, nq * 4));
        CHECK(cudaMalloc(&dout, nq * 4));
        const size_t wsb = kvd_workspace_size(&d);
        CHECK(cudaMalloc(&ws, wsb > 0 ? wsb : 1));
        CHECK(cudaMemcpy(dq, q.data(), nq * 4, cudaMemcpyHostToDevice));
        CHECK(cudaMemcpy(dk, k.data(), nkv, cudaMemcpyHostToDevice));
        CHECK(cudaMemcpy(dv, v.data(), nkv, cudaMemcpyHostToDevice));
        CHECK(cudaMemcpy(dks, ks.data(), ns * 4, cudaMemcpyHostToDevice));
        CHECK(cudaMemcpy(dvs, vs.data(), ns * 4, cudaMemcpyHostToDevice));
        CHECK(kvd_decode_launch(&d, dq, dk, dv, dks, dvs, dref, ws, wsb, nullptr));
        std::vector<float> ref(nq), out(nq);
        CHECK(cudaMemcpy(ref.data(), dref, nq * 4, cudaMemcpyDeviceToHost));
        for (int call = 0; call < 2; ++call) {
            CHECK(cudaMemset(dout, 0xFF, nq * 4));
            CHECK(kvd_decode_launch_noalloc(&d, dq, dk, dv, dks, dvs, dout, nullptr));
            CHECK(cudaMemcpy(out.data(), dout, nq * 4, cudaMemcpyDeviceToHost));
            double worst = 0.0;
            for (size_t i = 0; i < nq; ++i) {
                const double err = std::fabs(double(out[i]) - double(ref[i]));
                if (!(err <= 2e-5 + 1e-4 * std::fabs(double(ref[i])))) ++failures;
                if (err > worst || std::isnan(err)) worst = std::isnan(err) ? INFINITY : err;
            }
            std::printf("round %d call %d: max |noalloc - workspace entry| = %.3g\n", round, call, worst);
        }
        int32_t st = -1;
        CHECK(kvd_device_status(&st));
        if (st != KVD_STATUS_OK) ++failures;
        CHECK(cudaDeviceReset());  // a new primary context for the next round
    }
    std::printf(failures ? "FAILED (%d)\n" : "ok\n", failures);
    return failures ? 1 : 0;
}
