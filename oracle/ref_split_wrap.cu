// Build glue for the reference's own split kernel file (test infrastructure).
//
// This translation unit contains no reference code: it includes
// kv_cache/KV_int8_split_optimized.cu from the reference checkout (path given
// by -DKVREF_SPLIT_SRC at build time, see oracle/Makefile), renames its
// exported symbols so they cannot clash with the product library, and adds
// plain-pointer entry points around the file's static fp32 host loop
// `cpu_reference` (KV_int8_split_optimized.cu:385-437) so tests and the
// reference leg of bench.py can call it. Only tests/ and bench.py load the
// resulting oracle/_ref/libkvref_split.so.
#define main kvref_split_main
#define solve kvref_split_solve
#define kv_int8_split_launch kvref_split_launch
#include KVREF_SPLIT_SRC
#undef main
#undef solve
#undef kv_int8_split_launch

#include <chrono>
#include <thread>

namespace {
struct CpuJob {
    std::vector<float> Q, ks, vs, out;
    std::vector<int8_t> K, V;
    int H = 0, S = 0, D = 0;
};
}  // namespace

extern "C" void* kvref_cpu_prepare(const float* Q, const int8_t* K, const int8_t* V,
                                   const float* ks, const float* vs, int H, int S, int D) {
    CpuJob* j = new CpuJob;
    const size_t qn = size_t(H) * D, kvn = size_t(H) * S * D, sn = size_t(H) * S;
    j->Q.assign(Q, Q + qn);
    j->K.assign(K, K + kvn);
    j->V.assign(V, V + kvn);
    j->ks.assign(ks, ks + sn);
    j->vs.assign(vs, vs + sn);
    j->out.assign(qn, 0.0f);
    j->H = H; j->S = S; j->D = D;
    return j;
}

extern "C" void kvref_cpu_run(void* job) {
    CpuJob* j = static_cast<CpuJob*>(job);
    cpu_reference(j->Q, j->K, j->V, j->ks, j->vs, j->out, j->H, j->S, j->D);
}

extern "C" void kvref_cpu_output(void* job, float* out) {
    CpuJob* j = static_cast<CpuJob*>(job);
    std::copy(j->out.begin(), j->out.end(), out);
}

extern "C" void kvref_cpu_free(void* job) { delete static_cast<CpuJob*>(job); }

// Runs every job once, each on its own host thread; returns wall seconds.
extern "C" double kvref_cpu_run_parallel(void** jobs, int n) {
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<std::thread> threads;
    threads.reserve(n);
    for (int i = 0; i < n; ++i) threads.emplace_back(kvref_cpu_run, jobs[i]);
    for (auto& t : threads) t.join();
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

// One-shot convenience: the reference host loop on plain pointers.
extern "C" void kvref_cpu_reference(const float* Q, const int8_t* K, const int8_t* V,
                                    const float* ks, const float* vs, float* out,
                                    int H, int S, int D) {
    void* j = kvref_cpu_prepare(Q, K, V, ks, vs, H, S, D);
    kvref_cpu_run(j);
    kvref_cpu_output(j, out);
    kvref_cpu_free(j);
}
