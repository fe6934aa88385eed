// Test support: drives kvd::OrderedWorkspace (cuda-operators_b200/csrc/kvd_workspace.h),
// the stream-ordered scratch owner that restates mur::OrderedWorkspace
// (common/ordered_workspace.cuh:10-58 of the reference), through two decodes
// that share one workspace on two streams.
//
// Owner 1: allocated on stream A, decode on A, handoff(B) -- B now waits for
// A's work through an event -- decode on B into a second output, explicit
// close() (one cudaFreeAsync on B). Owner 2 is moved into a new owner and
// released by the destructor alone. Without the handoff the decode on B would
// overwrite A's split records while A still reads them. Built by
// tests/test_workspace_gpu.py into tests/native/_build, linked against
// libkvdecode_b200.so.
#include <cuda_runtime.h>

#include "kvd_workspace.h"
#include "kvdecode.h"

// result[0..2] = Audit {allocations, free_submissions, cleanup_errors};
// result[3] = 1 if the owner's last stream was B after the handoff;
// result[4] = 1 if a second handoff to the owning stream is a no-op.
// Returns the first CUDA error.
extern "C" int kvd_workspace_probe(const kvd_decode_desc* d, const void* Q, const int8_t* K, const int8_t* V,
                                   const float* ks, const float* vs, void* out_a, void* out_b, void* out_c,
                                   int* result) {
    cudaStream_t a = nullptr, b = nullptr;
    cudaError_t e = cudaStreamCreateWithFlags(&a, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&b, cudaStreamNonBlocking);
    kvd::OrderedWorkspace::Audit audit;
    const size_t bytes = kvd_workspace_size(d);
    if (e == cudaSuccess) {
        kvd::OrderedWorkspace ws(bytes, a, &audit);
        e = ws.status();
        if (e == cudaSuccess) e = kvd_decode_launch(d, Q, K, V, ks, vs, out_a, ws.data(), ws.bytes(), a);
        if (e == cudaSuccess) e = ws.handoff(b);
        result[3] = ws.last_stream() == b ? 1 : 0;
        if (e == cudaSuccess) e = ws.handoff(b);
        result[4] = ws.last_stream() == b ? 1 : 0;
        if (e == cudaSuccess) e = kvd_decode_launch(d, Q, K, V, ks, vs, out_b, ws.data(), ws.bytes(), b);
        const cudaError_t c = ws.close();
        if (e == cudaSuccess) e = c;
    }
    if (e == cudaSuccess) {
        kvd::OrderedWorkspace first(bytes, b, &audit);
        kvd::OrderedWorkspace owner(std::move(first));  // the moved-from owner frees nothing
        e = owner.status();
        if (e == cudaSuccess) e = kvd_decode_launch(d, Q, K, V, ks, vs, out_c, owner.data(), owner.bytes(), b);
    }  // destructor: cudaFreeAsync on b
    if (a) {
        const cudaError_t s = cudaStreamSynchronize(a);
        if (e == cudaSuccess) e = s;
    }
    if (b) {
        const cudaError_t s = cudaStreamSynchronize(b);
        if (e == cudaSuccess) e = s;
    }
    if (a) cudaStreamDestroy(a);
    if (b) cudaStreamDestroy(b);
    result[0] = audit.allocations;
    result[1] = audit.free_submissions;
    result[2] = audit.cleanup_errors;
    return static_cast<int>(e);
}
