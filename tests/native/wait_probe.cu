// Test support: exercises the bounded mbarrier wait of the decode kernels
// (kvd::mbar_wait in cuda-operators_b200/csrc/kvd_common.cuh) on a barrier
// that nothing ever arrives at. The wait must give up after its time limit,
// record KVD_STATUS_WAIT_TIMEOUT and let the kernel return normally, leaving
// the CUDA context usable. Built into tests/native/_build by tests/conftest.py.
#include "kvd_common.cuh"

namespace kvd {
__device__ int32_t g_status = 0;  // this probe library's own status word
}

__global__ void wait_probe_kernel(int32_t* out) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        kvd::mbar_init(&bar, 1);
        kvd::fence_mbar_init();
    }
    __syncthreads();
    const bool completed = kvd::mbar_wait(&bar, 0);  // phase 0 never completes
    __syncthreads();
    if (threadIdx.x == 0) {
        out[0] = completed ? 1 : 0;
        out[1] = kvd::g_status;
    }
}

// Launches the probe (one block of 64 threads), waits for it, and returns
// {completed, status} through `result`; the return value is the CUDA error.
extern "C" int kvd_wait_probe(int32_t* result) {
    int32_t* d = nullptr;
    cudaError_t e = cudaMalloc(&d, 2 * sizeof(int32_t));
    if (e != cudaSuccess) return e;
    const int32_t init[2] = {-1, -1};
    e = cudaMemcpy(d, init, sizeof(init), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        wait_probe_kernel<<<1, 64>>>(d);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(result, d, 2 * sizeof(int32_t), cudaMemcpyDeviceToHost);
    cudaFree(d);
    return e;
}
