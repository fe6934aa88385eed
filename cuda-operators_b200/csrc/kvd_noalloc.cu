// kvd_noalloc.cu -- a decode entry point that allocates no device memory.
//
// Who needs it: callers that may not allocate device memory when they decode.
// A host framework that owns all device memory and hands a plugin nothing but
// its input and output buffers is one; a serving loop that bans allocation on
// its hot path (cudaMalloc can synchronise the device and stall every other
// stream) is another. kvd_decode_launch needs a caller-provided workspace and
// solve() allocates one stream-ordered; this entry point instead keeps the
// scratch of the split-KV decode (the ragged tile plan and the partial
// (m, l, o) records of heads that span several CTAs) in one fixed array
// compiled into the library.
//
// Properties a caller must know:
//  * Size: KVD_NOALLOC_SCRATCH_BYTES (512 KiB). A descriptor whose
//    kvd_workspace_size() exceeds it is rejected with cudaErrorInvalidValue and
//    one line on stderr; nothing is launched. The size grows with the split
//    records of long sequences: on a B200 a dense head_dim-128 decode of 4,096
//    tokens fits (about 312 KiB), but long contexts do not -- 4 sequences x 32
//    heads x 131,072 tokens plans 37 splits per head, 2.5 MB of records -- nor
//    do very large ragged batches, whose plan arrays alone outgrow the array.
//  * Memory: the array is a static __device__ object, so every GPU that loads
//    this library holds 512 KiB for it until the process exits.
//  * Set-up: the first call on each device (with that device current) looks
//    up the array's device address with cudaGetSymbolAddress and caches it
//    together with the unique id of the CUDA context it belongs to. A call in
//    another context of that device (after cudaDeviceReset, or under a context
//    the caller made current) looks the address up again. The lookup may load
//    the library's device code, so make the first call on a device -- and the
//    first one after a reset -- outside any stream capture.
//  * Sharing: every call uses the same array and it keeps whatever the last
//    call wrote. Nothing in it has to start at zero -- each call writes every
//    record it later reads -- but two calls whose kernels overlap on the GPU
//    (different streams or host threads on one device) overwrite each other's
//    scratch and produce wrong results. Issue them in order on one stream, or
//    use kvd_decode_launch with a workspace per concurrent call.
//  * It calls no cudaMalloc, cudaFree or other allocating routine.
#include <cuda.h>

#include <cstdio>
#include <mutex>

#include "kvd_common.cuh"
#include "kvd_decode.cuh"

namespace kvd {
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[KVD_NOALLOC_SCRATCH_BYTES];

struct NoallocSlot {
    unsigned long long ctx_id;  // unique id of the context the address belongs to (0: none yet)
    void* addr;
};
std::mutex g_noalloc_mutex;
NoallocSlot g_noalloc_slots[kMaxDevices] = {};

// Device address of g_noalloc_scratch in the current context (host code sees
// only a host-side stand-in for the symbol; it must never be passed to a kernel).
cudaError_t noalloc_scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    NoallocSlot& slot = g_noalloc_slots[dev];
    const unsigned long long ctx = current_context_id();
    if (ctx == 0 || slot.ctx_id != ctx || slot.addr == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // binds the device's context if none was current
        if (e != cudaSuccess) return e;
        slot.addr = p;
        slot.ctx_id = current_context_id();
    }
    *out = slot.addr;
    return cudaSuccess;
}

}  // namespace
}  // namespace kvd

extern "C" cudaError_t kvd_decode_launch_noalloc(const kvd_decode_desc* desc, const void* Q, const int8_t* K,
                                                 const int8_t* V, const float* k_scale, const float* v_scale,
                                                 void* out, cudaStream_t stream) {
    if (desc == nullptr || !Q || !K || !V || !k_scale || !v_scale || !out) return cudaErrorInvalidValue;
    const size_t need = kvd_workspace_size(desc);
    if (need > KVD_NOALLOC_SCRATCH_BYTES) {
        std::fprintf(stderr,
                     "[kvdecode] kvd_decode_launch_noalloc: this decode needs %zu bytes of scratch, more than the "
                     "library's fixed %u-byte array; use kvd_decode_launch with a workspace\n",
                     need, static_cast<unsigned>(KVD_NOALLOC_SCRATCH_BYTES));
        return cudaErrorInvalidValue;
    }
    void* scratch = nullptr;
    const cudaError_t e = kvd::noalloc_scratch_address(&scratch);
    if (e != cudaSuccess) return e;
    return kvd_decode_launch(desc, Q, K, V, k_scale, v_scale, out, scratch, KVD_NOALLOC_SCRATCH_BYTES, stream);
}
