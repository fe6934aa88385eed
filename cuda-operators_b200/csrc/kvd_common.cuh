// kvd_common.cuh -- device helpers shared by the sm_100a decode kernels:
// mbarriers with bounded waits, 1-D bulk async copies (TMA engine, no tensor
// map, CTA-local destinations only), packed fp32x2 arithmetic and the exact INT8 -> fp32
// conversion used on the CUDA-core path.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kvdecode.h"

namespace kvd {

// Device status word (KVD_STATUS_*). Kernels OR a code into it instead of
// trapping; kvd_device_status() reads and clears it.
extern __device__ int32_t g_status;

constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s bound on every spin-wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void record_status(int32_t code) {
    atomicOr(&g_status, code);
}

// ------------------------------------------------- query / output element types
// Query element `off` of Q, whose type KVD_FLAG_Q_* in `flags` selects.
__device__ __forceinline__ float load_q(const void* Q, int64_t off, uint32_t flags) {
    if (flags & KVD_FLAG_Q_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(Q)[off]);
    if (flags & KVD_FLAG_Q_F16) return __half2float(static_cast<const __half*>(Q)[off]);
    return static_cast<const float*>(Q)[off];
}

// Stores a normalised output element in the type KVD_FLAG_OUT_* selects.
__device__ __forceinline__ void store_out(void* out, int64_t off, float v, uint32_t flags) {
    if (flags & KVD_FLAG_OUT_BF16) static_cast<__nv_bfloat16*>(out)[off] = __float2bfloat16_rn(v);
    else if (flags & KVD_FLAG_OUT_F16) static_cast<__half*>(out)[off] = __float2half_rn(v);
    else static_cast<float*>(out)[off] = v;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Raises the pending transaction count of the current phase without
// arriving (for copies whose number is only known while they are issued;
// the issuer arrives once after the last one).
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// As above, but lets the hardware suspend the warp for up to `hint_ns` until
// the phase completes, instead of returning at once: a waiting warp then
// spends no issue slots polling.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

constexpr uint32_t kSuspendHintNs = 1000000;  // 1 ms per suspended try

// Bounded wait for the phase with the given parity to complete. Returns false
// (and records KVD_STATUS_WAIT_TIMEOUT) if it has not completed within
// kWaitTimeoutNs; the caller then stops issuing work and drains.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait_suspend(bar, parity, kSuspendHintNs)) return true;
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
            record_status(KVD_STATUS_WAIT_TIMEOUT);
            return false;
        }
    }
}

// ------------------------------------------------------------- bulk copies
// 1-D global -> shared copy on the TMA engine, completion counted on `bar`.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Named barrier over `count` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ------------------------------------------------- INT8 -> fp32, exactly
// Four signed codes packed in one 32-bit word. Flipping the sign bit of each
// byte gives u = x + 128 in [1, 255]; placing u in the low mantissa byte of
// 2^23 (bit pattern 0x4B0000uu) is the float 2^23 + u exactly, and subtracting
// 2^23 + 128 (exact) returns x. One PRMT per code and one packed add per two.
constexpr float kMagic = 8388736.0f;  // 2^23 + 128

__device__ __forceinline__ void dequant4(uint32_t w, float2& lo, float2& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650));
    const float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651));
    const float f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652));
    const float f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653));
    const float2 m = make_float2(-kMagic, -kMagic);
    lo = __fadd2_rn(make_float2(f0, f1), m);
    hi = __fadd2_rn(make_float2(f2, f3), m);
}

// Programmatic dependent launch. A kernel launched with the programmatic
// stream-serialization attribute may start while the kernel before it in the
// stream is still running; grid_dependency_wait() blocks until that kernel has
// completed and its memory writes are visible (a no-op without the attribute).
// allow_dependents() lets such a dependent kernel begin launching early.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float fast_exp2(float x) {
    return exp2f(x);
}

}  // namespace kvd
