// kvd_quant.cuh -- the symmetric per-token INT8 quantiser of the cache
// (scale = max|x| / 127 in IEEE fp32, code = clamp(rint(x / scale), -127, 127),
// all-zero row -> scale 0, codes 0), shared by the append kernels and the
// fused append of the tensor-core decode so both write the same bits. It must
// not be built with fast-math: both divisions are IEEE, round to nearest even.
#pragma once

#include <cstdint>

namespace kvd {

// One warp quantises one row of `dim` floats.
__device__ __forceinline__ void quantize_row_warp(const float* __restrict__ x, int dim,
                                                  int8_t* __restrict__ codes, float* __restrict__ scale,
                                                  int lane) {
    float amax = 0.f;
    for (int d = lane; d < dim; d += 32) amax = fmaxf(amax, fabsf(x[d]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (amax == 0.f) {
        for (int d = lane; d < dim; d += 32) codes[d] = 0;
        if (lane == 0) *scale = 0.f;
        return;
    }
    const float s = amax / 127.0f;
    for (int d = lane; d < dim; d += 32) {
        float r = rintf(x[d] / s);
        r = fminf(fmaxf(r, -127.0f), 127.0f);
        codes[d] = static_cast<int8_t>(r);
    }
    if (lane == 0) *scale = s;
}

// The same rule for one 128-float row held in registers, lane l holding
// elements 4l..4l+3 (one 16-byte load per lane instead of a strided loop).
// The maximum does not depend on the order of its operands and each code is
// computed from its own element, so the bits equal quantize_row_warp's.
// `codes` must be 4-byte aligned.
__device__ __forceinline__ uint32_t quantize4(float v0, float v1, float v2, float v3, float s) {
    auto q = [s](float v) {
        float r = rintf(v / s);
        r = fminf(fmaxf(r, -127.0f), 127.0f);
        return static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(r)));
    };
    return q(v0) | (q(v1) << 8) | (q(v2) << 16) | (q(v3) << 24);
}

__device__ __forceinline__ void quantize_row128_regs(float4 x, int8_t* __restrict__ codes,
                                                     float* __restrict__ scale, int lane) {
    float amax = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float s = 0.f;
    uint32_t packed = 0u;
    if (amax != 0.f) {
        s = amax / 127.0f;
        packed = quantize4(x.x, x.y, x.z, x.w, s);
    }
    reinterpret_cast<uint32_t*>(codes)[lane] = packed;
    if (lane == 0) *scale = s;
}

}  // namespace kvd
