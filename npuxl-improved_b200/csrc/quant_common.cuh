// quant_common.cuh - the QUANTIZE_I8 arithmetic shared by the quantize and
// the fused norm/activation + quantize kernels (src/kernels/llm.cpp:387-411):
// scale = maxabs/127 (IEEE divide; 1.0 when <= 0 or not finite), q =
// roundf(x * (1/scale)) clamped to [-128, 127]; NaN never wins the max.
#pragma once

#include <cstdint>

namespace vnpu_b200 {
namespace {

__device__ __forceinline__ float scale_from_absmax(float m) {
    float s = __fdiv_rn(m, 127.0f);
    if (s <= 0.0f || !isfinite(s)) s = 1.0f;
    return s;
}

__device__ __forceinline__ int8_t quantize_value(float x, float inv) {
    float q = roundf(__fmul_rn(x, inv));
    q = q > 127.0f ? 127.0f : q;
    q = q < -128.0f ? -128.0f : q;
    return static_cast<int8_t>(static_cast<int>(q));
}

__device__ __forceinline__ uint32_t pack4(float a, float b, float c, float d, float inv) {
    return (static_cast<uint32_t>(static_cast<uint8_t>(quantize_value(a, inv)))) |
           (static_cast<uint32_t>(static_cast<uint8_t>(quantize_value(b, inv))) << 8) |
           (static_cast<uint32_t>(static_cast<uint8_t>(quantize_value(c, inv))) << 16) |
           (static_cast<uint32_t>(static_cast<uint8_t>(quantize_value(d, inv))) << 24);
}

__device__ __forceinline__ float block_max(float v, float *red) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < (blockDim.x >> 5) ? red[lane] : 0.0f;
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) red[0] = v;
    }
    __syncthreads();
    const float r = red[0];
    __syncthreads();
    return r;
}

}  // namespace
}  // namespace vnpu_b200
