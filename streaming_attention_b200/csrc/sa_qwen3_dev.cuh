// sa_qwen3_dev.cuh -- device helpers shared by the Qwen3 kernels and the
// prompt GEMM's fused epilogues.
#pragma once
#include <cuda_bf16.h>
#include <cstdint>

namespace sa {
namespace qd {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// RMS-normalise one 128-wide head held by a warp (lane l: elements 4l..4l+3)
// with gain nw (eps 1e-6 inside the sqrt, qwen3_ops.cpp:355-369), then
// rotate-half RoPE with the position's cos/sin rows (qwen3_ops.cpp:110-188):
// element i pairs with i + 64, held by lane l ^ 16.
__device__ __forceinline__ float4 head_norm_rope(const float (&e_in)[4], const float* nw, const float* cr,
                                                 const float* sr, int lane) {
    constexpr int D = 128;
    float e[4] = {e_in[0], e_in[1], e_in[2], e_in[3]};
    float ss = e[0] * e[0] + e[1] * e[1] + e[2] * e[2] + e[3] * e[3];
    ss = warp_sum(ss);
    const float rms = sqrtf(ss / (float)D + 1e-6f);
#pragma unroll
    for (int j = 0; j < 4; ++j) e[j] = (e[j] / rms) * nw[4 * lane + j];
    float p[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) p[j] = __shfl_xor_sync(0xffffffffu, e[j], 16);
    const bool first = lane < 16;
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int i = (4 * lane + j) & (D / 2 - 1);
        const float c = cr[i], s = sr[i];
        // first half: x1*c + (-x2)*s ; second half: x2*c + x1*s
        o[j] = first ? e[j] * c + (-p[j]) * s : e[j] * c + p[j] * s;
    }
    return make_float4(o[0], o[1], o[2], o[3]);
}

// Four floats as bf16 (round to nearest), 8 bytes.
__device__ __forceinline__ uint2 bf16x4(float4 v) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    return u;
}

}  // namespace qd
}  // namespace sa
