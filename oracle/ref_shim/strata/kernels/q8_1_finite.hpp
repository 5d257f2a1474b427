// Q8_1 block rules for building the reference's src/fused_gdn.cu into the test-only oracle/_ref library.
// The reference's own header is not in its tree; these are this project's written rules (the ones the CUDA
// kernels and the CPU oracle share):
//   d = amax / 127, clamped to 65504 when NaN, infinite or above the fp16 maximum;
//   q = 0 for an all-zero block, else roundf(x / d) clamped to [-127, 127];
//   stored {half(d), half(sum clamped to +-65504, NaN -> 0)}.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace strata::kernels {

__device__ __forceinline__ float q8_1_finite(float d) { return d <= 65504.0f ? d : 65504.0f; }

__device__ __forceinline__ int8_t q8_1_quant(float x, float d, float amax) {
    if (amax == 0.0f) return 0;
    const float q = fminf(fmaxf(roundf(__fdiv_rn(x, d)), -127.0f), 127.0f);
    return (int8_t) (int) q;
}

__device__ __forceinline__ __half2 q8_1_ds(float d, float sum) {
    const float s = sum != sum ? 0.0f : fminf(fmaxf(sum, -65504.0f), 65504.0f);
    return __halves2half2(__float2half_rn(d), __float2half_rn(s));
}

}  // namespace strata::kernels
