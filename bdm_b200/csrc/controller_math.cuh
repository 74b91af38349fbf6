// Element-wise controller math of the reference (_parameters.py:189-220, heads.py:11-22),
// shared by the controller epilogue (controllers.cu) and the fused decode step (decode.cu) so
// both round and approximate identically.
#pragma once

#include "common.cuh"

namespace bdm {
namespace ctl {

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }
// Wide activations use the hardware exp and an approximate divide (relative error
// ~1e-6: below one BF16 ulp and far below the FP32 tolerance).
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

// Scale of the q / k normalisation of one head from the sum of squares of its SiLU'd row:
// 'nvidia' x * rsqrt(sum x^2 + 1e-6), 'original' x / max(|x|, 1e-12) (_parameters.py:214-220).
__device__ __forceinline__ float qk_scale(float sum_sq, int nvidia) {
    return nvidia ? 1.0f / sqrtf(sum_sq + 1e-6f) : 1.0f / fmaxf(sqrtf(sum_sq), 1e-12f);
}

// Decay gate g = -exp(A_log[h]) * softplus(f + dt_bias) in FP32 (_parameters.py:207-210).
__device__ __forceinline__ float decay_gate(float a_log, float f, float dt_bias) {
    return -expf(a_log) * softplus_f(f + dt_bias);
}

}  // namespace ctl
}  // namespace bdm
