// Output normalisation and sigmoid gate of the reference's output interface
// (_parameters.py:222-232 _project_bank_output: LayerNorm or RMS of the combined reads, times
// dtype(sigmoid(gate))), element by element with explicit roundings (no multiply-add
// contraction).  Shared by the combine kernels (combine.cu, combine_project.cu) and the decode
// steps (decode.cu), so every path hands o_proj the same values.
#pragma once

#include "common.cuh"

namespace bdm {
namespace ng {

// dtype(sigmoid(x)): BF16 rows on the fast exponential and divide, FP32 rows on expf and an
// IEEE divide.
template <typename T> __device__ __forceinline__ float gate_sigmoid(float x) {
    if constexpr (sizeof(T) == 2) return rnd<T>(__fdividef(1.0f, 1.0f + __expf(-x)));
    else return rnd<T>(1.0f / (1.0f + expf(-x)));
}

// One term of the LayerNorm variance: acc + (x - mean)^2.
__device__ __forceinline__ float sq_dev(float x, float mean, float acc) {
    const float d = __fsub_rn(x, mean);
    return fmaf(d, d, acc);
}

// LayerNorm output of one column: (x - mean) * rstd * w (+ b).
__device__ __forceinline__ float layer_norm_col(float x, float mean, float rstd, float w, const float *b) {
    const float y = __fmul_rn(__fmul_rn(__fsub_rn(x, mean), rstd), w);
    return b ? __fadd_rn(y, *b) : y;
}

// 1 / sqrt(var + eps) of the LayerNorm; the RMS scale is this rounded to the dtype.
__device__ __forceinline__ float inv_std(float var, float eps) { return 1.0f / sqrtf(var + eps); }

// RMS-normalised column: dtype(dtype(x * sc) * w).
template <typename T> __device__ __forceinline__ float rms_col(float x, float sc, float w) {
    return rnd<T>(__fmul_rn(rnd<T>(__fmul_rn(x, sc)), w));
}

}  // namespace ng
}  // namespace bdm
