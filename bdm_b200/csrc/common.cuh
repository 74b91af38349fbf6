// Shared helpers for the BDM sm_100a kernels: element types, rounding, status plumbing.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/bdm_b200.h"

namespace bdm {

// ------------------------------------------------------------------ status

// Records the CUDA error of the last failing call on this host thread.
void set_last_cuda_error(cudaError_t e);
// Counts kernel launches issued by this library (process-wide).
void count_launch();

// Call once after every kernel launch.
inline int launch_status() {
    count_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return BDM_ERR_CUDA;
    }
    return BDM_OK;
}

inline int cuda_status(cudaError_t e) {
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return BDM_ERR_CUDA;
    }
    return BDM_OK;
}

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

// ------------------------------------------------------------ element types

using bf16 = __nv_bfloat16;

template <typename T> struct Elem;
template <> struct Elem<float> {
    __device__ __forceinline__ static float load(const float *p) { return *p; }
    __device__ __forceinline__ static float to_float(float x) { return x; }
    __device__ __forceinline__ static float from_float(float x) { return x; }
    // value rounded to this type, returned as float
    __device__ __forceinline__ static float round(float x) { return x; }
};
template <> struct Elem<bf16> {
    __device__ __forceinline__ static float load(const bf16 *p) { return __bfloat162float(*p); }
    __device__ __forceinline__ static float to_float(bf16 x) { return __bfloat162float(x); }
    __device__ __forceinline__ static bf16 from_float(float x) { return __float2bfloat16_rn(x); }
    __device__ __forceinline__ static float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
};

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

template <typename T> __device__ __forceinline__ float ld_f(const T *p, int64_t i) { return Elem<T>::to_float(p[i]); }
template <typename T> __device__ __forceinline__ void st_f(T *p, int64_t i, float x) { p[i] = Elem<T>::from_float(x); }
template <typename T> __device__ __forceinline__ float rnd(float x) { return Elem<T>::round(x); }

// Read-only global load through the non-coherent path.
template <typename T> __device__ __forceinline__ T ldg(const T *p) { return __ldg(p); }

// Dispatch a templated launcher on the runtime dtype code.
#define BDM_DISPATCH_DTYPE(code, T, ...)                \
    do {                                                \
        if ((code) == BDM_BF16) {                       \
            using T = ::bdm::bf16;                      \
            __VA_ARGS__;                                \
        } else if ((code) == BDM_F32) {                 \
            using T = float;                            \
            __VA_ARGS__;                                \
        } else {                                        \
            return BDM_ERR_DTYPE;                       \
        }                                               \
    } while (0)

inline bool valid_dtype(int code) { return code == BDM_BF16 || code == BDM_F32; }

constexpr int kNumSMs = 148;  // B200: 2 dies x 74 SMs

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Warp helpers ---------------------------------------------------------------
__device__ __forceinline__ unsigned lane_id() { return threadIdx.x & 31u; }

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

}  // namespace bdm
