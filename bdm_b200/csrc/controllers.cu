// Controller epilogue over the fused input projection (one warp per token).
//
// The six controller projections of the reference (_parameters.py:189-212;
// per-head heads.py:11-22) run as ONE GEMM in the caller
// (hidden @ [Wq; Wk; Wv; Wf1; Wb; Ww; Wread; Wwrite; Wgate]^T); this kernel
// applies what follows them, rounding to the activation dtype where the
// reference materialises a tensor in it:
//   q, k = normalize(silu(.)) per head   (nvidia: x*rsqrt(sum x^2 + 1e-6), _parameters.py:214-220)
//   v = silu(.), b = sigmoid(.), w = sigmoid(.)
//   g = -exp(A_log[h]) * softplus(f_proj.1(f1) + dt_bias)   in FP32 (_parameters.py:207-209)
// The second f_proj layer (dv -> H*S) is a per-token mat-vec: its weight is
// staged transposed in shared memory once per CTA, each lane owns output
// columns, and the token's f1 row is broadcast from shared memory.
#include "common.cuh"

namespace bdm {
namespace {

constexpr int kCtlWarps = 8;

// Accurate forms for the narrow controllers (q, k, b, g); the wide v / w
// activations use the hardware exp and reciprocal (relative error ~1e-6, below
// one BF16 ulp and far below the FP32 tolerance).
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

// 8 consecutive elements as one 16-byte (bf16) or two 16-byte (float) accesses.
template <typename T> struct Pack8;
template <> struct Pack8<bf16> {
    __device__ __forceinline__ static void load(const bf16 *p, float *x) {
        uint4 u = *reinterpret_cast<const uint4 *>(p);
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 f = __bfloat1622float2(h[i]);
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
        }
    }
    __device__ __forceinline__ static void store(bf16 *p, const float *x) {
        uint4 u;
        __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
        *reinterpret_cast<uint4 *>(p) = u;
    }
};
template <> struct Pack8<float> {
    __device__ __forceinline__ static void load(const float *p, float *x) {
        float4 a = reinterpret_cast<const float4 *>(p)[0], b = reinterpret_cast<const float4 *>(p)[1];
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
    __device__ __forceinline__ static void store(float *p, const float *x) {
        reinterpret_cast<float4 *>(p)[0] = make_float4(x[0], x[1], x[2], x[3]);
        reinterpret_cast<float4 *>(p)[1] = make_float4(x[4], x[5], x[6], x[7]);
    }
};

template <typename T>
__global__ void __launch_bounds__(kCtlWarps * 32)
controllers_kernel(const T *__restrict__ proj, int64_t ntok, int64_t ld, int64_t col_q, int64_t col_k, int64_t col_v,
                   int64_t col_f, int64_t col_b, int64_t col_w, const T *__restrict__ f2, const float *__restrict__ a_log,
                   const float *__restrict__ dt_bias, int H, int S, int dv, int qk_norm, int vec,
                   T *__restrict__ q, T *__restrict__ k, T *__restrict__ v, float *__restrict__ g,
                   T *__restrict__ b, T *__restrict__ w) {
    extern __shared__ float sm[];
    const int HS = H * S;
    float *f2t = sm;                         // [dv][HS] transposed second f_proj layer
    float *f1s = sm + (size_t)dv * HS;       // [kCtlWarps][dv]
    const int warp = threadIdx.x >> 5;
    const int lane = (int)lane_id();
    for (int i = threadIdx.x; i < dv * HS; i += blockDim.x) {
        const int o = i / dv, c = i % dv;
        f2t[c * HS + o] = Elem<T>::to_float(f2[i]);
    }
    __syncthreads();
    float *f1 = f1s + warp * dv;
    const int64_t V = (int64_t)H * dv;
    for (int64_t t = (int64_t)blockIdx.x * kCtlWarps + warp; t < ntok; t += (int64_t)gridDim.x * kCtlWarps) {
        const T *row = proj + t * ld;
        // q and k: one (role, head) pair per lane; silu rounds to dtype before the norm.
        for (int task = lane; task < 2 * H; task += 32) {
            const int h = task >> 1;
            const T *src = row + ((task & 1) ? col_k : col_q) + (int64_t)h * S;
            T *dst = ((task & 1) ? k : q) + t * HS + (int64_t)h * S;
            float x[16];
            float ss = 0.f;
            for (int s = 0; s < S; ++s) {
                x[s] = rnd<T>(silu_f(Elem<T>::to_float(src[s])));
                ss += x[s] * x[s];
            }
            const float scale = qk_norm ? 1.0f / sqrtf(ss + 1e-6f) : 1.0f / fmaxf(sqrtf(ss), 1e-12f);
            for (int s = 0; s < S; ++s) dst[s] = Elem<T>::from_float(x[s] * scale);
        }
        // g: f2 = f_proj.1(f1) rounded to dtype, then the FP32 gate; b = sigmoid.
        for (int c = lane; c < dv; c += 32) f1[c] = Elem<T>::to_float(row[col_f + c]);
        __syncwarp();
        for (int o0 = 2 * lane; o0 < HS; o0 += 64) {
            float2 acc = make_float2(0.f, 0.f);
            const bool pair = o0 + 1 < HS;
#pragma unroll 8
            for (int c = 0; c < dv; ++c) {
                const float x = f1[c];
                if (pair && (HS % 2 == 0)) {
                    const float2 w2 = *reinterpret_cast<const float2 *>(f2t + c * HS + o0);
                    acc.x = fmaf(x, w2.x, acc.x);
                    acc.y = fmaf(x, w2.y, acc.y);
                } else {
                    acc.x = fmaf(x, f2t[c * HS + o0], acc.x);
                    if (pair) acc.y = fmaf(x, f2t[c * HS + o0 + 1], acc.y);
                }
            }
            for (int i = 0; i < 2 && o0 + i < HS; ++i) {
                const int o = o0 + i;
                const float f = rnd<T>(i ? acc.y : acc.x);
                g[t * HS + o] = -expf(a_log[o / S]) * softplus_f(f + dt_bias[o]);
                b[t * HS + o] = Elem<T>::from_float(sigmoid_f(Elem<T>::to_float(row[col_b + o])));
            }
        }
        __syncwarp();
        // v = silu, w = sigmoid over the full value width, 8 elements per lane access.
        if (vec) {
            for (int64_t c = (int64_t)lane * 8; c < V; c += 32 * 8) {
                float xv[8], xw[8];
                Pack8<T>::load(row + col_v + c, xv);
                Pack8<T>::load(row + col_w + c, xw);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    xv[i] = silu_fast(xv[i]);
                    xw[i] = sigmoid_fast(xw[i]);
                }
                Pack8<T>::store(v + t * V + c, xv);
                Pack8<T>::store(w + t * V + c, xw);
            }
        } else {
            for (int64_t c = lane; c < V; c += 32) {
                v[t * V + c] = Elem<T>::from_float(silu_fast(Elem<T>::to_float(row[col_v + c])));
                w[t * V + c] = Elem<T>::from_float(sigmoid_fast(Elem<T>::to_float(row[col_w + c])));
            }
        }
    }
}

}  // namespace
}  // namespace bdm

extern "C" int bdm_controllers(const void *proj, int64_t ntok, int64_t ld, int64_t col_q, int64_t col_k, int64_t col_v,
                               int64_t col_f, int64_t col_b, int64_t col_w, const void *f2_weight, const float *a_log,
                               const float *dt_bias, int heads, int bank_size, int head_value_width, int qk_norm,
                               int dtype, void *q, void *k, void *v, float *g, void *b, void *w, void *stream) {
    using namespace bdm;
    if (ntok < 0 || heads <= 0 || bank_size <= 0 || head_value_width <= 0) return BDM_ERR_INVALID;
    if (bank_size > 16) return BDM_ERR_UNSUPPORTED;
    if (ntok == 0) return BDM_OK;
    if (!proj || !f2_weight || !a_log || !dt_bias || !q || !k || !v || !g || !b || !w) return BDM_ERR_INVALID;
    const int64_t HS = (int64_t)heads * bank_size, V = (int64_t)heads * head_value_width;
    if (col_q < 0 || col_k < 0 || col_v < 0 || col_f < 0 || col_b < 0 || col_w < 0 || col_q + HS > ld ||
        col_k + HS > ld || col_v + V > ld || col_f + head_value_width > ld || col_b + HS > ld || col_w + V > ld)
        return BDM_ERR_INVALID;
    const size_t smem = ((size_t)head_value_width * HS + (size_t)kCtlWarps * head_value_width) * sizeof(float);
    if (smem > 200 * 1024) return BDM_ERR_UNSUPPORTED;
    int64_t blocks = ceil_div(ntok, kCtlWarps);
    if (blocks > 8 * kNumSMs) blocks = 8 * kNumSMs;
    BDM_DISPATCH_DTYPE(dtype, T, {
        // 16-byte row accesses need 8-element aligned columns and row stride
        const uintptr_t mis = (reinterpret_cast<uintptr_t>(proj) | reinterpret_cast<uintptr_t>(v) |
                               reinterpret_cast<uintptr_t>(w)) & 15;
        const int vec = !mis && (ld % 8 == 0) && (col_v % 8 == 0) && (col_w % 8 == 0) && (V % 8 == 0);
        auto kern = controllers_kernel<T>;
        if (smem > 48 * 1024) {
            int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            if (rc) return rc;
        }
        kern<<<(unsigned)blocks, kCtlWarps * 32, smem, as_stream(stream)>>>(
            static_cast<const T *>(proj), ntok, ld, col_q, col_k, col_v, col_f, col_b, col_w,
            static_cast<const T *>(f2_weight), a_log, dt_bias, heads, bank_size, head_value_width, qk_norm, vec,
            static_cast<T *>(q), static_cast<T *>(k), static_cast<T *>(v), g, static_cast<T *>(b),
            static_cast<T *>(w));
    });
    return launch_status();
}
