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
// The second f_proj layer (dv -> H*S) is a per-token mat-vec done here.
#include "common.cuh"

namespace bdm {
namespace {

constexpr int kCtlWarps = 8;

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

template <typename T>
__global__ void __launch_bounds__(kCtlWarps * 32)
controllers_kernel(const T *__restrict__ proj, int64_t ntok, int64_t ld, int64_t col_q, int64_t col_k, int64_t col_v,
                   int64_t col_f, int64_t col_b, int64_t col_w, const T *__restrict__ f2, const float *__restrict__ a_log,
                   const float *__restrict__ dt_bias, int H, int S, int dv, int qk_norm, T *__restrict__ q,
                   T *__restrict__ k, T *__restrict__ v, float *__restrict__ g, T *__restrict__ b, T *__restrict__ w) {
    extern __shared__ float f1s[];  // [kCtlWarps][dv]
    const int warp = threadIdx.x >> 5;
    const int lane = (int)lane_id();
    float *f1 = f1s + warp * dv;
    const int HS = H * S;
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
            float scale = qk_norm ? 1.0f / sqrtf(ss + 1e-6f) : 1.0f / fmaxf(sqrtf(ss), 1e-12f);
            for (int s = 0; s < S; ++s) dst[s] = Elem<T>::from_float(x[s] * scale);
        }
        // b = sigmoid
        for (int o = lane; o < HS; o += 32) b[t * HS + o] = Elem<T>::from_float(sigmoid_f(Elem<T>::to_float(row[col_b + o])));
        // g: f2 = f_proj.1(f1) rounded to dtype, then the FP32 gate.
        for (int c = lane; c < dv; c += 32) f1[c] = Elem<T>::to_float(row[col_f + c]);
        __syncwarp();
        for (int o = 0; o < HS; ++o) {
            const T *wrow = f2 + (int64_t)o * dv;
            float part = 0.f;
            for (int c = lane; c < dv; c += 32) part = fmaf(f1[c], Elem<T>::to_float(wrow[c]), part);
            part = warp_sum(part);
            if (lane == (o & 31)) {
                float f = rnd<T>(part);
                g[t * HS + o] = -expf(a_log[o / S]) * softplus_f(f + dt_bias[o]);
            }
        }
        __syncwarp();
        // v = silu, w = sigmoid over the full value width.
        for (int64_t c = lane; c < V; c += 32) {
            v[t * V + c] = Elem<T>::from_float(silu_f(Elem<T>::to_float(row[col_v + c])));
            w[t * V + c] = Elem<T>::from_float(sigmoid_f(Elem<T>::to_float(row[col_w + c])));
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
    size_t smem = (size_t)kCtlWarps * head_value_width * sizeof(float);
    if (smem > 200 * 1024) return BDM_ERR_UNSUPPORTED;
    int64_t blocks = ceil_div(ntok, kCtlWarps);
    if (blocks > 32 * kNumSMs) blocks = 32 * kNumSMs;
    BDM_DISPATCH_DTYPE(dtype, T, {
        auto kern = controllers_kernel<T>;
        if (smem > 48 * 1024) {
            int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            if (rc) return rc;
        }
        kern<<<(unsigned)blocks, kCtlWarps * 32, smem, as_stream(stream)>>>(
            static_cast<const T *>(proj), ntok, ld, col_q, col_k, col_v, col_f, col_b, col_w,
            static_cast<const T *>(f2_weight), a_log, dt_bias, heads, bank_size, head_value_width, qk_norm,
            static_cast<T *>(q), static_cast<T *>(k), static_cast<T *>(v), g, static_cast<T *>(b), static_cast<T *>(w));
    });
    return launch_status();
}
