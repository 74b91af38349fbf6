// Controller epilogue over the fused input projection (element-parallel).
//
// The controller projections of the reference (_parameters.py:189-212; per
// head heads.py:11-22) run as ONE GEMM in the caller
// (hidden @ [Wq; Wk; Wv; Wf1; Wb; Ww; Wread; Wwrite; Wgate]^T), followed by the
// small f_proj.1 GEMM (f = f1 @ Wf2^T; with few tokens, as in decode, this kernel
// computes f itself from f1 and Wf2).  This kernel applies everything after
// them, rounding to the activation dtype where the reference materialises a
// tensor in it:
//   q, k = normalize(silu(.)) per head   (nvidia: x*rsqrt(sum x^2 + 1e-6), _parameters.py:214-220)
//   b = sigmoid(.), g = -exp(A_log[h]) * softplus(f + dt_bias) in FP32 (_parameters.py:207-210)
//   v = silu(.), w = sigmoid(.)
// Three independent index ranges in one launch: one thread per (token, head) for
// q and k (per-head norms), one per (token, head*S + s) for b and the decay gate
// g (and f_proj.1's dot product when the kernel computes f), one per 8-element
// chunk of the wide v / w rows (streamed with 16-byte accesses).
#include "common.cuh"
#include "controller_math.cuh"

namespace bdm {
namespace {

constexpr int kCtlThreads = 256;
constexpr int kMaxS = 16;

using namespace ctl;

struct CtlArgs {
    const void *proj;
    int64_t ntok, ld, col_q, col_k, col_v, col_b, col_w;
    const void *f;
    int64_t ldf;
    const void *wf2;  // f_proj.1 weight [H*S, f1_width] when f is computed here (f == null)
    int64_t col_f1;
    int f1_width;
    const float *a_log, *dt_bias;
    int H, S, dv, qk_norm, vec;
    void *q, *k, *v, *b, *w;
    float *g;
    int64_t narrow_blocks, gate_blocks;
};

template <typename T>
__device__ __forceinline__ void narrow_item(const CtlArgs &a, int64_t t, int h) {
    const T *row = static_cast<const T *>(a.proj) + t * a.ld;
    const int S = a.S, HS = a.H * a.S;
    const int64_t o = t * HS + (int64_t)h * S;
    float x[kMaxS];
#pragma unroll
    for (int role = 0; role < 2; ++role) {  // q then k
        const T *src = row + (role ? a.col_k : a.col_q) + (int64_t)h * S;
        float ss = 0.f;
        for (int s = 0; s < S; ++s) {
            x[s] = rnd<T>(silu_f(Elem<T>::to_float(src[s])));
            ss = fmaf(x[s], x[s], ss);
        }
        const float scale = qk_scale(ss, a.qk_norm);
        T *dst = static_cast<T *>(role ? a.k : a.q) + o;
        for (int s = 0; s < S; ++s) dst[s] = Elem<T>::from_float(x[s] * scale);
    }
}

// b = sigmoid, g = -exp(A_log[h]) * softplus(f + dt_bias) for one (token, head*S + s);
// f from the given f_proj output, or computed here as dtype(f1 . Wf2[hs]) (FP32 accumulation).
template <typename T>
__device__ __forceinline__ void gate_item(const CtlArgs &a, int64_t t, int hs) {
    const T *row = static_cast<const T *>(a.proj) + t * a.ld;
    const int64_t o = t * (int64_t)a.H * a.S + hs;
    float fv;
    if (a.f) {
        fv = Elem<T>::to_float(static_cast<const T *>(a.f)[t * a.ldf + hs]);
    } else {
        const T *f1 = row + a.col_f1;
        const T *wrow = static_cast<const T *>(a.wf2) + (int64_t)hs * a.f1_width;
        float acc = 0.f;
        for (int j = 0; j < a.f1_width; ++j) acc = fmaf(Elem<T>::to_float(f1[j]), Elem<T>::to_float(wrow[j]), acc);
        fv = rnd<T>(acc);
    }
    const int h = hs / a.S;
    static_cast<T *>(a.b)[o] = Elem<T>::from_float(sigmoid_f(Elem<T>::to_float(row[a.col_b + hs])));
    a.g[o] = decay_gate(a.a_log[h], fv, a.dt_bias[hs]);
}

template <typename T>
__device__ __forceinline__ void wide_item(const CtlArgs &a, int64_t i) {
    const int64_t V = (int64_t)a.H * a.dv;
    if (a.vec) {  // BF16, 16-byte aligned rows: one chunk of 8 columns of v and of w
        const int64_t per = V / 8;
        const int64_t t = i / per, c = (i % per) * 8;
        const T *row = static_cast<const T *>(a.proj) + t * a.ld;
        const uint4 rv = *reinterpret_cast<const uint4 *>(row + a.col_v + c);
        const uint4 rw = *reinterpret_cast<const uint4 *>(row + a.col_w + c);
        const __nv_bfloat162 *hv = reinterpret_cast<const __nv_bfloat162 *>(&rv);
        const __nv_bfloat162 *hw = reinterpret_cast<const __nv_bfloat162 *>(&rw);
        uint4 ov, ow;
        __nv_bfloat162 *pv = reinterpret_cast<__nv_bfloat162 *>(&ov);
        __nv_bfloat162 *pw = reinterpret_cast<__nv_bfloat162 *>(&ow);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 fv = __bfloat1622float2(hv[j]), fw = __bfloat1622float2(hw[j]);
            pv[j] = __floats2bfloat162_rn(silu_fast(fv.x), silu_fast(fv.y));
            pw[j] = __floats2bfloat162_rn(sigmoid_fast(fw.x), sigmoid_fast(fw.y));
        }
        *reinterpret_cast<uint4 *>(static_cast<T *>(a.v) + t * V + c) = ov;
        *reinterpret_cast<uint4 *>(static_cast<T *>(a.w) + t * V + c) = ow;
    } else {  // one element of v and of w
        const int64_t t = i / V, c = i % V;
        const T *row = static_cast<const T *>(a.proj) + t * a.ld;
        static_cast<T *>(a.v)[t * V + c] = Elem<T>::from_float(silu_fast(Elem<T>::to_float(row[a.col_v + c])));
        static_cast<T *>(a.w)[t * V + c] = Elem<T>::from_float(sigmoid_fast(Elem<T>::to_float(row[a.col_w + c])));
    }
}

template <typename T>
__global__ void __launch_bounds__(kCtlThreads) controllers_kernel(const CtlArgs a) {
    const int64_t blk = blockIdx.x;
    if (blk < a.narrow_blocks) {
        const int64_t item = blk * kCtlThreads + threadIdx.x;
        if (item < a.ntok * a.H) narrow_item<T>(a, item / a.H, (int)(item % a.H));
    } else if (blk < a.narrow_blocks + a.gate_blocks) {
        const int64_t item = (blk - a.narrow_blocks) * kCtlThreads + threadIdx.x;
        const int HS = a.H * a.S;
        if (item < a.ntok * HS) gate_item<T>(a, item / HS, (int)(item % HS));
    } else {
        const int64_t item = (blk - a.narrow_blocks - a.gate_blocks) * kCtlThreads + threadIdx.x;
        const int64_t V = (int64_t)a.H * a.dv;
        if (item < a.ntok * (a.vec ? V / 8 : V)) wide_item<T>(a, item);
    }
}

}  // namespace
}  // namespace bdm

extern "C" int bdm_controllers(const void *proj, int64_t ntok, int64_t ld, int64_t col_q, int64_t col_k, int64_t col_v,
                               int64_t col_b, int64_t col_w, const void *f, int64_t ldf, const void *wf2,
                               int64_t col_f1, int f1_width, const float *a_log,
                               const float *dt_bias, int heads, int bank_size, int head_value_width, int qk_norm,
                               int dtype, void *q, void *k, void *v, float *g, void *b, void *w, void *stream) {
    using namespace bdm;
    if (ntok < 0 || heads <= 0 || bank_size <= 0 || head_value_width <= 0) return BDM_ERR_INVALID;
    if (bank_size > kMaxS) return BDM_ERR_UNSUPPORTED;
    if (ntok == 0) return BDM_OK;
    if (!proj || (!f && !wf2) || !a_log || !dt_bias || !q || !k || !v || !g || !b || !w) return BDM_ERR_INVALID;
    const int64_t HS = (int64_t)heads * bank_size, V = (int64_t)heads * head_value_width;
    if (col_q < 0 || col_k < 0 || col_v < 0 || col_b < 0 || col_w < 0 || col_q + HS > ld || col_k + HS > ld ||
        col_v + V > ld || col_b + HS > ld || col_w + V > ld || (f && ldf < HS))
        return BDM_ERR_INVALID;
    if (!f && (f1_width <= 0 || col_f1 < 0 || col_f1 + f1_width > ld)) return BDM_ERR_INVALID;
    CtlArgs a{};
    a.proj = proj; a.ntok = ntok; a.ld = ld; a.col_q = col_q; a.col_k = col_k; a.col_v = col_v;
    a.col_b = col_b; a.col_w = col_w; a.f = f; a.ldf = ldf; a.a_log = a_log; a.dt_bias = dt_bias;
    a.wf2 = wf2; a.col_f1 = col_f1; a.f1_width = f1_width;
    a.H = heads; a.S = bank_size; a.dv = head_value_width; a.qk_norm = qk_norm;
    a.q = q; a.k = k; a.v = v; a.b = b; a.w = w; a.g = g;
    const uintptr_t mis = (reinterpret_cast<uintptr_t>(proj) | reinterpret_cast<uintptr_t>(v) |
                           reinterpret_cast<uintptr_t>(w)) & 15;
    a.vec = dtype == BDM_BF16 && !mis && ld % 8 == 0 && col_v % 8 == 0 && col_w % 8 == 0 && V % 8 == 0;
    a.narrow_blocks = ceil_div(ntok * heads, kCtlThreads);
    a.gate_blocks = ceil_div(ntok * HS, kCtlThreads);
    const int64_t wide_blocks = ceil_div(ntok * (a.vec ? V / 8 : V), kCtlThreads);
    if (a.narrow_blocks + a.gate_blocks + wide_blocks > 0x7fffffffLL) return BDM_ERR_UNSUPPORTED;
    BDM_DISPATCH_DTYPE(dtype, T, {
        controllers_kernel<T><<<(unsigned)(a.narrow_blocks + a.gate_blocks + wide_blocks), kCtlThreads, 0,
                                as_stream(stream)>>>(a);
    });
    return launch_status();
}
