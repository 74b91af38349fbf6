// Decode step: one token per batch row, reading and writing only its routed banks.
//
// Restates inference.step's bank kernels (inference.py:21-67,175-193):
//   _decode_write  every write bank of the row: load S x dv state, delta-rule
//                  update with the route-weighted controls, store in the cache dtype
//   _decode_read   after all writes: scale * M^T dtype(q*r), rounded to dtype
//   _decode_sum    reads summed in ascending bank order, rounding after each add
// One 1024-thread CTA per batch row runs all phases: every (write slot, column)
// and every (read slot, column) is one thread's task, so a row's bank tiles are
// read in one round of independent loads; the reads go through shared memory
// and are summed per column in ascending bank order.  Optionally the same CTA
// applies the output norm and sigmoid gate (bdm_combine_norm_gate's arithmetic)
// to the summed row.  HBM traffic per row is the KW bank tiles read and written
// plus the KR bank tiles read.
#include "common.cuh"

namespace bdm {
namespace {

constexpr int kDecThreads = 1024;  // one (slot, column) task per thread at H*dv = 128, KW = KR = 8
constexpr int kDecMaxK = 64;
constexpr int kDecMaxS = 16;

template <typename CT> __device__ __forceinline__ float ld_state(const void *p, int64_t i) {
    return Elem<CT>::to_float(static_cast<const CT *>(p)[i]);
}
template <typename CT> __device__ __forceinline__ void st_state(void *p, int64_t i, float x) {
    static_cast<CT *>(p)[i] = Elem<CT>::from_float(x);
}

__device__ __forceinline__ float dec_block_sum(float x, float *red) {
    x = warp_sum(x);
    const int warp = threadIdx.x >> 5, lane = (int)lane_id();
    const int nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = x;
    __syncthreads();
    const float t = lane < nw ? red[lane] : 0.f;
    return warp_sum(t);
}

// Output gate, as bdm_combine_norm_gate computes it: BF16 rows on the fast
// exponential and divide, FP32 rows on expf and an IEEE divide.
template <typename T> __device__ __forceinline__ float gate_sigmoid(float x) {
    if constexpr (sizeof(T) == 2) return rnd<T>(__fdividef(1.0f, 1.0f + __expf(-x)));
    else return rnd<T>(1.0f / (1.0f + expf(-x)));
}

struct DecNorm {
    const void *gate;  // null: write the combined reads to `raw` only
    int64_t ld_gate;
    const void *nw, *nb;
    float eps;
    int mode;  // 1 LayerNorm, 0 RMS
    void *out;
};

template <typename T, typename CT, int S>
__global__ void __launch_bounds__(kDecThreads)
decode_kernel(const T *__restrict__ q, const T *__restrict__ k, const T *__restrict__ v, const float *__restrict__ g,
              const T *__restrict__ b, const T *__restrict__ w, const int64_t *__restrict__ wi,
              const T *__restrict__ ww, const int64_t *__restrict__ ri, const T *__restrict__ rw, int64_t J, int H,
              int dv, int kw, int kr, int routed_decay, float scale, void *state, T *__restrict__ raw,
              const DecNorm nrm) {
    extern __shared__ float sm[];
    // [kw][H][S] x3 (exp(g_e), a, k), [kr][H][S] (q_e), then the reads [kr][V]
    const int HS = H * S;
    const int64_t V = (int64_t)H * dv;
    float *se = sm;
    float *sa = se + kw * HS;
    float *sk = sa + kw * HS;
    float *sq = sk + kw * HS;
    float *reads = sq + kr * HS;
    __shared__ int64_t wbank[kDecMaxK], rbank[kDecMaxK];
    __shared__ float wwt[kDecMaxK];
    __shared__ int rorder[kDecMaxK];
    __shared__ float red[32];

    const int64_t row = blockIdx.x;
    const int tid = threadIdx.x;
    if (tid < kw) {
        int64_t bk = wi[row * kw + tid];
        wbank[tid] = (bk >= 0 && bk < J) ? bk : -1;
        wwt[tid] = Elem<T>::to_float(ww[row * kw + tid]);
    }
    if (tid < kr) {
        int64_t bk = ri[row * kr + tid];
        rbank[tid] = (bk >= 0 && bk < J) ? bk : -1;
    }
    __syncthreads();
    if (tid < kr) {  // ascending bank order, ties by slot
        const int64_t bj = rbank[tid];
        int rank = 0;
        for (int i = 0; i < kr; ++i) rank += (rbank[i] < bj) || (rbank[i] == bj && i < tid);
        rorder[rank] = tid;
    }
    for (int task = tid; task < kw * HS; task += kDecThreads) {
        const int slot = task / HS, hs = task % HS;
        const float p = wwt[slot];
        const int64_t o = row * HS + hs;
        const float kk = Elem<T>::to_float(k[o]);
        const float ge = routed_decay ? g[o] * p : g[o];
        se[task] = expf(ge);
        sa[task] = rnd<T>(Elem<T>::to_float(b[o]) * p) * kk;
        sk[task] = kk;
    }
    for (int task = tid; task < kr * HS; task += kDecThreads) {
        const int slot = task / HS, hs = task % HS;
        const float r = Elem<T>::to_float(rw[row * kr + slot]);
        sq[task] = rnd<T>(Elem<T>::to_float(q[row * HS + hs]) * r);
    }
    __syncthreads();
    // ---------------------------------------------------------------- writes
    for (int64_t task = tid; task < (int64_t)kw * V; task += kDecThreads) {
        const int slot = (int)(task / V);
        const int64_t col = task % V;
        const int h = (int)(col / dv), c = (int)(col % dv);
        const int64_t bank = wbank[slot];
        if (bank < 0) continue;
        const int64_t base = ((row * J + bank) * H + h) * (int64_t)S * dv + c;
        const float *e = se + (slot * H + h) * S;
        const float *a = sa + (slot * H + h) * S;
        const float *kk = sk + (slot * H + h) * S;
        float hd[S];
        float erase = 0.f;
#pragma unroll
        for (int s = 0; s < S; ++s) {
            hd[s] = ld_state<CT>(state, base + (int64_t)s * dv) * e[s];
            erase = fmaf(a[s], hd[s], erase);
        }
        const float p = wwt[slot];
        const int64_t tv = row * V + col;
        const float u = rnd<T>(Elem<T>::to_float(w[tv]) * p) * Elem<T>::to_float(v[tv]) - erase;
#pragma unroll
        for (int s = 0; s < S; ++s) st_state<CT>(state, base + (int64_t)s * dv, fmaf(kk[s], u, hd[s]));
    }
    __syncthreads();  // block-wide visibility of the rewritten banks
    // ----------------------------------------------------------------- reads
    for (int64_t task = tid; task < (int64_t)kr * V; task += kDecThreads) {
        const int slot = (int)(task / V);
        const int64_t col = task % V;
        const int h = (int)(col / dv), c = (int)(col % dv);
        const int64_t bank = rbank[slot];
        float val = 0.f;
        if (bank >= 0) {
            const int64_t base = ((row * J + bank) * H + h) * (int64_t)S * dv + c;
            const float *qe = sq + (slot * H + h) * S;
            float x[S];
#pragma unroll
            for (int s = 0; s < S; ++s) x[s] = ld_state<CT>(state, base + (int64_t)s * dv) * qe[s];
            float sum;
            if constexpr (S == 8) {
                sum = ((x[0] + x[1]) + (x[4] + x[5])) + ((x[2] + x[3]) + (x[6] + x[7]));
            } else {
                sum = 0.f;
#pragma unroll
                for (int s = 0; s < S; ++s) sum += x[s];
            }
            val = rnd<T>(sum * scale);
        }
        reads[task] = val;
    }
    __syncthreads();
    // -------------------------------------- ascending-bank sum (+ norm, gate)
    const bool fuse = nrm.gate != nullptr;
    float sum1 = 0.f, sum2 = 0.f;
    for (int64_t col = tid; col < V; col += kDecThreads) {
        float acc = 0.f;
        for (int r = 0; r < kr; ++r) acc = rnd<T>(acc + reads[(int64_t)rorder[r] * V + col]);
        if (raw) raw[row * V + col] = Elem<T>::from_float(acc);
        reads[col] = acc;  // slot 0's row is no longer needed: keep the sums for the norm
        sum1 += acc;
    }
    if (!fuse) return;  // CTA-uniform
    __syncthreads();
    const float inv_w = 1.0f / (float)V;
    const T *nw = static_cast<const T *>(nrm.nw);
    const T *nb = static_cast<const T *>(nrm.nb);
    const T *gt = static_cast<const T *>(nrm.gate) + row * nrm.ld_gate;
    T *out = static_cast<T *>(nrm.out) + row * V;
    if (nrm.mode == 1) {
        const float mean = dec_block_sum(sum1, red) * inv_w;
        for (int64_t col = tid; col < V; col += kDecThreads) {
            const float d = reads[col] - mean;
            sum2 += d * d;
        }
        const float var = dec_block_sum(sum2, red) * inv_w;
        const float rstd = 1.0f / sqrtf(var + nrm.eps);
        for (int64_t col = tid; col < V; col += kDecThreads) {
            float y = (reads[col] - mean) * rstd * Elem<T>::to_float(nw[col]);
            if (nb) y += Elem<T>::to_float(nb[col]);
            out[col] = Elem<T>::from_float(rnd<T>(y) * gate_sigmoid<T>(Elem<T>::to_float(gt[col])));
        }
    } else {
        for (int64_t col = tid; col < V; col += kDecThreads) sum2 += reads[col] * reads[col];
        const float var = dec_block_sum(sum2, red) * inv_w;
        const float sc = rnd<T>(1.0f / sqrtf(var + nrm.eps));
        for (int64_t col = tid; col < V; col += kDecThreads) {
            const float n = rnd<T>(rnd<T>(reads[col] * sc) * Elem<T>::to_float(nw[col]));
            out[col] = Elem<T>::from_float(n * gate_sigmoid<T>(Elem<T>::to_float(gt[col])));
        }
    }
}

template <typename T, typename CT>
int launch_decode(const void *q, const void *k, const void *v, const float *g, const void *b, const void *w,
                  const int64_t *wi, const void *ww, const int64_t *ri, const void *rw, int64_t batch, int64_t J, int H,
                  int S, int dv, int kw, int kr, int routed_decay, float scale, void *state, void *raw,
                  const DecNorm &nrm, cudaStream_t st) {
    const size_t smem = (size_t)(3 * kw + kr) * H * S * sizeof(float) + (size_t)kr * H * dv * sizeof(float);
    if (smem > 200 * 1024) return BDM_ERR_UNSUPPORTED;
#define BDM_DEC_CASE(SS)                                                                                           \
    case SS: {                                                                                                     \
        auto kern = decode_kernel<T, CT, SS>;                                                                      \
        if (smem > 48 * 1024) {                                                                                    \
            int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
            if (rc) return rc;                                                                                     \
        }                                                                                                          \
        kern<<<(unsigned)batch, kDecThreads, smem, st>>>(                                                          \
            static_cast<const T *>(q), static_cast<const T *>(k), static_cast<const T *>(v), g,                   \
            static_cast<const T *>(b), static_cast<const T *>(w), wi, static_cast<const T *>(ww), ri,             \
            static_cast<const T *>(rw), J, H, dv, kw, kr, routed_decay, scale, state, static_cast<T *>(raw), nrm); \
        return launch_status();                                                                                    \
    }
    switch (S) {
        BDM_DEC_CASE(4)
        BDM_DEC_CASE(8)
        BDM_DEC_CASE(16)
        default: return BDM_ERR_UNSUPPORTED;
    }
#undef BDM_DEC_CASE
}

}  // namespace
}  // namespace bdm

extern "C" int bdm_decode_step(const void *q, const void *k, const void *v, const float *g, const void *b,
                               const void *w, const int64_t *write_idx, const void *write_w, const int64_t *read_idx,
                               const void *read_w, int64_t batch, int64_t bank_count, int heads, int bank_size,
                               int head_value_width, int kw, int kr, int dtype, int routed_decay, float scale,
                               void *state, int state_dtype, void *raw, const void *gate, int64_t ld_gate,
                               const void *norm_weight, const void *norm_bias, float eps, int norm_mode, void *out,
                               void *stream) {
    using namespace bdm;
    if (batch < 0 || bank_count <= 0 || heads <= 0 || head_value_width <= 0 || kw <= 0 || kr <= 0)
        return BDM_ERR_INVALID;
    if (kw > kDecMaxK || kr > kDecMaxK || bank_size > kDecMaxS) return BDM_ERR_UNSUPPORTED;
    if (batch == 0) return BDM_OK;
    if (batch > 0x7fffffffLL) return BDM_ERR_UNSUPPORTED;
    if (!q || !k || !v || !g || !b || !w || !write_idx || !write_w || !read_idx || !read_w || !state)
        return BDM_ERR_INVALID;
    if (!gate && !raw) return BDM_ERR_INVALID;  // nothing to write
    if (gate && (!norm_weight || !out || ld_gate < (int64_t)heads * head_value_width ||
                 (norm_mode != 0 && norm_mode != 1)))
        return BDM_ERR_INVALID;
    if (!valid_dtype(state_dtype)) return BDM_ERR_DTYPE;
    const DecNorm nrm{gate, ld_gate, norm_weight, norm_bias, eps, norm_mode, out};
    cudaStream_t st = as_stream(stream);
    BDM_DISPATCH_DTYPE(dtype, T, {
        if (state_dtype == BDM_BF16)
            return launch_decode<T, bf16>(q, k, v, g, b, w, write_idx, write_w, read_idx, read_w, batch, bank_count,
                                          heads, bank_size, head_value_width, kw, kr, routed_decay, scale, state, raw,
                                          nrm, st);
        return launch_decode<T, float>(q, k, v, g, b, w, write_idx, write_w, read_idx, read_w, batch, bank_count,
                                       heads, bank_size, head_value_width, kw, kr, routed_decay, scale, state, raw,
                                       nrm, st);
    });
    return BDM_OK;
}
