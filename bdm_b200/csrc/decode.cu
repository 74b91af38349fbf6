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
#include "controller_math.cuh"
#include "norm_gate.cuh"
#include "route_select.cuh"

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

// Output norm and gate: the combine kernels' arithmetic (norm_gate.cuh).
using ng::gate_sigmoid;
using ng::layer_norm_col;

// The arithmetic both step kernels share, with explicit roundings (no multiply-add
// contraction), so the fused step and the separate kernels agree bit for bit.
// u = dtype(w p) v - erase of a write.
template <typename T> __device__ __forceinline__ float write_u(float w, float p, float v, float erase) {
    return __fsub_rn(__fmul_rn(rnd<T>(__fmul_rn(w, p)), v), erase);
}
// dtype(scale * sum_s M_s q_s) of a read: the S = 8 pairwise tree of forward_rows.py:5-7.
template <typename T, int S> __device__ __forceinline__ float read_value(const float (&m)[S], const float *qe, float scale) {
    float x[S];
#pragma unroll
    for (int s = 0; s < S; ++s) x[s] = __fmul_rn(m[s], qe[s]);
    float sum;
    if constexpr (S == 8) {
        sum = __fadd_rn(__fadd_rn(__fadd_rn(x[0], x[1]), __fadd_rn(x[4], x[5])),
                        __fadd_rn(__fadd_rn(x[2], x[3]), __fadd_rn(x[6], x[7])));
    } else {
        sum = 0.f;
#pragma unroll
        for (int s = 0; s < S; ++s) sum = __fadd_rn(sum, x[s]);
    }
    return rnd<T>(__fmul_rn(sum, scale));
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
        const float u = write_u<T>(Elem<T>::to_float(w[tv]), p, Elem<T>::to_float(v[tv]), erase);
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
            float m[S];
#pragma unroll
            for (int s = 0; s < S; ++s) m[s] = ld_state<CT>(state, base + (int64_t)s * dv);
            val = read_value<T, S>(m, qe, scale);
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
            const float d = __fsub_rn(reads[col], mean);
            sum2 = fmaf(d, d, sum2);
        }
        const float var = dec_block_sum(sum2, red) * inv_w;
        const float rstd = 1.0f / sqrtf(var + nrm.eps);
        for (int64_t col = tid; col < V; col += kDecThreads) {
            const float bias = nb ? Elem<T>::to_float(nb[col]) : 0.f;
            const float y = layer_norm_col(reads[col], mean, rstd, Elem<T>::to_float(nw[col]), nb ? &bias : nullptr);
            out[col] = Elem<T>::from_float(rnd<T>(y) * gate_sigmoid<T>(Elem<T>::to_float(gt[col])));
        }
    } else {
        for (int64_t col = tid; col < V; col += kDecThreads) sum2 = fmaf(reads[col], reads[col], sum2);
        const float var = dec_block_sum(sum2, red) * inv_w;
        const float sc = rnd<T>(1.0f / sqrtf(var + nrm.eps));
        for (int64_t col = tid; col < V; col += kDecThreads) {
            const float n = rnd<T>(rnd<T>(reads[col] * sc) * Elem<T>::to_float(nw[col]));
            out[col] = Elem<T>::from_float(n * gate_sigmoid<T>(Elem<T>::to_float(gt[col])));
        }
    }
}

// ---------------------------------------------------------------------------
// Fused decode step: the controllers and both routers run in the same CTA as the bank
// step, from the token's row of the fused input projection, so a step is three launches
// (projection GEMM, this kernel, o_proj).  Every part uses the separate kernels' arithmetic
// (controller_math.cuh, route_select.cuh and the helpers above).  The bank tiles of the
// write banks and of every read bank that is not also a write bank of the row are loaded in
// one round before the writes; a read bank that this step also writes is read after them.
// ---------------------------------------------------------------------------
struct DecTokenArgs {
    const void *proj;
    int64_t ld, col_q, col_k, col_v, col_f1, col_b, col_w, col_read, col_write, col_gate;
    const void *wf2;
    int f1_width;
    const float *a_log, *dt_bias;
    int qk_norm, j1, j2, sub, count;
    int64_t J;
    int H, dv, routed_decay;
    float scale;
    void *state;
    const void *nw, *nb;
    float eps;
    int mode;
    void *out;
};

template <typename T, typename CT, int S>
__global__ void __launch_bounds__(kDecThreads) decode_token_kernel(const DecTokenArgs a) {
    extern __shared__ float sm[];
    const int H = a.H, dv = a.dv, HS = H * S, kw = a.count, kr = a.count;
    const int64_t V = (int64_t)H * dv;
    const int rsc = route::token_scratch_floats(a.j1, a.j2, a.sub, a.count);
    float *rowf = sm;                   // the projection row
    float *zsc = rowf + a.ld;           // router scratch, [2][rsc]
    float *cq = zsc + 2 * rsc;          // q, k, b, g [HS]; v, w [V]
    float *ck = cq + HS;
    float *cb = ck + HS;
    float *cg = cb + HS;
    float *cv = cg + HS;
    float *cw = cv + V;
    float *se = cw + V;                 // per write slot: exp(g_e), a, k [kw][HS]
    float *sa = se + kw * HS;
    float *sk = sa + kw * HS;
    float *sq = sk + kw * HS;           // per read slot: dtype(q r) [kr][HS]
    float *reads = sq + kr * HS;        // [kr][V]
    float *wf2s = reads + kr * V;       // f_proj.1's weight [HS][f1_width]
    __shared__ int64_t wbank[kDecMaxK], rbank[kDecMaxK];
    __shared__ float wwt[kDecMaxK], rwt[kDecMaxK];
    __shared__ int rorder[kDecMaxK];
    __shared__ float red[32];
    __shared__ int cand[route::kMaxCand];
    __shared__ int ncand_s;

    const int64_t row = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = (int)lane_id();
    const T *prow = static_cast<const T *>(a.proj) + row * a.ld;
    for (int64_t i = tid; i < a.ld; i += kDecThreads) rowf[i] = Elem<T>::to_float(prow[i]);
    for (int i = tid; i < HS * a.f1_width; i += kDecThreads)
        wf2s[i] = Elem<T>::to_float(static_cast<const T *>(a.wf2)[i]);
    if (tid == 0) ncand_s = route::staircase_candidates(a.sub, a.count, cand, route::kMaxCand);
    __syncthreads();
    // ------------------------------------------ routers (warps 0, 1) and controllers (the rest)
    if (warp < 2) {
        float *z = zsc + warp * rsc;
        const int64_t col = warp == 0 ? a.col_write : a.col_read;
        for (int i = lane; i < a.j1 + a.j2; i += 32) z[i] = rowf[col + i];
        int64_t index = -1;
        float weight = 0.f;
        if (route::route_token<T>(z, a.j1, a.j2, a.sub, a.count, cand, ncand_s, index, weight)) {
            const int64_t bank = (index >= 0 && index < a.J) ? index : -1;
            if (warp == 0) {
                wbank[lane] = bank;
                wwt[lane] = rnd<T>(weight);
            } else {
                rbank[lane] = bank;
                rwt[lane] = rnd<T>(weight);
            }
        }
    } else {
        const int n_narrow = 2 * H, n_gate = HS;
        for (int64_t item = tid - 64; item < n_narrow + n_gate + V; item += kDecThreads - 64) {
            if (item < n_narrow) {  // q (role 0) or k (role 1) of head h: normalize(silu(.))
                const int role = (int)(item / H), h = (int)(item % H);
                const float *src = rowf + (role ? a.col_k : a.col_q) + h * S;
                float x[S], ss = 0.f;
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    x[s] = rnd<T>(ctl::silu_f(src[s]));
                    ss = fmaf(x[s], x[s], ss);
                }
                const float scale = ctl::qk_scale(ss, a.qk_norm);
                float *dst = (role ? ck : cq) + h * S;
#pragma unroll
                for (int s = 0; s < S; ++s) dst[s] = rnd<T>(x[s] * scale);
            } else if (item < n_narrow + n_gate) {  // b and the decay gate of (h, s); f = dtype(f1 . Wf2[hs])
                const int hs = (int)(item - n_narrow), h = hs / S;
                const float *f1 = rowf + a.col_f1;
                const float *wrow = wf2s + (int64_t)hs * a.f1_width;
                float acc = 0.f;
                for (int j = 0; j < a.f1_width; ++j) acc = fmaf(f1[j], wrow[j], acc);
                cb[hs] = rnd<T>(ctl::sigmoid_f(rowf[a.col_b + hs]));
                cg[hs] = ctl::decay_gate(a.a_log[h], rnd<T>(acc), a.dt_bias[hs]);
            } else {  // v = silu, w = sigmoid of one column
                const int64_t c = item - n_narrow - n_gate;
                cv[c] = rnd<T>(ctl::silu_fast(rowf[a.col_v + c]));
                cw[c] = rnd<T>(ctl::sigmoid_fast(rowf[a.col_w + c]));
            }
        }
    }
    __syncthreads();
    // ------------------------------------------------ per-slot controls (decode_kernel's)
    if (tid < kr) {  // ascending bank order, ties by slot
        const int64_t bj = rbank[tid];
        int rank = 0;
        for (int i = 0; i < kr; ++i) rank += (rbank[i] < bj) || (rbank[i] == bj && i < tid);
        rorder[rank] = tid;
    }
    for (int task = tid; task < kw * HS; task += kDecThreads) {
        const int slot = task / HS, hs = task % HS;
        const float p = wwt[slot];
        const float kk = ck[hs];
        const float ge = a.routed_decay ? cg[hs] * p : cg[hs];
        se[task] = expf(ge);
        sa[task] = rnd<T>(cb[hs] * p) * kk;
        sk[task] = kk;
    }
    for (int task = tid; task < kr * HS; task += kDecThreads) {
        const int slot = task / HS, hs = task % HS;
        sq[task] = rnd<T>(cq[hs] * rwt[slot]);
    }
    __syncthreads();
    // -------------------------- read tiles that no write of this step touches: load now
    float pre[S];
    bool preloaded = false;
    if (tid < kr * V) {
        const int slot = (int)(tid / V);
        const int64_t col = tid % V;
        const int h = (int)(col / dv), c = (int)(col % dv);
        const int64_t bank = rbank[slot];
        bool hit = false;
        for (int i = 0; i < kw; ++i) hit |= wbank[i] == bank;
        if (bank >= 0 && !hit) {
            const int64_t base = ((row * a.J + bank) * H + h) * (int64_t)S * dv + c;
#pragma unroll
            for (int s = 0; s < S; ++s) pre[s] = ld_state<CT>(a.state, base + (int64_t)s * dv);
            preloaded = true;
        }
    }
    // ---------------------------------------------------------------- writes
    for (int64_t task = tid; task < (int64_t)kw * V; task += kDecThreads) {
        const int slot = (int)(task / V);
        const int64_t col = task % V;
        const int h = (int)(col / dv), c = (int)(col % dv);
        const int64_t bank = wbank[slot];
        if (bank < 0) continue;
        const int64_t base = ((row * a.J + bank) * H + h) * (int64_t)S * dv + c;
        const float *e = se + (slot * H + h) * S;
        const float *aa = sa + (slot * H + h) * S;
        const float *kk = sk + (slot * H + h) * S;
        float hd[S];
        float erase = 0.f;
#pragma unroll
        for (int s = 0; s < S; ++s) {
            hd[s] = ld_state<CT>(a.state, base + (int64_t)s * dv) * e[s];
            erase = fmaf(aa[s], hd[s], erase);
        }
        const float u = write_u<T>(cw[col], wwt[slot], cv[col], erase);
#pragma unroll
        for (int s = 0; s < S; ++s) st_state<CT>(a.state, base + (int64_t)s * dv, fmaf(kk[s], u, hd[s]));
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
            const int64_t base = ((row * a.J + bank) * H + h) * (int64_t)S * dv + c;
            const float *qe = sq + (slot * H + h) * S;
            float m[S];
            const bool use_pre = task == tid && preloaded;
#pragma unroll
            for (int s = 0; s < S; ++s) m[s] = use_pre ? pre[s] : ld_state<CT>(a.state, base + (int64_t)s * dv);
            val = read_value<T, S>(m, qe, a.scale);
        }
        reads[task] = val;
    }
    __syncthreads();
    // ------------------------------------ ascending-bank sum, norm, gate (decode_kernel's)
    float sum1 = 0.f, sum2 = 0.f;
    for (int64_t col = tid; col < V; col += kDecThreads) {
        float acc = 0.f;
        for (int r = 0; r < kr; ++r) acc = rnd<T>(acc + reads[(int64_t)rorder[r] * V + col]);
        reads[col] = acc;
        sum1 += acc;
    }
    __syncthreads();
    const float inv_w = 1.0f / (float)V;
    const T *nw = static_cast<const T *>(a.nw);
    const T *nb = static_cast<const T *>(a.nb);
    const float *gt = rowf + a.col_gate;
    T *out = static_cast<T *>(a.out) + row * V;
    if (a.mode == 1) {
        const float mean = dec_block_sum(sum1, red) * inv_w;
        for (int64_t col = tid; col < V; col += kDecThreads) {
            const float d = __fsub_rn(reads[col], mean);
            sum2 = fmaf(d, d, sum2);
        }
        const float var = dec_block_sum(sum2, red) * inv_w;
        const float rstd = 1.0f / sqrtf(var + a.eps);
        for (int64_t col = tid; col < V; col += kDecThreads) {
            const float bias = nb ? Elem<T>::to_float(nb[col]) : 0.f;
            const float y = layer_norm_col(reads[col], mean, rstd, Elem<T>::to_float(nw[col]), nb ? &bias : nullptr);
            out[col] = Elem<T>::from_float(rnd<T>(y) * gate_sigmoid<T>(gt[col]));
        }
    } else {
        for (int64_t col = tid; col < V; col += kDecThreads) sum2 = fmaf(reads[col], reads[col], sum2);
        const float var = dec_block_sum(sum2, red) * inv_w;
        const float sc = rnd<T>(1.0f / sqrtf(var + a.eps));
        for (int64_t col = tid; col < V; col += kDecThreads) {
            const float n = rnd<T>(rnd<T>(reads[col] * sc) * Elem<T>::to_float(nw[col]));
            out[col] = Elem<T>::from_float(n * gate_sigmoid<T>(gt[col]));
        }
    }
}

template <typename T, typename CT>
int launch_decode_token(const DecTokenArgs &a, int S, int64_t batch, cudaStream_t st) {
    const int64_t V = (int64_t)a.H * a.dv;
    const int HS = a.H * S;
    const size_t smem = ((size_t)a.ld + 2 * route::token_scratch_floats(a.j1, a.j2, a.sub, a.count) + 4 * HS +
                         2 * V + (size_t)4 * a.count * HS + (size_t)a.count * V + (size_t)HS * a.f1_width) *
                        sizeof(float);
    if (smem > 200 * 1024) return BDM_ERR_UNSUPPORTED;
#define BDM_DECT_CASE(SS)                                                                                          \
    case SS: {                                                                                                     \
        auto kern = decode_token_kernel<T, CT, SS>;                                                                \
        if (smem > 48 * 1024) {                                                                                    \
            int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
            if (rc) return rc;                                                                                     \
        }                                                                                                          \
        kern<<<(unsigned)batch, kDecThreads, smem, st>>>(a);                                                       \
        return launch_status();                                                                                    \
    }
    switch (S) {
        BDM_DECT_CASE(4)
        BDM_DECT_CASE(8)
        BDM_DECT_CASE(16)
        default: return BDM_ERR_UNSUPPORTED;
    }
#undef BDM_DECT_CASE
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

extern "C" int bdm_decode_token_step(const void *proj, int64_t batch, int64_t ld, int64_t col_q, int64_t col_k,
                                     int64_t col_v, int64_t col_f1, int64_t col_b, int64_t col_w, int64_t col_read,
                                     int64_t col_write, int64_t col_gate, const void *wf2, int f1_width,
                                     const float *a_log, const float *dt_bias, int qk_norm, int j1, int j2,
                                     int selected, int64_t bank_count, int heads, int bank_size,
                                     int head_value_width, int dtype, int routed_decay, float scale, void *state,
                                     int state_dtype, const void *norm_weight, const void *norm_bias, float eps,
                                     int norm_mode, void *out, void *stream) {
    using namespace bdm;
    if (batch < 0 || bank_count <= 0 || heads <= 0 || head_value_width <= 0 || selected <= 0 || j1 <= 0 ||
        j2 <= 0 || (int64_t)j1 * j2 != bank_count || f1_width <= 0 || (norm_mode != 0 && norm_mode != 1))
        return BDM_ERR_INVALID;
    if (batch == 0) return BDM_OK;
    if (!proj || !wf2 || !a_log || !dt_bias || !state || !norm_weight || !out) return BDM_ERR_INVALID;
    const int64_t HS = (int64_t)heads * bank_size, V = (int64_t)heads * head_value_width;
    const int64_t need[][2] = {{col_q, HS}, {col_k, HS}, {col_v, V}, {col_f1, f1_width}, {col_b, HS}, {col_w, V},
                               {col_read, j1 + j2}, {col_write, j1 + j2}, {col_gate, V}};
    for (const auto &n : need)
        if (n[0] < 0 || n[0] + n[1] > ld) return BDM_ERR_INVALID;
    int sub = selected < j1 ? selected : j1;
    sub = sub < j2 ? sub : j2;
    const int count = selected < sub * sub ? selected : sub * sub;
    if (j1 > 1024 || j2 > 1024 || sub > 32 || count > 32) return BDM_ERR_UNSUPPORTED;
    if (bank_size > kDecMaxS || batch > 0x7fffffffLL) return BDM_ERR_UNSUPPORTED;
    if (!valid_dtype(state_dtype)) return BDM_ERR_DTYPE;
    DecTokenArgs a{};
    a.proj = proj; a.ld = ld; a.col_q = col_q; a.col_k = col_k; a.col_v = col_v; a.col_f1 = col_f1;
    a.col_b = col_b; a.col_w = col_w; a.col_read = col_read; a.col_write = col_write; a.col_gate = col_gate;
    a.wf2 = wf2; a.f1_width = f1_width; a.a_log = a_log; a.dt_bias = dt_bias; a.qk_norm = qk_norm;
    a.j1 = j1; a.j2 = j2; a.sub = sub; a.count = count; a.J = bank_count; a.H = heads; a.dv = head_value_width;
    a.routed_decay = routed_decay; a.scale = scale; a.state = state; a.nw = norm_weight; a.nb = norm_bias;
    a.eps = eps; a.mode = norm_mode; a.out = out;
    cudaStream_t st = as_stream(stream);
    BDM_DISPATCH_DTYPE(dtype, T, {
        if (state_dtype == BDM_BF16) return launch_decode_token<T, bf16>(a, bank_size, batch, st);
        return launch_decode_token<T, float>(a, bank_size, batch, st);
    });
    return BDM_OK;
}
