// Product-key top-B router (one warp per token).
//
// Restates product_key_route (implementation/bdm/gdn2_banks.py:74-114):
//   top-sub per factor -> sub x sub pair sums in the logits dtype -> top-count
//   -> softmax in FP32, index = row * J2 + col.
// Every selection orders by (value desc, index asc), so equal scores resolve to
// the lower index -- the tie rule the reference leaves to torch.topk.  Short
// lists (factor widths <= 128, the pair "staircase") are ranked directly; wide
// factors use warp arg-max rounds over 64-bit keys (order-preserving value
// bits : inverted index).
#include "common.cuh"

namespace bdm {
namespace {

constexpr int kRouteWarps = 8;
constexpr int kRankMax = 128;  // factor widths ranked directly
constexpr int kMaxCand = 128;  // staircase pair candidates handled by ranking

__device__ __forceinline__ uint32_t ordered_bits(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Warp arg-max of (hi, lo) keys; every lane gets the winning key.
__device__ __forceinline__ void warp_argmax(uint32_t hi, uint32_t lo, uint32_t &wh, uint32_t &wl) {
    wh = __reduce_max_sync(0xffffffffu, hi);
    wl = __reduce_max_sync(0xffffffffu, hi == wh ? lo : 0u);
}

// Local best of the elements this lane owns (i = lane + 32*m), skipping taken ones.
__device__ __forceinline__ void lane_best(const float *vals, int n, uint32_t taken, uint32_t &bh, uint32_t &bl) {
    bh = 0u;
    bl = 0u;
    const int lane = (int)lane_id();
    for (int m = 0, i = lane; i < n; ++m, i += 32) {
        if (taken & (1u << m)) continue;
        uint32_t h = ordered_bits(vals[i]);
        uint32_t l = ~(uint32_t)i;
        if (h > bh || (h == bh && l > bl)) {
            bh = h;
            bl = l;
        }
    }
}

// Top-k of vals[0..n) (n <= 1024, k <= n) ordered by (value desc, index asc).
__device__ void warp_topk(const float *vals, int n, int k, float *out_v, int *out_i) {
    const int lane = (int)lane_id();
    uint32_t taken = 0u, bh, bl;
    lane_best(vals, n, taken, bh, bl);
    for (int r = 0; r < k; ++r) {
        uint32_t wh, wl;
        warp_argmax(bh, bl, wh, wl);
        int i = (int)(~wl);
        if (lane == 0) {
            out_v[r] = vals[i];
            out_i[r] = i;
        }
        if ((i & 31) == lane) {
            taken |= 1u << (i >> 5);
            lane_best(vals, n, taken, bh, bl);
        }
    }
    __syncwarp();
}

// Rank selection for short lists: element i's rank is the number of elements
// ordered before it by (value desc, index asc); ranks < k are written to
// out[rank].  n <= 4 * 32.
__device__ void warp_rank_select(const float *vals, int n, int k, float *out_v, int *out_i) {
    const int lane = (int)lane_id();
    for (int i = lane; i < n; i += 32) {
        const float x = vals[i];
        int rank = 0;
        for (int j = 0; j < n; ++j) {
            const float y = vals[j];
            rank += (y > x) || (y == x && j < i);
        }
        if (rank < k) {
            out_v[rank] = x;
            out_i[rank] = i;
        }
    }
    __syncwarp();
}

// Pairs (i, l) that can reach the top `count`: a pair is outranked by every
// (i', l') <= (i, l) componentwise (sums of descending lists, lower pair index),
// so only pairs with (i + 1) * (l + 1) <= count are candidates.  Returns the
// candidate count, or cap + 1 (list not filled) when more than `cap` exist.
__device__ int staircase_candidates(int sub, int count, int *cand, int cap) {
    int m = 0;
    for (int i = 0; i < sub; ++i) {
        const int width = min(sub, count / (i + 1));
        for (int l = 0; l < width; ++l) {
            if (m == cap) return cap + 1;
            cand[m++] = i * sub + l;
        }
    }
    return m;
}

// Two routers over the same rows in one launch: virtual token t < ntok routes the
// block at column 0 into (out_idx, out_w); t >= ntok routes the block at column
// `second` of row t - ntok into (out_idx2, out_w2).  second < 0: one router.
template <typename T>
__global__ void __launch_bounds__(kRouteWarps * 32)
route_kernel(const T *__restrict__ logits, int64_t ntok, int64_t ld, int j1, int j2, int sub, int count,
             int64_t *__restrict__ out_idx, T *__restrict__ out_w, int64_t second, int64_t *__restrict__ out_idx2,
             T *__restrict__ out_w2) {
    extern __shared__ float smem[];
    __shared__ int cand[kMaxCand];
    __shared__ int ncand_s;
    const int warp = threadIdx.x >> 5;
    const int lane = (int)lane_id();
    if (threadIdx.x == 0) ncand_s = staircase_candidates(sub, count, cand, kMaxCand);
    __syncthreads();
    const int ncand = ncand_s;
    const bool fast_pairs = ncand <= kMaxCand && ncand > 0;
    const int per_warp = j1 + j2 + 4 * sub + sub * sub + 2 * count;
    float *z = smem + warp * per_warp;
    float *fv = z + j1 + j2;
    float *sv = fv + sub;
    int *fi = reinterpret_cast<int *>(sv + sub);
    int *si = fi + sub;
    float *pv = reinterpret_cast<float *>(si + sub);
    float *cv = pv + sub * sub;
    int *ci = reinterpret_cast<int *>(cv + count);

    const int64_t nvirt = second >= 0 ? 2 * ntok : ntok;
    for (int64_t vt = (int64_t)blockIdx.x * kRouteWarps + warp; vt < nvirt; vt += (int64_t)gridDim.x * kRouteWarps) {
        const bool other = vt >= ntok;
        const int64_t t = other ? vt - ntok : vt;
        const T *row = logits + t * ld + (other ? second : 0);
        int64_t *oidx = other ? out_idx2 : out_idx;
        T *ow = other ? out_w2 : out_w;
        for (int i = lane; i < j1 + j2; i += 32) z[i] = Elem<T>::to_float(row[i]);
        __syncwarp();
        if (j1 <= kRankMax) warp_rank_select(z, j1, sub, fv, fi);
        else warp_topk(z, j1, sub, fv, fi);
        if (j2 <= kRankMax) warp_rank_select(z + j1, j2, sub, sv, si);
        else warp_topk(z + j1, j2, sub, sv, si);
        // Pair scores in the logits dtype, pair p = i*sub + l (gdn2_banks.py:106-110).
        if (fast_pairs) {
            for (int c = lane; c < ncand; c += 32) {
                const int p = cand[c];
                pv[c] = rnd<T>(fv[p / sub] + sv[p % sub]);
            }
            __syncwarp();
            for (int c = lane; c < ncand; c += 32) {
                const float x = pv[c];
                const int pc = cand[c];
                int rank = 0;
                for (int d = 0; d < ncand; ++d) {
                    const float y = pv[d];
                    rank += (y > x) || (y == x && cand[d] < pc);
                }
                if (rank < count) {
                    cv[rank] = x;
                    ci[rank] = pc;
                }
            }
            __syncwarp();
        } else {
            for (int p = lane; p < sub * sub; p += 32) pv[p] = rnd<T>(fv[p / sub] + sv[p % sub]);
            __syncwarp();
            warp_topk(pv, sub * sub, count, cv, ci);
        }
        // Softmax in FP32 over the descending selection: cv[0] is the maximum.
        float e = 0.f;
        if (lane < count) e = expf(cv[lane] - cv[0]);
        float sum = warp_sum(e);
        if (lane < count) {
            int p = ci[lane];
            oidx[t * count + lane] = (int64_t)fi[p / sub] * j2 + si[p % sub];
            ow[t * count + lane] = Elem<T>::from_float(e / sum);
        }
        __syncwarp();
    }
}

}  // namespace
}  // namespace bdm

namespace bdm {
namespace {

int route_launch(const void *logits, int64_t ntok, int64_t ld, int j1, int j2, int selected, int dtype,
                 int64_t *indices, void *weights, int64_t second, int64_t *indices2, void *weights2, void *stream) {
    int sub = selected < j1 ? selected : j1;
    sub = sub < j2 ? sub : j2;
    int count = selected < sub * sub ? selected : sub * sub;
    if (j1 > 1024 || j2 > 1024 || sub > 32 || count > 32) return BDM_ERR_UNSUPPORTED;
    size_t per_warp = (size_t)(j1 + j2 + 4 * sub + sub * sub + 2 * count) * sizeof(float);
    size_t smem = per_warp * kRouteWarps;
    if (smem > 200 * 1024) return BDM_ERR_UNSUPPORTED;
    int64_t blocks = ceil_div(second >= 0 ? 2 * ntok : ntok, kRouteWarps);
    if (blocks > 16 * kNumSMs) blocks = 16 * kNumSMs;
    BDM_DISPATCH_DTYPE(dtype, T, {
        auto kern = route_kernel<T>;
        if (smem > 48 * 1024) {
            int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            if (rc) return rc;
        }
        kern<<<(unsigned)blocks, kRouteWarps * 32, smem, as_stream(stream)>>>(
            static_cast<const T *>(logits), ntok, ld, j1, j2, sub, count, indices, static_cast<T *>(weights), second,
            indices2, static_cast<T *>(weights2));
    });
    return launch_status();
}

}  // namespace
}  // namespace bdm

extern "C" int bdm_route(const void *logits, int64_t ntok, int64_t ld, int j1, int j2, int selected, int dtype,
                         int64_t *indices, void *weights, void *stream) {
    using namespace bdm;
    if (ntok < 0 || j1 <= 0 || j2 <= 0 || selected <= 0 || ld < j1 + j2) return BDM_ERR_INVALID;
    if (ntok == 0) return BDM_OK;
    if (!logits || !indices || !weights) return BDM_ERR_INVALID;
    return route_launch(logits, ntok, ld, j1, j2, selected, dtype, indices, weights, -1, nullptr, nullptr, stream);
}

extern "C" int bdm_route_pair(const void *logits, int64_t ntok, int64_t ld, int64_t second, int j1, int j2,
                              int selected, int dtype, int64_t *indices, void *weights, int64_t *indices2,
                              void *weights2, void *stream) {
    using namespace bdm;
    if (ntok < 0 || j1 <= 0 || j2 <= 0 || selected <= 0 || second < 0 || ld < j1 + j2 || ld < second + j1 + j2)
        return BDM_ERR_INVALID;
    if (ntok == 0) return BDM_OK;
    if (!logits || !indices || !weights || !indices2 || !weights2) return BDM_ERR_INVALID;
    return route_launch(logits, ntok, ld, j1, j2, selected, dtype, indices, weights, second, indices2, weights2,
                        stream);
}
