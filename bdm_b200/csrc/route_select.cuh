// Product-key top-B selection for one token on one warp (restates product_key_route,
// implementation/bdm/gdn2_banks.py:74-114): top-sub per factor -> sub x sub pair sums in the
// logits dtype -> top-count -> FP32 softmax, index = row * J2 + col.  Every selection orders by
// (value desc, index asc), so equal scores resolve to the lower index -- the tie rule the
// reference leaves to torch.topk.  Short lists (factor widths <= 128, the pair "staircase") are
// sorted in registers (warp bitonic network over 64-bit keys: order-preserving value bits above
// the inverted index; both factors in one sort when together they fit 128 keys); wide factors use
// warp arg-max rounds over the same keys.  Shared by the router kernel (router.cu) and the fused
// decode step (decode.cu).
#pragma once

#include "common.cuh"

namespace bdm {
namespace route {

constexpr int kRankMax = 128;  // factor widths sorted in registers
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
__device__ __forceinline__ void warp_topk(const float *vals, int n, int k, float *out_v, int *out_i) {
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

// Selection key: order-preserving value bits above the inverted index, so the descending key
// order is (value desc, index asc); -0 and +0 are one value, as in a float comparison.
__device__ __forceinline__ unsigned long long sel_key(float v, int i) {
    if (v == 0.f) v = 0.f;
    return ((unsigned long long)ordered_bits(v) << 32) | (unsigned long long)(~(uint32_t)i);
}

// Sorts 32*M keys held as key[m] of lane l (element l + 32 m) into descending order across the
// warp (bitonic network: shuffles between lanes, exchanges inside a lane for strides >= 32).
template <int M>
__device__ __forceinline__ void warp_bitonic_desc(unsigned long long (&key)[M]) {
    const int lane = (int)lane_id();
#pragma unroll
    for (int k = 2; k <= 32 * M; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j >= 32) {
                const int mj = j / 32;
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    if (m & mj) continue;
                    const bool desc = ((lane + 32 * m) & k) == 0;
                    const unsigned long long a = key[m], b = key[m ^ mj];
                    const bool swap = desc ? (a < b) : (a > b);
                    key[m] = swap ? b : a;
                    key[m ^ mj] = swap ? a : b;
                }
            } else {
                const bool lower = (lane & j) == 0;
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    const bool desc = ((lane + 32 * m) & k) == 0;
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, key[m], j);
                    const bool keep_max = lower == desc;
                    key[m] = keep_max ? (key[m] > other ? key[m] : other) : (key[m] < other ? key[m] : other);
                }
            }
        }
    }
}

// Top-k (k <= 32) of vals[0..n), n <= 32 * M, by (value desc, index asc): keys sorted in registers.
template <int M>
__device__ __forceinline__ void warp_sort_select_m(const float *vals, int n, int k, float *out_v, int *out_i) {
    const int lane = (int)lane_id();
    unsigned long long key[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const int e = lane + 32 * m;
        key[m] = e < n ? sel_key(vals[e], e) : 0ull;
    }
    warp_bitonic_desc<M>(key);
    if (lane < k) {
        const int i = (int)(~(uint32_t)(key[0] & 0xffffffffu));
        out_v[lane] = vals[i];
        out_i[lane] = i;
    }
    __syncwarp();
}

__device__ __forceinline__ void warp_sort_select(const float *vals, int n, int k, float *out_v, int *out_i) {
    if (n <= 32) warp_sort_select_m<1>(vals, n, k, out_v, out_i);
    else if (n <= 64) warp_sort_select_m<2>(vals, n, k, out_v, out_i);
    else warp_sort_select_m<4>(vals, n, k, out_v, out_i);
}

// Top-sub of both factors at once: z[0, j1) and z[j1, j1 + j2), j1 + j2 <= 32 * M, in one sort.
// A key carries its factor above the selection key (value bits, inverted index within the
// factor), so factor 1 sorts ahead of factor 2 and each keeps the (value desc, index asc) order:
// factor 1's top-sub end at flat positions [0, sub), factor 2's at [j1, j1 + sub).
template <int M>
__device__ __forceinline__ void warp_sort_select_pair_m(const float *z, int j1, int j2, int sub, float *fv, int *fi,
                                                        float *sv, int *si) {
    const int lane = (int)lane_id();
    unsigned long long key[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const int e = lane + 32 * m;
        if (e < j1 + j2) {
            const bool first = e < j1;
            const int i = first ? e : e - j1;
            float v = z[e];
            if (v == 0.f) v = 0.f;
            key[m] = ((unsigned long long)(first ? 1u : 0u) << 63) | ((unsigned long long)ordered_bits(v) << 31) |
                     (unsigned long long)(~(uint32_t)i & 0x7fffffffu);
        } else {
            key[m] = 0ull;
        }
    }
    warp_bitonic_desc<M>(key);
    // factor 2's l-th key sits at flat position j1 + l: lane (j1 + l) % 32, register (j1 + l) / 32
    const int e2 = j1 + lane;
    unsigned long long k2 = 0ull;
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const unsigned long long t = __shfl_sync(0xffffffffu, key[m], e2 & 31);
        if ((e2 >> 5) == m) k2 = t;
    }
    if (lane < sub) {
        const int i1 = (int)(~(uint32_t)(key[0] & 0x7fffffffull) & 0x7fffffffu);
        const int i2 = (int)(~(uint32_t)(k2 & 0x7fffffffull) & 0x7fffffffu);
        fv[lane] = z[i1];
        fi[lane] = i1;
        sv[lane] = z[j1 + i2];
        si[lane] = i2;
    }
    __syncwarp();
}

// Pairs (i, l) that can reach the top `count`: a pair is outranked by every
// (i', l') <= (i, l) componentwise (sums of descending lists, lower pair index),
// so only pairs with (i + 1) * (l + 1) <= count are candidates.  Returns the
// candidate count, or cap + 1 (list not filled) when more than `cap` exist.
__device__ __forceinline__ int staircase_candidates(int sub, int count, int *cand, int cap) {
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

// Scratch floats of one warp's token, laid out as route_token expects.
__host__ __device__ constexpr int token_scratch_floats(int j1, int j2, int sub, int count) {
    return j1 + j2 + 4 * sub + sub * sub + 2 * count;
}

// Routes one token: scratch[0 .. j1 + j2) holds its logits; cand / ncand are the staircase
// candidates (staircase_candidates).  Lane i < count gets (index, weight) of the i-th selection in
// descending score order and returns true.
template <typename T>
__device__ __forceinline__ bool route_token(float *scratch, int j1, int j2, int sub, int count, const int *cand,
                                            int ncand, int64_t &index, float &weight) {
    const int lane = (int)lane_id();
    const bool fast_pairs = ncand <= kMaxCand && ncand > 0;
    float *z = scratch;
    float *fv = z + j1 + j2;
    float *sv = fv + sub;
    int *fi = reinterpret_cast<int *>(sv + sub);
    int *si = fi + sub;
    float *pv = reinterpret_cast<float *>(si + sub);
    float *cv = pv + sub * sub;
    int *ci = reinterpret_cast<int *>(cv + count);
    __syncwarp();
    if (j1 + j2 <= 32) {  // both factors in one register sort
        warp_sort_select_pair_m<1>(z, j1, j2, sub, fv, fi, sv, si);
    } else if (j1 + j2 <= 64) {
        warp_sort_select_pair_m<2>(z, j1, j2, sub, fv, fi, sv, si);
    } else if (j1 + j2 <= kRankMax) {
        warp_sort_select_pair_m<4>(z, j1, j2, sub, fv, fi, sv, si);
    } else {
        if (j1 <= kRankMax) warp_sort_select(z, j1, sub, fv, fi);
        else warp_topk(z, j1, sub, fv, fi);
        if (j2 <= kRankMax) warp_sort_select(z + j1, j2, sub, sv, si);
        else warp_topk(z + j1, j2, sub, sv, si);
    }
    // Pair scores in the logits dtype, pair p = i*sub + l (gdn2_banks.py:106-110).
    if (fast_pairs) {
        for (int c = lane; c < ncand; c += 32) {
            const int p = cand[c];
            pv[c] = rnd<T>(fv[p / sub] + sv[p % sub]);
        }
        __syncwarp();
        // candidates are listed in ascending pair index, so the slot c orders ties as p does
        if (ncand <= 32) {
            unsigned long long key[1] = {lane < ncand ? sel_key(pv[lane], lane) : 0ull};
            warp_bitonic_desc<1>(key);
            if (lane < count) {
                const int c = (int)(~(uint32_t)(key[0] & 0xffffffffu));
                cv[lane] = pv[c];
                ci[lane] = cand[c];
            }
        } else {
            unsigned long long key[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int c = lane + 32 * m;
                key[m] = c < ncand ? sel_key(pv[c], c) : 0ull;
            }
            warp_bitonic_desc<4>(key);
            if (lane < count) {
                const int c = (int)(~(uint32_t)(key[0] & 0xffffffffu));
                cv[lane] = pv[c];
                ci[lane] = cand[c];
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
    const float sum = warp_sum(e);
    bool mine = false;
    if (lane < count) {
        const int p = ci[lane];
        index = (int64_t)fi[p / sub] * j2 + si[p % sub];
        weight = e / sum;
        mine = true;
    }
    __syncwarp();
    return mine;
}

}  // namespace route
}  // namespace bdm
