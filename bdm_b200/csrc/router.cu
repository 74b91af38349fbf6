// Product-key top-B router (one warp per token): route_select.cuh's per-token selection
// (restating product_key_route, implementation/bdm/gdn2_banks.py:74-114) over every row.
#include "common.cuh"
#include "route_select.cuh"

namespace bdm {
namespace {

constexpr int kRouteWarps = 8;
// Two routers over the same rows in one launch: virtual token t < ntok routes the
// block at column 0 into (out_idx, out_w); t >= ntok routes the block at column
// `second` of row t - ntok into (out_idx2, out_w2).  second < 0: one router.
template <typename T>
__global__ void __launch_bounds__(kRouteWarps * 32)
route_kernel(const T *__restrict__ logits, int64_t ntok, int64_t ld, int j1, int j2, int sub, int count,
             int64_t *__restrict__ out_idx, T *__restrict__ out_w, int64_t second, int64_t *__restrict__ out_idx2,
             T *__restrict__ out_w2) {
    extern __shared__ float smem[];
    __shared__ int cand[route::kMaxCand];
    __shared__ int ncand_s;
    const int warp = threadIdx.x >> 5;
    const int lane = (int)lane_id();
    if (threadIdx.x == 0) ncand_s = route::staircase_candidates(sub, count, cand, route::kMaxCand);
    __syncthreads();
    const int ncand = ncand_s;
    float *z = smem + warp * route::token_scratch_floats(j1, j2, sub, count);

    const int64_t nvirt = second >= 0 ? 2 * ntok : ntok;
    for (int64_t vt = (int64_t)blockIdx.x * kRouteWarps + warp; vt < nvirt; vt += (int64_t)gridDim.x * kRouteWarps) {
        const bool other = vt >= ntok;
        const int64_t t = other ? vt - ntok : vt;
        const T *row = logits + t * ld + (other ? second : 0);
        for (int i = lane; i < j1 + j2; i += 32) z[i] = Elem<T>::to_float(row[i]);
        int64_t index;
        float weight;
        if (route::route_token<T>(z, j1, j2, sub, count, cand, ncand, index, weight)) {
            (other ? out_idx2 : out_idx)[t * count + lane] = index;
            (other ? out_w2 : out_w)[t * count + lane] = Elem<T>::from_float(weight);
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
    size_t per_warp = (size_t)route::token_scratch_floats(j1, j2, sub, count) * sizeof(float);
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
