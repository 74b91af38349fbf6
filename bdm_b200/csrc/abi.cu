// ABI utilities (status text, last CUDA error) and the product-key initial state.
#include <atomic>

#include "common.cuh"

namespace bdm {

static thread_local int g_last_cuda_error = 0;
static std::atomic<long long> g_launches{0};

void set_last_cuda_error(cudaError_t e) { g_last_cuda_error = (int)e; }
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

namespace {

// out[n, j, h, s, c] = round_factor(U[r / Q, c] + Z[r % Q, c]), r = (j*H + h)*S + s
// (_parameters.py:48-61; product_routed_update.py:10-16 rounds the FP32 sum to
// the factor dtype before widening).
template <typename FT, typename OT>
__global__ void product_state_kernel(const FT *__restrict__ U, const FT *__restrict__ Z, int64_t Q, int64_t batch,
                                     int64_t rows, int dv, OT *__restrict__ out) {
    const int64_t per_batch = rows * dv;
    const int64_t total = batch * per_batch;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t e = i % per_batch;
        const int64_t r = e / dv;
        const int c = (int)(e % dv);
        const float x = rnd<FT>(Elem<FT>::to_float(U[(r / Q) * dv + c]) + Elem<FT>::to_float(Z[(r % Q) * dv + c]));
        out[i] = Elem<OT>::from_float(x);
    }
}

__global__ void status_or_kernel(int *dst, const int *src) {
    const int bits = *src;
    if (bits) atomicOr(dst, bits);
}

}  // namespace
}  // namespace bdm

extern "C" int bdm_status_or(int *dst, const int *src, void *stream) {
    using namespace bdm;
    if (!dst || !src) return BDM_ERR_INVALID;
    status_or_kernel<<<1, 1, 0, as_stream(stream)>>>(dst, src);
    return launch_status();
}

extern "C" const char *bdm_status_string(int status) {
    switch (status) {
        case BDM_OK: return "ok";
        case BDM_ERR_INVALID: return "invalid argument (size, shape or null pointer)";
        case BDM_ERR_DTYPE: return "unsupported element type";
        case BDM_ERR_UNSUPPORTED: return "geometry not supported by the sm_100a kernels";
        case BDM_ERR_CUDA: return "CUDA launch or runtime error";
        case BDM_ERR_WORKSPACE: return "workspace missing or too small";
        default: return "unknown status";
    }
}

extern "C" int bdm_last_cuda_error(void) { return bdm::g_last_cuda_error; }

extern "C" int bdm_abi_version(void) { return 1; }

extern "C" long long bdm_kernel_launches(void) { return bdm::g_launches.load(std::memory_order_relaxed); }

extern "C" int bdm_product_state(const void *row_factor, const void *col_factor, int64_t rows_p, int64_t cols_q,
                                 int factor_dtype, int64_t batch, int64_t bank_count, int heads, int bank_size,
                                 int head_value_width, void *out, int out_dtype, void *stream) {
    using namespace bdm;
    if (rows_p <= 0 || cols_q <= 0 || batch < 0 || bank_count <= 0 || heads <= 0 || bank_size <= 0 ||
        head_value_width <= 0)
        return BDM_ERR_INVALID;
    const int64_t rows = bank_count * heads * bank_size;
    if (rows_p * cols_q != rows) return BDM_ERR_INVALID;
    if (batch == 0) return BDM_OK;
    if (!row_factor || !col_factor || !out) return BDM_ERR_INVALID;
    if (!valid_dtype(factor_dtype) || !valid_dtype(out_dtype)) return BDM_ERR_DTYPE;
    const int64_t total = batch * rows * head_value_width;
    int64_t blocks = ceil_div(total, 256);
    if (blocks > 64 * kNumSMs) blocks = 64 * kNumSMs;
    cudaStream_t st = as_stream(stream);
    BDM_DISPATCH_DTYPE(factor_dtype, FT, {
        if (out_dtype == BDM_BF16)
            product_state_kernel<FT, bf16><<<(unsigned)blocks, 256, 0, st>>>(
                static_cast<const FT *>(row_factor), static_cast<const FT *>(col_factor), cols_q, batch, rows,
                head_value_width, static_cast<bf16 *>(out));
        else
            product_state_kernel<FT, float><<<(unsigned)blocks, 256, 0, st>>>(
                static_cast<const FT *>(row_factor), static_cast<const FT *>(col_factor), cols_q, batch, rows,
                head_value_width, static_cast<float *>(out));
    });
    return launch_status();
}
