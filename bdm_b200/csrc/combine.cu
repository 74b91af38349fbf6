// Read combine + output normalisation + sigmoid gate (one CTA per token).
//
// Restates the token-order readout (gdn2_banks.py:265-283 scatter_bank_outputs,
// role_bank_dispatch.py:201-231 _readout) and the normalisation and gate of
// _project_bank_output (_parameters.py:222-232).  The KR read rows of a token
// are summed in ascending bank order -- the packed (bank) order the reference
// visits -- then LayerNorm (or RMS), then times dtype(sigmoid(gate)).
//
// Bank-sharded forward: bdm_combine_partial sums, per token, only the read rows
// of banks this rank owns (FP32, ascending bank order); the ranks' partials are
// summed by a reduce-scatter, and bdm_norm_gate_f32 rounds that FP32 sum once to
// the activation dtype (the forward's round-once combine) before norm and gate.
#include "common.cuh"
#include "norm_gate.cuh"

namespace bdm {
namespace {

constexpr int kCols = 8;  // columns per thread
constexpr int kMaxKR = 64;

// Load 8 consecutive elements (one 16-byte access for bf16 when `vec`).
template <typename T>
__device__ __forceinline__ void load8(const T *p, float *x, int64_t n_valid, bool vec) {
    if constexpr (sizeof(T) == 2) {
        if (vec && n_valid >= 8) {
            uint4 u = *reinterpret_cast<const uint4 *>(p);
            const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float2 f = __bfloat1622float2(h[i]);
                x[2 * i] = f.x;
                x[2 * i + 1] = f.y;
            }
            return;
        }
    }
#pragma unroll
    for (int i = 0; i < kCols; ++i) x[i] = i < n_valid ? Elem<T>::to_float(p[i]) : 0.f;
}

__device__ __forceinline__ void load8f(const float *p, float *x, int64_t n_valid, bool vec) {
    if (vec && n_valid >= 8) {
        const float4 a = *reinterpret_cast<const float4 *>(p), b = *reinterpret_cast<const float4 *>(p + 4);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
        return;
    }
#pragma unroll
    for (int i = 0; i < kCols; ++i) x[i] = i < n_valid ? p[i] : 0.f;
}

// slot_at[rank] = the slot of this token's rank-th smallest bank (ties: lower slot).
__device__ __forceinline__ void bank_order(const int64_t *ri, int64_t t, int kr, int64_t *banks, int *slot_at) {
    if ((int)threadIdx.x < kr) banks[threadIdx.x] = ri[t * kr + threadIdx.x];
    __syncthreads();
    if ((int)threadIdx.x < kr) {
        const int j = threadIdx.x;
        const int64_t bj = banks[j];
        int rank = 0;
        for (int i = 0; i < kr; ++i) rank += (banks[i] < bj) || (banks[i] == bj && i < j);
        slot_at[rank] = j;
    }
    __syncthreads();
}

__device__ __forceinline__ float block_sum(float x, float *red) {
    x = warp_sum(x);
    const int warp = threadIdx.x >> 5, lane = (int)lane_id();
    const int nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = x;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.f;
    return warp_sum(t);
}

template <typename T>
__global__ void combine_norm_gate_kernel(const T *__restrict__ reads, const int64_t *__restrict__ ri, int64_t ntok,
                                         int kr, int64_t width, const T *__restrict__ gate, int64_t ld_gate,
                                         const T *__restrict__ nw, const T *__restrict__ nb, float eps, int norm_mode,
                                         int round_each, int vec, T *__restrict__ out,
                                         const float *__restrict__ combined, T *__restrict__ raw_out) {
    __shared__ int64_t banks[kMaxKR];
    __shared__ int slot_at[kMaxKR];
    __shared__ float red[32];
    const int64_t t = blockIdx.x;
    if (t >= ntok) return;
    if (ri) bank_order(ri, t, kr, banks, slot_at);
    const int64_t c0 = (int64_t)threadIdx.x * kCols;
    float x[kCols];
#pragma unroll
    for (int i = 0; i < kCols; ++i) x[i] = 0.f;
    const bool act = c0 < width;
    const int64_t nv = width - c0;
    if (act) {
        if (ri) {
            // up to kBatchRows rows in flight per thread, summed in bank order
#ifndef BDM_COMBINE_ROWS
#define BDM_COMBINE_ROWS 1
#endif
            constexpr int kBatchRows = BDM_COMBINE_ROWS;
            for (int r0 = 0; r0 < kr; r0 += kBatchRows) {
                float y[kBatchRows][kCols];
#pragma unroll
                for (int r = 0; r < kBatchRows; ++r)
                    if (r0 + r < kr) load8<T>(reads + (t * kr + slot_at[r0 + r]) * width + c0, y[r], nv, vec);
#pragma unroll
                for (int r = 0; r < kBatchRows; ++r) {
                    if (r0 + r < kr) {
#pragma unroll
                        for (int i = 0; i < kCols; ++i) x[i] = round_each ? rnd<T>(x[i] + y[r][i]) : x[i] + y[r][i];
                    }
                }
            }
            if (!round_each) {
#pragma unroll
                for (int i = 0; i < kCols; ++i) x[i] = rnd<T>(x[i]);
            }
        } else if (combined) {
            load8f(combined + t * width + c0, x, nv, vec);
#pragma unroll
            for (int i = 0; i < kCols; ++i) x[i] = rnd<T>(x[i]);
        } else {
            load8<T>(reads + t * width + c0, x, nv, vec);
        }
        if (raw_out) {  // the combined read sum in the activation dtype (kept for the backward)
#pragma unroll
            for (int i = 0; i < kCols; ++i)
                if (c0 + i < width) raw_out[t * width + c0 + i] = Elem<T>::from_float(x[i]);
        }
    }
    const float inv_w = 1.0f / (float)width;
    float n[kCols];
    if (norm_mode == 1) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < kCols; ++i) s += x[i];
        const float mean = block_sum(s, red) * inv_w;
        float sq = 0.f;
#pragma unroll
        for (int i = 0; i < kCols; ++i)
            if (act && c0 + i < width) sq = ng::sq_dev(x[i], mean, sq);
        const float var = block_sum(sq, red) * inv_w;
        const float rstd = ng::inv_std(var, eps);
#pragma unroll
        for (int i = 0; i < kCols; ++i) {
            float y = 0.f;
            if (act && c0 + i < width) {
                const float b = nb ? Elem<T>::to_float(nb[c0 + i]) : 0.f;
                y = ng::layer_norm_col(x[i], mean, rstd, Elem<T>::to_float(nw[c0 + i]), nb ? &b : nullptr);
            }
            n[i] = rnd<T>(y);
        }
    } else {
        float sq = 0.f;
#pragma unroll
        for (int i = 0; i < kCols; ++i) sq = fmaf(x[i], x[i], sq);
        const float var = block_sum(sq, red) * inv_w;
        const float sc = rnd<T>(ng::inv_std(var, eps));
#pragma unroll
        for (int i = 0; i < kCols; ++i) {
            n[i] = 0.f;
            if (act && c0 + i < width) n[i] = ng::rms_col<T>(x[i], sc, Elem<T>::to_float(nw[c0 + i]));
        }
    }
    if (act) {
        float gv[kCols];
        load8<T>(gate + t * ld_gate + c0, gv, nv, vec);
        T *orow = out + t * width + c0;
        if constexpr (sizeof(T) == 2) {
            if (vec && nv >= 8) {
                uint4 u;
                __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&u);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    h[i] = __floats2bfloat162_rn(n[2 * i] * ng::gate_sigmoid<T>(gv[2 * i]),
                                                 n[2 * i + 1] * ng::gate_sigmoid<T>(gv[2 * i + 1]));
                *reinterpret_cast<uint4 *>(orow) = u;
                return;
            }
        }
#pragma unroll
        for (int i = 0; i < kCols; ++i) {
            if (c0 + i < width) orow[i] = Elem<T>::from_float(n[i] * ng::gate_sigmoid<T>(gv[i]));
        }
    }
}

// Per token: FP32 sum, in ascending bank order, of the read rows whose bank this
// rank owns; zero when it owns none of them.
template <typename T>
__global__ void combine_partial_kernel(const T *__restrict__ reads, const int64_t *__restrict__ ri, int64_t ntok,
                                       int kr, int64_t width, const int32_t *__restrict__ owner, int64_t J, int rank,
                                       int vec, float *__restrict__ out) {
    __shared__ int64_t banks[kMaxKR];
    __shared__ int slot_at[kMaxKR];
    const int64_t t = blockIdx.x;
    if (t >= ntok) return;
    bank_order(ri, t, kr, banks, slot_at);
    const int64_t c0 = (int64_t)threadIdx.x * kCols;
    if (c0 >= width) return;
    const int64_t nv = width - c0;
    float x[kCols];
#pragma unroll
    for (int i = 0; i < kCols; ++i) x[i] = 0.f;
    for (int r = 0; r < kr; ++r) {
        const int slot = slot_at[r];
        int64_t bank = banks[slot];
        bank = bank < 0 ? 0 : (bank >= J ? J - 1 : bank);
        if (owner[bank] != rank) continue;
        float y[kCols];
        load8<T>(reads + (t * kr + slot) * width + c0, y, nv, vec);
#pragma unroll
        for (int i = 0; i < kCols; ++i) x[i] += y[i];
    }
    float *orow = out + t * width + c0;
    if (vec && nv >= 8) {
        *reinterpret_cast<float4 *>(orow) = make_float4(x[0], x[1], x[2], x[3]);
        *reinterpret_cast<float4 *>(orow + 4) = make_float4(x[4], x[5], x[6], x[7]);
    } else {
        for (int i = 0; i < kCols && i < nv; ++i) orow[i] = x[i];
    }
}

int combine_threads(int64_t width, int64_t &threads) {
    threads = ceil_div(ceil_div(width, kCols), 32) * 32;
    if (threads < 64) threads = 64;
    return threads > 1024 ? BDM_ERR_UNSUPPORTED : BDM_OK;
}

}  // namespace
}  // namespace bdm

static int combine_norm_gate_impl(const void *reads, const int64_t *read_idx, int64_t ntok, int kr, int64_t width,
                                  const void *gate, int64_t ld_gate, const void *norm_weight, const void *norm_bias,
                                  float eps, int norm_mode, int round_each, int dtype, void *out, void *raw_out,
                                  void *stream) {
    using namespace bdm;
    if (ntok < 0 || width <= 0 || ld_gate < width) return BDM_ERR_INVALID;
    if (read_idx && (kr <= 0 || kr > kMaxKR)) return BDM_ERR_UNSUPPORTED;
    if (ntok == 0) return BDM_OK;
    if (!reads || !gate || !norm_weight || !out) return BDM_ERR_INVALID;
    if (norm_mode != 0 && norm_mode != 1) return BDM_ERR_INVALID;
    int64_t threads = 0;
    if (combine_threads(width, threads)) return BDM_ERR_UNSUPPORTED;
    if (ntok > 0x7fffffffLL) return BDM_ERR_UNSUPPORTED;
    const uintptr_t mis =
        (reinterpret_cast<uintptr_t>(reads) | reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(out)) & 15;
    const int vec = !mis && width % 8 == 0 && ld_gate % 8 == 0;
    BDM_DISPATCH_DTYPE(dtype, T, {
        combine_norm_gate_kernel<T><<<(unsigned)ntok, (unsigned)threads, 0, as_stream(stream)>>>(
            static_cast<const T *>(reads), read_idx, ntok, read_idx ? kr : 1, width, static_cast<const T *>(gate),
            ld_gate, static_cast<const T *>(norm_weight), static_cast<const T *>(norm_bias), eps, norm_mode,
            round_each, vec, static_cast<T *>(out), nullptr, static_cast<T *>(raw_out));
    });
    return launch_status();
}

extern "C" int bdm_combine_norm_gate(const void *reads, const int64_t *read_idx, int64_t ntok, int kr, int64_t width,
                                     const void *gate, int64_t ld_gate, const void *norm_weight, const void *norm_bias,
                                     float eps, int norm_mode, int round_each, int dtype, void *out, void *stream) {
    return combine_norm_gate_impl(reads, read_idx, ntok, kr, width, gate, ld_gate, norm_weight, norm_bias, eps,
                                  norm_mode, round_each, dtype, out, nullptr, stream);
}

extern "C" int bdm_combine_norm_gate_save(const void *reads, const int64_t *read_idx, int64_t ntok, int kr,
                                          int64_t width, const void *gate, int64_t ld_gate, const void *norm_weight,
                                          const void *norm_bias, float eps, int norm_mode, int round_each, int dtype,
                                          void *out, void *raw_out, void *stream) {
    if (ntok > 0 && !raw_out) return BDM_ERR_INVALID;
    return combine_norm_gate_impl(reads, read_idx, ntok, kr, width, gate, ld_gate, norm_weight, norm_bias, eps,
                                  norm_mode, round_each, dtype, out, raw_out, stream);
}

extern "C" int bdm_combine_partial(const void *reads, const int64_t *read_idx, int64_t ntok, int kr, int64_t width,
                                   const int32_t *owner, int64_t bank_count, int rank, int dtype, float *out,
                                   void *stream) {
    using namespace bdm;
    if (ntok < 0 || width <= 0 || bank_count <= 0 || rank < 0) return BDM_ERR_INVALID;
    if (kr <= 0 || kr > kMaxKR) return BDM_ERR_UNSUPPORTED;
    if (ntok == 0) return BDM_OK;
    if (!reads || !read_idx || !owner || !out) return BDM_ERR_INVALID;
    int64_t threads = 0;
    if (combine_threads(width, threads)) return BDM_ERR_UNSUPPORTED;
    if (ntok > 0x7fffffffLL) return BDM_ERR_UNSUPPORTED;
    const uintptr_t mis = (reinterpret_cast<uintptr_t>(reads) | reinterpret_cast<uintptr_t>(out)) & 15;
    const int vec = !mis && width % 8 == 0;
    BDM_DISPATCH_DTYPE(dtype, T, {
        combine_partial_kernel<T><<<(unsigned)ntok, (unsigned)threads, 0, as_stream(stream)>>>(
            static_cast<const T *>(reads), read_idx, ntok, kr, width, owner, bank_count, rank, vec, out);
    });
    return launch_status();
}

extern "C" int bdm_norm_gate_f32(const float *combined, int64_t ntok, int64_t width, const void *gate,
                                 int64_t ld_gate, const void *norm_weight, const void *norm_bias, float eps,
                                 int norm_mode, int dtype, void *out, void *stream) {
    using namespace bdm;
    if (ntok < 0 || width <= 0 || ld_gate < width) return BDM_ERR_INVALID;
    if (ntok == 0) return BDM_OK;
    if (!combined || !gate || !norm_weight || !out) return BDM_ERR_INVALID;
    if (norm_mode != 0 && norm_mode != 1) return BDM_ERR_INVALID;
    int64_t threads = 0;
    if (combine_threads(width, threads)) return BDM_ERR_UNSUPPORTED;
    if (ntok > 0x7fffffffLL) return BDM_ERR_UNSUPPORTED;
    const uintptr_t mis = (reinterpret_cast<uintptr_t>(combined) | reinterpret_cast<uintptr_t>(gate) |
                           reinterpret_cast<uintptr_t>(out)) & 15;
    const int vec = !mis && width % 8 == 0 && ld_gate % 8 == 0;
    BDM_DISPATCH_DTYPE(dtype, T, {
        combine_norm_gate_kernel<T><<<(unsigned)ntok, (unsigned)threads, 0, as_stream(stream)>>>(
            nullptr, nullptr, ntok, 1, width, static_cast<const T *>(gate), ld_gate,
            static_cast<const T *>(norm_weight), static_cast<const T *>(norm_bias), eps, norm_mode, 0, vec,
            static_cast<T *>(out), combined, nullptr);
    });
    return launch_status();
}
