// Per-bank GDN2 delta-rule recurrence in chunks, with the intra-chunk products on the
// tensor cores (tcgen05.mma kind::tf32, accumulators in tensor memory).
//
// Same recurrence as recurrence.cu (reference gdn2_banks.py:22-43 reference_packed_gdn2,
// role_bank_kernel.py:46-73 _role_forward, forward_rows.py:9-149, with the packing of
// gdn2_banks.py:196-224 / role_bank_dispatch.py:41-73 / routed_update.py:5-13 folded in),
// in its chunked (WY / UT) form.  Per event of one bank sequence, on the S x dv state M:
//     write:  M = diag(e) M ;  u = x - M^T a ;  M = M + k u^T      (x = dtype(w p) v, a = dtype(b p) k)
//     read:   o = scale * M^T q                                    (q = dtype(q r))
// Over a chunk of C events that starts from M0, with G_t the inclusive cumulative log-decay
// (per row) from the chunk start and reads given k = 0, x = 0 and a := q:
//     Z[t][j] = sum_s a_t[s] k_j[s] exp(G_t[s] - G_j[s])      (j < t, else 0)
//     zhat_t  = exp(G_t) * a_t,   T = (I + Z)^-1,   Y = T zhat
//     U       = T X - Y M0             (C x dv: u_t for writes, -o_t / scale for reads)
//     M_C     = exp(G_C) * M0 + sum_j exp(G_C - G_j) k_j u_j^T
// Every decay factor is exp of a non-positive number, so nothing overflows.  U is one
// tensor-core product per head: U^T (dv x C) = [X^T | M0^T] (dv x (C + S)) . [T | -Y]^T,
// M = 128 value columns, N = 16 events, K = C + S = 24 (three K = 8 tf32 instructions).
// The chunk length C is the reference's BF16 storage interval (16 for S <= 8, 8 for S = 16),
// so chunk starts are exactly the storage points where the state is rounded.
//
// One CTA = one warpgroup of 128 threads; thread i owns value column i of a 128-column tile
// and the S rows of it for P heads of one sequence (the heads share events and run in
// lockstep, so one MMA wait serves P heads).  Per chunk: the thread writes its chunk-start
// state into the K-groups of the A operand, one thread issues 3P MMAs and a commit, and
// while they run the CTA prepares the next chunk (event ids, control rows, the pair
// coefficients Z, the triangular inverse T, Y, and the gathered write values X) into the
// other half of a double buffer.  Then every thread loads its row of U from tensor memory,
// writes the reads and carries the state on in FP32 registers.
#include "common.cuh"
#include "scan.cuh"
#include "tcgen05.cuh"

#include <type_traits>

namespace bdm {
namespace {

constexpr int kChunkThreads = 128;
constexpr int kTile = 128;               // value columns per unit (MMA M)
constexpr int kMmaN = 16;                // MMA N: the chunk's events (U) or state rows (state MMA), padded
constexpr int kAGroup = kTile * 8;       // floats in one K-group of A (128 rows x 8)
constexpr int kBGroup = kMmaN * 8;       // floats in one K-group of B (16 rows x 8)
constexpr int kTmemPerHead = 2 * kMmaN;  // U, then the state carry, per head
constexpr float kFactorRange = 80.0f;    // largest chunk log-decay range the split pair factor takes
constexpr unsigned long long kMmaWaitNs = 1000000000ull;  // 1 s
constexpr int kChunkCtasPerSm = 4;       // resident CTAs per SM the launch is sized for

// Float index of the 16-byte chunk holding (row, k..k+3) of a K-group with R rows (k % 4 == 0).
template <int R> __device__ __forceinline__ int kgroup_index(int row, int k) {
    return (k >> 2) * (R * 4) + (row >> 3) * 32 + (row & 7) * 4;
}
// Float index of element (row, k) of a K-major operand with R rows (K-groups consecutive).
template <int R> __device__ __forceinline__ int operand_index(int row, int k) {
    return (k >> 3) * (R * 8) + kgroup_index<R>(row, k & 7) + (k & 3);
}

template <int S, int P> struct ChunkSmem {
    static constexpr int C = chunk_events(S);
    static constexpr int KX = C / 8;        // K-groups of write values (and of the state MMA)
    static constexpr int KM = (S + 7) / 8;  // K-groups of chunk-start state
    static_assert(KX + KM == 3, "three K-groups per head");
    alignas(128) float ax[2][P][KX * kAGroup];   // A: write values X (rows = value columns, k = events)
    alignas(128) float am[P][KM * kAGroup];      // A: chunk-start state (k = state rows)
    alignas(128) float bop[2][P][3 * kBGroup];   // B of U:  rows = events t, k = [T[t][.] | -Y[t][.]]
    alignas(128) float bst[2][P][KX * kBGroup];  // B of the state carry: rows = state rows s, k = events j
    float dend[2][P][S];
    float wt[2][C];
    int tok[2][C], rid[2][C];
    unsigned wmask[2], rmask[2];
    alignas(16) float zhat[P][C][S];
    alignas(16) float ktil[P][C][S];
    float araw[P][C][S], kraw[P][C][S], G[P][C][S];
    alignas(16) float Z[P][C][C];
    alignas(16) float Tm[P][C][C];
    uint64_t bar_u, bar_m;  // U complete; state carry complete
    long long item;
    uint32_t tmem;
};

template <typename T>
__device__ __forceinline__ float write_value(T w, T v, float wt);
template <>
__device__ __forceinline__ float write_value<bf16>(bf16 w, bf16 v, float wt) {
    // dtype(w * p) exactly as the reference rounds it, then an exact FP32 product with v
    return __bfloat162float(__hmul(w, __float2bfloat16_rn(wt))) * __bfloat162float(v);
}

// Chunk-start state of this thread's column: cache, product-key factors or zero, rounded
// to BF16 when the training storage policy is on (as load_initial_state in recurrence.cu).
template <int S, int P>
__device__ __forceinline__ void chunk_initial_state(const ScanParams &p, int64_t bidx, int64_t bank, int h0, int col,
                                                    float (&M)[P][S]) {
#pragma unroll
    for (int q = 0; q < P; ++q)
#pragma unroll
        for (int s = 0; s < S; ++s) M[q][s] = 0.f;
    if (p.cache) {
#pragma unroll
        for (int q = 0; q < P; ++q) {
            const int64_t off = ((bidx * p.J + bank) * p.H + h0 + q) * (int64_t)S * p.dv + col;
#pragma unroll
            for (int s = 0; s < S; ++s)
                M[q][s] = p.cache_dtype == BDM_BF16 ? __bfloat162float(static_cast<const bf16 *>(p.cache)[off + s * p.dv])
                                                    : static_cast<const float *>(p.cache)[off + s * p.dv];
        }
    } else if (p.row_factor) {
        int64_t gbank = bank;
        if (p.bank_ids) {
            gbank = p.bank_ids[bank];
            gbank = gbank < 0 ? 0 : (gbank >= p.total_banks ? p.total_banks - 1 : gbank);
        }
#pragma unroll
        for (int q = 0; q < P; ++q)
#pragma unroll
            for (int s = 0; s < S; ++s) {
                const int64_t r = (gbank * p.total_heads + p.head_offset + h0 + q) * S + s;
                const int64_t ou = (r / p.factor_cols) * p.dv + col, oz = (r % p.factor_cols) * p.dv + col;
                if (p.factor_dtype == BDM_BF16)
                    M[q][s] = bf16_round(__bfloat162float(static_cast<const bf16 *>(p.row_factor)[ou]) +
                                         __bfloat162float(static_cast<const bf16 *>(p.col_factor)[oz]));
                else
                    M[q][s] = static_cast<const float *>(p.row_factor)[ou] + static_cast<const float *>(p.col_factor)[oz];
            }
    }
    if (p.interval > 0) {
#pragma unroll
        for (int q = 0; q < P; ++q)
#pragma unroll
            for (int s = 0; s < S; ++s) M[q][s] = bf16_round(M[q][s]);
    }
}

// A chunk is prepared into buffer `bb` in two parts: its event ids (loaded two chunks ahead,
// decoded one chunk ahead, then published to shared memory); then the A operand's write values, the control rows
// and their decays, the pair coefficients Z, T, Y, the B operand [T | -Y] of U and the
// end-relative keys of the state carry (chunk_prepare_rest).
// Event ids of a chunk decoded into registers of threads [0, C) (token, read row, route weight),
// fetched one chunk ahead of their use so the id and route-weight loads are off the chain.
struct ChunkEvents {
    int tok = -1, rid = -1;
    float wt = 0.f;
    bool wr = false, rd = false;
};

// Raw event ids of a chunk (threads [0, C)), loaded two chunks ahead of their use.
struct ChunkIds {
    int64_t id = -1;
};

template <int C>
__device__ __forceinline__ ChunkIds chunk_load_ids(const ScanParams &p, int64_t base, int n) {
    ChunkIds r;
    const int tid = threadIdx.x;
    if (tid < C && tid < n) r.id = p.order[base + tid];
    return r;
}

// Decodes ids loaded a chunk earlier and starts the route-weight loads (consumed a chunk later).
template <typename T>
__device__ __forceinline__ ChunkEvents chunk_decode_ids(const ScanParams &p, const ChunkIds &r) {
    ChunkEvents ev;
    const int64_t id = r.id;
    if (id >= 0 && id < p.nw) {
        ev.tok = (int)(id / p.kw);
        ev.wr = true;
        ev.wt = Elem<T>::to_float(static_cast<const T *>(p.ww)[id]);
    } else if (id >= p.nw && id < p.E) {
        ev.rid = (int)(id - p.nw);
        ev.tok = ev.rid / p.kr;
        ev.rd = true;
        ev.wt = Elem<T>::to_float(static_cast<const T *>(p.rw)[ev.rid]);
    }
    if (ev.tok >= p.nt) {  // the weight is left as loaded (unused): resetting it would wait on the load
        ev.tok = ev.rid = -1;
        ev.wr = ev.rd = false;
    }
    return ev;
}

template <int S, int P>
__device__ __forceinline__ void chunk_publish_events(ChunkSmem<S, P> &sh, int bb, const ChunkEvents &ev) {
    constexpr int C = ChunkSmem<S, P>::C;
    const int tid = threadIdx.x;
    if (tid < C) {
        sh.tok[bb][tid] = ev.tok;
        sh.rid[bb][tid] = ev.rid;
        sh.wt[bb][tid] = ev.wt;
    }
    if (tid < 32) {
        const unsigned wm = __ballot_sync(0xffffffffu, ev.wr), rm = __ballot_sync(0xffffffffu, ev.rd);
        if (tid == 0) {
            sh.wmask[bb] = wm;
            sh.rmask[bb] = rm;
        }
    }
    __syncthreads();
}

template <typename T, int S, int P>
__device__ __forceinline__ void chunk_prepare_rest(const ScanParams &p, ChunkSmem<S, P> &sh, int bb, int h0, int col) {
    constexpr int C = ChunkSmem<S, P>::C;
    const int tid = threadIdx.x;
    const unsigned wmask = sh.wmask[bb];
    // 2) control rows: thread (s, e) of head q, so the C events of one row are C adjacent lanes
    constexpr int kElems = C * S;  // 128 for S = 8 and 16, 64 for S = 4
    const int e = tid % C, s = tid / C;
    float ctl_k[P], ctl_b[P], ctl_g[P];
    const int tok_e = sh.tok[bb][e];
    const float wt_e = sh.wt[bb][e];
    const bool w_e = (wmask >> e) & 1u;
    if (tid < kElems) {
#pragma unroll
        for (int q = 0; q < P; ++q) {
            ctl_k[q] = ctl_b[q] = ctl_g[q] = 0.f;
            if (tok_e >= 0) {
                const int64_t o = ((int64_t)tok_e * p.H + h0 + q) * S + s;
                if (w_e) {
                    ctl_k[q] = Elem<T>::to_float(static_cast<const T *>(p.k)[o]);
                    ctl_b[q] = Elem<T>::to_float(static_cast<const T *>(p.b)[o]);
                    ctl_g[q] = p.g[o];
                } else {
                    ctl_k[q] = Elem<T>::to_float(static_cast<const T *>(p.q)[o]);
                }
            }
        }
    }
    // 3) start the write events' value-row loads (consumed after the T solve): item (head,
    //    4 events, 4 columns) per thread, 8-byte loads of v and w
    constexpr int kXItems = P * (C / 4) * (kTile / 4);
    constexpr int kXPer = (kXItems + kChunkThreads - 1) / kChunkThreads;
    uint2 xv[kXPer][4], xw[kXPer][4];
    {
        const int64_t V = (int64_t)p.H * p.dv;
        const int tile0 = col - tid;  // first column of this unit's tile
#pragma unroll
        for (int k = 0; k < kXPer; ++k) {
            const int it = tid + k * kChunkThreads;
            const int cg = it % (kTile / 4), e4 = ((it / (kTile / 4)) % (C / 4)) * 4, q = it / ((kTile / 4) * (C / 4));
            const int64_t cbase = (int64_t)(h0 + q) * p.dv + tile0 + 4 * cg;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                xv[k][i] = xw[k][i] = make_uint2(0u, 0u);
                if (it < kXItems && ((wmask >> (e4 + i)) & 1u)) {
                    const int64_t o = (int64_t)sh.tok[bb][e4 + i] * V + cbase;
                    xv[k][i] = __ldg(reinterpret_cast<const uint2 *>(static_cast<const T *>(p.v) + o));
                    xw[k][i] = __ldg(reinterpret_cast<const uint2 *>(static_cast<const T *>(p.w) + o));
                }
            }
        }
    }
    // 4) per (head, row, event): log-decay scan over the chunk (shuffles within C lanes),
    //    decayed erase / query rows, end-relative keys, chunk decay
    bool wide = false;
    if (tid < kElems) {
#pragma unroll
        for (int q = 0; q < P; ++q) {
            float ge = 0.f, a = 0.f, kk = 0.f;
            if (tok_e >= 0) {
                if (w_e) {
                    kk = ctl_k[q];
                    ge = fmaxf(p.routed_decay ? ctl_g[q] * wt_e : ctl_g[q], kMinLogDecay);
                    a = rnd<T>(ctl_b[q] * wt_e) * kk;
                } else {
                    a = rnd<T>(ctl_k[q] * wt_e);
                }
            }
            float gc = ge;
#pragma unroll
            for (int d = 1; d < C; d <<= 1) {
                const float up = __shfl_up_sync(0xffffffffu, gc, d, C);
                if (e >= d) gc += up;
            }
            const float gend = __shfl_sync(0xffffffffu, gc, C - 1, C);
            wide |= -gend > kFactorRange;
            sh.zhat[q][e][s] = __expf(gc) * a;
            sh.ktil[q][e][s] = __expf(-gc) * kk;
            sh.araw[q][e][s] = a;
            sh.kraw[q][e][s] = kk;
            sh.G[q][e][s] = gc;
            sh.bst[bb][q][operand_index<kMmaN>(s, e)] = tc::to_tf32(__expf(gend - gc) * kk);
            if (e == 0) sh.dend[bb][q][s] = __expf(gend);
        }
    }
    wide = __syncthreads_or(wide);
    // 5) pair coefficients Z[t][j] (j < t, j a write): sum_s a_t k_j exp(G_t - G_j), split as
    //    zhat_t . ktil_j unless the chunk's decay range could overflow the split factors;
    //    item (head, t, 4 columns j) per thread
    for (int it = tid; it < P * C * (C / 4); it += kChunkThreads) {
        const int j4 = (it % (C / 4)) * 4, t = (it / (C / 4)) % C, q = it / (C * (C / 4));
        float z[4] = {0.f, 0.f, 0.f, 0.f};
        if (!wide) {
            float zt[S];
#pragma unroll
            for (int r = 0; r < S; r += 4) *reinterpret_cast<float4 *>(zt + r) = *reinterpret_cast<const float4 *>(&sh.zhat[q][t][r]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int j = j4 + i;
                if (j < t && ((wmask >> j) & 1u)) {
#pragma unroll
                    for (int r = 0; r < S; r += 4) {
                        const float4 kt = *reinterpret_cast<const float4 *>(&sh.ktil[q][j][r]);
                        z[i] = fmaf(zt[r], kt.x, fmaf(zt[r + 1], kt.y, fmaf(zt[r + 2], kt.z, fmaf(zt[r + 3], kt.w, z[i]))));
                    }
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int j = j4 + i;
                if (j < t && ((wmask >> j) & 1u)) {
#pragma unroll
                    for (int r = 0; r < S; ++r)
                        z[i] = fmaf(sh.araw[q][t][r] * sh.kraw[q][j][r], __expf(sh.G[q][t][r] - sh.G[q][j][r]), z[i]);
                }
            }
        }
        *reinterpret_cast<float4 *>(&sh.Z[q][t][j4]) = make_float4(z[0], z[1], z[2], z[3]);
    }
    __syncthreads();
    // 6) T = (I + Z)^-1 (unit lower triangular): lane (head, j) solves column j forward
    if (tid < P * C) {
        const int q = tid / C, j = tid % C;
        float colv[C];
#pragma unroll
        for (int t = 0; t < C; ++t) {
            float a0 = 0.f, a1 = 0.f;  // colv[i] = 0 for i < j
#pragma unroll
            for (int i4 = 0; i4 < t; i4 += 4) {
                const float4 z4 = *reinterpret_cast<const float4 *>(&sh.Z[q][t][i4]);
                a0 = fmaf(z4.x, colv[i4], a0);
                if (i4 + 1 < t) a1 = fmaf(z4.y, colv[i4 + 1], a1);
                if (i4 + 2 < t) a0 = fmaf(z4.z, colv[i4 + 2], a0);
                if (i4 + 3 < t) a1 = fmaf(z4.w, colv[i4 + 3], a1);
            }
            colv[t] = t == j ? 1.f : (t > j ? -(a0 + a1) : 0.f);
        }
#pragma unroll
        for (int t = 0; t < C; ++t) sh.Tm[q][t][j] = colv[t];
    }
    __syncthreads();
    // 6b) A operand write values from the rows loaded at the start
#pragma unroll
    for (int k = 0; k < kXPer; ++k) {
        const int it = tid + k * kChunkThreads;
        if (it < kXItems) {
            const int cg = it % (kTile / 4), e4 = ((it / (kTile / 4)) % (C / 4)) * 4, q = it / ((kTile / 4) * (C / 4));
            float x[4][4];  // [column][event]
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int ev = e4 + i;
#pragma unroll
                for (int c = 0; c < 4; ++c) x[c][i] = 0.f;
                if ((wmask >> ev) & 1u) {
                    const __nv_bfloat162 p2 = __float2bfloat162_rn(sh.wt[bb][ev]);
                    const float2 w01 = __bfloat1622float2(__hmul2(*reinterpret_cast<const __nv_bfloat162 *>(&xw[k][i].x), p2));
                    const float2 w23 = __bfloat1622float2(__hmul2(*reinterpret_cast<const __nv_bfloat162 *>(&xw[k][i].y), p2));
                    const float2 v01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&xv[k][i].x));
                    const float2 v23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&xv[k][i].y));
                    x[0][i] = tc::to_tf32(w01.x * v01.x);
                    x[1][i] = tc::to_tf32(w01.y * v01.y);
                    x[2][i] = tc::to_tf32(w23.x * v23.x);
                    x[3][i] = tc::to_tf32(w23.y * v23.y);
                }
            }
            float *aq = sh.ax[bb][q] + (e4 >> 3) * kAGroup;
#pragma unroll
            for (int c0 = 0; c0 < 4; ++c0) {
                const int c = (c0 + cg) & 3;  // rotated so a warp's stores spread over the banks
                float4 v4 = make_float4(x[0][0], x[0][1], x[0][2], x[0][3]);
#pragma unroll
                for (int cc = 1; cc < 4; ++cc)
                    if (cc == c) v4 = make_float4(x[cc][0], x[cc][1], x[cc][2], x[cc][3]);
                *reinterpret_cast<float4 *>(aq + kgroup_index<kTile>(4 * cg + c, e4 & 7)) = v4;
            }
        }
    }
    // 7) B operand of U, rows t < C: [T[t][0..C) | -Y[t][0..S)], Y = T zhat; item (head, t,
    //    4 columns of T) and (head, t, 2 state rows of Y) per thread
    for (int it = tid; it < P * C * (C / 4); it += kChunkThreads) {
        const int j4 = (it % (C / 4)) * 4, t = (it / (C / 4)) % C, q = it / (C * (C / 4));
        const float4 t4 = *reinterpret_cast<const float4 *>(&sh.Tm[q][t][j4]);
        *reinterpret_cast<float4 *>(sh.bop[bb][q] + operand_index<kMmaN>(t, j4)) =
            make_float4(tc::to_tf32(t4.x), tc::to_tf32(t4.y), tc::to_tf32(t4.z), tc::to_tf32(t4.w));
    }
    for (int it = tid; it < P * C * (S / 2); it += kChunkThreads) {
        const int s2 = (it % (S / 2)) * 2, t = (it / (S / 2)) % C, q = it / (C * (S / 2));
        float y0 = 0.f, y1 = 0.f;
#pragma unroll
        for (int j4 = 0; j4 < C; j4 += 4) {
            const float4 t4 = *reinterpret_cast<const float4 *>(&sh.Tm[q][t][j4]);  // T[t][j] = 0 for j > t
            const float tv[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 zh = *reinterpret_cast<const float2 *>(&sh.zhat[q][j4 + i][s2]);
                y0 = fmaf(tv[i], zh.x, y0);
                y1 = fmaf(tv[i], zh.y, y1);
            }
        }
        *reinterpret_cast<float2 *>(sh.bop[bb][q] + operand_index<kMmaN>(t, C + s2)) =
            make_float2(tc::to_tf32(-y0), tc::to_tf32(-y1));
    }
}

template <typename T, int S, int P>
__global__ void __launch_bounds__(kChunkThreads, 4) chunk_scan_kernel(const ScanParams p) {
    using Sm = ChunkSmem<S, P>;
    constexpr int C = Sm::C, KX = Sm::KX, KM = Sm::KM;
    constexpr uint32_t kCols = P * kTmemPerHead <= 32 ? 32 : (P * kTmemPerHead <= 64 ? 64 : 128);
    constexpr uint32_t kIdesc = tc::idesc_tf32(kTile, kMmaN);
    extern __shared__ __align__(1024) unsigned char chunk_smem[];
    Sm &sh = *reinterpret_cast<Sm *>(chunk_smem);
    const int tid = threadIdx.x, warp = tid >> 5;

    if (warp == 0) tc::tmem_alloc(&sh.tmem, kCols);
    if (tid == 0) {
        tc::mbar_init(&sh.bar_u, 1);
        tc::mbar_init(&sh.bar_m, 1);
        tc::mbar_fence_init();
    }
    // Operand padding no chunk writes (B rows C..15 when C = 8, K columns C+S..23 and state
    // rows S..15 when S = 4 or 8) must read as zero: clear the B operands and the state once.
    for (int i = tid; i < 2 * P * 3 * kBGroup; i += kChunkThreads) (&sh.bop[0][0][0])[i] = 0.f;
    for (int i = tid; i < 2 * P * KX * kBGroup; i += kChunkThreads) (&sh.bst[0][0][0])[i] = 0.f;
    for (int i = tid; i < P * KM * kAGroup; i += kChunkThreads) (&sh.am[0][0])[i] = 0.f;
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = sh.tmem;
    const uint32_t lane_base = tmem + (((uint32_t)warp * 32u) << 16);

    int64_t total = 0;
    for (int c = p.ws_classes; c < kLenClasses; ++c) total += p.counts[c];
    const int64_t per_seq = (int64_t)(p.H / P) * p.ctiles;
    total *= per_seq;
    const int64_t V = (int64_t)p.H * p.dv;
    unsigned phase = 0;
    bool failed = false;

    for (;;) {
        if (tid == 0) sh.item = (long long)atomicAdd(p.chunk_next, 1ull);
        __syncthreads();
        const int64_t item = sh.item;
        if (item >= total) break;  // CTA-uniform
        int64_t local = item / per_seq;
        int cls = p.ws_classes;
        while (cls < kLenClasses - 1 && local >= p.counts[cls]) local -= p.counts[cls++];
        const int64_t seq = p.lists[(int64_t)cls * p.nseq + local];
        const int64_t rem = item % per_seq;
        const int h0 = (int)(rem / p.ctiles) * P;
        const int col = (int)(rem % p.ctiles) * kTile + tid;
        const int64_t bidx = seq / p.J, bank = seq % p.J;
        const int64_t start = min(max(p.cu[seq], (int64_t)0), p.E);
        const int64_t end = min(max(p.cu[seq + 1], start), p.E);
        const int64_t nch = (end - start + C - 1) / C;

        float M[P][S];
        chunk_initial_state<S, P>(p, bidx, bank, h0, col, M);
        auto ids_of = [&](int64_t c) {
            const int64_t b0 = start + c * C;
            return chunk_load_ids<C>(p, b0, (int)min((int64_t)C, end - b0));
        };
        ChunkEvents ev_next;
        ChunkIds id_next;
        if (nch > 0) {
            chunk_publish_events<S, P>(sh, 0, chunk_decode_ids<T>(p, ids_of(0)));
            if (nch > 1) ev_next = chunk_decode_ids<T>(p, ids_of(1));
            if (nch > 2) id_next = ids_of(2);
            chunk_prepare_rest<T, S, P>(p, sh, 0, h0, col);
        }

        for (int64_t ci = 0; ci < nch; ++ci) {
            const int bb = (int)(ci & 1);
            if (ci > 0 && p.interval > 0) {  // storage point: the reference rounds the state here
#pragma unroll
                for (int q = 0; q < P; ++q)
#pragma unroll
                    for (int s = 0; s < S; ++s) M[q][s] = bf16_round(M[q][s]);
            }
            // chunk-start state into the A operand (K-major, 4 rows per 16-byte store)
#pragma unroll
            for (int q = 0; q < P; ++q)
#pragma unroll
                for (int s4 = 0; s4 < S; s4 += 4)
                    *reinterpret_cast<float4 *>(sh.am[q] + (s4 >> 3) * kAGroup + kgroup_index<kTile>(tid, s4 & 7)) =
                        make_float4(tc::to_tf32(M[q][s4]), tc::to_tf32(M[q][s4 + 1]), tc::to_tf32(M[q][s4 + 2]),
                                    tc::to_tf32(M[q][s4 + 3]));
            tc::fence_async_smem();
            tc::fence_before_sync();
            __syncthreads();
            tc::fence_after_sync();
            if (tid == 0) {  // U^T = [X^T | M0^T] [T | -Y]^T
#pragma unroll
                for (int q = 0; q < P; ++q) {
                    const uint32_t tu = tmem + (uint32_t)(q * kTmemPerHead);
#pragma unroll
                    for (int kg = 0; kg < 3; ++kg) {
                        const float *a = kg < KX ? sh.ax[bb][q] + kg * kAGroup : sh.am[q] + (kg - KX) * kAGroup;
                        tc::mma_tf32(tu, tc::smem_desc(tc::smem_u32(a), kTile * 16, 128),
                                     tc::smem_desc(tc::smem_u32(sh.bop[bb][q] + kg * kBGroup), kMmaN * 16, 128),
                                     kIdesc, kg > 0 ? 1u : 0u);
                    }
                }
                tc::mma_commit(&sh.bar_u);
            }
            // The state carry reads U back from tensor memory as its A operand, so it is issued
            // once U is complete; the next chunk's preparation overlaps both.
            const bool more = ci + 1 < nch;
            if (more) {
                chunk_publish_events<S, P>(sh, bb ^ 1, ev_next);
                ev_next = ci + 2 < nch ? chunk_decode_ids<T>(p, id_next) : ChunkEvents();
                id_next = ci + 3 < nch ? ids_of(ci + 3) : ChunkIds();
            }
            if (tid == 0) {
                if (tc::mbar_wait(&sh.bar_u, phase, kMmaWaitNs)) {
                    tc::fence_after_sync();
#pragma unroll
                    for (int q = 0; q < P; ++q) {
                        const uint32_t tu = tmem + (uint32_t)(q * kTmemPerHead), tm = tu + kMmaN;
#pragma unroll
                        for (int kg = 0; kg < KX; ++kg)
                            tc::mma_tf32_tmem_a(
                                tm, tu + (uint32_t)(kg * 8),
                                tc::smem_desc(tc::smem_u32(sh.bst[bb][q] + kg * kBGroup), kMmaN * 16, 128), kIdesc,
                                kg > 0 ? 1u : 0u);
                    }
                    tc::mma_commit(&sh.bar_m);
                }
            }
            if (more) chunk_prepare_rest<T, S, P>(p, sh, bb ^ 1, h0, col);
            const bool ok = tc::mbar_wait(&sh.bar_m, phase, kMmaWaitNs);
            phase ^= 1u;
            if (__syncthreads_or(!ok)) {
                failed = true;
                break;
            }
            tc::fence_after_sync();
            float U[P][16], D[P][S > 8 ? 16 : 8];
#pragma unroll
            for (int q = 0; q < P; ++q) {
                const uint32_t tu = lane_base + (uint32_t)(q * kTmemPerHead);
                tc::tmem_ld16(tu, U[q]);
                if constexpr (S > 8) tc::tmem_ld16(tu + kMmaN, D[q]);
                else tc::tmem_ld8(tu + kMmaN, D[q]);
            }
            tc::tmem_wait_ld();
            // reads: o = scale * q^T M = -scale * U[t]
            const unsigned rmask = sh.rmask[bb];
#pragma unroll
            for (int t = 0; t < C; ++t) {
                if ((rmask >> t) & 1u) {
                    T *o = static_cast<T *>(p.reads) + (int64_t)sh.rid[bb][t] * V + (int64_t)h0 * p.dv + col;
#pragma unroll
                    for (int q = 0; q < P; ++q) o[(int64_t)q * p.dv] = Elem<T>::from_float(-p.scale * U[q][t]);
                }
            }
            // state carry: M = exp(G_C) M + sum_j exp(G_C - G_j) k_j u_j
#pragma unroll
            for (int q = 0; q < P; ++q)
#pragma unroll
                for (int s = 0; s < S; ++s) M[q][s] = fmaf(sh.dend[bb][q][s], M[q][s], D[q][s]);
        }
        if (failed) break;
        if (p.store_final && p.cache) {
#pragma unroll
            for (int q = 0; q < P; ++q) {
                const int64_t off = ((bidx * p.J + bank) * p.H + h0 + q) * (int64_t)S * p.dv + col;
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    if (p.cache_dtype == BDM_BF16) static_cast<bf16 *>(p.cache)[off + s * p.dv] = __float2bfloat16_rn(M[q][s]);
                    else static_cast<float *>(p.cache)[off + s * p.dv] = M[q][s];
                }
            }
        }
        __syncthreads();  // every thread has read sh.item before the next unit is taken
    }
    if (failed) {
        // a tensor-core wait gave up: record it, give the MMAs in flight one more bounded
        // wait, then release tensor memory and leave (this CTA's outputs are unspecified)
        if (tid == 0) atomicOr(p.status, BDM_SCAN_ERR_TIMEOUT);
        tc::mbar_wait(&sh.bar_u, phase ^ 1u, kMmaWaitNs);
        tc::mbar_wait(&sh.bar_m, phase ^ 1u, kMmaWaitNs);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, kCols);
}

template <int S, int P>
int launch_chunk(const ScanParams &p0, cudaStream_t st, bool programmatic) {
    ScanParams p = p0;
    p.ctiles = p.dv / kTile;
    auto kern = chunk_scan_kernel<bf16, S, P>;
    const int smem = (int)sizeof(ChunkSmem<S, P>);
    int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    if (rc) return rc;
    // all of the unified L1 / shared array as shared memory, so several CTAs fit per SM
    rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                          (int)cudaSharedmemCarveoutMaxShared));
    if (rc) return rc;
    int dev = 0, sms = kNumSMs, per_sm = 1;
    rc = cuda_status(cudaGetDevice(&dev));
    if (rc) return rc;
    rc = cuda_status(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if (rc) return rc;
    rc = cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kChunkThreads, smem));
    if (rc) return rc;
    // persistent CTAs: as many as fit (by shared memory and registers; tensor memory holds 512
    // columns per SM, far more than fit), each taking units from the work counter
    const int64_t units = p.batch * p.J * (p.H / P) * p.ctiles;
    const int64_t blocks = max((int64_t)1, min(units, (int64_t)sms * max(per_sm, kChunkCtasPerSm)));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(kChunkThreads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = programmatic ? 1 : 0;
    rc = cuda_status(cudaLaunchKernelEx(&cfg, kern, p));
    count_launch();
    return rc;
}

}  // namespace

bool chunk_scan_eligible(const ScanParams &p, int dtype, int S) {
    if (dtype != BDM_BF16 || p.ckpt) return false;
    if (S != 4 && S != 8 && S != 16) return false;
    if (p.dv % kTile != 0) return false;
    return p.interval == 0 || p.interval == chunk_events(S);
}

int launch_chunk_scan(const ScanParams &p, int S, cudaStream_t st, bool programmatic) {
    const bool pair = p.H % 2 == 0;
    switch (S) {
        case 4: return pair ? launch_chunk<4, 2>(p, st, programmatic) : launch_chunk<4, 1>(p, st, programmatic);
        case 8: return pair ? launch_chunk<8, 2>(p, st, programmatic) : launch_chunk<8, 1>(p, st, programmatic);
        case 16: return pair ? launch_chunk<16, 2>(p, st, programmatic) : launch_chunk<16, 1>(p, st, programmatic);
        default: return BDM_ERR_UNSUPPORTED;
    }
}

}  // namespace bdm
