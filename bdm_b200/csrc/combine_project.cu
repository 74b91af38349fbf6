// Read combine + output normalisation + sigmoid gate fused into the output projection (o_proj).
//
// Restates, for BF16 activations, the token-order readout (role_bank_dispatch.py:201-216 _readout,
// gdn2_banks.py:265-283: the KR read rows of a token summed in ascending bank order) followed by
// _project_bank_output (_parameters.py:222-232: LayerNorm or RMS, times dtype(sigmoid(gate)), then
// o_proj = x W^T + b).  One persistent CTA per SM walks tiles of 64 tokens:
//
//   combine warps (12) sum each token's read rows, normalise and gate them with the arithmetic of
//     bdm_combine_norm_gate (norm_gate.cuh), and write the BF16 o_proj input of the tile straight
//     into shared memory as the MMA's B operand (K-major, 128-byte swizzle): the normalised
//     tensor never reaches global memory;
//   one thread streams the o_proj weight W [D, V] by TMA in boxes of 128 rows x 64 columns through
//     a ring of shared-memory stages (tensor map over this GPU's memory, no multicast), and issues
//     tcgen05.mma kind::f16 with M = 128 output features and N = 64 tokens (K = 16 per
//     instruction), so out^T = W . a^T for all D <= 1024 features of the tile accumulates in
//     tensor memory (D / 128 accumulators of 64 FP32 columns, 512 columns);
//   the combine warps then read the accumulators back (tcgen05.ld), add the bias, round to BF16,
//     stage the output rows in the (now free) token tile and store them with 16-byte accesses,
//     before combining their next tile.
//
// The token tile and the accumulators are single-buffered: a tile's MMAs start once its combine
// is done and the previous tile's accumulators have been read; the weight ring runs ahead across
// tiles.  Each CTA starts its sweep of W at a different box, so the SMs do not all request the
// same L2 lines at once.  Every mbarrier wait is bounded (BDM_CP_ERR_TIMEOUT in the caller's
// status word; the CTA drains its copies and MMAs in flight and returns).
#include "common.cuh"
#include "norm_gate.cuh"
#include "tcgen05.cuh"

#include <cuda.h>

#include <mutex>

namespace bdm {
namespace {

constexpr int kTileTok = 64;   // tokens per tile: the MMA's N
constexpr int kFeat = 128;     // output features per MMA: the MMA's M
constexpr int kAtomK = 64;     // BF16 columns in one 128-byte swizzle row
constexpr int kAtomBytes = kTileTok * 128;   // one 64-column slice of the token tile
constexpr int kStageBytes = kFeat * 128;     // one weight box
constexpr int kCombineWarps = 12;
// warp 0: tensor memory, weight loads (TMA) and MMAs; warps 1..12 combine + epilogue.  13 warps
// keep the register limit at 128 per thread (two rows of loads in flight per combine thread).
constexpr int kCpThreads = (1 + kCombineWarps) * 32;
constexpr int kMaxStages = 8;
constexpr int kMaxFusedKR = 16;
constexpr int kSmemMax = 232448;  // opt-in shared memory per CTA on sm_100
constexpr unsigned long long kCpWaitNs = 2000000000ull;  // 2 s
constexpr int BDM_CP_ERR_TIMEOUT = 2;
constexpr unsigned kPhaseSleepNs = 256;  // poll interval of the waits that span a whole phase
constexpr int kOrderBar = 9;  // named barrier of the combine warps (token groups use 1..8)

struct CpParams {
    const bf16 *reads;   // [ntok * kr, width]
    const int64_t *ri;   // [ntok, kr] bank of each read slot
    int64_t ntok;
    int kr, width, out_dim, stages;
    const bf16 *gate;    // [ntok, >= width], row stride ld_gate
    int64_t ld_gate;
    const bf16 *nw, *nb;
    float eps;
    int norm_mode, round_each;
    const bf16 *bias;    // [out_dim] or null
    bf16 *out;           // [ntok, out_dim], row stride ld_out
    int64_t ld_out;
    int64_t ntiles;
    int *status;         // error bits (ORed), may be null
};

struct CpCtl {
    uint64_t full[kMaxStages], empty[kMaxStages];
    uint64_t a_full, acc_full, acc_empty, drain;
    uint32_t tmem;
    int abort;
    float red1[kCombineWarps], red2[kCombineWarps];
    uint8_t order[kTileTok][kMaxFusedKR];  // per tile row: read slots in ascending bank order
};

constexpr int cp_a_bytes(int width) { return (width / kAtomK) * kAtomBytes; }
constexpr int cp_smem_bytes(int width, int stages) {
    return 1024 + cp_a_bytes(width) + stages * kStageBytes + (int)sizeof(CpCtl);
}

// Bounded wait on a phase; gives up after kCpWaitNs (or once another thread of the CTA gave up),
// recording the error.  sleep_ns > 0 backs off between polls: long waits (a whole combine or MMA
// phase) then leave the issue slots to the warps that do the work.
__device__ bool cp_wait(CpCtl &c, uint64_t *bar, unsigned parity, int *status, unsigned sleep_ns = 0) {
    if (tc::mbar_test(bar, parity)) return true;
    const unsigned long long t0 = tc::global_ns();
    for (long long i = 0; i < (1ll << 32); ++i) {
        if (sleep_ns) __nanosleep(sleep_ns);
        if (tc::mbar_test(bar, parity)) return true;
        if ((i & 63) == 63) {
            if (*reinterpret_cast<volatile int *>(&c.abort)) return false;
            if (tc::global_ns() - t0 > kCpWaitNs) break;
        }
    }
    *reinterpret_cast<volatile int *>(&c.abort) = 1;
    if (status) atomicOr(status, BDM_CP_ERR_TIMEOUT);
    return false;
}

__device__ __forceinline__ void named_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}

// Sum over the warps of one token's group, in the order of combine.cu's block_sum (warp sums,
// then the warp totals summed by one warp_sum with zeros past the group).
__device__ __forceinline__ float group_sum(float x, float *red, int first_warp, int wpg, int gw, int bar_id) {
    const int lane = (int)lane_id();
    x = warp_sum(x);
    if (lane == 0) red[first_warp + gw] = x;
    named_sync(bar_id, wpg * 32);
    const float t = lane < wpg ? red[first_warp + lane] : 0.f;
    return warp_sum(t);
}

__device__ __forceinline__ void unpack8(const uint4 &u, float (&f)[8]) {
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 v = __bfloat1622float2(h[i]);
        f[2 * i] = v.x;
        f[2 * i + 1] = v.y;
    }
}

// Loads of one tile row, 8 columns: its read rows j0 .. j0 + 7 (< kr, in ascending bank order) and,
// with j0 == 0, its gate.
__device__ __forceinline__ void load_row(const CpParams &p, const CpCtl &c, int64_t tile, int r, int c0, int j0,
                                         uint4 (&y)[8], uint4 &g) {
    const int64_t t = tile * kTileTok + r;
    if (t >= p.ntok) return;
    const bf16 *rrow = p.reads + t * p.kr * (int64_t)p.width + c0;
    const uint64_t once = tc::l2_evict_first();  // read rows and gates are read once: keep W in L2
#pragma unroll
    for (int j = 0; j < 8; ++j)
        if (j0 + j < p.kr) y[j] = tc::ldg_hint(rrow + (int64_t)c.order[r][j0 + j] * p.width, once);
    if (j0 == 0) g = tc::ldg_hint(p.gate + t * p.ld_gate + c0, once);
}

// x += read rows j0 .. j0 + 7 (< kr) in order; round_each rounds to BF16 after every add.
__device__ __forceinline__ void accumulate(const CpParams &p, int j0, const uint4 (&y)[8], float (&x)[8]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        if (j0 + j < p.kr) {
            float f[8];
            unpack8(y[j], f);
#pragma unroll
            for (int i = 0; i < 8; ++i) x[i] = p.round_each ? bf16_round(x[i] + f[i]) : x[i] + f[i];
        }
    }
}

// Norm and gate of one tile row from its read sum x; stores the BF16 o_proj input into the token
// tile (row r, 64-column slice c0 / 64, swizzled 16-byte chunk).  Zeros for rows past the tokens.
__device__ __forceinline__ void finish_row(const CpParams &p, CpCtl &c, unsigned char *abuf, int64_t tile, int r,
                                           int gi, int gw, int wpg, int c0, float (&x)[8], const uint4 &g) {
    const int64_t t = tile * kTileTok + r;
    uint4 packed = make_uint4(0u, 0u, 0u, 0u);
    if (t < p.ntok) {  // uniform over the group
        const int bar_id = 1 + gi;
        const float inv_w = 1.0f / (float)p.width;
        if (!p.round_each) {
#pragma unroll
            for (int i = 0; i < 8; ++i) x[i] = bf16_round(x[i]);
        }
        // this thread's 8 columns of the norm weight / bias (L1-resident after the first row)
        float wn[8], bn[8];
        unpack8(__ldg(reinterpret_cast<const uint4 *>(p.nw + c0)), wn);
        if (p.nb) unpack8(__ldg(reinterpret_cast<const uint4 *>(p.nb + c0)), bn);
        float n[8];
        if (p.norm_mode == 1) {
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) s += x[i];
            const float mean = group_sum(s, c.red1, gi * wpg, wpg, gw, bar_id) * inv_w;
            float sq = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) sq = ng::sq_dev(x[i], mean, sq);
            const float var = group_sum(sq, c.red2, gi * wpg, wpg, gw, bar_id) * inv_w;
            const float rstd = ng::inv_std(var, p.eps);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                n[i] = bf16_round(ng::layer_norm_col(x[i], mean, rstd, wn[i], p.nb ? &bn[i] : nullptr));
        } else {
            float sq = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) sq = fmaf(x[i], x[i], sq);
            const float var = group_sum(sq, c.red1, gi * wpg, wpg, gw, bar_id) * inv_w;
            const float sc = bf16_round(ng::inv_std(var, p.eps));
#pragma unroll
            for (int i = 0; i < 8; ++i) n[i] = ng::rms_col<bf16>(x[i], sc, wn[i]);
            named_sync(bar_id, wpg * 32);  // red1 is rewritten by the next row
        }
        float gv[8];
        unpack8(g, gv);
        __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&packed);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            h[i] = __floats2bfloat162_rn(n[2 * i] * ng::gate_sigmoid<bf16>(gv[2 * i]),
                                         n[2 * i + 1] * ng::gate_sigmoid<bf16>(gv[2 * i + 1]));
    }
    const int kb = c0 >> 6, ch = (c0 >> 3) & 7;
    *reinterpret_cast<uint4 *>(abuf + kb * kAtomBytes + r * 128 + ((ch ^ (r & 7)) << 4)) = packed;
}

__device__ __forceinline__ void zero8(float (&x)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = 0.f;
}

// The rows gi, gi + ngroups, ... of a tile for one token group.  kr <= 8: the next row's loads are
// in flight while the current row is normalised (two register buffers).  kr <= 16: one row at a
// time, its read rows in two batches of 8.
__device__ __forceinline__ void combine_rows(const CpParams &p, CpCtl &c, unsigned char *abuf, int64_t tile, int gi,
                                             int gw, int wpg, int ngroups, int c0) {
    uint4 y0[8], y1[8], g0 = make_uint4(0u, 0u, 0u, 0u), g1 = g0;
    float x[8];
    if (p.kr <= 8) {
        int r = gi;
        load_row(p, c, tile, r, c0, 0, y0, g0);
        for (; r < kTileTok; r += 2 * ngroups) {
            const int r1 = r + ngroups, r2 = r + 2 * ngroups;
            if (r1 < kTileTok) load_row(p, c, tile, r1, c0, 0, y1, g1);
            zero8(x);
            accumulate(p, 0, y0, x);
            finish_row(p, c, abuf, tile, r, gi, gw, wpg, c0, x, g0);
            if (r1 >= kTileTok) break;
            if (r2 < kTileTok) load_row(p, c, tile, r2, c0, 0, y0, g0);
            zero8(x);
            accumulate(p, 0, y1, x);
            finish_row(p, c, abuf, tile, r1, gi, gw, wpg, c0, x, g1);
        }
    } else {
        for (int r = gi; r < kTileTok; r += ngroups) {
            load_row(p, c, tile, r, c0, 0, y0, g0);
            load_row(p, c, tile, r, c0, 8, y1, g1);
            zero8(x);
            accumulate(p, 0, y0, x);
            accumulate(p, 8, y1, x);
            finish_row(p, c, abuf, tile, r, gi, gw, wpg, c0, x, g0);
        }
    }
}

// Position in a CTA's sweep of the weight boxes: ring stage and how often the ring wrapped; the
// column slice and feature block, both as a position in this CTA's order (kbi, mti) and rotated by
// its starting box (kb, mt).  Feature blocks run fastest.
struct Sweep {
    int s = 0;
    uint32_t round = 0;
    int kbi = 0, mti = 0, kb, mt;
    __device__ Sweep(int rot_kb, int rot_mt) : kb(rot_kb), mt(rot_mt) {}
    __device__ __forceinline__ void next(int stages, int nkb, int nmt, int rot_kb, int rot_mt) {
        if (++s == stages) {
            s = 0;
            ++round;
        }
        if (++mt == nmt) mt = 0;
        if (++mti == nmt) {
            mti = 0;
            mt = rot_mt;
            if (++kb == nkb) kb = 0;
            if (++kbi == nkb) {
                kbi = 0;
                kb = rot_kb;
            }
        }
    }
};

__global__ void __launch_bounds__(kCpThreads, 1)
combine_project_kernel(const CpParams p, const __grid_constant__ CUtensorMap wmap) {
    extern __shared__ unsigned char cp_smem_raw[];
    // the swizzled operands need 1024-byte alignment
    unsigned char *base = cp_smem_raw + ((1024u - (tc::smem_u32(cp_smem_raw) & 1023u)) & 1023u);
    unsigned char *abuf = base;
    unsigned char *wbuf = base + cp_a_bytes(p.width);
    CpCtl &c = *reinterpret_cast<CpCtl *>(wbuf + p.stages * kStageBytes);
    const int warp = threadIdx.x >> 5, lane = (int)lane_id();
    const int nkb = p.width / kAtomK, nmt = p.out_dim / kFeat;
    const int stages = p.stages;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            tc::mbar_init(&c.full[s], 1);
            tc::mbar_init(&c.empty[s], 1);
        }
        tc::mbar_init(&c.a_full, kCombineWarps);
        tc::mbar_init(&c.acc_full, 1);
        tc::mbar_init(&c.acc_empty, kCombineWarps);
        tc::mbar_init(&c.drain, 1);
        c.abort = 0;
        tc::mbar_fence_init();
    }
    if (warp == 0) tc::tmem_alloc(&c.tmem, 512);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = c.tmem;

    if (warp == 0) {
        // ------------------------------------------------- weight loads (TMA) + MMA issue
        // One thread: step q consumes weight box q (tile-major, then 64-column slice, then
        // 128-feature block) from ring stage q mod stages; box q + stages - 1 is loaded once step q - 1's
        // MMAs have released its stage, so stages - 1 boxes stay in flight and the tensor pipe keeps
        // step q queued while the thread waits.
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_bf16(kFeat, kTileTok);
            const uint32_t per_tile = (uint32_t)(nkb * nmt);
            // CTAs start their sweep of W at different boxes (column slice and feature block), so
            // the SMs do not all request the same L2 lines at once
            const int rot_kb = (int)(blockIdx.x % nkb), rot_mt = (int)((blockIdx.x / nkb) % nmt);
            const uint64_t keep = tc::l2_evict_last();  // every tile of every CTA reads all of W
            int64_t my_tiles = 0;
            for (int64_t tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x) ++my_tiles;
            const uint32_t total = (uint32_t)my_tiles * per_tile;
            // boxes are walked with incremental counters: one thread issues everything, and integer
            // divisions by runtime values would dominate its loop
            Sweep lc(rot_kb, rot_mt), qc(rot_kb, rot_mt);  // next box to load / to consume
            uint32_t loaded = 0;
            auto load = [&]() {
                tc::mbar_arrive_expect_tx(&c.full[lc.s], kStageBytes);
                tc::tma_load_2d_hint(wbuf + lc.s * kStageBytes, &wmap, lc.kb * kAtomK, lc.mt * kFeat, &c.full[lc.s],
                                     keep);
                lc.next(stages, nkb, nmt, rot_kb, rot_mt);
                ++loaded;
            };
            while (loaded < total && loaded + 1 < (uint32_t)stages) load();
            bool ok = true;
            for (int it = 0; it < my_tiles && ok; ++it) {
                ok = cp_wait(c, &c.a_full, it & 1, p.status, kPhaseSleepNs);
                if (ok && it > 0) ok = cp_wait(c, &c.acc_empty, (it - 1) & 1, p.status);
                if (!ok) break;
                tc::fence_after_sync();
                for (uint32_t r = 0; r < per_tile; ++r) {
                    if (!cp_wait(c, &c.full[qc.s], qc.round & 1, p.status)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint32_t wa = tc::smem_u32(wbuf + qc.s * kStageBytes);
                    const uint32_t ab = tc::smem_u32(abuf + qc.kb * kAtomBytes);
                    const uint32_t d = tmem + (uint32_t)(qc.mt * kTileTok);
#pragma unroll
                    for (int kk = 0; kk < kAtomK / 16; ++kk)
                        tc::mma_bf16(d, tc::smem_desc_sw128(wa + kk * 32), tc::smem_desc_sw128(ab + kk * 32), idesc,
                                     (qc.kbi | kk) != 0);
                    tc::mma_commit(&c.empty[qc.s]);  // the stage is free once these MMAs have read it
                    qc.next(stages, nkb, nmt, rot_kb, rot_mt);
                    if (loaded < total) {
                        // the next box reuses the stage of the step `stages` before it (step q - 1)
                        if (lc.round > 0 && !cp_wait(c, &c.empty[lc.s], (lc.round - 1) & 1, p.status)) {
                            ok = false;
                            break;
                        }
                        load();
                    }
                }
                if (ok) tc::mma_commit(&c.acc_full);  // the tile's accumulators are complete
            }
            // every MMA issued has completed, and every box loaded has landed, before the CTA
            // releases tensor memory and shared memory
            tc::mma_commit(&c.drain);
            tc::mbar_wait(&c.drain, 0, kCpWaitNs);
            for (uint32_t j = loaded > (uint32_t)stages ? loaded - stages : 0; j < loaded; ++j)
                tc::mbar_wait(&c.full[j % stages], (j / stages) & 1, kCpWaitNs);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ combine + epilogue
        const int cw = warp - 1;
        const int wpg = p.width / 256;  // warps per token row (8 columns per thread)
        const int ngroups = kCombineWarps / wpg;
        const int gi = cw / wpg, gw = cw % wpg;
        const bool member = gi < ngroups;
        const int c0 = (gw * 32 + lane) * 8;
        const int lw = warp & 3;  // tensor-memory lane quarter this warp may read
        const int tq = cw >> 2;   // first 16-token slice of the tile this warp stores (then + 3)
        int it = 0;
        for (int64_t tile = blockIdx.x;; tile += gridDim.x, ++it) {
            if (it > 0) {
                // the previous tile: its MMAs are done (token tile free), accumulators ready
                if (!cp_wait(c, &c.acc_full, (it - 1) & 1, p.status, kPhaseSleepNs)) break;
                tc::fence_after_sync();
                // The token tile is free: stage the output rows there in chunks of `fc` features
                // (tokens x fc BF16), then store whole rows with 16-byte accesses.
                const int64_t tbase = (tile - gridDim.x) * kTileTok;
                const int fc = p.out_dim < p.width ? p.out_dim : p.width;
                bf16 *stage = reinterpret_cast<bf16 *>(abuf);
                for (int f0 = 0; f0 < p.out_dim; f0 += fc) {
                    for (int sl = tq; sl < kTileTok / 16; sl += kCombineWarps / 4) {
                        for (int mt = f0 / kFeat; mt < (f0 + fc) / kFeat; ++mt) {
                            float v[16];
                            tc::tmem_ld16(tmem + ((uint32_t)(lw * 32) << 16) + (uint32_t)(mt * kTileTok + sl * 16), v);
                            tc::tmem_wait_ld();
                            const int f = mt * kFeat + lw * 32 + lane;
                            const float b = p.bias ? __bfloat162float(p.bias[f]) : 0.f;
#pragma unroll
                            for (int i = 0; i < 16; ++i)
                                stage[(sl * 16 + i) * fc + (f - f0)] =
                                    __float2bfloat16_rn(p.bias ? __fadd_rn(v[i], b) : v[i]);
                        }
                    }
                    if (f0 + fc >= p.out_dim) {  // every accumulator has been read: the next tile's MMAs may run
                        tc::fence_before_sync();
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive(&c.acc_empty);
                    }
                    named_sync(kOrderBar, kCombineWarps * 32);
                    const int vec_per_row = fc / 8;
                    for (int idx = cw * 32 + lane; idx < kTileTok * vec_per_row; idx += kCombineWarps * 32) {
                        const int row = idx / vec_per_row, v8 = idx % vec_per_row;
                        const int64_t t = tbase + row;
                        if (t < p.ntok)
                            *reinterpret_cast<uint4 *>(p.out + t * p.ld_out + f0 + v8 * 8) =
                                *reinterpret_cast<const uint4 *>(stage + row * fc + v8 * 8);
                    }
                    named_sync(kOrderBar, kCombineWarps * 32);  // the staging area is rewritten next
                }
            }
            if (tile >= p.ntiles) break;
            // ascending-bank order of every row's read slots (ties: lower slot first), one
            // (row, slot) item per thread
            for (int item = cw * 32 + lane; item < kTileTok * p.kr; item += kCombineWarps * 32) {
                const int row = item / p.kr, j = item % p.kr;
                const int64_t t = tile * kTileTok + row;
                if (t < p.ntok) {
                    const int64_t *rb = p.ri + t * p.kr;
                    const int64_t bj = rb[j];
                    int rank = 0;
                    for (int i = 0; i < p.kr; ++i) {
                        const int64_t bi = rb[i];
                        rank += (bi < bj) || (bi == bj && i < j);
                    }
                    c.order[row][rank] = (uint8_t)j;
                }
            }
            named_sync(kOrderBar, kCombineWarps * 32);
            if (member) combine_rows(p, c, abuf, tile, gi, gw, wpg, ngroups, c0);
            tc::fence_async_smem();  // the tile's generic-proxy writes become visible to the MMAs
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&c.a_full);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 512);
    }
}

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_tiled() {
    static EncodeTiled fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<EncodeTiled>(nullptr);
        return reinterpret_cast<EncodeTiled>(f);
    }();
    return fn;
}

constexpr int kMaxDevices = 64;
std::mutex g_cp_mu;
bool g_cp_attr_set[kMaxDevices];
int g_cp_sms[kMaxDevices];

}  // namespace
}  // namespace bdm

// Shapes the fused kernel takes (the caller runs bdm_combine_norm_gate and its own GEMM otherwise).
static int combine_project_geometry(int64_t width, int64_t out_dim, int kr, int dtype, int &stages) {
    using namespace bdm;
    if (dtype != BDM_BF16) return BDM_ERR_UNSUPPORTED;
    if (width < 512 || width > 1024 || width % 256 != 0) return BDM_ERR_UNSUPPORTED;
    if (out_dim <= 0 || out_dim > 1024 || out_dim % kFeat != 0) return BDM_ERR_UNSUPPORTED;
    if (kr <= 0 || kr > kMaxFusedKR) return BDM_ERR_UNSUPPORTED;
    stages = (kSmemMax - cp_smem_bytes((int)width, 0)) / kStageBytes;
    if (stages > kMaxStages) stages = kMaxStages;
    return stages >= 2 ? BDM_OK : BDM_ERR_UNSUPPORTED;
}

extern "C" int bdm_combine_project_supported(int64_t width, int64_t out_dim, int kr, int dtype) {
    int stages = 0;
    return combine_project_geometry(width, out_dim, kr, dtype, stages) == BDM_OK ? 1 : 0;
}

extern "C" int bdm_combine_project(const void *reads, const int64_t *read_idx, int64_t ntok, int kr, int64_t width,
                                   const void *gate, int64_t ld_gate, const void *norm_weight, const void *norm_bias,
                                   float eps, int norm_mode, int round_each, const void *o_weight, const void *o_bias,
                                   int64_t out_dim, int dtype, void *out, int64_t ld_out, int *status, void *stream) {
    using namespace bdm;
    if (ntok < 0 || width <= 0 || out_dim <= 0 || ld_gate < width || ld_out < out_dim) return BDM_ERR_INVALID;
    if (norm_mode != 0 && norm_mode != 1) return BDM_ERR_INVALID;
    if (!valid_dtype(dtype)) return BDM_ERR_DTYPE;
    int stages = 0;
    if (int rc = combine_project_geometry(width, out_dim, kr, dtype, stages)) return rc;
    if (ntok == 0) return BDM_OK;
    if (!reads || !read_idx || !gate || !norm_weight || !o_weight || !out) return BDM_ERR_INVALID;
    const uintptr_t mis = (reinterpret_cast<uintptr_t>(reads) | reinterpret_cast<uintptr_t>(gate) |
                           reinterpret_cast<uintptr_t>(o_weight) | reinterpret_cast<uintptr_t>(norm_weight) |
                           reinterpret_cast<uintptr_t>(norm_bias) | reinterpret_cast<uintptr_t>(out)) & 15;
    if (mis || ld_gate % 8 != 0 || ld_out % 8 != 0) return BDM_ERR_UNSUPPORTED;
    EncodeTiled encode = encode_tiled();
    if (!encode) return BDM_ERR_UNSUPPORTED;
    CUtensorMap wmap;
    const cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)out_dim};
    const cuuint64_t strides[1] = {(cuuint64_t)width * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kAtomK, (cuuint32_t)kFeat}, estr[2] = {1, 1};
    if (encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(o_weight), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return BDM_ERR_UNSUPPORTED;
    int dev = 0;
    if (int rc = cuda_status(cudaGetDevice(&dev))) return rc;
    if (dev < 0 || dev >= kMaxDevices) return BDM_ERR_UNSUPPORTED;
    const int smem = cp_smem_bytes((int)width, stages);
    {
        std::lock_guard<std::mutex> lock(g_cp_mu);
        if (!g_cp_attr_set[dev]) {
            if (int rc = cuda_status(
                    cudaFuncSetAttribute(combine_project_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax)))
                return rc;
            if (int rc = cuda_status(cudaDeviceGetAttribute(&g_cp_sms[dev], cudaDevAttrMultiProcessorCount, dev)))
                return rc;
            g_cp_attr_set[dev] = true;
        }
    }
    CpParams p{};
    p.reads = static_cast<const bf16 *>(reads);
    p.ri = read_idx;
    p.ntok = ntok;
    p.kr = kr;
    p.width = (int)width;
    p.out_dim = (int)out_dim;
    p.stages = stages;
    p.gate = static_cast<const bf16 *>(gate);
    p.ld_gate = ld_gate;
    p.nw = static_cast<const bf16 *>(norm_weight);
    p.nb = static_cast<const bf16 *>(norm_bias);
    p.eps = eps;
    p.norm_mode = norm_mode;
    p.round_each = round_each;
    p.bias = static_cast<const bf16 *>(o_bias);
    p.out = static_cast<bf16 *>(out);
    p.ld_out = ld_out;
    p.ntiles = ceil_div(ntok, kTileTok);
    p.status = status;
    const int64_t grid = p.ntiles < g_cp_sms[dev] ? p.ntiles : g_cp_sms[dev];
    combine_project_kernel<<<(unsigned)grid, kCpThreads, smem, as_stream(stream)>>>(p, wmap);
    return launch_status();
}
