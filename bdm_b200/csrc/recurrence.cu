// Per-bank GDN2 delta-rule recurrence over dispatched events.
//
// Restates the reference recurrence (gdn2_banks.py:22-43 reference_packed_gdn2,
// role_bank_kernel.py:46-73 _role_forward, forward_rows.py:9-149) together with
// the route-weighted packing it consumes (gdn2_banks.py:196-224,
// role_bank_dispatch.py:41-73, routed_update.py:5-13), without materialising
// packed event tensors: every event is gathered from token storage by id.
//
// Work unit = one warp = (batch*bank sequence, head, tile of 32*NC value
// columns).  The S x dv bank state is column-separable: each lane owns NC
// columns and keeps all S rows of them in FP32 registers (f32x2 packed math on
// sm_100), so reductions over rows need no shuffles.
//
// Deferred decay.  Reference step for a write event (per row s, per column):
//     M = e * M ;  u = w_e*v - sum_s a_s M_s ;  M = M + k u
// with e = exp(g_e), a = dtype(b*p)*k.  Inside a segment of events the kernel
// keeps N = M / D, D_s = prod of e_s since the segment start, so one event is
//     u = w_e*v - sum_s (a_s D_s) N_s ;  N_s += (k_s / D_s) u
// and a read is  out = scale * sum_s (q_s D_s) N_s.  The per-event row
// coefficients a*D, k/D, q*D come from a segmented prefix sum of log-decays
// across the lanes of the warp (lane = event), computed while the previous
// batch runs.  N is multiplied back by D (materialised) at every segment end:
// the end of a batch, a BF16 state-storage point (gdn2_banks.py:35-36), or
// where the cumulative log-decay would leave the FP32 range (the batch is cut).
#include "common.cuh"
#include "scan.cuh"

#include <atomic>
#include <type_traits>

namespace bdm {
namespace {

#ifndef BDM_SCAN_MIN_BLOCKS
#define BDM_SCAN_MIN_BLOCKS 4  // resident CTAs per SM the register allocation targets (measured best)
#endif
#ifndef BDM_SCAN_MIN_BLOCKS_G2
#define BDM_SCAN_MIN_BLOCKS_G2 3  // the same with two heads per warp (twice the state registers per lane)
#endif
#ifndef BDM_SCAN_G2
#define BDM_SCAN_G2 1  // 1: even head counts run two heads per warp in the short kernel
#endif
#ifndef BDM_SCAN_LONG
#define BDM_SCAN_LONG 1  // 1: long sequences run on warp-specialised CTAs; 0: every unit on one warp
#endif
#ifndef BDM_SCAN_LONG_CTAS_PER_SM
#define BDM_SCAN_LONG_CTAS_PER_SM 2  // warp-specialised CTAs per SM (persistent over the long units)
#endif
#ifndef BDM_SCAN_DYNAMIC
#define BDM_SCAN_DYNAMIC 0  // 1: persistent CTAs take work items from an atomic counter; 0: one item per CTA
#endif
#ifndef BDM_SCAN_PREFETCH
#define BDM_SCAN_PREFETCH 4  // value-row prefetch distance (events)
#endif

constexpr int kScanWarps = 4;
constexpr int kPrefetch = BDM_SCAN_PREFETCH;
// With two heads per warp the value rows are twice as wide: two events ahead keep the registers
// within 3 CTAs per SM (measured faster than four events at 3 CTAs or 4 CTAs with spills).
#ifndef BDM_SCAN_PREFETCH_G2
#define BDM_SCAN_PREFETCH_G2 2
#endif
constexpr int kPrefetchG2 = BDM_SCAN_PREFETCH_G2;

// Lower bounds of classes 1..3; class 0 starts at the launch's long-sequence bound.
__device__ __constant__ int kLenLower[kLenClasses] = {0, 2048, 512, 1};

template <int BYTES> struct VecOf;
template <> struct VecOf<4> { using type = uint32_t; };
template <> struct VecOf<8> { using type = uint2; };
template <> struct VecOf<16> { using type = uint4; };

// NC consecutive elements of T moved as one vector (two for 32 bytes).
template <typename T, int NC> struct Row {
    static constexpr int kBytes = NC * (int)sizeof(T);
    T x[NC];
};

template <typename T, int NC>
__device__ __forceinline__ void load_row(Row<T, NC> &r, const T *p) {
    constexpr int B = Row<T, NC>::kBytes;
    if constexpr (B == 32) {
        const uint4 *src = reinterpret_cast<const uint4 *>(p);
        uint4 *dst = reinterpret_cast<uint4 *>(r.x);
        dst[0] = __ldg(src);
        dst[1] = __ldg(src + 1);
    } else {
        using V = typename VecOf<B>::type;
        *reinterpret_cast<V *>(r.x) = __ldg(reinterpret_cast<const V *>(p));
    }
}

template <typename T, int NC>
__device__ __forceinline__ void store_row(T *p, const Row<T, NC> &r) {
    constexpr int B = Row<T, NC>::kBytes;
    if constexpr (B == 32) {
        uint4 *dst = reinterpret_cast<uint4 *>(p);
        const uint4 *src = reinterpret_cast<const uint4 *>(r.x);
        dst[0] = src[0];
        dst[1] = src[1];
    } else {
        using V = typename VecOf<B>::type;
        *reinterpret_cast<V *>(p) = *reinterpret_cast<const V *>(r.x);
    }
}

__device__ __forceinline__ float2 dup(float x) { return make_float2(x, x); }

template <typename T> __device__ __forceinline__ float2 load_pair(const T *x);
template <> __device__ __forceinline__ float2 load_pair<float>(const float *x) { return make_float2(x[0], x[1]); }
template <> __device__ __forceinline__ float2 load_pair<bf16>(const bf16 *x) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(x));
}

template <typename T> __device__ __forceinline__ void store_pair(T *x, float2 v);
template <> __device__ __forceinline__ void store_pair<float>(float *x, float2 v) {
    x[0] = v.x;
    x[1] = v.y;
}
template <> __device__ __forceinline__ void store_pair<bf16>(bf16 *x, float2 v) {
    *reinterpret_cast<__nv_bfloat162 *>(x) = __floats2bfloat162_rn(v.x, v.y);
}

__device__ __forceinline__ float2 bf16_round_pair(float2 x) {
    return __bfloat1622float2(__floats2bfloat162_rn(x.x, x.y));
}

// u = dtype(w * p) * v - erase for a column pair.  The product of two BF16
// values is exact in FP32, so one packed BF16 multiply (RNE) reproduces the
// reference's rounded w*p, and one FMA forms u exactly as mul-then-subtract does.
template <typename T> struct WriteValue;
template <> struct WriteValue<bf16> {
    __device__ __forceinline__ static float2 apply(const bf16 *w, const bf16 *v, float2 pp, float2 minus_erase) {
        const __nv_bfloat162 p2 = *reinterpret_cast<const __nv_bfloat162 *>(&pp.x);
        const __nv_bfloat162 we = __hmul2(*reinterpret_cast<const __nv_bfloat162 *>(w), p2);
        return __ffma2_rn(__bfloat1622float2(we), load_pair<bf16>(v), minus_erase);
    }
};
template <> struct WriteValue<float> {
    __device__ __forceinline__ static float2 apply(const float *w, const float *v, float2 pp, float2 minus_erase) {
        const float2 we = __fmul2_rn(load_pair<float>(w), pp);
        return __ffma2_rn(we, load_pair<float>(v), minus_erase);
    }
};

// Route weight as the pair operand WriteValue expects (BF16: bf16x2 bits in .x).
template <typename T> __device__ __forceinline__ float2 weight_pair(float p);
template <> __device__ __forceinline__ float2 weight_pair<float>(float p) { return dup(p); }
template <> __device__ __forceinline__ float2 weight_pair<bf16>(float p) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(p, p);
    float2 r;
    r.x = *reinterpret_cast<const float *>(&h);
    r.y = 0.f;
    return r;
}

// Asynchronous global -> shared copy of BYTES (16-byte chunks when possible).
template <int BYTES>
__device__ __forceinline__ void cp_async(void *smem, const void *gmem) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    const char *g = static_cast<const char *>(gmem);
    if constexpr (BYTES % 16 == 0) {
#pragma unroll
        for (int i = 0; i < BYTES / 16; ++i)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s + 16 * i), "l"(g + 16 * i));
    } else if constexpr (BYTES == 8) {
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(g));
    } else {
        static_assert(BYTES == 4, "unsupported copy size");
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(g));
    }
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// Raw control rows of one event copied from token storage: k | b (dtype) and
// g (float) for a write; q (dtype) in the k slot for a read.
template <typename T, int S> struct RawLayout {
    static constexpr int kBytes = S * (int)sizeof(T);
    static constexpr int gBytes = S * 4;
    static constexpr int kOff = 0, bOff = kBytes, gOff = 2 * kBytes;
    static constexpr int size = 2 * kBytes + gBytes;
};

// Per-event controls as duplicated pairs: [a*D or q_e*D | k/D | p, pad | D before the event].
template <int S> struct CtlLayout {
    static constexpr int c = 0, kd = S, p = 2 * S, dprev = 2 * S + 2, size = 3 * S + 2;
};

// Per-event record of a staged batch, written by the lane that staged the event: the event's row
// offset in token storage (write: token * V for its value / write-gate rows; read: read id * V for
// its output row) and its kind.  The event loop reads one record per event instead of decoding ids
// and masks itself: the staging does that work one event per lane, the loop one event per warp
// instruction.
struct __align__(16) EvRec {
    long long off;
    int kind;
    int pad;
};
constexpr int kEvWrite = 1, kEvRead = 2, kEvRound = 4, kEvCk = 8;

#ifndef BDM_SCAN_EB_S16
#define BDM_SCAN_EB_S16 16  // events per staged batch when S = 16 (32 otherwise)
#endif
template <int S> struct EvBatch { static constexpr int value = S >= 16 ? BDM_SCAN_EB_S16 : 32; };


// Initial state of a unit's columns: the cache, the product-key factors (bank
// mapped into the full table on sharded ranks, head offset for head groups),
// or zero; rounded to BF16 when the training storage policy is on.
template <int S, int NP>
__device__ __forceinline__ void load_initial_state(const ScanParams &p, int64_t bank, int hh, int col0, bool active,
                                                   int64_t state_off, float2 (&N)[S][NP]) {
#pragma unroll
    for (int s = 0; s < S; ++s)
#pragma unroll
        for (int j = 0; j < NP; ++j) N[s][j] = make_float2(0.f, 0.f);
    if (!active) return;
    if (p.cache) {
#pragma unroll
        for (int s = 0; s < S; ++s)
#pragma unroll
            for (int j = 0; j < NP; ++j) {
                const int64_t o = state_off + (int64_t)s * p.dv + 2 * j;
                N[s][j] = p.cache_dtype == BDM_BF16 ? load_pair<bf16>(static_cast<const bf16 *>(p.cache) + o)
                                                    : load_pair<float>(static_cast<const float *>(p.cache) + o);
            }
    } else if (p.row_factor) {
        int64_t gbank = bank;
        if (p.bank_ids) {
            gbank = p.bank_ids[bank];
            gbank = gbank < 0 ? 0 : (gbank >= p.total_banks ? p.total_banks - 1 : gbank);
        }
#pragma unroll
        for (int s = 0; s < S; ++s) {
            const int64_t r = (gbank * p.total_heads + p.head_offset + hh) * S + s;
            const int64_t ou = (r / p.factor_cols) * p.dv + col0, oz = (r % p.factor_cols) * p.dv + col0;
#pragma unroll
            for (int j = 0; j < NP; ++j) {
                if (p.factor_dtype == BDM_BF16) {
                    const float2 u = load_pair<bf16>(static_cast<const bf16 *>(p.row_factor) + ou + 2 * j);
                    const float2 z = load_pair<bf16>(static_cast<const bf16 *>(p.col_factor) + oz + 2 * j);
                    N[s][j] = bf16_round_pair(make_float2(u.x + z.x, u.y + z.y));
                } else {
                    const float2 u = load_pair<float>(static_cast<const float *>(p.row_factor) + ou + 2 * j);
                    const float2 z = load_pair<float>(static_cast<const float *>(p.col_factor) + oz + 2 * j);
                    N[s][j] = make_float2(u.x + z.x, u.y + z.y);
                }
            }
        }
    }
    if (p.interval > 0) {
#pragma unroll
        for (int s = 0; s < S; ++s)
#pragma unroll
            for (int j = 0; j < NP; ++j) N[s][j] = bf16_round_pair(N[s][j]);
    }
}

// One staged event on a lane's columns.  Coefficients come two at a time
// (128-bit shared loads of duplicated pairs); dot products run in NCH
// independent chains per column pair.
template <typename T, int S, int NC>
__device__ __forceinline__ void event_step(const float2 *row, bool round_point, bool is_write, bool is_read,
                                           bool active, const Row<T, NC> &vr, const Row<T, NC> &wr, float scale,
                                           T *out_row, float2 (&N)[S][NC / 2], bool ck_point = false,
                                           float *ck_row = nullptr, int64_t ck_stride = 0) {
    using Ctl = CtlLayout<S>;
    constexpr int NP = NC / 2;
    // independent FMA chains per column pair: with 4 or more pairs the pairs alone give the ILP
    constexpr int NCH = NP >= 4 ? 1 : (NP >= 2 ? 2 : 4);
    if (round_point) {  // storage point: materialise, round to BF16
#pragma unroll
        for (int s = 0; s < S; ++s) {
            const float2 d2 = row[Ctl::dprev + s];
#pragma unroll
            for (int c = 0; c < NP; ++c) N[s][c] = bf16_round_pair(__fmul2_rn(N[s][c], d2));
        }
    } else if (ck_point) {  // checkpoint only: materialise
#pragma unroll
        for (int s = 0; s < S; ++s) {
            const float2 d2 = row[Ctl::dprev + s];
#pragma unroll
            for (int c = 0; c < NP; ++c) N[s][c] = __fmul2_rn(N[s][c], d2);
        }
    }
    if (ck_point && active) {  // the state before this event, for the recurrence backward
#pragma unroll
        for (int s = 0; s < S; ++s)
#pragma unroll
            for (int c = 0; c < NP; ++c) store_pair<float>(ck_row + (int64_t)s * ck_stride + 2 * c, N[s][c]);
    }
    const float4 *crow = reinterpret_cast<const float4 *>(row + Ctl::c);
    if (is_write) {
        float2 mer[NP];
#pragma unroll
        for (int c = 0; c < NP; ++c) {
            float2 ch[NCH];
#pragma unroll
            for (int i = 0; i < NCH; ++i) ch[i] = make_float2(0.f, 0.f);
#pragma unroll
            for (int s = 0; s < S; s += 2) {
                const float4 cc = crow[s / 2];
                const int i = (s / 2) % NCH;
                ch[i] = __ffma2_rn(make_float2(cc.x, cc.y), N[s][c], ch[i]);
                ch[(i + NCH / 2) % NCH] = __ffma2_rn(make_float2(cc.z, cc.w), N[s + 1][c], ch[(i + NCH / 2) % NCH]);
            }
#pragma unroll
            for (int i = 1; i < NCH; ++i) ch[0] = __fadd2_rn(ch[0], ch[i]);
            mer[c] = make_float2(-ch[0].x, -ch[0].y);
        }
        const float2 pw = row[Ctl::p];
        float2 u[NP];
#pragma unroll
        for (int c = 0; c < NP; ++c) u[c] = WriteValue<T>::apply(wr.x + 2 * c, vr.x + 2 * c, pw, mer[c]);
        const float4 *krow = reinterpret_cast<const float4 *>(row + Ctl::kd);
#pragma unroll
        for (int s = 0; s < S; s += 2) {
            const float4 kk = krow[s / 2];
#pragma unroll
            for (int c = 0; c < NP; ++c) {
                N[s][c] = __ffma2_rn(make_float2(kk.x, kk.y), u[c], N[s][c]);
                N[s + 1][c] = __ffma2_rn(make_float2(kk.z, kk.w), u[c], N[s + 1][c]);
            }
        }
    } else if (is_read) {
        float2 acc[NP][NCH];
#pragma unroll
        for (int c = 0; c < NP; ++c)
#pragma unroll
            for (int i = 0; i < NCH; ++i) acc[c][i] = make_float2(0.f, 0.f);
#pragma unroll
        for (int s = 0; s < S; s += 2) {
            const float4 cc = crow[s / 2];
            const int i = (s / 2) % NCH;
#pragma unroll
            for (int c = 0; c < NP; ++c) {
                acc[c][i] = __ffma2_rn(make_float2(cc.x, cc.y), N[s][c], acc[c][i]);
                acc[c][(i + NCH / 2) % NCH] =
                    __ffma2_rn(make_float2(cc.z, cc.w), N[s + 1][c], acc[c][(i + NCH / 2) % NCH]);
            }
        }
        if (active) {
            Row<T, NC> o;
#pragma unroll
            for (int c = 0; c < NP; ++c) {
#pragma unroll
                for (int i = 1; i < NCH; ++i) acc[c][0] = __fadd2_rn(acc[c][0], acc[c][i]);
                store_pair<T>(o.x + 2 * c, __fmul2_rn(acc[c][0], dup(scale)));
            }
            store_row<T, NC>(out_row, o);
        }
    }
}

// Short sequences: one warp per (sequence, group of G heads, column tile) unit, kScanWarps
// units per CTA; each warp stages and runs its own batches.  Takes the length
// classes from p.ws_classes on (all of them when the long kernel does not run).
// G = 2: the two halves of the warp run two heads of the same sequence (16 lanes x NC columns
// each); the events, their records and the loop control are shared by both heads, and the
// staging runs one (event, head) pair per lane over batches of 16 events.
// CK: the launch writes the recurrence backward's state checkpoints (training forwards only;
// the inference instantiation keeps none of that code).
template <typename T, int S, int NC, bool CK, int G>
__global__ void __launch_bounds__(kScanWarps * 32, G == 2 ? BDM_SCAN_MIN_BLOCKS_G2 : BDM_SCAN_MIN_BLOCKS)
bank_scan_kernel(const ScanParams p) {
    constexpr int NP = NC / 2;
    constexpr int LPG = 32 / G;  // lanes per head
    // two heads per warp: 16 events per batch (one (event, head) pair per lane), 8 at S = 16 (its
    // coefficient rows are twice as long; 48 KB of static shared memory)
    constexpr int EBG = G == 2 ? (S >= 16 ? 8 : 16) : 32;
    constexpr int EB = EvBatch<S>::value < EBG ? EvBatch<S>::value : EBG;
    constexpr int PD = G == 2 ? kPrefetchG2 : kPrefetch;
    using Raw = RawLayout<T, S>;
    using Ctl = CtlLayout<S>;
    static_assert(EB % PD == 0 && LPG % EB == 0 && EB <= LPG && S % 2 == 0 && (G == 1 || G == 2), "batch layout");
    __shared__ __align__(16) float2 ctl_all[kScanWarps][EB][G][Ctl::size];
    __shared__ __align__(16) float2 dend_all[kScanWarps][G][S];
    __shared__ __align__(16) unsigned char raw_all[kScanWarps][G == 1 ? EB : 32][Raw::size];
    // EB records per batch plus PD empty ones, so prefetches past the batch need no bounds check
    __shared__ EvRec ev_all[kScanWarps][EB + PD];
    __shared__ unsigned long long item_shared;

    const int warp = threadIdx.x >> 5;
    const int lane = (int)lane_id();
    const int el = lane % LPG, hl = lane / LPG;  // staging: event el of the batch, head hl of the group
    float2(*ctl)[G][Ctl::size] = ctl_all[warp];
    float2(*dend)[S] = dend_all[warp];
    unsigned char(*raw)[Raw::size] = raw_all[warp];
    EvRec *ev_s = ev_all[warp];
    if (lane < PD) ev_s[EB + lane] = EvRec{0, 0, 0};
    const int64_t per_seq = (int64_t)(p.H / G) * p.ctiles;
    int64_t total = 0;  // units of the classes this kernel runs (the long classes go to the long kernel)
#pragma unroll
    for (int c = 0; c < kLenClasses; ++c) total += c >= p.ws_classes ? p.counts[c] : 0;
    total *= per_seq;

    // CTAs take kScanWarps consecutive (sequence, head, column tile) units at a
    // time, so the warps of a CTA work on the heads of one sequence and share
    // its control rows in L1.
    unsigned long long static_item = blockIdx.x;
    for (;;) {
    __syncthreads();
    if (threadIdx.x == 0) item_shared = BDM_SCAN_DYNAMIC ? atomicAdd(p.next, 1ull) : static_item;
    __syncthreads();
    static_item += gridDim.x;
    const unsigned long long item_s = item_shared;
    const int64_t item = (int64_t)item_s * kScanWarps + warp;
    if ((int64_t)item_s * kScanWarps >= total) break;  // CTA-uniform
    if (item >= total) continue;
    int64_t local = (int64_t)item / per_seq;
    int cls = p.ws_classes;
    while (cls < kLenClasses - 1 && local >= p.counts[cls]) local -= p.counts[cls++];
    const int64_t seq = p.lists[(int64_t)cls * p.nseq + local];
    const int64_t rem = (int64_t)item % per_seq;
    const int hh = (int)(rem / p.ctiles) * G + hl;  // this lane's head
    const int ct = (int)(rem % p.ctiles);
    const int64_t bidx = seq / p.J, bank = seq % p.J;
    const int col0 = ct * LPG * NC + el * NC;
    const bool active = col0 < p.dv;
    const int HS = p.H * S;
    const int64_t V = (int64_t)p.H * p.dv;
    const int nw = (int)p.nw, kw = p.kw, kr = p.kr, nt = (int)p.nt, E = (int)p.E;

    const T *qp = static_cast<const T *>(p.q);
    const T *kp = static_cast<const T *>(p.k);
    const T *vp = static_cast<const T *>(p.v) + (int64_t)hh * p.dv + col0;
    const T *bp = static_cast<const T *>(p.b);
    const T *wp = static_cast<const T *>(p.w) + (int64_t)hh * p.dv + col0;
    const T *wwp = static_cast<const T *>(p.ww);
    const T *rwp = static_cast<const T *>(p.rw);
    T *outp = static_cast<T *>(p.reads) + (int64_t)hh * p.dv + col0;

    // ---------------------------------------------------------- initial state
    float2 N[S][NP];
    const int64_t state_off = ((bidx * p.J + bank) * p.H + hh) * (int64_t)S * p.dv + col0;
    load_initial_state<S, NP>(p, bank, hh, col0, active, state_off, N);

    // Clamp caller-provided bounds so a malformed cu_seqlens cannot index past `order`.
    const int64_t start = min(max(p.cu[seq], (int64_t)0), p.E);
    const int64_t end = min(max(p.cu[seq + 1], start), p.E);

    // ------------------------------------------------------ batch staging
    // Lane i owns event i of a batch.  stage_issue decodes its id and starts the
    // asynchronous copy of its control rows; stage_finish turns them into the
    // deferred-decay coefficients.
    int my_tok = -1, my_rid = -1;
    bool my_write = false;
    float my_wt = 0.f;
    auto stage_issue = [&](int64_t bbase, int bn) {
        my_tok = -1;
        my_rid = -1;
        my_write = false;
        my_wt = 0.f;
        if (el < bn) {
            const int64_t id = p.order[bbase + el];
            if (id >= 0 && id < nw) {
                my_tok = (int)id / kw;
                my_write = true;
                my_wt = Elem<T>::to_float(wwp[id]);
            } else if (id >= nw && id < E) {
                my_rid = (int)id - nw;
                my_tok = my_rid / kr;
                my_wt = Elem<T>::to_float(rwp[my_rid]);
            }
            if (my_tok >= nt) {
                my_tok = -1;
                my_write = false;
                my_rid = -1;
            }
        }
        if (my_tok >= 0) {
            const int64_t o = (int64_t)my_tok * HS + (int64_t)hh * S;
            if (my_write) {
                cp_async<Raw::kBytes>(raw[lane] + Raw::kOff, kp + o);
                cp_async<Raw::kBytes>(raw[lane] + Raw::bOff, bp + o);
                cp_async<Raw::gBytes>(raw[lane] + Raw::gOff, p.g + o);
            } else {
                cp_async<Raw::kBytes>(raw[lane] + Raw::kOff, qp + o);
            }
        }
        cp_async_commit();
    };
    // pos0 = position of the batch's first event in its sequence.  Sets the
    // number of events to run (<= bn, cut where the log-decay range ends), the
    // storage-point mask, and returns the write mask.
    auto stage_finish = [&](int64_t pos0, int bn, int &n_out, unsigned &round_out, unsigned &ck_out) -> unsigned {
        cp_async_wait_all();
        const bool valid = el < bn;
        const int64_t pos = pos0 + el;
        const bool head = valid && p.interval > 0 && pos > 0 && (pos % p.interval) == 0;
        const bool ckp = CK && valid && pos > 0 && (pos % p.ckpt_block) == 0;
        const T *rk = reinterpret_cast<const T *>(raw[lane] + Raw::kOff);
        const float *rg = reinterpret_cast<const float *>(raw[lane] + Raw::gOff);
        // segmented inclusive scan of log-decays; segments start at lane 0 and at storage points
        float L[S];
#pragma unroll
        for (int s = 0; s < S; ++s) {
            float ge = 0.f;
            if (my_write && my_tok >= 0) ge = fmaxf(p.routed_decay ? rg[s] * my_wt : rg[s], kMinLogDecay);
            L[s] = ge;
        }
        bool f = head || ckp || el == 0;
#pragma unroll
        for (int d = 1; d < LPG; d <<= 1) {
            const bool fu = __shfl_up_sync(0xffffffffu, f, d, LPG);
            const bool take = el >= d && !f;
#pragma unroll
            for (int s = 0; s < S; ++s) {
                const float lu = __shfl_up_sync(0xffffffffu, L[s], d, LPG);
                if (take) L[s] += lu;
            }
            f = f || (el >= d && fu);
        }
        // cut the batch before the first event whose segment would leave the FP32 range
        float lmin = 0.f;
#pragma unroll
        for (int s = 0; s < S; ++s) lmin = fminf(lmin, L[s]);
        unsigned over = __ballot_sync(0xffffffffu, valid && lmin < kMinLogDecay);
        if (G == 2) over = (over | (over >> 16)) & 0xffffu;  // either head's range ends the batch
        const int n = over ? (__ffs(over) - 1) : bn;  // >= 1: a single event is floored above
        const bool use = el < n;
        float D[S];
#pragma unroll
        // the hardware exponential: L >= -60, so its relative error stays near 5e-6, far inside
        // the FP32 tolerance, and it is a fraction of expf's instructions
        for (int s = 0; s < S; ++s) D[s] = __expf(L[s]);
        if (use && my_tok >= 0) {
            if (my_write) {
                const T *rb = reinterpret_cast<const T *>(raw[lane] + Raw::bOff);
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    const float kk = Elem<T>::to_float(rk[s]);
                    const float a = rnd<T>(Elem<T>::to_float(rb[s]) * my_wt) * kk;
                    ctl[el][hl][Ctl::c + s] = dup(a * D[s]);
                    ctl[el][hl][Ctl::kd + s] = dup(kk * __expf(-L[s]));
                }
                ctl[el][hl][Ctl::p] = weight_pair<T>(my_wt);
            } else {
#pragma unroll
                for (int s = 0; s < S; ++s)
                    ctl[el][hl][Ctl::c + s] = dup(rnd<T>(Elem<T>::to_float(rk[s]) * my_wt) * D[s]);
            }
        }
        // D before a storage point (materialise there), D after the last event (batch end)
#pragma unroll
        for (int s = 0; s < S; ++s) {
            const float before = __shfl_up_sync(0xffffffffu, D[s], 1, LPG);
            if (use && (head || ckp)) ctl[el][hl][Ctl::dprev + s] = dup(el == 0 ? 1.0f : before);
            if (el == n - 1) dend[hl][s] = dup(D[s]);
        }
        if (hl == 0 && el < EB) {
            EvRec r{0, 0, 0};
            if (use && my_tok >= 0) {
                r.kind = my_write ? kEvWrite : kEvRead;
                r.off = (long long)(my_write ? my_tok : my_rid) * V;
            }
            if (use && head) r.kind |= kEvRound;
            if (use && ckp) r.kind |= kEvCk;
            ev_s[el] = r;
        }
        n_out = n;
        round_out = __ballot_sync(0xffffffffu, hl == 0 && use && head);
        ck_out = __ballot_sync(0xffffffffu, hl == 0 && use && ckp);
        const unsigned wm = __ballot_sync(0xffffffffu, hl == 0 && use && my_write && my_tok >= 0);
        __syncwarp();
        return wm;
    };

    int n = 0;
    unsigned wmask = 0, rmask = 0, cmask = 0;
    {
        const int bn = (int)min((int64_t)EB, end - start);
        if (bn > 0) {
            stage_issue(start, bn);
            wmask = stage_finish(0, bn, n, rmask, cmask);
        }
    }
    Row<T, NC> vr[PD], wr[PD];

    for (int64_t base = start; base < end;) {
        const int64_t nbase = base + n;
        const int nn = (int)min((int64_t)EB, end - nbase);
        // events past n have empty records: no loads, and event_step does nothing for them
        auto prefetch = [&](int ev, int slot) {
            const EvRec r = ev_s[ev];
            if ((r.kind & kEvWrite) && active) {
                load_row<T, NC>(vr[slot], vp + r.off);
                load_row<T, NC>(wr[slot], wp + r.off);
            }
        };
#pragma unroll
        for (int j = 0; j < PD; ++j) prefetch(j, j);
        bool issued = false;
        for (int e0 = 0; e0 < n; e0 += PD) {
            if (e0 == EB / 2 && nn > 0) {  // stage the next batch under the second half
                stage_issue(nbase, nn);
                issued = true;
            }
#pragma unroll
            for (int j = 0; j < PD; ++j) {  // a group past n runs empty records (no-ops)
                const int ev = e0 + j;
                const EvRec r = ev_s[ev];
                float *ck_row = nullptr;
                const bool ck_here = CK && (r.kind & kEvCk);
                if (ck_here) {
                    const int64_t pos = base - start + ev;
                    ck_row = p.ckpt + ((start / p.ckpt_block + seq + pos / p.ckpt_block) * p.H + hh) * (int64_t)S * p.dv +
                             col0;
                }
                event_step<T, S, NC>(ctl[ev][hl], r.kind & kEvRound, r.kind & kEvWrite, r.kind & (kEvWrite | kEvRead),
                                     active, vr[j], wr[j], p.scale, outp + r.off, N, ck_here, ck_row, p.dv);
                prefetch(ev + PD, j);
            }
        }
        // segment end: materialise N = D * N for the next batch (or the final state)
#pragma unroll
        for (int s = 0; s < S; ++s) {
            const float2 d2 = dend[hl][s];
#pragma unroll
            for (int c = 0; c < NP; ++c) N[s][c] = __fmul2_rn(N[s][c], d2);
        }
        if (nn > 0) {
            if (!issued) stage_issue(nbase, nn);
            __syncwarp();
            wmask = stage_finish(nbase - start, nn, n, rmask, cmask);
        }
        base = nbase;
    }

    if (p.store_final && p.cache && active) {
#pragma unroll
        for (int s = 0; s < S; ++s)
#pragma unroll
            for (int j = 0; j < NP; ++j) {
                const int64_t o = state_off + (int64_t)s * p.dv + 2 * j;
                if (p.cache_dtype == BDM_BF16) store_pair<bf16>(static_cast<bf16 *>(p.cache) + o, N[s][j]);
                else store_pair<float>(static_cast<float *>(p.cache) + o, N[s][j]);
            }
    }
    __syncwarp();  // staging buffers are reused by the next unit
    }
}

// ===========================================================================
// Long sequences: warp-specialised CTAs.
//
// A sequence with thousands of events is a serial chain; its latency, not the
// GPU's throughput, bounds a launch whose router is skewed.  The first
// p.ws_ctas CTAs of a launch take the units (sequence, head) of the long
// length classes and split each across warps:
//   warp 0 (producer) stages a batch of EB events: ids, route weights, async
//     copies of the k|b|g / q rows and of the lanes' v / w values, the
//     segmented log-decay scan and the deferred-decay coefficients;
//   warps 1..T (consumers, one per value-column tile) run the state math from
//     shared memory only.
// The producer stages batch i+1 while the consumers run batch i, so a batch
// costs about max(staging, math) instead of their sum, the tiles of a head
// share one staging pass, and the consumers never wait on global memory.
//
// Handoff through a two-slot ring: mbarriers full[slot] (32 producer
// arrivals) and empty[slot] (32*T consumer arrivals), waited by phase parity.
// The value rows of batch i+1 are copied once its slot is free (after the
// consumers finish batch i-1, while they run batch i).  Every wait is bounded:
// after kWaitPolls polls or kWaitNs nanoseconds it records
// BDM_SCAN_ERR_TIMEOUT in the status word, raises the CTA's abort flag and
// returns; the other warps then fail their own bounded waits and return.
// ===========================================================================
constexpr int kWsMaxTiles = kScanWarps - 1;  // consumers per CTA
// Ring depth and batch size: two slots of 32 events (~67 KB at S = 16, two
// column tiles), so two long CTAs and two short CTAs share an SM.
#ifndef BDM_SCAN_LONG_SLOTS
#define BDM_SCAN_LONG_SLOTS 2
#endif
#ifndef BDM_SCAN_LONG_BATCH
#define BDM_SCAN_LONG_BATCH 32
#endif
constexpr int kWsSlots = BDM_SCAN_LONG_SLOTS;
constexpr long long kWaitPolls = 1ll << 22;
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t *bar, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;\n" : "=l"(t));
    return t;
}
// Bounded wait for the phase of `parity` to complete; false on timeout (after limit_ns).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity, unsigned long long limit_ns) {
    if (mbar_test(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (long long i = 0; i < kWaitPolls; ++i) {
        if (mbar_test(bar, parity)) return true;
        if ((i & 255) == 255 && global_ns() - t0 > limit_ns) break;
    }
    return false;
}

// Shared memory of a warp-specialised CTA: the ring (fixed part), the
// producer's raw row buffers, then the staged value rows (sized at launch by
// the number of column tiles).
constexpr int kWsBatch = BDM_SCAN_LONG_BATCH;  // events per staged batch in long mode (every S)
template <typename T, int S> struct WsShared {
    static constexpr int EB = kWsBatch;
    float2 ctl[kWsSlots][EB][CtlLayout<S>::size];
    float2 dend[kWsSlots][S];
    int tok[kWsSlots][EB], rid[kWsSlots][EB];
    int n[kWsSlots];
    unsigned wmask[kWsSlots], rmask[kWsSlots];
    uint64_t full[kWsSlots], empty[kWsSlots];
    long long item;
    int abort;
    __align__(16) unsigned char raw[2][EB][RawLayout<T, S>::size];
};
template <typename T, int S, int NC>
__host__ __device__ constexpr int64_t ws_value_bytes(int tiles) {  // v and w rows of a slot's events
    return (int64_t)kWsSlots * kWsBatch * tiles * 2 * 32 * NC * (int64_t)sizeof(T);
}
template <typename T, int S> __host__ __device__ constexpr int64_t ws_fixed_bytes() {
    return ((int64_t)sizeof(WsShared<T, S>) + 15) / 16 * 16;
}

struct Staged {
    int tok, rid;
    bool write;
    float wt;
};

// Ring slot of the it-th batch and the phase parity of its n-th use.
__device__ __forceinline__ int ring_slot(unsigned it) { return (int)(it % kWsSlots); }
__device__ __forceinline__ unsigned use_parity(unsigned it) { return (it / kWsSlots) & 1u; }

template <typename T, int S, int NC>
__device__ __forceinline__ void scan_long_units(const ScanParams &p, unsigned char *smem) {
    constexpr int NP = NC / 2;
    constexpr int EB = kWsBatch;
    using Raw = RawLayout<T, S>;
    using Ctl = CtlLayout<S>;
    constexpr int kRowElems = 32 * NC;  // one tile's columns of a v or w row
    WsShared<T, S> &sh = *reinterpret_cast<WsShared<T, S> *>(smem);
    T *vw = reinterpret_cast<T *>(smem + ws_fixed_bytes<T, S>());  // [slot][event][tile][v|w][kRowElems]

    const int warp = threadIdx.x >> 5;
    const int lane = (int)lane_id();
    const int tiles = p.ctiles;
    int64_t long_seqs = 0;
    for (int c = 0; c < p.ws_classes; ++c) long_seqs += p.counts[c];
    const int64_t total = long_seqs * p.H;
    if ((int64_t)blockIdx.x >= total) return;  // CTA-uniform
    if (threadIdx.x == 0) {
        for (int b = 0; b < kWsSlots; ++b) {
            mbar_init(&sh.full[b], 32);
            mbar_init(&sh.empty[b], 32 * tiles);
        }
        sh.abort = 0;
    }
    __syncthreads();

    volatile int *abort_flag = &sh.abort;
    const unsigned long long wait_ns = p.wait_ns ? p.wait_ns : kWaitNs;
    bool withhold = p.test_fault == 1;  // diagnostics: skip the first hand-off of this CTA
    auto fail = [&]() {
        if (lane == 0) atomicOr(p.status, BDM_SCAN_ERR_TIMEOUT);
        *abort_flag = 1;
    };
    auto slot_values = [&](int slot, int ev, int tile, int which) {
        return vw + ((((int64_t)slot * EB + ev) * tiles + tile) * 2 + which) * kRowElems;
    };
    const int HS = p.H * S;
    const int64_t V = (int64_t)p.H * p.dv;
    const int nw = (int)p.nw, kw = p.kw, kr = p.kr, nt = (int)p.nt, E = (int)p.E;
    unsigned it = 0;  // batches handed through the ring (same count on every warp)

    for (;;) {
        // units in LPT order: the next longest unit goes to the next free CTA
        __syncthreads();
        if (threadIdx.x == 0) sh.item = (long long)atomicAdd(p.long_next, 1ull);
        __syncthreads();
        const int64_t item = sh.item;
        if (item >= total || *abort_flag) break;
        int64_t local = item / p.H;
        int cls = 0;
        while (cls < kLenClasses - 1 && local >= p.counts[cls]) local -= p.counts[cls++];
        const int64_t seq = p.lists[(int64_t)cls * p.nseq + local];
        const int hh = (int)(item % p.H);
        const int64_t bidx = seq / p.J, bank = seq % p.J;
        const int64_t start = min(max(p.cu[seq], (int64_t)0), p.E);
        const int64_t end = min(max(p.cu[seq + 1], start), p.E);

        if (warp == 0) {
            // ------------------------------------------------------- producer
            const T *qp = static_cast<const T *>(p.q);
            const T *kp = static_cast<const T *>(p.k);
            const T *bp = static_cast<const T *>(p.b);
            const T *wwp = static_cast<const T *>(p.ww);
            const T *rwp = static_cast<const T *>(p.rw);
            // ids, weights and k|b|g / q rows of events [bbase, bbase + bn): lane = event
            // id and route weight of each lane's event in the batch after the one
            // being issued, loaded one batch ahead (nothing waits on them until then)
            int64_t pre_base = -1, pre_id = -1;
            T pre_wt = Elem<T>::from_float(0.f);
            auto weight_of = [&](int64_t id) -> T {
                if (id >= 0 && id < nw) return wwp[id];
                if (id >= nw && id < E) return rwp[id - nw];
                return Elem<T>::from_float(0.f);
            };
            auto issue_rows = [&](int64_t bbase, int bn, unsigned char (*rawb)[Raw::size], Staged &st) {
                st.tok = -1;
                st.rid = -1;
                st.write = false;
                st.wt = 0.f;
                int64_t my_id = -1;
                T my_wt = Elem<T>::from_float(0.f);
                if (bbase == pre_base) {
                    my_id = pre_id;
                    my_wt = pre_wt;
                } else if (lane < bn) {
                    my_id = p.order[bbase + lane];
                    my_wt = weight_of(my_id);
                }
                pre_base = bbase + bn;
                pre_id = (lane < EB && pre_base + lane < end) ? p.order[pre_base + lane] : -1;
                pre_wt = weight_of(pre_id);
                if (lane < bn) {
                    const int64_t id = my_id;
                    if (id >= 0 && id < nw) {
                        st.tok = (int)id / kw;
                        st.write = true;
                        st.wt = Elem<T>::to_float(my_wt);
                    } else if (id >= nw && id < E) {
                        st.rid = (int)id - nw;
                        st.tok = st.rid / kr;
                        st.wt = Elem<T>::to_float(my_wt);
                    }
                    if (st.tok >= nt) {
                        st.tok = -1;
                        st.write = false;
                        st.rid = -1;
                    }
                }
                if (st.tok >= 0) {
                    const int64_t o = (int64_t)st.tok * HS + (int64_t)hh * S;
                    if (st.write) {
                        cp_async<Raw::kBytes>(rawb[lane] + Raw::kOff, kp + o);
                        cp_async<Raw::kBytes>(rawb[lane] + Raw::bOff, bp + o);
                        cp_async<Raw::gBytes>(rawb[lane] + Raw::gOff, p.g + o);
                    } else {
                        cp_async<Raw::kBytes>(rawb[lane] + Raw::kOff, qp + o);
                    }
                }
            };
            // v / w columns of the batch's writes into ring slot `slot` (all lanes per event)
            // each lane copies its own write event's v and w columns (every tile)
            auto issue_values = [&](int bn, const Staged &st, int slot) {
                constexpr int kPiece = 16;
                const int row_bytes = kRowElems * (int)sizeof(T);
                const int64_t dv_bytes = (int64_t)p.dv * sizeof(T);
                if (lane >= bn || !st.write || st.tok < 0) return;
                const int64_t head_off = ((int64_t)st.tok * V + (int64_t)hh * p.dv) * sizeof(T);
                for (int which = 0; which < 2; ++which) {
                    const char *src = static_cast<const char *>(which ? p.w : p.v) + head_off;
                    for (int tile = 0; tile < tiles; ++tile) {
                        char *dst = reinterpret_cast<char *>(slot_values(slot, lane, tile, which));
                        for (int off = 0; off < row_bytes; off += kPiece) {
                            const int64_t col_bytes = (int64_t)tile * row_bytes + off;
                            if (col_bytes < dv_bytes) cp_async<kPiece>(dst + off, src + col_bytes);
                        }
                    }
                }
            };
            // coefficients of a staged batch into ring slot b; returns the events to run
            auto finish = [&](int64_t pos0, int bn, const unsigned char (*rawb)[Raw::size], const Staged &st, int b,
                              bool newer_pending) -> int {
                if (newer_pending) asm volatile("cp.async.wait_group 1;\n" ::: "memory");
                else cp_async_wait_all();
                float2(*ctl)[Ctl::size] = sh.ctl[b];
                const bool valid = lane < bn;
                const int64_t pos = pos0 + lane;
                const bool head = valid && p.interval > 0 && pos > 0 && (pos % p.interval) == 0;
                const T *rk = reinterpret_cast<const T *>(rawb[lane] + Raw::kOff);
                const float *rg = reinterpret_cast<const float *>(rawb[lane] + Raw::gOff);
                float L[S];
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    float ge = 0.f;
                    if (st.write && st.tok >= 0) ge = fmaxf(p.routed_decay ? rg[s] * st.wt : rg[s], kMinLogDecay);
                    L[s] = ge;
                }
                bool f = head || lane == 0;
#pragma unroll
                for (int d = 1; d < EB; d <<= 1) {
                    const bool fu = __shfl_up_sync(0xffffffffu, f, d);
                    const bool take = lane >= d && !f;
#pragma unroll
                    for (int s = 0; s < S; ++s) {
                        const float lu = __shfl_up_sync(0xffffffffu, L[s], d);
                        if (take) L[s] += lu;
                    }
                    f = f || (lane >= d && fu);
                }
                float lmin = 0.f;
#pragma unroll
                for (int s = 0; s < S; ++s) lmin = fminf(lmin, L[s]);
                const unsigned over = __ballot_sync(0xffffffffu, valid && lmin < kMinLogDecay);
                const int n = over ? (__ffs(over) - 1) : bn;  // >= 1: one event's decay is floored above
                const bool use = lane < n;
                float D[S];
#pragma unroll
                for (int s = 0; s < S; ++s) D[s] = expf(L[s]);
                if (use && st.tok >= 0) {
                    if (st.write) {
                        const T *rb = reinterpret_cast<const T *>(rawb[lane] + Raw::bOff);
#pragma unroll
                        for (int s = 0; s < S; ++s) {
                            const float kk = Elem<T>::to_float(rk[s]);
                            const float a = rnd<T>(Elem<T>::to_float(rb[s]) * st.wt) * kk;
                            ctl[lane][Ctl::c + s] = dup(a * D[s]);
                            ctl[lane][Ctl::kd + s] = dup(kk * expf(-L[s]));
                        }
                        ctl[lane][Ctl::p] = weight_pair<T>(st.wt);
                    } else {
#pragma unroll
                        for (int s = 0; s < S; ++s) {
                            ctl[lane][Ctl::c + s] = dup(rnd<T>(Elem<T>::to_float(rk[s]) * st.wt) * D[s]);
                            ctl[lane][Ctl::kd + s] = make_float2(0.f, 0.f);
                        }
                        ctl[lane][Ctl::p] = make_float2(0.f, 0.f);
                    }
                } else if (use) {
#pragma unroll
                    for (int s = 0; s < S; ++s) {
                        ctl[lane][Ctl::c + s] = make_float2(0.f, 0.f);
                        ctl[lane][Ctl::kd + s] = make_float2(0.f, 0.f);
                    }
                    ctl[lane][Ctl::p] = make_float2(0.f, 0.f);
                }
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    const float before = __shfl_up_sync(0xffffffffu, D[s], 1);
                    if (use && head) ctl[lane][Ctl::dprev + s] = dup(lane == 0 ? 1.0f : before);
                    if (lane == n - 1) sh.dend[b][s] = dup(D[s]);
                }
                if (lane < EB) {
                    sh.tok[b][lane] = use ? st.tok : -1;
                    sh.rid[b][lane] = use ? st.rid : -1;
                }
                const unsigned rm = __ballot_sync(0xffffffffu, use && head);
                const unsigned wm = __ballot_sync(0xffffffffu, use && st.write && st.tok >= 0);
                if (lane == 0) {
                    sh.n[b] = n;
                    sh.wmask[b] = wm;
                    sh.rmask[b] = rm;
                }
                __syncwarp();
                return n;
            };

            Staged cur{-1, -1, false, 0.f}, nxt{-1, -1, false, 0.f};
            int64_t base = start;
            int bn = (int)min((int64_t)EB, end - base);
            bool ok = true;
            // A batch's slot frees when the consumers finish the batch kWsSlots before it.
            auto acquire = [&](unsigned j) {
                return j < kWsSlots || mbar_wait(&sh.empty[ring_slot(j)], use_parity(j - kWsSlots), wait_ns);
            };
            issue_rows(base, bn, sh.raw[it & 1], cur);
            if (!acquire(it)) ok = false;
            if (ok) issue_values(bn, cur, ring_slot(it));
            cp_async_commit();
            while (ok && base < end) {
                const int64_t sbase = base + bn;  // next batch if this one is not cut
                const int sbn = (int)min((int64_t)EB, end - sbase);
                if (sbn > 0) {
                    issue_rows(sbase, sbn, sh.raw[(it + 1) & 1], nxt);
                    cp_async_commit();
                }
                const int b = ring_slot(it);
                const int n = finish(base - start, bn, sh.raw[it & 1], cur, b, sbn > 0);
                if (withhold) withhold = false;  // the consumers' wait for this batch runs out
                else mbar_arrive(&sh.full[b]);
                if (n < bn) {  // cut: the next batch starts right after the n-th event
                    cp_async_wait_all();
                    base += n;
                    bn = (int)min((int64_t)EB, end - base);
                    if (bn > 0) issue_rows(base, bn, sh.raw[(it + 1) & 1], nxt);
                } else {
                    base = sbase;
                    bn = sbn;
                }
                ++it;
                if (base < end) {
                    if (!acquire(it)) {
                        ok = false;
                        break;
                    }
                    issue_values(bn, nxt, ring_slot(it));
                    cp_async_commit();
                }
                cur = nxt;
            }
            cp_async_wait_all();
            if (!ok) fail();
        } else {
            // ------------------------------------------------------ consumers
            const int ct = warp - 1;
            const int col0 = ct * 32 * NC + lane * NC;
            const bool active = col0 < p.dv;
            T *outp = static_cast<T *>(p.reads) + (int64_t)hh * p.dv + col0;
            float2 N[S][NP];
            const int64_t state_off = ((bidx * p.J + bank) * p.H + hh) * (int64_t)S * p.dv + col0;
            load_initial_state<S, NP>(p, bank, hh, col0, active, state_off, N);
            int64_t base = start;
            bool ok = true;
            while (base < end) {
                const int b = ring_slot(it);
                if (!mbar_wait(&sh.full[b], use_parity(it), wait_ns)) {
                    ok = false;
                    break;
                }
                const int n = sh.n[b];
                const unsigned wmask = sh.wmask[b], rmask = sh.rmask[b];
                const float2(*ctl)[Ctl::size] = sh.ctl[b];
                // Every event runs the same straight-line code (reads have zero k/D rows
                // and a zeroed update), so consecutive events pipeline.
                for (int ev = 0; ev < n; ++ev) {
                    if ((rmask >> ev) & 1u) {  // storage point: materialise, round to BF16
#pragma unroll
                        for (int s = 0; s < S; ++s) {
                            const float2 d2 = ctl[ev][Ctl::dprev + s];
#pragma unroll
                            for (int c = 0; c < NP; ++c) N[s][c] = bf16_round_pair(__fmul2_rn(N[s][c], d2));
                        }
                    }
                    const bool wr_ev = (wmask >> ev) & 1u;
                    const float4 *crow = reinterpret_cast<const float4 *>(ctl[ev] + Ctl::c);
                    const float4 *krow = reinterpret_cast<const float4 *>(ctl[ev] + Ctl::kd);
                    const Row<T, NC> vr = *reinterpret_cast<const Row<T, NC> *>(slot_values(b, ev, ct, 0) + lane * NC);
                    const Row<T, NC> wr = *reinterpret_cast<const Row<T, NC> *>(slot_values(b, ev, ct, 1) + lane * NC);
                    // same chains and summation order as event_step (a sequence gives the
                    // same bits whichever kernel runs it)
                    constexpr int NCH = NP >= 2 ? 2 : 4;
                    float2 dot[NP][NCH];
#pragma unroll
                    for (int c = 0; c < NP; ++c)
#pragma unroll
                        for (int i = 0; i < NCH; ++i) dot[c][i] = make_float2(0.f, 0.f);
#pragma unroll
                    for (int s = 0; s < S; s += 2) {
                        const float4 cc = crow[s / 2];
                        const int i = (s / 2) % NCH;
#pragma unroll
                        for (int c = 0; c < NP; ++c) {
                            dot[c][i] = __ffma2_rn(make_float2(cc.x, cc.y), N[s][c], dot[c][i]);
                            dot[c][(i + NCH / 2) % NCH] =
                                __ffma2_rn(make_float2(cc.z, cc.w), N[s + 1][c], dot[c][(i + NCH / 2) % NCH]);
                        }
                    }
                    const float2 pw = ctl[ev][Ctl::p];
                    float2 u[NP];
#pragma unroll
                    for (int c = 0; c < NP; ++c) {
#pragma unroll
                        for (int i = 1; i < NCH; ++i) dot[c][0] = __fadd2_rn(dot[c][0], dot[c][i]);
                        const float2 d = dot[c][0];
                        const float2 uw = WriteValue<T>::apply(wr.x + 2 * c, vr.x + 2 * c, pw, make_float2(-d.x, -d.y));
                        u[c] = wr_ev ? uw : make_float2(0.f, 0.f);
                    }
#pragma unroll
                    for (int s = 0; s < S; s += 2) {
                        const float4 kk = krow[s / 2];
#pragma unroll
                        for (int c = 0; c < NP; ++c) {
                            N[s][c] = __ffma2_rn(make_float2(kk.x, kk.y), u[c], N[s][c]);
                            N[s + 1][c] = __ffma2_rn(make_float2(kk.z, kk.w), u[c], N[s + 1][c]);
                        }
                    }
                    if (!wr_ev && sh.tok[b][ev] >= 0 && active) {
                        Row<T, NC> o;
#pragma unroll
                        for (int c = 0; c < NP; ++c) store_pair<T>(o.x + 2 * c, __fmul2_rn(dot[c][0], dup(p.scale)));
                        store_row<T, NC>(outp + (int64_t)sh.rid[b][ev] * V, o);
                    }
                }
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    const float2 d2 = sh.dend[b][s];
#pragma unroll
                    for (int c = 0; c < NP; ++c) N[s][c] = __fmul2_rn(N[s][c], d2);
                }
                __syncwarp();
                mbar_arrive(&sh.empty[b]);
                base += n;
                ++it;
            }
            if (!ok) fail();
            if (ok && p.store_final && p.cache && active) {
#pragma unroll
                for (int s = 0; s < S; ++s)
#pragma unroll
                    for (int j = 0; j < NP; ++j) {
                        const int64_t o = state_off + (int64_t)s * p.dv + 2 * j;
                        if (p.cache_dtype == BDM_BF16) store_pair<bf16>(static_cast<bf16 *>(p.cache) + o, N[s][j]);
                        else store_pair<float>(static_cast<float *>(p.cache) + o, N[s][j]);
                    }
            }
        }
    }
}

template <typename T, int S, int NC>
__global__ void __launch_bounds__(kScanWarps * 32, BDM_SCAN_MIN_BLOCKS)
bank_scan_long_kernel(const ScanParams p) {
    // The short-sequence kernel is this kernel's programmatic dependent: it may
    // start once every CTA here has started, i.e. after the long chains hold
    // their SM slots.  It reads nothing this kernel writes.
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    extern __shared__ __align__(16) unsigned char scan_smem[];
    scan_long_units<T, S, NC>(p, scan_smem);
}

// Work list: every non-empty sequence goes to the list of its length class, in
// ascending sequence order (one CTA: per-thread contiguous chunks + block scans).
constexpr int kListThreads = 1024;
constexpr int kMaxSortedLong = 4096;  // long sequences sorted by length (more stay in sequence order)

__device__ __forceinline__ int len_class(const int64_t *cu, int64_t s, int64_t E, int64_t long_min) {
    const int64_t a = min(max(cu[s], (int64_t)0), E), b = min(max(cu[s + 1], a), E);
    const int64_t len = b - a;
    if (len <= 0) return -1;
    if (len >= long_min) return 0;
    int c = 1;
    while (c < kLenClasses - 1 && len < kLenLower[c]) ++c;
    return c;
}

__global__ void __launch_bounds__(kListThreads)
build_worklist(const int64_t *__restrict__ cu, int64_t nseq, int64_t E, int64_t unit_factor, int64_t slots,
               int *__restrict__ lists,
               int *__restrict__ counts) {
    // long-sequence bound of this launch: the (event, head, tile) work of the
    // events it runs (cu[nseq]; fewer than E on a bank-sharded rank) over the
    // GPU's warp slots, and at least kLongEvents; unit_factor 0 disables it
    const int64_t ran = min(max(cu[nseq], (int64_t)0), E);
    const int64_t long_min = unit_factor > 0 ? max(kLongEvents, ran * unit_factor / slots) : ((int64_t)1 << 62);
    __shared__ int warp_tot[kLenClasses][32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t chunk = (nseq + kListThreads - 1) / kListThreads;
    const int64_t lo = min((int64_t)tid * chunk, nseq), hi = min(lo + chunk, nseq);
    int cnt[kLenClasses] = {0, 0, 0, 0};
    for (int64_t s = lo; s < hi; ++s) {
        const int c = len_class(cu, s, E, long_min);
        if (c >= 0) ++cnt[c];
    }
    int off[kLenClasses];
#pragma unroll
    for (int c = 0; c < kLenClasses; ++c) {  // exclusive scan of cnt[c] over threads
        int x = cnt[c];
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, d);
            if (lane >= d) x += y;
        }
        if (lane == 31) warp_tot[c][warp] = x;
        off[c] = x - cnt[c];
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int c = 0; c < kLenClasses; ++c) {
            const int t = warp_tot[c][lane];
            int x = t;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, d);
                if (lane >= d) x += y;
            }
            warp_tot[c][lane] = x - t;
            if (lane == 31) counts[c] = x;
        }
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < kLenClasses; ++c) off[c] += warp_tot[c][warp];
    for (int64_t s = lo; s < hi; ++s) {
        const int c = len_class(cu, s, E, long_min);
        if (c >= 0) lists[(int64_t)c * nseq + off[c]++] = (int)s;
    }
    // Long sequences longest first (bitonic sort of (length desc, sequence asc)),
    // so the long kernel's CTAs take them in LPT order.
    __shared__ unsigned long long keys[kMaxSortedLong];
    __syncthreads();
    const int nlong = counts[0];
    if (nlong > 1 && nlong <= kMaxSortedLong) {
        int n2 = 1;
        while (n2 < nlong) n2 <<= 1;
        for (int i = tid; i < n2; i += kListThreads) {
            unsigned long long key = ~0ull;
            if (i < nlong) {
                const int sq = lists[i];
                const int64_t a = min(max(cu[sq], (int64_t)0), E), b = min(max(cu[sq + 1], a), E);
                key = ((unsigned long long)(0xffffffffu - (unsigned)min(b - a, (int64_t)0xffffffff)) << 32) |
                      (unsigned)sq;
            }
            keys[i] = key;
        }
        __syncthreads();
        for (int k = 2; k <= n2; k <<= 1) {
            for (int j = k >> 1; j > 0; j >>= 1) {
                for (int i = tid; i < n2; i += kListThreads) {
                    const int ixj = i ^ j;
                    if (ixj > i) {
                        const unsigned long long x = keys[i], y = keys[ixj];
                        if ((x > y) == ((i & k) == 0)) {
                            keys[i] = y;
                            keys[ixj] = x;
                        }
                    }
                }
                __syncthreads();
            }
        }
        for (int i = tid; i < nlong; i += kListThreads) lists[i] = (int)(keys[i] & 0xffffffffu);
    }
}

template <typename T, int S, int NC>
int launch_scan(const ScanParams &p, cudaStream_t st) {
    ScanParams q = p;
    q.ctiles = (int)ceil_div(p.dv, 32 * NC);
    q.units = p.batch * p.J * p.H * q.ctiles;
    if (q.units == 0) return BDM_OK;
    int dev = 0, sms = kNumSMs;
    int rc = cuda_status(cudaGetDevice(&dev));
    if (rc) return rc;
    rc = cuda_status(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if (rc) return rc;
    // A sequence is long when its serial chain would outlast its share of the
    // launch: more events than the launch's (event, head, tile) work over the
    // GPU's warp slots (and at least kLongEvents; decided on the device, which
    // knows how many events the launch runs).  Long sequences run on
    // warp-specialised CTAs in their own kernel, started first; with a long
    // launch (plenty of work to hide a chain) there are none.
    const bool long_mode = BDM_SCAN_LONG && q.ctiles <= kWsMaxTiles;
    build_worklist<<<1, kListThreads, 0, st>>>(p.cu, p.nseq, p.E, long_mode ? (int64_t)p.H * q.ctiles : 0,
                                               (int64_t)sms * 32, const_cast<int *>(p.lists),
                                               const_cast<int *>(p.counts));
    rc = launch_status();
    if (rc) return rc;
    q.ws_classes = long_mode ? kWsClasses : 0;
    if (long_mode) {
        // Long units first: at most BDM_SCAN_LONG_CTAS_PER_SM persistent CTAs per SM
        // (the rest of each SM stays free for short CTAs from the start).
        q.ws_ctas = min(ceil_div(p.E, kLongEvents) * p.H, (int64_t)sms * BDM_SCAN_LONG_CTAS_PER_SM);
        const size_t smem = (size_t)(ws_fixed_bytes<T, S>() + ws_value_bytes<T, S, NC>(q.ctiles));
        auto lk = bank_scan_long_kernel<T, S, NC>;
        rc = cuda_status(cudaFuncSetAttribute(lk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        if (rc) return rc;
        lk<<<(unsigned)q.ws_ctas, 32 * (1 + q.ctiles), smem, st>>>(q);
        rc = launch_status();
        if (rc) return rc;
    }
    // bdm_bank_scan_chunked: the remaining classes on the tensor-core chunked kernel
    // (chunk_scan.cu), as the long kernel's programmatic dependent.
    if (q.chunked) return launch_chunk_scan(q, S, st, long_mode);
    // Even head counts run two heads per warp (twice the columns per lane): BF16 with at most 8
    // columns per lane (the doubled state and value rows fit the registers of 3 CTAs per SM, the
    // staging arrays the 48 KB of static shared memory), heads split into whole column tiles.
    constexpr bool kG2Fits = sizeof(T) == 2 && NC <= 4 && S * NC <= 32;
    constexpr int NC2 = kG2Fits ? 2 * NC : NC, G2 = kG2Fits ? 2 : 1;
    const bool g2 = BDM_SCAN_G2 && kG2Fits && p.H % 2 == 0 && p.dv % (32 * NC) == 0;
    int per_sm = 1;
    void (*sk)(const ScanParams) = p.ckpt ? bank_scan_kernel<T, S, NC, true, 1> : bank_scan_kernel<T, S, NC, false, 1>;
    if (g2) sk = p.ckpt ? bank_scan_kernel<T, S, NC2, true, G2> : bank_scan_kernel<T, S, NC2, false, G2>;
    rc = cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sk, kScanWarps * 32, 0));
    if (rc) return rc;
    const int64_t want = ceil_div(q.units / (g2 ? 2 : 1), kScanWarps);
    const int64_t blocks = BDM_SCAN_DYNAMIC ? min((int64_t)sms * (per_sm > 0 ? per_sm : 1), want)
                                            : min(want, (int64_t)0x7fffffff);
    // With long units the short kernel is a programmatic dependent launch of the
    // long kernel (starts once the long CTAs are resident; work after it in the
    // stream still waits for both).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(kScanWarps * 32);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = long_mode ? 1 : 0;
    rc = cuda_status(cudaLaunchKernelEx(&cfg, sk, q));
    count_launch();
    return rc;
}

template <typename T>
int launch_scan_shape(const ScanParams &p, int S, cudaStream_t st) {
    const bool narrow = p.dv < 128;
    switch (S) {
        case 4: return narrow ? launch_scan<T, 4, 2>(p, st) : launch_scan<T, 4, 8>(p, st);
        case 8: return narrow ? launch_scan<T, 8, 2>(p, st) : launch_scan<T, 8, 4>(p, st);
        case 16: return launch_scan<T, 16, 2>(p, st);
        default: return BDM_ERR_UNSUPPORTED;
    }
}

}  // namespace
}  // namespace bdm

namespace bdm {
namespace {
// Diagnostics set by bdm_scan_test_fault (process-wide; off unless a test turns them on).
std::atomic<unsigned long long> g_scan_wait_ns{0};
std::atomic<int> g_scan_test_fault{0};
// Workspace: 256-byte header [counts (kLenClasses int32) at 0 | dynamic counters (uint64) at 64
// (short kernel), 72 (long kernel) and 80 (chunked kernel) | status word (int32, BDM_SCAN_ERR_* bits) at 128], then the lists.
constexpr int64_t kWsHeader = 256;
inline int64_t scan_workspace_bytes(int64_t nseq) { return kWsHeader + (int64_t)kLenClasses * nseq * 4; }
}  // namespace
}  // namespace bdm

extern "C" int64_t bdm_bank_scan_workspace_bytes(int64_t batch, int64_t bank_count) {
    if (batch <= 0 || bank_count <= 0) return -1;
    return bdm::scan_workspace_bytes(batch * bank_count);
}

namespace {
int bank_scan_impl(bool chunked, const void *q, const void *k, const void *v, const float *g, const void *b, const void *w,
                             const int64_t *write_idx, const void *write_w, const int64_t *read_idx,
                             const void *read_w, const int64_t *order, const int64_t *cu_seqlens, int64_t batch,
                             int64_t time, int64_t bank_count, int heads, int bank_size, int head_value_width, int kw,
                             int kr, int dtype, int routed_decay, float scale, const void *row_factor,
                             const void *col_factor, int64_t factor_cols, int factor_dtype,
                             const int32_t *bank_ids, int64_t total_banks, int head_offset, int total_heads,
                             void *cache, int cache_dtype,
                             int store_final, int state_interval, void *reads, void *workspace,
                             int64_t workspace_bytes, float *checkpoints, int checkpoint_block, void *stream) {
    using namespace bdm;
    if (batch <= 0 || time <= 0 || bank_count <= 0 || heads <= 0 || head_value_width <= 0 || kw <= 0 || kr <= 0)
        return BDM_ERR_INVALID;
    if (!q || !k || !v || !g || !b || !w || !write_idx || !write_w || !read_idx || !read_w || !order || !cu_seqlens ||
        !reads)
        return BDM_ERR_INVALID;
    if (bank_size != 4 && bank_size != 8 && bank_size != 16) return BDM_ERR_UNSUPPORTED;
    if (head_value_width % 8) return BDM_ERR_UNSUPPORTED;
    if (state_interval < 0 || (store_final && !cache)) return BDM_ERR_INVALID;
    if (!valid_dtype(dtype) || (cache && !valid_dtype(cache_dtype))) return BDM_ERR_DTYPE;
    if (batch * time * (int64_t)(kw + kr) >= ((int64_t)1 << 31)) return BDM_ERR_UNSUPPORTED;
    if (batch * bank_count >= ((int64_t)1 << 31)) return BDM_ERR_UNSUPPORTED;
    if (bank_ids && total_banks < bank_count) return BDM_ERR_INVALID;
    if (total_heads == 0) total_heads = heads;
    if (head_offset < 0 || head_offset + heads > total_heads || (cache && total_heads != heads))
        return BDM_ERR_INVALID;
    const int64_t table_banks = bank_ids ? total_banks : bank_count;
    if (!cache && row_factor) {
        if (!col_factor || factor_cols <= 0 || !valid_dtype(factor_dtype)) return BDM_ERR_INVALID;
        if ((table_banks * total_heads * bank_size) % factor_cols) return BDM_ERR_INVALID;
    }
    const int64_t nseq = batch * bank_count;
    if (!workspace || workspace_bytes < scan_workspace_bytes(nseq)) return BDM_ERR_WORKSPACE;
    if (checkpoints && (checkpoint_block <= 0 || cache || bank_ids || head_offset != 0 || total_heads != heads))
        return BDM_ERR_INVALID;
    ScanParams p{};
    p.q = q; p.k = k; p.v = v; p.g = g; p.b = b; p.w = w;
    p.wi = write_idx; p.ri = read_idx; p.ww = write_w; p.rw = read_w;
    p.order = order; p.cu = cu_seqlens;
    p.batch = batch; p.time = time; p.J = bank_count; p.nt = batch * time; p.nw = p.nt * kw;
    p.E = p.nt * (kw + kr);
    p.H = heads; p.dv = head_value_width; p.kw = kw; p.kr = kr; p.routed_decay = routed_decay;
    p.scale = scale;
    p.row_factor = cache ? nullptr : row_factor;
    p.col_factor = cache ? nullptr : col_factor;
    p.factor_cols = factor_cols; p.factor_dtype = factor_dtype;
    p.bank_ids = bank_ids; p.total_banks = table_banks;
    p.head_offset = head_offset; p.total_heads = total_heads;
    p.cache = cache; p.cache_dtype = cache_dtype; p.store_final = store_final; p.interval = state_interval;
    p.reads = reads;
    p.ckpt = checkpoints;
    p.ckpt_block = checkpoints ? checkpoint_block : 0;
    p.chunked = chunked ? 1 : 0;
    p.wait_ns = g_scan_wait_ns.load(std::memory_order_relaxed);
    p.test_fault = g_scan_test_fault.load(std::memory_order_relaxed);
    if (chunked && !chunk_scan_eligible(p, dtype, bank_size)) return BDM_ERR_UNSUPPORTED;
    char *ws = static_cast<char *>(workspace);
    int *counts = reinterpret_cast<int *>(ws);
    int *lists = reinterpret_cast<int *>(ws + kWsHeader);
    p.counts = counts;
    p.next = reinterpret_cast<unsigned long long *>(ws + 64);
    p.status = reinterpret_cast<int *>(ws + 128);
    p.long_next = reinterpret_cast<unsigned long long *>(ws + 72);
    p.chunk_next = reinterpret_cast<unsigned long long *>(ws + 80);
    p.lists = lists;
    p.nseq = nseq;
    cudaStream_t st = as_stream(stream);
    int rc = cuda_status(cudaMemsetAsync(workspace, 0, kWsHeader, st));
    if (rc) return rc;
    BDM_DISPATCH_DTYPE(dtype, T, { return launch_scan_shape<T>(p, bank_size, st); });
    return BDM_OK;
}
}  // namespace

#define BDM_SCAN_ARGS                                                                                                  \
    const void *q, const void *k, const void *v, const float *g, const void *b, const void *w,                         \
        const int64_t *write_idx, const void *write_w, const int64_t *read_idx, const void *read_w,                    \
        const int64_t *order, const int64_t *cu_seqlens, int64_t batch, int64_t time, int64_t bank_count, int heads,   \
        int bank_size, int head_value_width, int kw, int kr, int dtype, int routed_decay, float scale,                 \
        const void *row_factor, const void *col_factor, int64_t factor_cols, int factor_dtype,                         \
        const int32_t *bank_ids, int64_t total_banks, int head_offset, int total_heads, void *cache, int cache_dtype,  \
        int store_final, int state_interval, void *reads, void *workspace, int64_t workspace_bytes,                    \
        float *checkpoints, int checkpoint_block, void *stream
#define BDM_SCAN_PASS                                                                                                  \
    q, k, v, g, b, w, write_idx, write_w, read_idx, read_w, order, cu_seqlens, batch, time, bank_count, heads,         \
        bank_size, head_value_width, kw, kr, dtype, routed_decay, scale, row_factor, col_factor, factor_cols,          \
        factor_dtype, bank_ids, total_banks, head_offset, total_heads, cache, cache_dtype, store_final,                \
        state_interval, reads, workspace, workspace_bytes, checkpoints, checkpoint_block, stream

extern "C" int bdm_bank_scan(BDM_SCAN_ARGS) { return bank_scan_impl(false, BDM_SCAN_PASS); }
extern "C" int bdm_bank_scan_chunked(BDM_SCAN_ARGS) { return bank_scan_impl(true, BDM_SCAN_PASS); }

extern "C" int bdm_scan_test_fault(int fault, unsigned long long wait_ns) {
    if (fault != 0 && fault != 1) return BDM_ERR_INVALID;
    bdm::g_scan_test_fault.store(fault, std::memory_order_relaxed);
    bdm::g_scan_wait_ns.store(wait_ns, std::memory_order_relaxed);
    return BDM_OK;
}
