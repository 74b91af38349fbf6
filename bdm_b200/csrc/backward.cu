// Training backward of the BDM bank path.
//
// Restates the reference's training derivatives:
//   recurrence      role_bank_kernel.py:76-150 (_role_backward: checkpoint replay, then the
//                   reverse per-event chain), routed_update.py:31-49 (decay_transform's dp term)
//   event VJP       role_bank_dispatch.py:76-132 (_vjp: per-token gather of the event
//                   gradients, rounded to the parameter dtype where the reference stores them)
//   initial state   product_routed_update.py:51-76 (factor gradients = sums of the state gradient)
//   router          autograd of product_key_route (gdn2_banks.py:74-114)
//   controllers     autograd of _controllers (_parameters.py:189-220, heads.py:11-22)
//   output          autograd of _project_bank_output (_parameters.py:222-232)
//
// Recurrence backward, per event of one (sequence, head) on one state column x
// (h0 = state before the event, dh = adjoint of the state after it):
//   write:  hd = h0*e (e = exp(g_e)), u = w_e*v - sum_s a_s hd_s (a = b_e*k),
//           du = sum_s dh_s k_s,  c_s = hd_s du,  A_s = dh_s u,  dh'_s = dh_s - a_s du,
//           G_s = dh'_s hd_s,  dh <- dh' * e
//   read:   o_s = h0_s do (do = output gradient of the read's token), dh += scale * q_e do
// The per-event S-vectors A, c, G (write) and o (read) are sums over the columns;
// dk_e = A - b_e c, db_e = -k c, dg_e = G, dq_e = scale * o follow in the VJP.
//
// One warp per (sequence, head, tile of 32 or 64 columns), one or two columns per
// lane, so a column's S rows stay in registers.  A first forward sweep writes the
// state to HBM every kBlock events; the reverse sweep takes the blocks last to
// first: it replays a block from its checkpoint into a lane-private shared-memory
// history of the state before each event, then walks the block backwards.  Each
// pass over a block first stages the block's event controls in shared memory (all
// of the block's loads in flight at once), so replay and reverse read only shared
// memory, and the loops stay rolled (compact code, no instruction-cache misses).
#include <type_traits>
#include "common.cuh"
#include "scan.cuh"

namespace bdm {
namespace {

constexpr unsigned kFull = 0xffffffffu;

// ------------------------------------------------------------ warp reductions

// Sums N per-lane values across the warp.  While the live count is even, a butterfly
// level halves it: a lane keeps one half of its live values (the upper half on lanes
// whose OFF bit is set) and adds the partner's copy of that half.  Once it is odd, the
// remaining levels add the partner's copy of every live value.  Every value is summed
// over the same tree (lane bits 16, 8, 4, 2, 1 in that order) whatever N is, so padding
// N to a power of two would change only the cost.  Independent adds run as FP32x2 pairs.
constexpr int reduce_live(int live, int off) { return (off >= 1 && live % 2 == 0) ? reduce_live(live / 2, off / 2) : live; }
constexpr unsigned reduce_bfly(int live, int off) {
    return off < 1 ? 0u : (live % 2 == 0 ? reduce_bfly(live / 2, off / 2) : (unsigned)(2 * off - 1));
}

template <int H, int N>
__device__ __forceinline__ void add_pairs(float (&v)[N], const float (&a)[H], const float (&b)[H]) {
#pragma unroll
    for (int i = 0; i + 1 < H; i += 2) {
        const float2 r = __fadd2_rn(make_float2(a[i], a[i + 1]), make_float2(b[i], b[i + 1]));
        v[i] = r.x;
        v[i + 1] = r.y;
    }
    if constexpr (H % 2 == 1) v[H - 1] = a[H - 1] + b[H - 1];
}

template <int LIVE, int OFF, int N> struct SplitReduce {
    static __device__ __forceinline__ void run(float (&v)[N], unsigned lane, int &base) {
        if constexpr (OFF >= 1) {
            if constexpr (LIVE % 2 == 0) {
                constexpr int H = LIVE / 2;
                const bool up = (lane & OFF) != 0;
                float keep[H], recv[H];
#pragma unroll
                for (int i = 0; i < H; ++i) {
                    const float send = up ? v[i] : v[i + H];
                    keep[i] = up ? v[i + H] : v[i];
                    recv[i] = __shfl_xor_sync(kFull, send, OFF);
                }
                add_pairs<H, N>(v, keep, recv);
                if (up) base += H;
                SplitReduce<H, OFF / 2, N>::run(v, lane, base);
            } else {
                float own[LIVE], recv[LIVE];
#pragma unroll
                for (int i = 0; i < LIVE; ++i) {
                    own[i] = v[i];
                    recv[i] = __shfl_xor_sync(kFull, v[i], OFF);
                }
                add_pairs<LIVE, N>(v, own, recv);
                SplitReduce<LIVE, OFF / 2, N>::run(v, lane, base);
            }
        }
    }
};

// Sums the N per-lane values across the warp and stores the N totals to out[0..N).
template <int N>
__device__ __forceinline__ void reduce_store(float (&v)[N], float *out) {
    constexpr int kLive = reduce_live(N, 16);
    constexpr unsigned kBfly = reduce_bfly(N, 16);
    const unsigned lane = lane_id();
    int base = 0;
    SplitReduce<N, 16, N>::run(v, lane, base);
    if constexpr (kBfly + 1 >= kLive) {  // the lanes holding one window store one total each
        const int q = (int)(lane & kBfly);
        float x = v[0];
#pragma unroll
        for (int i = 1; i < kLive; ++i) x = q == i ? v[i] : x;
        if (q < kLive) out[base + q] = x;
    } else if ((lane & kBfly) == 0) {
#pragma unroll
        for (int i = 0; i < kLive; ++i) out[base + i] = v[i];
    }
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(kFull, x, o));
    return x;
}

// ------------------------------------------------------- recurrence backward

struct ScanBwdParams {
    const void *q, *k, *v;
    const float *g;
    const void *b, *w, *ww, *rw;
    const int64_t *order, *cu;
    int64_t nseq, J, nt, nw, E, units;
    int H, dv, kw, kr, routed_decay, interval, tiles;
    float scale;
    const void *row_factor, *col_factor;
    int64_t factor_cols;
    int factor_dtype;
    const void *dread;  // [nt, H*dv] gradient of the combined read output (activation dtype)
    float *ckpt;        // [slots, H, S, dv] states at block starts
    float *evg;         // [tiles, E, H, 3S] per-(event, head) column sums (A | c | G; o for reads)
    float *du;          // [nt*kw, H*dv] write-event du per column
    float *dinit;       // [nseq, H, S, dv] gradient of each sequence's initial state
    int ckpt_ready;     // the forward recurrence wrote the block checkpoints (sequences < kLongSeq events)
};

// Sequences the forward may run on its long-sequence kernel, which writes no checkpoints: the
// forward's long bound is at least kLongEvents, so every shorter sequence has them.
constexpr int64_t kLongSeq = kLongEvents;

template <int S, int COLS> struct BwdGeom {
    static constexpr int kBlock = 128 / (S * COLS);  // events between HBM checkpoints (16 KB of history)
    static constexpr int kRec = 3 * S;               // floats per (event, head) record
    static constexpr int kTileCols = 32 * COLS;      // value columns per warp (lane l: l, l+32, ...)
};

// One block of events staged in shared memory by the warp that owns the unit:
// lane-uniform rows [k | a | e] per event (a = dtype(b*p)*k, e = exp(g_e); a read
// keeps q_e = dtype(q*r) in the k slot), the lane's column values per event
// (write: dtype(w*p)*v; read: the output gradient), the event ids, and the
// lane-private history of the states before each event of the block.  States are
// held as (s, s+1) pairs: every per-row operation of the recurrence and of its
// reverse runs along s, so one packed FP32x2 instruction does two rows with the
// same per-component rounding as the scalar instruction.
template <int S, int COLS> struct BlockStage {
    using G = BwdGeom<S, COLS>;
    float2 hist[G::kBlock][S / 2][COLS][32];
    alignas(16) float uni[G::kBlock][3 * S];
    float col[G::kBlock][COLS][32];
    int id[G::kBlock];  // event ids < 2^31 (checked on the host)
    int tok[G::kBlock];
};

__device__ __forceinline__ float2 pair(float x) { return make_float2(x, x); }
__device__ __forceinline__ float2 upair(const float *u, int s) { return *reinterpret_cast<const float2 *>(u + s); }

template <typename T, int S, int COLS>
__device__ __forceinline__ void stage_block(const ScanBwdParams &p, BlockStage<S, COLS> &st, int64_t pos0, int n,
                                            int h, int col0, bool want_dout) {
    const unsigned lane = lane_id();
    const int64_t V = (int64_t)p.H * p.dv;
    __syncwarp();
    for (int i = (int)lane; i < n; i += 32) {  // lanes over events: ids and the lane-uniform rows
        const int64_t id = __ldg(p.order + pos0 + i);
        st.id[i] = (int)id;
        float *u = st.uni[i];
        if (id < p.nw) {
            const int64_t tok = (uint32_t)id / (uint32_t)p.kw;  // event ids < 2^31 (checked on the host)
            st.tok[i] = (int)tok;
            const float pw = ld_f(static_cast<const T *>(p.ww), id);
            const int64_t base = (tok * p.H + h) * S;
#pragma unroll
            for (int s = 0; s < S; ++s) {
                const float kk = ld_f(static_cast<const T *>(p.k), base + s);
                const float gg = p.g[base + s];
                u[s] = kk;
                u[S + s] = rnd<T>(ld_f(static_cast<const T *>(p.b), base + s) * pw) * kk;
                u[2 * S + s] = expf(p.routed_decay ? gg * pw : gg);
            }
        } else if (want_dout) {  // reads matter only to the reverse pass
            const int64_t rid = id - p.nw;
            const int rtok = (int)((uint32_t)rid / (uint32_t)p.kr);
            st.tok[i] = rtok;
            const int64_t base = ((int64_t)rtok * p.H + h) * S;
            const float r = ld_f(static_cast<const T *>(p.rw), rid);
#pragma unroll
            for (int s = 0; s < S; ++s) u[s] = rnd<T>(ld_f(static_cast<const T *>(p.q), base + s) * r);
        }
    }
    __syncwarp();
    const int64_t hc = (int64_t)h * p.dv + col0;  // the lane's first column within a token row
    const T *wl = static_cast<const T *>(p.w) + hc, *vl = static_cast<const T *>(p.v) + hc;
    const T *dl = static_cast<const T *>(p.dread) + hc;
    const int nw = (int)p.nw;
#pragma unroll 4
    for (int i = 0; i < n; ++i) {  // every lane over the events: its own columns
        const int id = st.id[i];
        const bool wr = id < nw;
        if (!wr && !want_dout) continue;
        const uint64_t row = (uint64_t)(uint32_t)st.tok[i] * (uint32_t)V;
        const float pw = wr ? ld_f(static_cast<const T *>(p.ww), id) : 0.f;
#pragma unroll
        for (int c = 0; c < COLS; ++c) {
            float val = 0.f;
            if (col0 + 32 * c < p.dv) {
                const uint64_t o = row + 32 * c;
                if (wr)
                    val = rnd<T>(ld_f(wl, o) * pw) * ld_f(vl, o);
                else if (want_dout)
                    val = ld_f(dl, o);
            }
            st.col[i][c][lane] = val;
        }
    }
    __syncwarp();
}

// Replays events [0, n) of the staged block from hs.  With `save` the state before each
// event (after its storage rounding) goes to the block history; `rpos` = position of
// event 0 modulo the storage interval.  hs[sp][c] = (state[2sp][c], state[2sp+1][c]);
// the even / odd halves of the a.h sum are the two components of er[c].
template <int S, int COLS>
__device__ __forceinline__ void replay_block(const ScanBwdParams &p, BlockStage<S, COLS> &st, int n, int rpos,
                                             bool save, float2 (&hs)[S / 2][COLS]) {
    const unsigned lane = lane_id();
#pragma unroll 1
    for (int i = 0; i < n; ++i) {
        if (p.interval > 0) {
            if (rpos == 0) {
#pragma unroll
                for (int sp = 0; sp < S / 2; ++sp)
#pragma unroll
                    for (int c = 0; c < COLS; ++c)
                        hs[sp][c] = make_float2(bf16_round(hs[sp][c].x), bf16_round(hs[sp][c].y));
            }
            rpos = rpos + 1 == p.interval ? 0 : rpos + 1;
        }
        if (save) {
#pragma unroll
            for (int sp = 0; sp < S / 2; ++sp)
#pragma unroll
                for (int c = 0; c < COLS; ++c) st.hist[i][sp][c][lane] = hs[sp][c];
        }
        if (st.id[i] >= (int)p.nw) continue;  // reads leave the state unchanged
        const float *u = st.uni[i];
        float2 er[COLS];
#pragma unroll
        for (int c = 0; c < COLS; ++c) er[c] = make_float2(0.f, 0.f);
#pragma unroll
        for (int sp = 0; sp < S / 2; ++sp) {
            const float2 e = upair(u, 2 * S + 2 * sp), a = upair(u, S + 2 * sp);
#pragma unroll
            for (int c = 0; c < COLS; ++c) {
                hs[sp][c] = __fmul2_rn(hs[sp][c], e);
                er[c] = __ffma2_rn(a, hs[sp][c], er[c]);
            }
        }
#pragma unroll
        for (int c = 0; c < COLS; ++c) {
            const float2 uu = pair(st.col[i][c][lane] - (er[c].x + er[c].y));
#pragma unroll
            for (int sp = 0; sp < S / 2; ++sp) hs[sp][c] = __ffma2_rn(upair(u, 2 * sp), uu, hs[sp][c]);
        }
    }
}

// Initial state of the lane's columns: product-key factors (rounded to their dtype), or
// zero; rounded to BF16 under the training storage policy.
template <int S, int COLS>
__device__ __forceinline__ void initial_columns(const ScanBwdParams &p, int64_t seq, int h, int col0,
                                                float2 (&hs)[S / 2][COLS]) {
    const int64_t bank = seq % p.J;
#pragma unroll
    for (int s = 0; s < S; ++s) {
        const int64_t r = (bank * p.H + h) * S + s;
#pragma unroll
        for (int c = 0; c < COLS; ++c) {
            const int cc = col0 + 32 * c;
            float x = 0.f;
            if (cc < p.dv && p.row_factor) {
                const int64_t ou = (r / p.factor_cols) * p.dv + cc, oz = (r % p.factor_cols) * p.dv + cc;
                if (p.factor_dtype == BDM_BF16)
                    x = bf16_round(ld_f(static_cast<const bf16 *>(p.row_factor), ou) +
                                   ld_f(static_cast<const bf16 *>(p.col_factor), oz));
                else
                    x = static_cast<const float *>(p.row_factor)[ou] + static_cast<const float *>(p.col_factor)[oz];
                if (p.interval > 0) x = bf16_round(x);
            }
            if (s & 1) hs[s / 2][c].y = x;
            else hs[s / 2][c].x = x;
        }
    }
}

// Reverse pass over events [0, n) of the staged block (descending), from the history.
template <int S, int COLS>
__device__ __forceinline__ void reverse_block(const ScanBwdParams &p, const BlockStage<S, COLS> &st, int n, int tile,
                                              int h, int col0, float2 (&dh)[S / 2][COLS]) {
    using G = BwdGeom<S, COLS>;
    constexpr int P = S / 2;
    const unsigned lane = lane_id();
    float *const rec0 = p.evg + ((int64_t)tile * p.E * p.H + h) * G::kRec;  // record of event 0
    const uint32_t rec_stride = (uint32_t)p.H * G::kRec;
    const uint32_t V = (uint32_t)p.H * (uint32_t)p.dv;
    float *const du0 = p.du + (int64_t)h * p.dv + col0;
    const int nw = (int)p.nw;
#pragma unroll 1
    for (int i = n - 1; i >= 0; --i) {
        const int id = st.id[i];
        const float *u = st.uni[i];
        float *rec = rec0 + (uint64_t)(uint32_t)id * rec_stride;
        if (id < nw) {
            float2 hd[P][COLS], er[COLS], du[COLS];
            float uu[COLS], dus[COLS];
#pragma unroll
            for (int c = 0; c < COLS; ++c) er[c] = du[c] = make_float2(0.f, 0.f);
#pragma unroll
            for (int sp = 0; sp < P; ++sp) {
                const float2 e = upair(u, 2 * S + 2 * sp), a = upair(u, S + 2 * sp), k = upair(u, 2 * sp);
#pragma unroll
                for (int c = 0; c < COLS; ++c) {
                    hd[sp][c] = __fmul2_rn(st.hist[i][sp][c][lane], e);
                    er[c] = __ffma2_rn(a, hd[sp][c], er[c]);
                    du[c] = __ffma2_rn(dh[sp][c], k, du[c]);
                }
            }
#pragma unroll
            for (int c = 0; c < COLS; ++c) {
                uu[c] = st.col[i][c][lane] - (er[c].x + er[c].y);
                dus[c] = du[c].x + du[c].y;
            }
            float red[3 * S];
#pragma unroll
            for (int sp = 0; sp < P; ++sp) {
                const float2 e = upair(u, 2 * S + 2 * sp), a = upair(u, S + 2 * sp);
                const float2 na = make_float2(-a.x, -a.y);
                float2 A = make_float2(0.f, 0.f), C = A, Gs = A;
#pragma unroll
                for (int c = 0; c < COLS; ++c) {
                    const float2 ds = pair(dus[c]);
                    A = __ffma2_rn(dh[sp][c], pair(uu[c]), A);
                    C = __ffma2_rn(hd[sp][c], ds, C);
                    const float2 dp = __ffma2_rn(na, ds, dh[sp][c]);
                    Gs = __ffma2_rn(dp, hd[sp][c], Gs);
                    dh[sp][c] = __fmul2_rn(dp, e);
                }
                red[2 * sp] = A.x;
                red[2 * sp + 1] = A.y;
                red[S + 2 * sp] = C.x;
                red[S + 2 * sp + 1] = C.y;
                red[2 * S + 2 * sp] = Gs.x;
                red[2 * S + 2 * sp + 1] = Gs.y;
            }
            float *dur = du0 + (uint64_t)(uint32_t)id * V;
#pragma unroll
            for (int c = 0; c < COLS; ++c)
                if (col0 + 32 * c < p.dv) dur[32 * c] = dus[c];
            reduce_store<3 * S>(red, rec);
        } else {
            float red[S];
            const float2 sc = pair(p.scale);
#pragma unroll
            for (int sp = 0; sp < P; ++sp) {
                const float2 k = upair(u, 2 * sp);
                float2 o = make_float2(0.f, 0.f);
#pragma unroll
                for (int c = 0; c < COLS; ++c) {
                    const float2 cv = pair(st.col[i][c][lane]);
                    o = __ffma2_rn(st.hist[i][sp][c][lane], cv, o);
                    dh[sp][c] = __ffma2_rn(__fmul2_rn(k, cv), sc, dh[sp][c]);
                }
                red[2 * sp] = o.x;
                red[2 * sp + 1] = o.y;
            }
            reduce_store<S>(red, rec);
        }
    }
}

// One warp (one CTA) per (sequence, head, tile of 32*COLS columns).
template <typename T, int S, int COLS>
__global__ void __launch_bounds__(32) scan_backward_kernel(const ScanBwdParams p) {
    using G = BwdGeom<S, COLS>;
    constexpr int P = S / 2;
    __shared__ BlockStage<S, COLS> st;
    const unsigned lane = lane_id();
    const int64_t unit = blockIdx.x;
    if (unit >= p.units) return;
    const int tile = (int)(unit % p.tiles);
    const int h = (int)((unit / p.tiles) % p.H);
    const int64_t seq = unit / ((int64_t)p.tiles * p.H);
    const int col0 = tile * G::kTileCols + (int)lane;
    const int64_t start = p.cu[seq], L = p.cu[seq + 1] - start;
    float2 dh[P][COLS];
#pragma unroll
    for (int sp = 0; sp < P; ++sp)
#pragma unroll
        for (int c = 0; c < COLS; ++c) dh[sp][c] = make_float2(0.f, 0.f);
    const int64_t stride_state = (int64_t)S * p.dv;
    const int interval = p.interval > 0 ? p.interval : 1;
    if (L > 0) {
        const int64_t nblk = (L + G::kBlock - 1) / G::kBlock;
        const int64_t slot0 = start / G::kBlock + seq;  // disjoint slot ranges across sequences
        float2 hs[P][COLS];
        if (nblk > 1 && (!p.ckpt_ready || L >= kLongSeq)) {  // sweep 1: checkpoints at blocks 1 .. nblk-1
            initial_columns<S, COLS>(p, seq, h, col0, hs);
#pragma unroll 1
            for (int64_t m = 0; m + 1 < nblk; ++m) {
                const int64_t e0 = m * G::kBlock;
                stage_block<T, S, COLS>(p, st, start + e0, G::kBlock, h, col0, false);
                replay_block<S, COLS>(p, st, G::kBlock, (int)(e0 % interval), false, hs);
                float *ck = p.ckpt + ((slot0 + m + 1) * p.H + h) * stride_state;
#pragma unroll
                for (int sp = 0; sp < P; ++sp)
#pragma unroll
                    for (int c = 0; c < COLS; ++c)
                        if (col0 + 32 * c < p.dv) {
                            ck[(int64_t)(2 * sp) * p.dv + col0 + 32 * c] = hs[sp][c].x;
                            ck[(int64_t)(2 * sp + 1) * p.dv + col0 + 32 * c] = hs[sp][c].y;
                        }
            }
        }
#pragma unroll 1
        for (int64_t m = nblk - 1; m >= 0; --m) {  // sweep 2: blocks in reverse
            if (m == 0) {
                initial_columns<S, COLS>(p, seq, h, col0, hs);
            } else {
                const float *ck = p.ckpt + ((slot0 + m) * p.H + h) * stride_state;
#pragma unroll
                for (int sp = 0; sp < P; ++sp)
#pragma unroll
                    for (int c = 0; c < COLS; ++c) {
                        const bool on = col0 + 32 * c < p.dv;
                        hs[sp][c] = on ? make_float2(ck[(int64_t)(2 * sp) * p.dv + col0 + 32 * c],
                                                     ck[(int64_t)(2 * sp + 1) * p.dv + col0 + 32 * c])
                                       : make_float2(0.f, 0.f);
                    }
            }
            const int64_t e0 = m * G::kBlock;
            const int blen = (int)min((int64_t)G::kBlock, L - e0);
            stage_block<T, S, COLS>(p, st, start + e0, blen, h, col0, true);
            replay_block<S, COLS>(p, st, blen, (int)(e0 % interval), true, hs);
            reverse_block<S, COLS>(p, st, blen, tile, h, col0, dh);
        }
    }
    float *di = p.dinit + (seq * p.H + h) * stride_state;
#pragma unroll
    for (int sp = 0; sp < P; ++sp)
#pragma unroll
        for (int c = 0; c < COLS; ++c)
            if (col0 + 32 * c < p.dv) {
                di[(int64_t)(2 * sp) * p.dv + col0 + 32 * c] = dh[sp][c].x;
                di[(int64_t)(2 * sp + 1) * p.dv + col0 + 32 * c] = dh[sp][c].y;
            }
}

template <typename T, int S, int COLS>
int launch_scan_backward(const ScanBwdParams &p, cudaStream_t st) {
    if (p.units > 0x7fffffffLL) return BDM_ERR_UNSUPPORTED;
    scan_backward_kernel<T, S, COLS><<<(unsigned)p.units, 32, 0, st>>>(p);
    return launch_status();
}

// Columns per lane: two for heads of 64 or more value columns with S <= 8 (one warp per
// 64-column tile), else one.
int scan_cols(int S, int dv) { return (S <= 8 && dv >= 64) ? 2 : 1; }

int64_t block_events(int S, int dv) {
    if (scan_cols(S, dv) == 2) return S == 4 ? BwdGeom<4, 2>::kBlock : BwdGeom<8, 2>::kBlock;
    return S == 4 ? BwdGeom<4, 1>::kBlock : S == 8 ? BwdGeom<8, 1>::kBlock : BwdGeom<16, 1>::kBlock;
}

int scan_tiles(int S, int dv) { return (int)ceil_div(dv, 32 * scan_cols(S, dv)); }


// ------------------------------------------------------------------ event VJP

struct VjpParams {
    const void *q, *k, *v;
    const float *g;
    const void *b, *w, *ww, *rw;
    const float *evg, *du;
    int64_t nt, nw, E, items;
    int H, dv, kw, kr, routed_decay, tiles;
    float scale;
    void *dq, *dk, *dv_out, *db, *dw_out;
    void *dww_h, *drw_h;  // [nt, H, kw] / [nt, H, kr] per-head route-weight gradients
    float *dg;
};

// Warp total of x when only lanes < W (a power of two, at most 16) can hold non-zero values:
// warp_sum's levels at offsets >= W only add +0 there, which turns -0 into +0 and changes
// nothing else, so one add of +0 and the levels below W give the same value on lane 0.
template <int W> __device__ __forceinline__ float warp_sum_low(float x) {
    x = __fadd_rn(x, 0.f);
#pragma unroll
    for (int o = W / 2; o > 0; o >>= 1) x += __shfl_xor_sync(kFull, x, o);
    return x;
}

constexpr int kVjpWarps = 4;
#ifndef BDM_VJP_BATCH
#define BDM_VJP_BATCH 4  // slots per load batch of the event VJP at <= 2 value columns per lane
#endif

// One warp per (token, head).  Mirrors _vjp's per-token loop over the write slots,
// then the read slots, with its rounding points.  The route-weight gradients stay
// per head (the reference runs one routed update per head); the router backward
// sums them over heads.  CPL = value columns per lane (lane l: l, l+32, ...).
// The loads of a batch of JB slots (event gradient rows, tile-0 records, route
// weights) are all issued before any of that batch's arithmetic, so a warp keeps
// a batch of independent requests in flight instead of one dependent round trip
// per slot; the arithmetic itself runs slot by slot in the reference's order.
// G = 2: the two half-warps take two heads of the token (16 lanes each, lane el:
// columns el, el+16, ...), so the per-slot work of the S lanes and the reductions
// serve two heads at once.  Columns el + 32i (even positions) and el + 16 + 32i (odd
// positions) are what lanes el and el + 16 hold at G = 1; their two partial sums,
// added, are warp_sum's first level, so every total keeps warp_sum's tree.
// Minimum CTAs per SM: the register budgets that measured fastest (no spills).
template <int G, int CPL> constexpr int vjp_min_blocks() { return G == 2 ? 5 : (CPL <= 2 ? 6 : 5); }

template <typename T, int S, int CPL, int G>
__global__ void __launch_bounds__(32 * kVjpWarps, (vjp_min_blocks<G, CPL>())) event_vjp_kernel(const VjpParams p) {
    constexpr int LPH = 32 / G;  // lanes per head
    const int64_t item = (int64_t)blockIdx.x * kVjpWarps + (threadIdx.x >> 5);
    const int HG = p.H / G;
    if (item >= p.nt * HG) return;
    const int64_t t = item / HG;
    const int lane = (int)lane_id();
    const int el = G == 2 ? (lane & 15) : lane;
    const int h = (int)(item % HG) * G + (G == 2 ? (lane >> 4) : 0);
    const int dv = p.dv;
    const int64_t V = (int64_t)p.H * dv;
    const int64_t hs0 = (t * p.H + h) * S;
    const bool nl = el < S;
    constexpr int R = 3 * S;
    constexpr int JB = CPL <= 2 ? BDM_VJP_BATCH : (CPL == 4 ? 4 : 2);  // slots per load batch
    const T *__restrict__ ww = static_cast<const T *>(p.ww);
    const T *__restrict__ rwp = static_cast<const T *>(p.rw);
    const float *__restrict__ evg = p.evg;
    float k0 = 0.f, b0 = 0.f, g0 = 0.f, q0 = 0.f;
    if (nl) {
        k0 = ld_f(static_cast<const T *>(p.k), hs0 + el);
        b0 = ld_f(static_cast<const T *>(p.b), hs0 + el);
        g0 = p.g[hs0 + el];
        q0 = ld_f(static_cast<const T *>(p.q), hs0 + el);
    }
    const int64_t vrow = t * V + (int64_t)h * dv;
    float v0[CPL], w0[CPL], accv[CPL], accw[CPL];
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
        const int c = el + LPH * i;
        const bool on = c < dv;
        v0[i] = on ? ld_f(static_cast<const T *>(p.v), vrow + c) : 0.f;
        w0[i] = on ? ld_f(static_cast<const T *>(p.w), vrow + c) : 0.f;
        accv[i] = accw[i] = 0.f;
    }
    // BF16 with an even number of columns per lane: the lane's columns (i, i+1) run as BF16x2
    // pairs.  Each BF16 result below is the same value as the FP32 expression rounded once:
    // a product of two BF16 values is exact in FP32; a sum of two BF16 values is exact in
    // FP32 unless their exponents differ by more than 16, and then both roundings return the
    // larger operand.  The FP32 x BF16 products stay FP32 (packed FP32x2) and are rounded by
    // one paired conversion.  The _rn forms never contract into a fused multiply-add.
    constexpr bool kPair = std::is_same<T, bf16>::value && CPL % 2 == 0;
    constexpr int NQ = CPL / 2 > 0 ? CPL / 2 : 1;
    __nv_bfloat162 w2[NQ], accv2[NQ], accw2[NQ];
    float2 v2[NQ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
        if constexpr (kPair) {
            w2[q] = __floats2bfloat162_rn(w0[2 * q], w0[2 * q + 1]);  // exact: BF16 values
            v2[q] = make_float2(v0[2 * q], v0[2 * q + 1]);
            accv2[q] = accw2[q] = __floats2bfloat162_rn(0.f, 0.f);
        }
    }
    float dk_acc = 0.f, db_acc = 0.f, dg_acc = 0.f, dq_acc = 0.f;
    T *dwwh = static_cast<T *>(p.dww_h) + (t * p.H + h) * p.kw;
    T *drwh = static_cast<T *>(p.drw_h) + (t * p.H + h) * p.kr;
    for (int j0 = 0; j0 < p.kw; j0 += JB) {
        float dub[JB][CPL], pwb[JB], ra[JB], rc[JB], rg[JB];
#pragma unroll
        for (int u = 0; u < JB; ++u) {
            const int j = j0 + u;
            const bool js = j < p.kw;
            const int64_t id = t * p.kw + j;
            pwb[u] = js ? ld_f(ww, id) : 0.f;
            const float *durow = p.du + id * V + (int64_t)h * dv;
#pragma unroll
            for (int i = 0; i < CPL; ++i) {
                const int c = el + LPH * i;
                dub[u][i] = (js && c < dv) ? __ldg(durow + c) : 0.f;
            }
            const float *rec = evg + (id * p.H + h) * R;
            const bool rs = js && nl;
            ra[u] = rs ? __ldg(rec + el) : 0.f;
            rc[u] = rs ? __ldg(rec + S + el) : 0.f;
            rg[u] = rs ? __ldg(rec + 2 * S + el) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < JB; ++u) {
            const int j = j0 + u;
            if (j >= p.kw) break;
            const int64_t id = t * p.kw + j;
            const float pw = pwb[u];
            float wvp = 0.f, wvp_odd = 0.f;  // G = 2: sums of the even / odd column positions
            float &wvp2 = G == 2 ? wvp_odd : wvp;
            if constexpr (kPair) {
                const __nv_bfloat162 pw2 = __float2bfloat162_rn(pw);  // exact: a BF16 route weight
#pragma unroll
                for (int q = 0; q < NQ; ++q) {
                    const float2 du = make_float2(dub[u][2 * q], dub[u][2 * q + 1]);
                    const float2 a = __bfloat1622float2(__hmul2_rn(w2[q], pw2));                  // dtype(w*p)
                    const __nv_bfloat162 dve = __float22bfloat162_rn(__fmul2_rn(du, a));      // dv of the event
                    const __nv_bfloat162 dwe = __float22bfloat162_rn(__fmul2_rn(du, v2[q]));  // dw of the event
                    accv2[q] = __hadd2_rn(accv2[q], dve);
                    accw2[q] = __hadd2_rn(accw2[q], __hmul2_rn(dwe, pw2));
                    const float2 x = __bfloat1622float2(__hmul2_rn(dwe, w2[q]));
                    if (el + 2 * LPH * q < dv) wvp += x.x;
                    if (el + 2 * LPH * q + LPH < dv) wvp2 += x.y;
                }
            } else {
#pragma unroll
                for (int i = 0; i < CPL; ++i) {
                    const int c = el + LPH * i;
                    if (c < dv) {
                        const float du = dub[u][i];
                        const float dve = rnd<T>(du * rnd<T>(w0[i] * pw));  // dv of the event (stored as dtype)
                        const float dwe = rnd<T>(du * v0[i]);                // dw of the event (stored as dtype)
                        accv[i] = rnd<T>(accv[i] + dve);
                        accw[i] = rnd<T>(accw[i] + rnd<T>(dwe * pw));
                        (i % 2 ? wvp2 : wvp) += rnd<T>(dwe * w0[i]);
                    }
                }
            }
            float wbp = 0.f, dec = 0.f;
            if (nl) {
                float A = 0.f, C = 0.f, Gs = 0.f;
                A += ra[u];
                C += rc[u];
                Gs += rg[u];
                for (int tile = 1; tile < p.tiles; ++tile) {
                    const float *rec = evg + (((int64_t)tile * p.E + id) * p.H + h) * R;
                    A += rec[el];
                    C += rec[S + el];
                    Gs += rec[2 * S + el];
                }
                const float be = rnd<T>(b0 * pw);
                const float dke = rnd<T>(A - be * C);
                const float dbe = rnd<T>(-k0 * C);
                dk_acc += dke;
                db_acc += rnd<T>(dbe * pw);
                if (p.routed_decay) {
                    dg_acc += Gs * pw;
                    dec = Gs * g0;
                } else {
                    dg_acc += Gs;
                }
                wbp = rnd<T>(dbe * b0);
            }
            float wv;
            if constexpr (G == 2) {
                float x = wvp + wvp_odd;  // warp_sum's level 16
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) x += __shfl_xor_sync(kFull, x, o);
                wv = rnd<T>(x);
            } else {
                wv = rnd<T>(warp_sum(wvp));
            }
            const float wb = rnd<T>(warp_sum_low<S>(wbp));  // wbp, dec: non-zero on lanes < S only
            const float decs = warp_sum_low<S>(dec);
            if (el == 0) dwwh[j] = Elem<T>::from_float(rnd<T>(wb + wv) + decs);
        }
    }
    for (int j0 = 0; j0 < p.kr; j0 += JB) {
        float ob[JB], rb[JB];
#pragma unroll
        for (int u = 0; u < JB; ++u) {
            const int j = j0 + u;
            const bool js = j < p.kr;
            const int64_t rid = t * p.kr + j;
            rb[u] = js ? ld_f(rwp, rid) : 0.f;
            ob[u] = (js && nl) ? __ldg(evg + ((p.nw + rid) * p.H + h) * R + el) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < JB; ++u) {
            const int j = j0 + u;
            if (j >= p.kr) break;
            const int64_t id = p.nw + t * p.kr + j;
            const float r = rb[u];
            float wrp = 0.f;
            if (nl) {
                float o = 0.f;
                o += ob[u] * p.scale;
                for (int tile = 1; tile < p.tiles; ++tile)
                    o += evg[(((int64_t)tile * p.E + id) * p.H + h) * R + el] * p.scale;
                const float dqe = rnd<T>(o);
                dq_acc += rnd<T>(dqe * r);
                wrp = rnd<T>(dqe * q0);
            }
            const float wr = warp_sum_low<S>(wrp);  // non-zero on lanes < S only
            if (el == 0) drwh[j] = Elem<T>::from_float(wr);
        }
    }
    if (nl) {
        st_f(static_cast<T *>(p.dq), hs0 + el, dq_acc);
        st_f(static_cast<T *>(p.dk), hs0 + el, dk_acc);
        st_f(static_cast<T *>(p.db), hs0 + el, db_acc);
        p.dg[hs0 + el] = dg_acc;
    }
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
        const int c = el + LPH * i;
        if (c < dv) {
            if constexpr (kPair) {
                const __nv_bfloat162 av = accv2[i / 2], aw = accw2[i / 2];
                static_cast<bf16 *>(p.dv_out)[vrow + c] = i % 2 ? __high2bfloat16(av) : __low2bfloat16(av);
                static_cast<bf16 *>(p.dw_out)[vrow + c] = i % 2 ? __high2bfloat16(aw) : __low2bfloat16(aw);
            } else {
                st_f(static_cast<T *>(p.dv_out), vrow + c, accv[i]);
                st_f(static_cast<T *>(p.dw_out), vrow + c, accw[i]);
            }
        }
    }
}

#ifndef BDM_VJP_G2
#define BDM_VJP_G2 1  // two heads per warp in the event VJP when the head count is even
#endif

template <typename T, int S>
void launch_vjp(const VjpParams &p, int cpl, cudaStream_t st) {
    if (BDM_VJP_G2 && p.H % 2 == 0 && cpl <= 4) {  // two heads per warp: 2 x cpl columns per lane
        const unsigned blocks = (unsigned)ceil_div(p.nt * (p.H / 2), kVjpWarps);
        if (cpl <= 1) event_vjp_kernel<T, S, 2, 2><<<blocks, 32 * kVjpWarps, 0, st>>>(p);
        else if (cpl == 2) event_vjp_kernel<T, S, 4, 2><<<blocks, 32 * kVjpWarps, 0, st>>>(p);
        else event_vjp_kernel<T, S, 8, 2><<<blocks, 32 * kVjpWarps, 0, st>>>(p);
        return;
    }
    const unsigned blocks = (unsigned)ceil_div(p.items, kVjpWarps);
    if (cpl <= 1) event_vjp_kernel<T, S, 1, 1><<<blocks, 32 * kVjpWarps, 0, st>>>(p);
    else if (cpl == 2) event_vjp_kernel<T, S, 2, 1><<<blocks, 32 * kVjpWarps, 0, st>>>(p);
    else if (cpl <= 4) event_vjp_kernel<T, S, 4, 1><<<blocks, 32 * kVjpWarps, 0, st>>>(p);
    else event_vjp_kernel<T, S, 8, 1><<<blocks, 32 * kVjpWarps, 0, st>>>(p);
}

// ------------------------------------------------------- initial-state factors

// ds[r][x] = dtype(sum_b dtype(dinit[b][r][x])): the state gradient of one logical row,
// rounded per sequence as the reference rounds each routed update's state gradient.
template <typename T>
__global__ void state_rows_kernel(const float *__restrict__ dinit, int64_t batch, int64_t rows, int dv,
                                  float *__restrict__ ds) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * dv) return;
    float acc = 0.f;
    for (int64_t b = 0; b < batch; ++b) acc += rnd<T>(dinit[b * rows * dv + i]);
    ds[i] = rnd<T>(acc);
}

// dU[p][x] = sum_q ds[p*Q+q][x] and dZ[q][x] = sum_p ds[p*Q+q][x], each rounded once.
template <typename T>
__global__ void factor_sums_kernel(const float *__restrict__ ds, int64_t P, int64_t Q, int dv,
                                   float *__restrict__ du, float *__restrict__ dz) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < P * dv) {
        const int64_t pp = i / dv, x = i % dv;
        float acc = 0.f;
        for (int64_t q = 0; q < Q; ++q) acc += ds[(pp * Q + q) * dv + x];
        du[i] = rnd<T>(acc);
    } else if (i < (P + Q) * dv) {
        const int64_t j = i - P * dv;
        const int64_t qq = j / dv, x = j % dv;
        float acc = 0.f;
        for (int64_t pp = 0; pp < P; ++pp) acc += ds[(pp * Q + qq) * dv + x];
        dz[j] = rnd<T>(acc);
    }
}

// ---------------------------------------------------------------- router

struct RouteBwdParams {
    const void *logits;  // [ntok, ld] holding both blocks
    void *dlogits;       // [ntok, ldd]
    int64_t ntok, ld, ldd, first, second;
    int j1, j2, count, heads;
    const int64_t *idx1, *idx2;
    const void *dw1, *dw2;  // [ntok, heads, count] per-head weight gradients
};

// One warp per (token, block).  Weights = softmax over the selected pair scores
// dtype(L1[row] + L2[col]); their gradient is softmax's backward, rounded to the
// logits dtype, then summed onto each selected row of the first factor and each
// selected column of the second (in selection order); all other logits get 0.
template <typename T>
__global__ void route_backward_kernel(const RouteBwdParams p) {
    const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= 2 * p.ntok) return;
    const int lane = (int)lane_id();
    const int64_t t = item >> 1;
    const int blk = (int)(item & 1);
    const int64_t off = blk ? p.second : p.first;
    const T *lg = static_cast<const T *>(p.logits) + t * p.ld + off;
    T *out = static_cast<T *>(p.dlogits) + t * p.ldd + off;
    const int64_t *idx = (blk ? p.idx2 : p.idx1) + t * p.count;
    const T *dw = static_cast<const T *>(blk ? p.dw2 : p.dw1) + t * p.heads * p.count;
    for (int i = lane; i < p.j1 + p.j2; i += 32) out[i] = Elem<T>::from_float(0.f);
    __syncwarp();
    const bool on = lane < p.count;
    int row = -1, colj = -1;
    float val = -INFINITY, dwc = 0.f;
    if (on) {
        const int64_t id = idx[lane];
        row = (int)(id / p.j2);
        colj = (int)(id % p.j2);
        val = rnd<T>(ld_f(lg, row) + ld_f(lg, p.j1 + colj));
        dwc = ld_f(dw, lane);  // the heads' weight gradients, summed in ascending head order
        for (int hh = 1; hh < p.heads; ++hh) dwc = rnd<T>(dwc + ld_f(dw, (int64_t)hh * p.count + lane));
    }
    const float m = warp_max(val);
    const float ex = on ? expf(val - m) : 0.f;
    const float tot = warp_sum(ex);
    const float wgt = on ? ex / tot : 0.f;
    const float dot = warp_sum(wgt * dwc);
    const float dval = on ? rnd<T>(wgt * (dwc - dot)) : 0.f;
    float trow = 0.f, tcol = 0.f;
    bool frow = on, fcol = on;
    for (int c = 0; c < p.count; ++c) {
        const int rc = __shfl_sync(kFull, row, c), cc = __shfl_sync(kFull, colj, c);
        const float dc = __shfl_sync(kFull, dval, c);
        if (rc == row) {
            trow += dc;
            if (c < lane) frow = false;
        }
        if (cc == colj) {
            tcol += dc;
            if (c < lane) fcol = false;
        }
    }
    if (frow) out[row] = Elem<T>::from_float(trow);
    if (fcol) out[p.j1 + colj] = Elem<T>::from_float(tcol);
}

// ------------------------------------------------------------- controllers

constexpr int kCtlThreads = 256;
constexpr int kMaxS = 16;
constexpr int kGateTokens = 64;  // tokens per thread in the b / g range (parameter partial sums)

__device__ __forceinline__ float sigmoid_ieee(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu_grad(float z) {
    const float s = sigmoid_ieee(z);
    return s * (1.0f + z * (1.0f - s));
}

struct CtlBwdArgs {
    const void *proj;
    int64_t ntok, ld, col_q, col_k, col_v, col_b, col_w;
    const void *f;
    int64_t ldf;
    const float *a_log, *dt_bias, *g;
    const void *b, *w;                 // forward outputs (sigmoid results)
    const void *dq, *dk, *dvv, *db, *dw;
    const float *dg;
    void *dproj;
    int64_t ldd;
    void *df;                          // [ntok, H*S]
    float *part_dt, *part_a;           // [chunks, H*S]
    int H, S, dv, qk_norm;
    int64_t narrow_blocks, gate_blocks, chunks;
};

// q and k of one (token, head): normalize(silu(z)) backward, then silu's.
template <typename T>
__device__ __forceinline__ void ctl_narrow(const CtlBwdArgs &a, int64_t t, int h) {
    const T *row = static_cast<const T *>(a.proj) + t * a.ld;
    T *drow = static_cast<T *>(a.dproj) + t * a.ldd;
    const int S = a.S;
    const int64_t o = (t * a.H + h) * S;
#pragma unroll
    for (int role = 0; role < 2; ++role) {
        const int64_t col = (role ? a.col_k : a.col_q) + (int64_t)h * S;
        const T *dy = static_cast<const T *>(role ? a.dk : a.dq) + o;
        float z[kMaxS], x[kMaxS];
        float ss = 0.f, xdy = 0.f;
        for (int s = 0; s < S; ++s) {
            z[s] = Elem<T>::to_float(row[col + s]);
            x[s] = rnd<T>(z[s] / (1.0f + expf(-z[s])));
            ss += x[s] * x[s];
            xdy += x[s] * ld_f(dy, s);
        }
        float scale, cube;
        if (a.qk_norm) {  // x * rsqrt(sum x^2 + 1e-6)
            scale = 1.0f / sqrtf(ss + 1e-6f);
            cube = scale * scale * scale;
        } else {          // x / max(|x|, 1e-12)
            const float n = sqrtf(ss);
            scale = 1.0f / fmaxf(n, 1e-12f);
            cube = n > 1e-12f ? scale * scale * scale : 0.f;
        }
        for (int s = 0; s < S; ++s) {
            const float dx = rnd<T>(scale * ld_f(dy, s) - x[s] * cube * xdy);
            drow[col + s] = Elem<T>::from_float(dx * silu_grad(z[s]));
        }
    }
}

// b and the decay gate of one head*S + s over a chunk of tokens; FP32 partial sums of
// the dt_bias gradient and of dg * g (the A_log gradient) per chunk.
template <typename T>
__device__ __forceinline__ void ctl_gate(const CtlBwdArgs &a, int64_t chunk, int hs) {
    const int HS = a.H * a.S;
    const int h = hs / a.S;
    const float na = -expf(a.a_log[h]);
    const float dtb = a.dt_bias[hs];
    float pdt = 0.f, pa = 0.f;
    const int64_t t1 = min(a.ntok, (chunk + 1) * kGateTokens);
    for (int64_t t = chunk * kGateTokens; t < t1; ++t) {
        const int64_t o = t * HS + hs;
        const float bo = ld_f(static_cast<const T *>(a.b), o);
        const float dbv = ld_f(static_cast<const T *>(a.db), o);
        st_f(static_cast<T *>(a.dproj), t * a.ldd + a.col_b + hs, dbv * (1.0f - bo) * bo);
        const float z = ld_f(static_cast<const T *>(a.f), t * a.ldf + hs) + dtb;
        const float dgv = a.dg[o];
        const float dz = dgv * na * (z > 20.0f ? 1.0f : sigmoid_ieee(z));
        st_f(static_cast<T *>(a.df), o, dz);
        pdt += dz;
        pa += dgv * a.g[o];
    }
    a.part_dt[chunk * HS + hs] = pdt;
    a.part_a[chunk * HS + hs] = pa;
}

template <typename T>
__device__ __forceinline__ void ctl_wide(const CtlBwdArgs &a, int64_t i) {
    const int64_t V = (int64_t)a.H * a.dv;
    const int64_t t = i / V, c = i % V;
    const T *row = static_cast<const T *>(a.proj) + t * a.ld;
    T *drow = static_cast<T *>(a.dproj) + t * a.ldd;
    const float zv = Elem<T>::to_float(row[a.col_v + c]);
    drow[a.col_v + c] = Elem<T>::from_float(ld_f(static_cast<const T *>(a.dvv), i) * silu_grad(zv));
    const float wo = ld_f(static_cast<const T *>(a.w), i);
    drow[a.col_w + c] = Elem<T>::from_float(ld_f(static_cast<const T *>(a.dw), i) * (1.0f - wo) * wo);
}

template <typename T>
__global__ void __launch_bounds__(kCtlThreads) controllers_backward_kernel(const CtlBwdArgs a) {
    const int64_t blk = blockIdx.x;
    if (blk < a.narrow_blocks) {
        const int64_t item = blk * kCtlThreads + threadIdx.x;
        if (item < a.ntok * a.H) ctl_narrow<T>(a, item / a.H, (int)(item % a.H));
    } else if (blk < a.narrow_blocks + a.gate_blocks) {
        const int64_t item = (blk - a.narrow_blocks) * kCtlThreads + threadIdx.x;
        const int HS = a.H * a.S;
        if (item < a.chunks * HS) ctl_gate<T>(a, item / HS, (int)(item % HS));
    } else {
        const int64_t item = (blk - a.narrow_blocks - a.gate_blocks) * kCtlThreads + threadIdx.x;
        if (item < a.ntok * a.H * a.dv) ctl_wide<T>(a, item);
    }
}

// ----------------------------------------------------------- output interface

constexpr int kNgCols = 8;
constexpr int kNgTokens = 16;  // tokens per CTA (norm-parameter partial sums)

template <typename T> __device__ __forceinline__ float gate_sigmoid(float x);
template <> __device__ __forceinline__ float gate_sigmoid<bf16>(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
template <> __device__ __forceinline__ float gate_sigmoid<float>(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float ng_block_sum(float x, float *red) {
    x = warp_sum(x);
    const int warp = threadIdx.x >> 5, lane = (int)lane_id();
    const int nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = x;
    __syncthreads();
    float s = lane < nw ? red[lane] : 0.f;
    return warp_sum(s);
}

struct NgBwdArgs {
    const void *dout, *raw, *gate, *nw, *nb;
    int64_t ntok, width, ld_gate, ldd;
    float eps;
    int norm_mode;
    void *draw, *dgate;
    float *part_w, *part_b;  // [blocks, width]
};

// Backward of  out = norm(raw) * dtype(sigmoid(gate_logit))  for kNgTokens tokens per
// CTA, each thread on 8 columns; norm = LayerNorm (mode 1) or the reference's RMS
// form dtype(dtype(raw * dtype(rsqrt(mean raw^2 + eps))) * weight) (mode 0).
template <typename T>
__global__ void norm_gate_backward_kernel(const NgBwdArgs a) {
    __shared__ float red[32];
    const int64_t c0 = (int64_t)threadIdx.x * kNgCols;
    const bool act = c0 < a.width;
    const float inv_w = 1.0f / (float)a.width;
    float gw[kNgCols], gb[kNgCols], wv[kNgCols], bv[kNgCols];
#pragma unroll
    for (int i = 0; i < kNgCols; ++i) {
        const bool on = act && c0 + i < a.width;
        gw[i] = gb[i] = 0.f;
        wv[i] = on ? ld_f(static_cast<const T *>(a.nw), c0 + i) : 0.f;
        bv[i] = on && a.nb ? ld_f(static_cast<const T *>(a.nb), c0 + i) : 0.f;
    }
    const int64_t t0 = (int64_t)blockIdx.x * kNgTokens;
    const int64_t t1 = min(a.ntok, t0 + kNgTokens);
    // a token's loads are issued one token ahead, so they overlap the previous token's reductions
    float xn[kNgCols], dyn[kNgCols], gln[kNgCols];
    auto load_token = [&](int64_t t) {
#pragma unroll
        for (int i = 0; i < kNgCols; ++i) {
            const bool on = act && c0 + i < a.width;
            xn[i] = on ? ld_f(static_cast<const T *>(a.raw), t * a.width + c0 + i) : 0.f;
            dyn[i] = on ? ld_f(static_cast<const T *>(a.dout), t * a.width + c0 + i) : 0.f;
            gln[i] = on ? ld_f(static_cast<const T *>(a.gate), t * a.ld_gate + c0 + i) : 0.f;
        }
    };
    if (t0 < t1) load_token(t0);
    for (int64_t t = t0; t < t1; ++t) {
        float x[kNgCols], dy[kNgCols], gt[kNgCols];
#pragma unroll
        for (int i = 0; i < kNgCols; ++i) {
            const bool on = act && c0 + i < a.width;
            x[i] = xn[i];
            dy[i] = dyn[i];
            gt[i] = on ? rnd<T>(gate_sigmoid<T>(gln[i])) : 0.f;
        }
        if (t + 1 < t1) load_token(t + 1);
        float n[kNgCols], dn[kNgCols], dx[kNgCols];
        if (a.norm_mode == 1) {
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < kNgCols; ++i) s += x[i];
            const float mean = ng_block_sum(s, red) * inv_w;
            float sq = 0.f;
#pragma unroll
            for (int i = 0; i < kNgCols; ++i)
                if (act && c0 + i < a.width) sq += (x[i] - mean) * (x[i] - mean);
            const float rstd = 1.0f / sqrtf(ng_block_sum(sq, red) * inv_w + a.eps);
            float xh[kNgCols], s1 = 0.f, s2 = 0.f;
#pragma unroll
            for (int i = 0; i < kNgCols; ++i) {
                const bool on = act && c0 + i < a.width;
                xh[i] = on ? (x[i] - mean) * rstd : 0.f;
                n[i] = on ? rnd<T>(xh[i] * wv[i] + bv[i]) : 0.f;
                dn[i] = rnd<T>(dy[i] * gt[i]);
                const float dxh = dn[i] * wv[i];
                s1 += dxh;
                s2 += dxh * xh[i];
                gw[i] += dn[i] * xh[i];
                gb[i] += dn[i];
            }
            s1 = ng_block_sum(s1, red);
            s2 = ng_block_sum(s2, red);
#pragma unroll
            for (int i = 0; i < kNgCols; ++i)
                dx[i] = rnd<T>(rstd * inv_w * ((float)a.width * dn[i] * wv[i] - s1 - xh[i] * s2));
        } else {
            float sq = 0.f;
#pragma unroll
            for (int i = 0; i < kNgCols; ++i) sq += x[i] * x[i];
            const float rs32 = 1.0f / sqrtf(ng_block_sum(sq, red) * inv_w + a.eps);
            const float rs = rnd<T>(rs32);
            float n1[kNgCols], dn1[kNgCols], drs = 0.f;
#pragma unroll
            for (int i = 0; i < kNgCols; ++i) {
                n1[i] = rnd<T>(x[i] * rs);
                n[i] = rnd<T>(n1[i] * wv[i]);
                dn[i] = rnd<T>(dy[i] * gt[i]);
                gw[i] += rnd<T>(dn[i] * n1[i]);
                dn1[i] = rnd<T>(dn[i] * wv[i]);
                drs += rnd<T>(dn1[i] * x[i]);
            }
            drs = rnd<T>(ng_block_sum(drs, red));
            const float dvar = drs * -0.5f * rs32 * rs32 * rs32;
#pragma unroll
            for (int i = 0; i < kNgCols; ++i)
                dx[i] = rnd<T>(rnd<T>(dn1[i] * rs) + rnd<T>(dvar * 2.0f * x[i] * inv_w));
        }
        if (act) {
#pragma unroll
            for (int i = 0; i < kNgCols; ++i) {
                if (c0 + i < a.width) {
                    st_f(static_cast<T *>(a.draw), t * a.width + c0 + i, dx[i]);
                    const float dgt = rnd<T>(dy[i] * n[i]);
                    st_f(static_cast<T *>(a.dgate), t * a.ldd + c0 + i, dgt * gt[i] * (1.0f - gt[i]));
                }
            }
        }
    }
    if (act) {
#pragma unroll
        for (int i = 0; i < kNgCols; ++i) {
            if (c0 + i < a.width) {
                a.part_w[(int64_t)blockIdx.x * a.width + c0 + i] = gw[i];
                if (a.part_b) a.part_b[(int64_t)blockIdx.x * a.width + c0 + i] = gb[i];
            }
        }
    }
}

// out[c] = sum over rows r of in[r*ld + c] (ascending r inside 8 interleaved groups, then
// the groups in order): deterministic column sums of partial-sum tables.
__global__ void column_sums_kernel(const float *__restrict__ in, int64_t rows, int64_t cols, int64_t ld,
                                   float *__restrict__ out) {
    __shared__ float part[8][32];
    const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
    const int64_t c = (int64_t)blockIdx.x * 32 + lane;
    float acc = 0.f;
    if (c < cols)
        for (int64_t r = grp; r < rows; r += 8) acc += in[r * ld + c];
    part[grp][lane] = acc;
    __syncthreads();
    if (grp == 0 && c < cols) {
        float s = 0.f;
        for (int i = 0; i < 8; ++i) s += part[i][lane];
        out[c] = s;
    }
}

int column_sums(const float *in, int64_t rows, int64_t cols, int64_t ld, float *out, cudaStream_t st) {
    if (cols <= 0) return BDM_OK;
    column_sums_kernel<<<(unsigned)ceil_div(cols, 32), 256, 0, st>>>(in, rows, cols, ld, out);
    return launch_status();
}

// out[i] = sum_{j < len} in[i*len + j] (ascending j): per-head sums of per-row totals.
__global__ void segment_sums_kernel(const float *__restrict__ in, int nseg, int len, float *__restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nseg) return;
    float s = 0.f;
    for (int j = 0; j < len; ++j) s += in[(int64_t)i * len + j];
    out[i] = s;
}

}  // namespace
}  // namespace bdm

// ------------------------------------------------------------------ C ABI

extern "C" int64_t bdm_scan_backward_checkpoint_bytes(int64_t batch, int64_t time, int kw, int kr, int64_t bank_count,
                                                      int heads, int bank_size, int head_value_width) {
    using namespace bdm;
    if (batch < 0 || time < 0 || kw <= 0 || kr <= 0 || bank_count <= 0 || heads <= 0 || head_value_width <= 0)
        return -1;
    if (bank_size != 4 && bank_size != 8 && bank_size != 16) return -1;
    const int64_t E = batch * time * (kw + kr);
    const int64_t slots = E / block_events(bank_size, head_value_width) + batch * bank_count + 1;
    return slots * heads * bank_size * head_value_width * (int64_t)sizeof(float);
}

extern "C" int bdm_scan_backward_block_events(int bank_size, int head_value_width) {
    if ((bank_size != 4 && bank_size != 8 && bank_size != 16) || head_value_width <= 0) return -1;
    return (int)bdm::block_events(bank_size, head_value_width);
}

extern "C" int bdm_scan_backward_tiles(int bank_size, int head_value_width) {
    if ((bank_size != 4 && bank_size != 8 && bank_size != 16) || head_value_width <= 0) return -1;
    return bdm::scan_tiles(bank_size, head_value_width);
}

extern "C" int bdm_scan_backward(const void *q, const void *k, const void *v, const float *g, const void *b,
                                 const void *w, const void *write_w, const void *read_w, const int64_t *order,
                                 const int64_t *cu_seqlens, int64_t batch, int64_t time, int64_t bank_count, int heads,
                                 int bank_size, int head_value_width, int kw, int kr, int dtype, int routed_decay,
                                 float scale, const void *row_factor, const void *col_factor, int64_t factor_cols,
                                 int factor_dtype, int state_interval, const void *d_read, float *event_grads,
                                 float *d_write_value, float *d_initial, float *checkpoints, int64_t checkpoint_bytes,
                                 int checkpoints_ready, void *stream) {
    using namespace bdm;
    if (batch < 0 || time < 0 || bank_count <= 0 || heads <= 0 || head_value_width <= 0 || kw <= 0 || kr <= 0 ||
        state_interval < 0)
        return BDM_ERR_INVALID;
    if (bank_size != 4 && bank_size != 8 && bank_size != 16) return BDM_ERR_UNSUPPORTED;
    if (!valid_dtype(dtype)) return BDM_ERR_DTYPE;
    if (row_factor && (!col_factor || factor_cols <= 0 || !valid_dtype(factor_dtype))) return BDM_ERR_INVALID;
    const int64_t need = bdm_scan_backward_checkpoint_bytes(batch, time, kw, kr, bank_count, heads, bank_size,
                                                            head_value_width);
    if (batch * time == 0) return BDM_OK;
    if (!q || !k || !v || !g || !b || !w || !write_w || !read_w || !order || !cu_seqlens || !d_read ||
        !event_grads || !d_write_value || !d_initial)
        return BDM_ERR_INVALID;
    if (!checkpoints || checkpoint_bytes < need) return BDM_ERR_WORKSPACE;
    if (batch * time * (kw + kr) > 0x7fffffffLL) return BDM_ERR_UNSUPPORTED;  // 32-bit event ids in the kernel
    ScanBwdParams p{};
    p.q = q; p.k = k; p.v = v; p.g = g; p.b = b; p.w = w; p.ww = write_w; p.rw = read_w;
    p.order = order; p.cu = cu_seqlens;
    p.nseq = batch * bank_count; p.J = bank_count; p.nt = batch * time; p.nw = p.nt * kw;
    p.E = p.nt * (kw + kr);
    p.H = heads; p.dv = head_value_width; p.kw = kw; p.kr = kr; p.routed_decay = routed_decay;
    p.interval = state_interval; p.tiles = scan_tiles(bank_size, head_value_width); p.scale = scale;
    p.row_factor = row_factor; p.col_factor = col_factor; p.factor_cols = factor_cols; p.factor_dtype = factor_dtype;
    p.dread = d_read; p.ckpt = checkpoints; p.evg = event_grads; p.du = d_write_value; p.dinit = d_initial;
    p.ckpt_ready = checkpoints_ready;
    p.units = p.nseq * heads * p.tiles;
    const cudaStream_t st = as_stream(stream);
    const bool two = scan_cols(bank_size, head_value_width) == 2;
    BDM_DISPATCH_DTYPE(dtype, T, {
        if (bank_size == 4) return two ? launch_scan_backward<T, 4, 2>(p, st) : launch_scan_backward<T, 4, 1>(p, st);
        if (bank_size == 8) return two ? launch_scan_backward<T, 8, 2>(p, st) : launch_scan_backward<T, 8, 1>(p, st);
        return launch_scan_backward<T, 16, 1>(p, st);
    });
    return BDM_ERR_UNSUPPORTED;
}

extern "C" int bdm_event_vjp(const void *q, const void *k, const void *v, const float *g, const void *b, const void *w,
                             const void *write_w, const void *read_w, const float *event_grads,
                             const float *d_write_value, int64_t ntok, int heads, int bank_size, int head_value_width,
                             int kw, int kr, int dtype, int routed_decay, float scale, void *dq, void *dk, void *dv,
                             float *dg, void *db, void *dw, void *d_write_w_heads, void *d_read_w_heads,
                             void *stream) {
    using namespace bdm;
    if (ntok < 0 || heads <= 0 || head_value_width <= 0 || kw <= 0 || kr <= 0) return BDM_ERR_INVALID;
    if (bank_size != 4 && bank_size != 8 && bank_size != 16) return BDM_ERR_UNSUPPORTED;
    if (head_value_width > 256) return BDM_ERR_UNSUPPORTED;
    if (!valid_dtype(dtype)) return BDM_ERR_DTYPE;
    if (ntok == 0) return BDM_OK;
    if (!q || !k || !v || !g || !b || !w || !write_w || !read_w || !event_grads || !d_write_value || !dq || !dk ||
        !dv || !dg || !db || !dw || !d_write_w_heads || !d_read_w_heads)
        return BDM_ERR_INVALID;
    VjpParams p{};
    p.q = q; p.k = k; p.v = v; p.g = g; p.b = b; p.w = w; p.ww = write_w; p.rw = read_w;
    p.evg = event_grads; p.du = d_write_value;
    p.nt = ntok; p.nw = ntok * kw; p.E = ntok * (kw + kr); p.items = ntok * heads;
    p.H = heads; p.dv = head_value_width; p.kw = kw; p.kr = kr; p.routed_decay = routed_decay;
    p.tiles = scan_tiles(bank_size, head_value_width); p.scale = scale;
    p.dq = dq; p.dk = dk; p.dv_out = dv; p.db = db; p.dw_out = dw; p.dww_h = d_write_w_heads;
    p.drw_h = d_read_w_heads; p.dg = dg;
    const int64_t blocks = ceil_div(p.items, kVjpWarps);
    if (blocks > 0x7fffffffLL) return BDM_ERR_UNSUPPORTED;
    const int cpl = (int)ceil_div(head_value_width, 32);
    const cudaStream_t st = as_stream(stream);
    BDM_DISPATCH_DTYPE(dtype, T, {
        if (bank_size == 4) launch_vjp<T, 4>(p, cpl, st);
        else if (bank_size == 8) launch_vjp<T, 8>(p, cpl, st);
        else launch_vjp<T, 16>(p, cpl, st);
    });
    return launch_status();
}

extern "C" int bdm_product_state_backward(const float *d_initial, int64_t batch, int64_t rows_p, int64_t cols_q,
                                          int head_value_width, int factor_dtype, float *d_rows, float *d_row_factor,
                                          float *d_col_factor, void *stream) {
    using namespace bdm;
    if (batch < 0 || rows_p <= 0 || cols_q <= 0 || head_value_width <= 0) return BDM_ERR_INVALID;
    if (!valid_dtype(factor_dtype)) return BDM_ERR_DTYPE;
    if (!d_initial || !d_rows || !d_row_factor || !d_col_factor) return BDM_ERR_INVALID;
    const int64_t rows = rows_p * cols_q;
    const cudaStream_t st = as_stream(stream);
    const int64_t n1 = rows * head_value_width, n2 = (rows_p + cols_q) * head_value_width;
    if (ceil_div(n1, 256) > 0x7fffffffLL) return BDM_ERR_UNSUPPORTED;
    BDM_DISPATCH_DTYPE(factor_dtype, T, {
        state_rows_kernel<T><<<(unsigned)ceil_div(n1, 256), 256, 0, st>>>(d_initial, batch, rows, head_value_width,
                                                                          d_rows);
        int rc = launch_status();
        if (rc != BDM_OK) return rc;
        factor_sums_kernel<T><<<(unsigned)ceil_div(n2, 256), 256, 0, st>>>(d_rows, rows_p, cols_q, head_value_width,
                                                                          d_row_factor, d_col_factor);
    });
    return launch_status();
}

extern "C" int bdm_route_backward(const void *logits, int64_t ntok, int64_t ld, int64_t first, int64_t second, int j1,
                                  int j2, int count, int heads, const int64_t *idx_first, const void *dw_first,
                                  const int64_t *idx_second, const void *dw_second, int dtype, void *d_logits,
                                  int64_t ldd, void *stream) {
    using namespace bdm;
    if (ntok < 0 || j1 <= 0 || j2 <= 0 || count <= 0 || heads <= 0 || first < 0 || second < first + j1 + j2 ||
        ld < second + j1 + j2 || ldd < second + j1 + j2)
        return BDM_ERR_INVALID;
    if (count > 32) return BDM_ERR_UNSUPPORTED;
    if (!valid_dtype(dtype)) return BDM_ERR_DTYPE;
    if (ntok == 0) return BDM_OK;
    if (!logits || !idx_first || !dw_first || !idx_second || !dw_second || !d_logits) return BDM_ERR_INVALID;
    RouteBwdParams p{};
    p.logits = logits; p.dlogits = d_logits; p.ntok = ntok; p.ld = ld; p.ldd = ldd; p.first = first;
    p.second = second; p.j1 = j1; p.j2 = j2; p.count = count; p.heads = heads; p.idx1 = idx_first;
    p.idx2 = idx_second;
    p.dw1 = dw_first; p.dw2 = dw_second;
    const int64_t blocks = ceil_div(2 * ntok, 8);
    if (blocks > 0x7fffffffLL) return BDM_ERR_UNSUPPORTED;
    BDM_DISPATCH_DTYPE(dtype, T, {
        route_backward_kernel<T><<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(p);
    });
    return launch_status();
}

extern "C" int64_t bdm_controllers_backward_partial_floats(int64_t ntok, int heads, int bank_size) {
    if (ntok < 0 || heads <= 0 || bank_size <= 0) return -1;
    return (2 * bdm::ceil_div(ntok, bdm::kGateTokens) + 1) * heads * bank_size;
}

extern "C" int bdm_controllers_backward(const void *proj, int64_t ntok, int64_t ld, int64_t col_q, int64_t col_k,
                                        int64_t col_v, int64_t col_b, int64_t col_w, const void *f, int64_t ldf,
                                        const float *a_log, const float *dt_bias, const float *g, const void *b,
                                        const void *w, const void *dq, const void *dk, const void *dv, const float *dg,
                                        const void *db, const void *dw, int heads, int bank_size,
                                        int head_value_width, int qk_norm, int dtype, void *d_proj, int64_t ldd,
                                        void *df, float *partials, float *d_dt_bias, float *d_a_log, void *stream) {
    using namespace bdm;
    if (ntok < 0 || heads <= 0 || bank_size <= 0 || head_value_width <= 0) return BDM_ERR_INVALID;
    if (bank_size > kMaxS) return BDM_ERR_UNSUPPORTED;
    if (!valid_dtype(dtype)) return BDM_ERR_DTYPE;
    const int64_t HS = (int64_t)heads * bank_size, V = (int64_t)heads * head_value_width;
    if (col_q < 0 || col_k < 0 || col_v < 0 || col_b < 0 || col_w < 0 || col_q + HS > ld || col_k + HS > ld ||
        col_v + V > ld || col_b + HS > ld || col_w + V > ld || ldf < HS || ldd < ld)
        return BDM_ERR_INVALID;
    if (!d_dt_bias || !d_a_log) return BDM_ERR_INVALID;
    const cudaStream_t st = as_stream(stream);
    if (ntok == 0) {
        int rc = cuda_status(cudaMemsetAsync(d_dt_bias, 0, sizeof(float) * HS, st));
        if (rc != BDM_OK) return rc;
        return cuda_status(cudaMemsetAsync(d_a_log, 0, sizeof(float) * heads, st));
    }
    if (!proj || !f || !a_log || !dt_bias || !g || !b || !w || !dq || !dk || !dv || !dg || !db || !dw || !d_proj ||
        !df || !partials)
        return BDM_ERR_INVALID;
    CtlBwdArgs a{};
    a.proj = proj; a.ntok = ntok; a.ld = ld; a.col_q = col_q; a.col_k = col_k; a.col_v = col_v; a.col_b = col_b;
    a.col_w = col_w; a.f = f; a.ldf = ldf; a.a_log = a_log; a.dt_bias = dt_bias; a.g = g; a.b = b; a.w = w;
    a.dq = dq; a.dk = dk; a.dvv = dv; a.db = db; a.dw = dw; a.dg = dg; a.dproj = d_proj; a.ldd = ldd; a.df = df;
    a.H = heads; a.S = bank_size; a.dv = head_value_width; a.qk_norm = qk_norm;
    a.chunks = ceil_div(ntok, kGateTokens);
    a.part_dt = partials;
    a.part_a = partials + a.chunks * HS;
    a.narrow_blocks = ceil_div(ntok * heads, kCtlThreads);
    a.gate_blocks = ceil_div(a.chunks * HS, kCtlThreads);
    const int64_t wide_blocks = ceil_div(ntok * V, kCtlThreads);
    if (a.narrow_blocks + a.gate_blocks + wide_blocks > 0x7fffffffLL) return BDM_ERR_UNSUPPORTED;
    BDM_DISPATCH_DTYPE(dtype, T, {
        controllers_backward_kernel<T><<<(unsigned)(a.narrow_blocks + a.gate_blocks + wide_blocks), kCtlThreads, 0,
                                         st>>>(a);
    });
    int rc = launch_status();
    if (rc != BDM_OK) return rc;
    // dt_bias: column sums over the chunks; A_log[h]: the same, then summed over the head's S columns
    rc = column_sums(a.part_dt, a.chunks, HS, HS, d_dt_bias, st);
    if (rc != BDM_OK) return rc;
    float *a_rows = a.part_a + a.chunks * HS;  // [HS] scratch after the two partial tables
    rc = column_sums(a.part_a, a.chunks, HS, HS, a_rows, st);
    if (rc != BDM_OK) return rc;
    segment_sums_kernel<<<(unsigned)ceil_div(heads, 128), 128, 0, st>>>(a_rows, heads, bank_size, d_a_log);
    return launch_status();
}

extern "C" int64_t bdm_norm_gate_backward_partial_floats(int64_t ntok, int64_t width) {
    if (ntok < 0 || width <= 0) return -1;
    return 2 * bdm::ceil_div(ntok, bdm::kNgTokens) * width;
}

extern "C" int bdm_norm_gate_backward(const void *d_out, const void *raw, int64_t ntok, int64_t width,
                                      const void *gate, int64_t ld_gate, const void *norm_weight,
                                      const void *norm_bias, float eps, int norm_mode, int dtype, void *d_raw,
                                      void *d_gate, int64_t ld_d_gate, float *partials, float *d_norm_weight,
                                      float *d_norm_bias, void *stream) {
    using namespace bdm;
    if (ntok < 0 || width <= 0 || ld_gate < width || ld_d_gate < width) return BDM_ERR_INVALID;
    if (norm_mode != 0 && norm_mode != 1) return BDM_ERR_INVALID;
    if (!valid_dtype(dtype)) return BDM_ERR_DTYPE;
    if (width > 1024 * kNgCols) return BDM_ERR_UNSUPPORTED;
    if (!d_norm_weight || (norm_mode == 1 && norm_bias && !d_norm_bias)) return BDM_ERR_INVALID;
    const cudaStream_t st = as_stream(stream);
    const bool want_b = norm_bias != nullptr && d_norm_bias != nullptr;
    if (ntok == 0) {
        int rc = cuda_status(cudaMemsetAsync(d_norm_weight, 0, sizeof(float) * width, st));
        if (rc != BDM_OK || !want_b) return rc;
        return cuda_status(cudaMemsetAsync(d_norm_bias, 0, sizeof(float) * width, st));
    }
    if (!d_out || !raw || !gate || !norm_weight || !d_raw || !d_gate || !partials) return BDM_ERR_INVALID;
    NgBwdArgs a{};
    a.dout = d_out; a.raw = raw; a.gate = gate; a.nw = norm_weight; a.nb = norm_bias; a.ntok = ntok;
    a.width = width; a.ld_gate = ld_gate; a.ldd = ld_d_gate; a.eps = eps; a.norm_mode = norm_mode;
    a.draw = d_raw; a.dgate = d_gate;
    const int64_t blocks = ceil_div(ntok, kNgTokens);
    a.part_w = partials;
    a.part_b = want_b ? partials + blocks * width : nullptr;
    const int threads = (int)(ceil_div(ceil_div(width, kNgCols), 32) * 32);
    if (blocks > 0x7fffffffLL) return BDM_ERR_UNSUPPORTED;
    BDM_DISPATCH_DTYPE(dtype, T, {
        norm_gate_backward_kernel<T><<<(unsigned)blocks, threads, 0, st>>>(a);
    });
    int rc = launch_status();
    if (rc != BDM_OK) return rc;
    rc = column_sums(a.part_w, blocks, width, width, d_norm_weight, st);
    if (rc != BDM_OK || !want_b) return rc;
    return column_sums(a.part_b, blocks, width, width, d_norm_bias, st);
}
