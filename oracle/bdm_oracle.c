/*
 * bdm_oracle.c -- CPU restatement of the Block Delta Memory (BDM) layer hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * product in bdm_b200/.  Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline / reference arm may load it.  The product path never calls it.
 *
 * Every function restates one piece of the reference (p0rc314in/bdm,
 * implementation/bdm/...) in plain C, following the reference's operation
 * order so that results agree bit-for-bit on integer work (routing indices,
 * dispatch order) and to the last few ulps on floating-point work:
 *
 *   oracle_route        gdn2_banks.py:74-114   product_key_route
 *                       (ties broken to the LOWER index at both top-k stages;
 *                        torch.topk leaves tie order unspecified)
 *   oracle_dispatch     gdn2_banks.py:174-185,237-246  pack_bank_events keys,
 *                       argsort, bincount -> cu_seqlens; role_bank_dispatch.py:15-24
 *   oracle_recurrence   gdn2_banks.py:196-224 (route-weighted packing) +
 *                       gdn2_banks.py:22-43 reference_packed_gdn2 (BF16 state
 *                       storage every `interval` events) +
 *                       inference.py:134-158 (interval 0: no rounding, prefill)
 *   oracle_combine      gdn2_banks.py:265-283 scatter_bank_outputs: reads summed
 *                       in ascending packed (bank) order; FP32 accumulation as
 *                       the CPU index_add_ does, or a rounding after every add
 *                       as the GPU readouts do (role_bank_dispatch.py:201-216)
 *   oracle_decode_step  inference.py:21-67,161-194 (_decode_write/_read/_sum)
 *
 * Parity is pinned by tests/test_oracle_golden.py against vectors produced by
 * the reference itself (tests/golden/make_golden.py).
 *
 * Threads: plain pthreads (oracle_set_threads); work is split over
 * independent tokens or (sequence, head) pairs, so results do not depend on
 * the thread count.
 *
 * Build: oracle/Makefile (-O2 -ffp-contract=off: the reference multiplies
 * and adds as separate roundings, so no FMA contraction here).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define ORACLE_OK 0
#define ORACLE_EINVAL 1
#define ORACLE_ENOMEM 2

/* ------------------------------------------------------------------ threads */

static int g_threads = 1;

int oracle_set_threads(int n) {
    if (n <= 0) {
        long c = sysconf(_SC_NPROCESSORS_ONLN);
        n = c > 0 ? (int)c : 1;
    }
    g_threads = n > 256 ? 256 : n;
    return g_threads;
}

int oracle_num_threads(void) { return g_threads; }

typedef void (*range_fn)(int64_t lo, int64_t hi, void *ctx);

typedef struct {
    range_fn fn;
    void *ctx;
    int64_t n, grain;
    int64_t next; /* guarded by mu */
    pthread_mutex_t mu;
} par_job;

static void *par_worker(void *arg) {
    par_job *job = (par_job *)arg;
    for (;;) {
        pthread_mutex_lock(&job->mu);
        int64_t lo = job->next;
        job->next += job->grain;
        pthread_mutex_unlock(&job->mu);
        if (lo >= job->n) break;
        int64_t hi = lo + job->grain < job->n ? lo + job->grain : job->n;
        job->fn(lo, hi, job->ctx);
    }
    return NULL;
}

/* Run fn over [0, n) in chunks of `grain` on g_threads threads (caller included). */
static void par_for(int64_t n, int64_t grain, range_fn fn, void *ctx) {
    if (n <= 0) return;
    if (grain < 1) grain = 1;
    int nt = g_threads;
    if ((int64_t)nt > (n + grain - 1) / grain) nt = (int)((n + grain - 1) / grain);
    if (nt <= 1) {
        fn(0, n, ctx);
        return;
    }
    par_job job = {fn, ctx, n, grain, 0, PTHREAD_MUTEX_INITIALIZER};
    pthread_t tids[256];
    int started = 0;
    for (int i = 0; i < nt - 1; ++i)
        if (pthread_create(&tids[started], NULL, par_worker, &job) == 0) ++started;
    par_worker(&job);
    for (int i = 0; i < started; ++i) pthread_join(tids[i], NULL);
    pthread_mutex_destroy(&job.mu);
}

/* ----------------------------------------------------------------- rounding */

/* Round-to-nearest-even float -> bfloat16 -> float (what torch's .to(bfloat16) does). */
static inline float bf16r(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) {
        if (u & 0x007fffffu) u |= 0x00400000u; /* keep NaN quiet */
        u &= 0xffff0000u;
    } else {
        u += 0x7fffu + ((u >> 16) & 1u);
        u &= 0xffff0000u;
    }
    memcpy(&x, &u, 4);
    return x;
}

static inline float rnd(float x, int bf16) { return bf16 ? bf16r(x) : x; }

float oracle_bf16_round(float x) { return bf16r(x); }

/* ------------------------------------------------------------------ routing */

/* Select the k largest of vals[0..n) ordered by (value desc, index asc). */
static void stable_topk(const float *vals, int n, int k, unsigned char *taken, float *out_v, int *out_i) {
    memset(taken, 0, (size_t)n);
    for (int r = 0; r < k; ++r) {
        int best = -1;
        for (int i = 0; i < n; ++i) {
            if (taken[i]) continue;
            if (best < 0 || vals[i] > vals[best]) best = i; /* strict: earlier index wins ties */
        }
        taken[best] = 1;
        out_v[r] = vals[best];
        out_i[r] = best;
    }
}

typedef struct {
    const float *logits;
    int J1, J2, sub, count, bf16;
    int64_t *out_idx;
    float *out_w;
    int err;
} route_ctx;

static void route_range(int64_t lo, int64_t hi, void *arg) {
    route_ctx *c = (route_ctx *)arg;
    const int J1 = c->J1, J2 = c->J2, sub = c->sub, count = c->count, npairs = sub * sub;
    int nmax = J1 > J2 ? J1 : J2;
    if (npairs > nmax) nmax = npairs;
    unsigned char *taken = (unsigned char *)malloc((size_t)nmax);
    float *fv = (float *)malloc(sizeof(float) * (size_t)sub * 2);
    int *fi = (int *)malloc(sizeof(int) * (size_t)sub * 2);
    float *pv = (float *)malloc(sizeof(float) * (size_t)npairs);
    float *cv = (float *)malloc(sizeof(float) * (size_t)count);
    int *ci = (int *)malloc(sizeof(int) * (size_t)count);
    float *ex = (float *)malloc(sizeof(float) * (size_t)count);
    if (!taken || !fv || !fi || !pv || !cv || !ci || !ex) {
        c->err = ORACLE_ENOMEM;
    } else {
        float *sv = fv + sub;
        int *si = fi + sub;
        for (int64_t t = lo; t < hi; ++t) {
            const float *z = c->logits + t * (int64_t)(J1 + J2);
            stable_topk(z, J1, sub, taken, fv, fi);
            stable_topk(z + J1, J2, sub, taken, sv, si);
            /* pair sums in the logits dtype, pair index i*sub + l (gdn2_banks.py:106-110) */
            for (int i = 0; i < sub; ++i)
                for (int l = 0; l < sub; ++l) pv[i * sub + l] = rnd(fv[i] + sv[l], c->bf16);
            stable_topk(pv, npairs, count, taken, cv, ci);
            /* softmax in FP32 (gdn2_banks.py:114) */
            float mx = cv[0];
            for (int r = 1; r < count; ++r) mx = cv[r] > mx ? cv[r] : mx;
            float sum = 0.f;
            for (int r = 0; r < count; ++r) {
                ex[r] = expf(cv[r] - mx);
                sum += ex[r];
            }
            for (int r = 0; r < count; ++r) {
                int row = fi[ci[r] / sub];
                int col = si[ci[r] % sub];
                c->out_idx[t * count + r] = (int64_t)row * J2 + col;
                c->out_w[t * count + r] = rnd(ex[r] / sum, c->bf16);
            }
        }
    }
    free(taken); free(fv); free(fi); free(pv); free(cv); free(ci); free(ex);
}

/*
 * Product-key top-B routing (gdn2_banks.py:74-114).
 * logits [ntok, J1+J2] hold values already representable in the logits dtype.
 * Outputs: out_idx [ntok, count] int64, out_w [ntok, count] (softmax in FP32,
 * then rounded to the logits dtype), count = min(B, sub*sub), sub = min(B, J1, J2).
 */
int oracle_route(const float *logits, int64_t ntok, int J1, int J2, int B, int bf16, int64_t *out_idx,
                 float *out_w) {
    if (ntok < 0 || J1 <= 0 || J2 <= 0 || B <= 0) return ORACLE_EINVAL;
    int sub = B < J1 ? B : J1;
    sub = sub < J2 ? sub : J2;
    int count = B < sub * sub ? B : sub * sub;
    route_ctx c = {logits, J1, J2, sub, count, bf16, out_idx, out_w, ORACLE_OK};
    par_for(ntok, 256, route_range, &c);
    return c.err;
}

/* ----------------------------------------------------------------- dispatch */

/*
 * Causal bank dispatch (gdn2_banks.py:174-185, 237-246).
 * Event ids: write (token, slot) -> token*KW + slot; read -> NT*KW + token*KR + slot.
 * Key ((b*J + bank)*T + t)*2 + role; events are ordered by key.  Equal keys
 * (only possible when one role names a bank twice for a token) keep event-id
 * order.  Outputs: order[E] (event id at each packed position), inverse[E],
 * tokens[E] (token of each packed position), cu[batch*J + 1].
 */
int oracle_dispatch(const int64_t *wi, const int64_t *ri, int64_t batch, int64_t time, int KW, int KR,
                    int64_t J, int64_t *order, int64_t *inverse, int64_t *tokens, int64_t *cu) {
    int64_t nt = batch * time;
    int64_t nseq = batch * J;
    for (int64_t i = 0; i < nt * KW; ++i)
        if (wi[i] < 0 || wi[i] >= J) return ORACLE_EINVAL;
    for (int64_t i = 0; i < nt * KR; ++i)
        if (ri[i] < 0 || ri[i] >= J) return ORACLE_EINVAL;
    int64_t *fill = (int64_t *)calloc((size_t)nseq + 1, sizeof(int64_t));
    if (!fill) return ORACLE_ENOMEM;
    memset(cu, 0, sizeof(int64_t) * (size_t)(nseq + 1));
    for (int64_t tok = 0; tok < nt; ++tok) {
        int64_t b = tok / time;
        for (int s = 0; s < KW; ++s) cu[b * J + wi[tok * KW + s] + 1]++;
        for (int s = 0; s < KR; ++s) cu[b * J + ri[tok * KR + s] + 1]++;
    }
    for (int64_t s = 0; s < nseq; ++s) cu[s + 1] += cu[s];
    for (int64_t tok = 0; tok < nt; ++tok) {
        int64_t b = tok / time;
        for (int role = 0; role < 2; ++role) {
            int K = role ? KR : KW;
            const int64_t *idx = role ? ri : wi;
            for (int s = 0; s < K; ++s) {
                int64_t seq = b * J + idx[tok * K + s];
                int64_t pos = cu[seq] + fill[seq]++;
                int64_t id = role ? nt * KW + tok * KR + s : tok * KW + s;
                order[pos] = id;
                inverse[id] = pos;
                tokens[pos] = tok;
            }
        }
    }
    free(fill);
    return ORACLE_OK;
}

/* --------------------------------------------------------------- recurrence */

typedef struct {
    const float *q, *k, *v, *g, *b, *w, *ww, *rw, *init;
    const int64_t *order, *cu;
    int64_t init_batch, nt, J;
    int H, S, dv, KW, KR, bf16, routed_decay, interval;
    float scale;
    float *reads, *final_state;
    int err;
} rec_ctx;

static void rec_range(int64_t lo, int64_t hi, void *arg) {
    rec_ctx *c = (rec_ctx *)arg;
    const int H = c->H, S = c->S, dv = c->dv, KW = c->KW, KR = c->KR, bf16 = c->bf16;
    const int64_t nt = c->nt, J = c->J, V = (int64_t)H * dv, se = (int64_t)S * dv;
    float *st = (float *)malloc(sizeof(float) * (size_t)se);
    float *a = (float *)malloc(sizeof(float) * (size_t)S);
    float *ge = (float *)malloc(sizeof(float) * (size_t)S);
    float *qe = (float *)malloc(sizeof(float) * (size_t)S);
    float *er = (float *)malloc(sizeof(float) * (size_t)dv);
    if (!st || !a || !ge || !qe || !er) {
        c->err = ORACLE_ENOMEM;
        free(st); free(a); free(ge); free(qe); free(er);
        return;
    }
    for (int64_t task = lo; task < hi; ++task) {
        int64_t seq = task / H;
        int h = (int)(task % H);
        int64_t bb = seq / J, bank = seq % J;
        const float *src = c->init + ((((bb % c->init_batch) * J + bank) * H + h) * se);
        for (int64_t i = 0; i < se; ++i) st[i] = c->interval > 0 ? bf16r(src[i]) : src[i];
        int64_t start = c->cu[seq], end = c->cu[seq + 1];
        for (int64_t pos = start; pos < end; ++pos) {
            /* stored-state precision (gdn2_banks.py:35-36) */
            if (c->interval > 0 && (pos - start) % c->interval == 0)
                for (int64_t i = 0; i < se; ++i) st[i] = bf16r(st[i]);
            int64_t id = c->order[pos];
            if (id < nt * KW) {
                int64_t tok = id / KW;
                float p = c->ww[id];
                const float *kk = c->k + (tok * H + h) * S;
                const float *gg = c->g + (tok * H + h) * S;
                const float *bt = c->b + (tok * H + h) * S;
                const float *vv = c->v + (tok * H + h) * dv;
                const float *wt = c->w + (tok * H + h) * dv;
                for (int s = 0; s < S; ++s) {
                    ge[s] = c->routed_decay ? gg[s] * p : gg[s];
                    a[s] = rnd(bt[s] * p, bf16) * kk[s];
                }
                for (int s = 0; s < S; ++s) {
                    float d = expf(ge[s]);
                    float *row = st + (int64_t)s * dv;
                    for (int x = 0; x < dv; ++x) row[x] = row[x] * d;
                }
                for (int x = 0; x < dv; ++x) er[x] = 0.f;
                for (int s = 0; s < S; ++s) {
                    const float *row = st + (int64_t)s * dv;
                    for (int x = 0; x < dv; ++x) er[x] = er[x] + a[s] * row[x];
                }
                for (int x = 0; x < dv; ++x) er[x] = rnd(wt[x] * p, bf16) * vv[x] - er[x];
                for (int s = 0; s < S; ++s) {
                    float *row = st + (int64_t)s * dv;
                    for (int x = 0; x < dv; ++x) row[x] = row[x] + kk[s] * er[x];
                }
            } else {
                int64_t rid = id - nt * KW;
                int64_t tok = rid / KR;
                float r = c->rw[rid];
                const float *qq = c->q + (tok * H + h) * S;
                for (int s = 0; s < S; ++s) qe[s] = rnd(qq[s] * r, bf16);
                for (int x = 0; x < dv; ++x) er[x] = 0.f;
                for (int s = 0; s < S; ++s) {
                    const float *row = st + (int64_t)s * dv;
                    for (int x = 0; x < dv; ++x) er[x] = er[x] + qe[s] * row[x];
                }
                float *out = c->reads + rid * V + (int64_t)h * dv;
                for (int x = 0; x < dv; ++x) out[x] = rnd(c->scale * er[x], bf16);
            }
        }
        if (c->final_state) memcpy(c->final_state + (((bb * J + bank) * H + h) * se), st, sizeof(float) * (size_t)se);
    }
    free(st); free(a); free(ge); free(qe); free(er);
}

/*
 * Bank recurrence over dispatched events (pack_bank_events + reference_packed_gdn2).
 *
 * Token-level inputs (values already representable in the activation dtype):
 *   q,k,b,g [NT, H, S]   v,w [NT, H, dv]   wi,ww [NT, KW]   ri,rw [NT, KR]
 *   init [init_batch, J, H, S, dv] (init_batch 1 broadcasts over the batch)
 * Packing (gdn2_banks.py:201-224), rounded to the activation dtype:
 *   read  q_e = q*r                  write b_e = b*p, w_e = w*p (per value column)
 *   write g_e = g*p in FP32 when routed_decay, else g
 * Recurrence (gdn2_banks.py:34-42), FP32, per event of one (batch, bank, head):
 *   if interval > 0 and i % interval == 0: state = bf16(state)   (storage policy)
 *   write: state *= exp(g_e); erase = sum_s (b_e*k)[s]*state[s,:];
 *          state += k (x) (w_e*v - erase)
 *   read:  out = scale * sum_s q_e[s]*state[s,:]   (rounded to activation dtype)
 * Read events leave the state unchanged (their packed g, b, w are zero).
 * Read outputs land at reads[(token*KR + slot), h*dv + c]; final_state (may be
 * NULL) receives the FP32 state after the last event [batch, J, H, S, dv].
 */
int oracle_recurrence(const float *q, const float *k, const float *v, const float *g, const float *b,
                      const float *w, const int64_t *wi, const float *ww, const int64_t *ri, const float *rw,
                      const float *init, int64_t init_batch, int64_t batch, int64_t time, int64_t J, int H,
                      int S, int dv, int KW, int KR, int bf16, int routed_decay, int interval, float scale,
                      float *reads, float *final_state) {
    int64_t nt = batch * time;
    int64_t E = nt * (KW + KR);
    int64_t nseq = batch * J;
    if (S <= 0 || S > 256 || dv <= 0 || H <= 0 || (init_batch != 1 && init_batch != batch)) return ORACLE_EINVAL;
    size_t ecap = (size_t)(E ? E : 1);
    int64_t *order = (int64_t *)malloc(sizeof(int64_t) * ecap);
    int64_t *inverse = (int64_t *)malloc(sizeof(int64_t) * ecap);
    int64_t *tokens = (int64_t *)malloc(sizeof(int64_t) * ecap);
    int64_t *cu = (int64_t *)malloc(sizeof(int64_t) * (size_t)(nseq + 1));
    int rc = ORACLE_ENOMEM;
    if (order && inverse && tokens && cu) rc = oracle_dispatch(wi, ri, batch, time, KW, KR, J, order, inverse, tokens, cu);
    if (rc == ORACLE_OK) {
        rec_ctx c = {q, k, v, g, b, w, ww, rw, init, order, cu, init_batch, nt, J, H, S, dv, KW, KR,
                     bf16, routed_decay, interval, scale, reads, final_state, ORACLE_OK};
        par_for(nseq * H, 4, rec_range, &c);
        rc = c.err;
    }
    free(order); free(inverse); free(tokens); free(cu);
    return rc;
}

/* ------------------------------------------------------------------ combine */

typedef struct {
    const float *reads;
    const int64_t *ri;
    int KR, bf16, round_each;
    int64_t V;
    float *raw;
} comb_ctx;

static void comb_range(int64_t lo, int64_t hi, void *arg) {
    comb_ctx *c = (comb_ctx *)arg;
    const int KR = c->KR;
    const int64_t V = c->V;
    int slots[256];
    for (int64_t t = lo; t < hi; ++t) {
        for (int s = 0; s < KR; ++s) slots[s] = s;
        for (int i = 1; i < KR; ++i) { /* insertion sort: stable */
            int cur = slots[i], j = i - 1;
            while (j >= 0 && c->ri[t * KR + slots[j]] > c->ri[t * KR + cur]) {
                slots[j + 1] = slots[j];
                --j;
            }
            slots[j + 1] = cur;
        }
        float *out = c->raw + t * V;
        for (int64_t x = 0; x < V; ++x) out[x] = 0.f;
        for (int s = 0; s < KR; ++s) {
            const float *row = c->reads + (t * KR + slots[s]) * V;
            for (int64_t x = 0; x < V; ++x) out[x] = rnd(out[x] + row[x], c->bf16 && c->round_each);
        }
        if (c->bf16 && !c->round_each)
            for (int64_t x = 0; x < V; ++x) out[x] = bf16r(out[x]);
    }
}

/*
 * Per-token read combine: sum the KR read rows of a token in ascending bank
 * order (ties: lower slot first), starting from zero.
 *   round_each = 0: FP32 accumulation, one rounding to the activation dtype at
 *     the end.  This is what the CPU reference's BF16 index_add_ does
 *     (gdn2_banks.py:265-283, checked against torch on CPU).
 *   round_each = 1: rounding after every add, as the reference's GPU readouts
 *     do (role_bank_dispatch.py:201-216, inference.py:53-85).
 * reads [ntok, KR, V] -> raw [ntok, V].
 */
int oracle_combine(const float *reads, const int64_t *ri, int64_t ntok, int KR, int64_t V, int bf16, int round_each,
                   float *raw) {
    if (KR <= 0 || KR > 256) return ORACLE_EINVAL;
    comb_ctx c = {reads, ri, KR, bf16, round_each, V, raw};
    par_for(ntok, 64, comb_range, &c);
    return ORACLE_OK;
}

/* ------------------------------------------------------------------- decode */

/* Eight-term tree used by the reference decode read (forward_rows.py:5-7). */
static inline float sum8(const float *x) { return ((x[0] + x[1]) + (x[4] + x[5])) + ((x[2] + x[3]) + (x[6] + x[7])); }

typedef struct {
    const float *q, *k, *v, *g, *b, *w, *ww, *rw;
    const int64_t *wi, *ri;
    float *state, *reads;
    int64_t J;
    int H, S, dv, KW, KR, bf16, cache_bf16, routed_decay;
    float scale;
} dec_ctx;

static void dec_range(int64_t lo, int64_t hi, void *arg) {
    dec_ctx *c = (dec_ctx *)arg;
    const int H = c->H, S = c->S, dv = c->dv, KW = c->KW, KR = c->KR, bf16 = c->bf16;
    const int64_t J = c->J, V = (int64_t)H * dv, se = (int64_t)S * dv;
    float a[256], ge[256], qe[256], hd[256], prod[256];
    for (int64_t bb = lo; bb < hi; ++bb) {
        for (int j = 0; j < KW; ++j) {
            int64_t bank = c->wi[bb * KW + j];
            float p = c->ww[bb * KW + j];
            for (int h = 0; h < H; ++h) {
                float *st = c->state + ((bb * J + bank) * H + h) * se;
                const float *kk = c->k + (bb * H + h) * S, *gg = c->g + (bb * H + h) * S;
                const float *bt = c->b + (bb * H + h) * S;
                const float *vv = c->v + (bb * H + h) * dv, *wt = c->w + (bb * H + h) * dv;
                for (int s = 0; s < S; ++s) {
                    ge[s] = c->routed_decay ? gg[s] * p : gg[s];
                    a[s] = rnd(bt[s] * p, bf16) * kk[s];
                }
                for (int x = 0; x < dv; ++x) {
                    float erase = 0.f;
                    for (int s = 0; s < S; ++s) hd[s] = st[(int64_t)s * dv + x] * expf(ge[s]);
                    for (int s = 0; s < S; ++s) erase = erase + a[s] * hd[s];
                    float u = rnd(wt[x] * p, bf16) * vv[x] - erase;
                    for (int s = 0; s < S; ++s) st[(int64_t)s * dv + x] = rnd(hd[s] + kk[s] * u, c->cache_bf16);
                }
            }
        }
        for (int j = 0; j < KR; ++j) {
            int64_t bank = c->ri[bb * KR + j];
            float r = c->rw[bb * KR + j];
            for (int h = 0; h < H; ++h) {
                const float *st = c->state + ((bb * J + bank) * H + h) * se;
                const float *qq = c->q + (bb * H + h) * S;
                for (int s = 0; s < S; ++s) qe[s] = rnd(qq[s] * r, bf16);
                float *out = c->reads + (bb * KR + j) * V + (int64_t)h * dv;
                for (int x = 0; x < dv; ++x) {
                    float acc;
                    for (int s = 0; s < S; ++s) prod[s] = st[(int64_t)s * dv + x] * qe[s];
                    if (S == 8) {
                        acc = sum8(prod);
                    } else {
                        acc = 0.f;
                        for (int s = 0; s < S; ++s) acc = acc + prod[s];
                    }
                    out[x] = rnd(acc * c->scale, bf16);
                }
            }
        }
    }
}

/*
 * One decode token per batch row (inference.py:161-194).
 *   token-level q,k,b,g [batch, H, S], v,w [batch, H, dv], routes [batch, KW|KR]
 *   state [batch, J, H, S, dv] holds cache-dtype values and is updated in place.
 * All B write banks of a row update first (distinct banks), each stored back in
 * the cache dtype (inference.py:21-34); then reads q_e = q*r (activation
 * dtype) see the updated banks (inference.py:37-50), each rounded to the
 * activation dtype, and are summed in ascending bank order with a rounding
 * after each add (inference.py:53-67).  raw [batch, H*dv].
 */
int oracle_decode_step(const float *q, const float *k, const float *v, const float *g, const float *b,
                       const float *w, const int64_t *wi, const float *ww, const int64_t *ri, const float *rw,
                       float *state, int64_t batch, int64_t J, int H, int S, int dv, int KW, int KR, int bf16,
                       int cache_bf16, int routed_decay, float scale, float *raw) {
    if (S <= 0 || S > 256 || KR <= 0 || KR > 256 || KW <= 0 || KW > 256) return ORACLE_EINVAL;
    const int64_t V = (int64_t)H * dv;
    float *reads = (float *)malloc(sizeof(float) * (size_t)(batch * KR * V));
    if (!reads) return ORACLE_ENOMEM;
    dec_ctx c = {q, k, v, g, b, w, ww, rw, wi, ri, state, reads, J, H, S, dv, KW, KR, bf16, cache_bf16,
                 routed_decay, scale};
    par_for(batch, 1, dec_range, &c);
    int rc = oracle_combine(reads, ri, batch, KR, V, bf16, 1, raw);
    free(reads);
    return rc;
}
