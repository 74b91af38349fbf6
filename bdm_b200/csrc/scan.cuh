// Launch parameters and work-list constants shared by the bank recurrence kernels
// (per-event kernels in recurrence.cu, chunked tensor-core kernel in chunk_scan.cu)
// and the recurrence backward (backward.cu).
#pragma once

#include "common.cuh"

namespace bdm {

struct ScanParams {
    const void *q, *k, *v;
    const float *g;
    const void *b, *w;
    const int64_t *wi, *ri;
    const void *ww, *rw;
    const int64_t *order, *cu;
    int64_t batch, time, J, nt, nw, E;
    int H, dv, kw, kr, routed_decay, ctiles;
    float scale;
    const void *row_factor, *col_factor;
    int64_t factor_cols;
    int factor_dtype;
    const int32_t *bank_ids;  // local bank -> bank of the full table (bank-sharded ranks), or null
    int64_t total_banks;
    int head_offset, total_heads;  // this call's heads are [head_offset, head_offset + H) of total_heads
    void *cache;
    int cache_dtype, store_final, interval;
    void *reads;
    int64_t units;        // (sequence, head, column tile) units when every sequence runs
    // Work list: non-empty sequences grouped by length class, longest class first.
    const int *lists;     // kLenClasses lists of capacity nseq
    const int *counts;    // [kLenClasses] list lengths
    unsigned long long *next;  // dynamic work counter (zero at launch)
    unsigned long long *long_next;  // the long kernel's work counter (zero at launch)
    unsigned long long *chunk_next;  // the chunked kernel's work counter (zero at launch)
    int *status;               // error bits (BDM_SCAN_ERR_*), zero at launch
    int ws_classes;            // length classes run by warp-specialised CTAs (0: none)
    int64_t ws_ctas;           // CTAs [0, ws_ctas) run those units
    int64_t nseq;
    // Training: the state before every ckpt_block-th event of a sequence (position > 0) is
    // written to ckpt[(start / ckpt_block + seq + pos / ckpt_block), head, S, dv] for the
    // recurrence backward (short-kernel sequences only; null / 0 when off).
    float *ckpt;
    int ckpt_block;
    int chunked;  // run the non-long classes on the tensor-core chunked kernel (chunk_scan.cu)
    // Diagnostics (bdm_scan_test_fault): the long kernel's bounded-wait limit in ns (0: 2 s) and
    // a test fault (1: its producer withholds the first batch hand-off, so the waits run out).
    unsigned long long wait_ns;
    int test_fault;
};

// Length classes of the work list (events per sequence, lower bounds), longest first.
// Inside a class sequences keep ascending (batch, bank) order, so warps running
// at the same time mostly read the same batch row's token rows (L2 locality).
constexpr int kLenClasses = 4;
constexpr int kWsClasses = 1;           // class 0 (the long sequences) runs warp-specialised
constexpr int64_t kLongEvents = 2048;   // a long sequence has at least this many events
constexpr int BDM_SCAN_ERR_TIMEOUT = 1;  // a producer/consumer or tensor-core wait gave up
constexpr float kMinLogDecay = -60.0f;  // floor of one event's log-decay (and of a deferred-decay segment)

// Events per chunk of the tensor-core recurrence: the BF16 state-storage interval of the
// reference (role_bank_kernel.py:153, model.py:131: min(16, max(4, 128 / next_pow2(S)))),
// so every chunk start is a storage point.
__host__ __device__ constexpr int chunk_events(int S) { return S >= 16 ? 8 : 16; }

// Whether the tensor-core chunked recurrence can take a launch (BF16 operands, 128-column tiles,
// storage points at chunk starts or none, no backward checkpoints), and its launcher: runs the
// work-list classes [p.ws_classes, kLenClasses) on the caller's stream.
bool chunk_scan_eligible(const ScanParams &p, int dtype, int S);
int launch_chunk_scan(const ScanParams &p, int S, cudaStream_t st, bool programmatic);

}  // namespace bdm
