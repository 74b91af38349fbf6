// Causal bank dispatch: a stable counting sort of routed events by (batch, bank).
//
// The reference builds the key ((b*J + bank)*T + t)*2 + role for every event
// and runs a full 64-bit torch.sort (role_bank_dispatch.py:15-24,143-153;
// gdn2_banks.py:181-185).  Enumerating events in (batch, t, role, slot) order
// makes that order the stable order of the sequence id b*J + bank alone, so
// this file sorts only ceil(log2(batch*J)) bits with LSD radix passes of at
// most 11 bits:
//   upsweep    per-tile digit histogram in shared memory -> tile table
//   scan       exclusive scan of the digit-major tile table
//   downsweep  per-warp counts (warp match_any aggregation), cross-warp
//              offsets, then a stable scatter ranked with match_any/popc
// cu_seqlens comes from a lower-bound search per sequence over the sorted
// sequence ids (the reference's _bounds, role_bank_dispatch.py:27-38).
//
// Bank-sharded ranks sort with an ownership map instead: an event whose bank
// this rank owns gets the sequence id b*J_local + slot(bank); every other event
// gets the id one past the last sequence, so it sorts after all owned events
// and cu_seqlens[B*J_local] is the owned event count.
#include "common.cuh"

#include <mutex>

namespace bdm {
namespace {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kItemsPerThread = 16;
constexpr int kTile = kSortThreads * kItemsPerThread;  // 4096 items per tile
constexpr int kWarpItems = kTile / kSortWarps;           // 512 items per warp
constexpr int kMaxRadixBits = 11;

constexpr int kScanThreads = 1024;
constexpr int kScanItems = 4;
constexpr int kScanBlock = kScanThreads * kScanItems;   // 4096
constexpr int64_t kScanMax = (int64_t)kScanBlock * kScanBlock;

// Pass-0 source: events enumerated in (token, role, slot) order.
struct EventSource {
    const int64_t *wi, *ri;
    int64_t nt, time, J;
    int kw, kr;
    int32_t *err;
    // Optional ownership map: owner[bank] == rank selects the event, slot[bank] is
    // its local bank; unselected events get sequence id `sentinel`.
    const int32_t *owner, *slot;
    int rank;
    int64_t local_banks, sentinel;
    __device__ __forceinline__ void get(int64_t i, uint32_t &seq, uint32_t &id, bool count_errors) const {
        const int per = kw + kr;
        int64_t tok = i / per;
        int r = (int)(i - tok * per);
        int64_t bank;
        if (r < kw) {
            bank = wi[tok * kw + r];
            id = (uint32_t)(tok * kw + r);
        } else {
            bank = ri[tok * kr + (r - kw)];
            id = (uint32_t)(nt * kw + tok * kr + (r - kw));
        }
        if (bank < 0 || bank >= J) {
            if (count_errors && err) atomicAdd(err, 1);
            bank = bank < 0 ? 0 : J - 1;  // keep the output a permutation
        }
        if (owner) {
            int64_t l = owner[bank] == rank ? (int64_t)slot[bank] : -1;
            if (l >= local_banks) {
                if (count_errors && err) atomicAdd(err, 1);
                l = -1;
            }
            seq = (uint32_t)(l < 0 ? sentinel : (tok / time) * local_banks + l);
        } else {
            seq = (uint32_t)((tok / time) * J + bank);
        }
    }
};

struct BufferSource {
    const uint32_t *keys, *vals;
    __device__ __forceinline__ void get(int64_t i, uint32_t &seq, uint32_t &id, bool) const {
        seq = keys[i];
        id = vals[i];
    }
};

struct BufferSink {
    uint32_t *keys, *vals;
    __device__ __forceinline__ void put(uint32_t pos, uint32_t seq, uint32_t id) const {
        keys[pos] = seq;
        vals[pos] = id;
    }
};

struct FinalSink {
    uint32_t *keys;
    int64_t *order, *inverse, *tokens;
    int64_t write_events;
    int kw, kr;
    __device__ __forceinline__ void put(uint32_t pos, uint32_t seq, uint32_t id) const {
        keys[pos] = seq;
        order[pos] = id;
        if (inverse) inverse[id] = pos;
        if (tokens) tokens[pos] = (int64_t)id < write_events ? (int64_t)id / kw : ((int64_t)id - write_events) / kr;
    }
};

template <class Src>
__global__ void __launch_bounds__(kSortThreads)
radix_upsweep(Src src, int64_t E, int shift, int rbits, int num_tiles, uint32_t *__restrict__ table, int count_errors) {
    extern __shared__ uint32_t hist[];
    const int radix = 1 << rbits;
    for (int d = threadIdx.x; d < radix; d += kSortThreads) hist[d] = 0;
    __syncthreads();
    const int64_t base = (int64_t)blockIdx.x * kTile;
#pragma unroll 4
    for (int j = 0; j < kItemsPerThread; ++j) {
        int64_t i = base + (int64_t)j * kSortThreads + threadIdx.x;
        if (i < E) {
            uint32_t seq, id;
            src.get(i, seq, id, count_errors != 0);
            atomicAdd(&hist[(seq >> shift) & (uint32_t)(radix - 1)], 1u);
        }
    }
    __syncthreads();
    for (int d = threadIdx.x; d < radix; d += kSortThreads) table[(int64_t)d * num_tiles + blockIdx.x] = hist[d];
}

template <class Src, class Sink>
__global__ void __launch_bounds__(kSortThreads)
radix_downsweep(Src src, Sink sink, int64_t E, int shift, int rbits, int num_tiles,
                const uint32_t *__restrict__ offsets) {
    extern __shared__ uint32_t cnt[];  // [kSortWarps][radix]
    const int radix = 1 << rbits;
    const uint32_t mask = (uint32_t)(radix - 1);
    for (int d = threadIdx.x; d < kSortWarps * radix; d += kSortThreads) cnt[d] = 0;
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    const unsigned lane = lane_id();
    const unsigned lt_mask = (1u << lane) - 1u;
    uint32_t *wc = cnt + warp * radix;
    const int64_t wbase = (int64_t)blockIdx.x * kTile + (int64_t)warp * kWarpItems;
    // A: per-warp digit counts, aggregated over equal digits with match_any.
    for (int c = 0; c < kWarpItems / 32; ++c) {
        int64_t i = wbase + c * 32 + lane;
        bool valid = i < E;
        uint32_t seq = 0, id = 0, d = 0xffffffffu;
        if (valid) {
            src.get(i, seq, id, false);
            d = (seq >> shift) & mask;
        }
        unsigned peers = __match_any_sync(0xffffffffu, d);
        if (valid && (unsigned)(__ffs(peers) - 1) == lane) wc[d] += (uint32_t)__popc(peers);
    }
    __syncthreads();
    // B: exclusive offsets across warps, seeded with this tile's global digit offset.
    for (int d = threadIdx.x; d < radix; d += kSortThreads) {
        uint32_t run = offsets[(int64_t)d * num_tiles + blockIdx.x];
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) {
            uint32_t t = cnt[w * radix + d];
            cnt[w * radix + d] = run;
            run += t;
        }
    }
    __syncthreads();
    // C: stable scatter in item order.
    for (int c = 0; c < kWarpItems / 32; ++c) {
        int64_t i = wbase + c * 32 + lane;
        bool valid = i < E;
        uint32_t seq = 0, id = 0, d = 0xffffffffu;
        if (valid) {
            src.get(i, seq, id, false);
            d = (seq >> shift) & mask;
        }
        unsigned peers = __match_any_sync(0xffffffffu, d);
        if (valid) sink.put(wc[d] + (uint32_t)__popc(peers & lt_mask), seq, id);
        __syncwarp();
        if (valid && (unsigned)(__ffs(peers) - 1) == lane) wc[d] += (uint32_t)__popc(peers);
        __syncwarp();
    }
}

// ----------------------------------------------------------------- scan

// Exclusive scan of one value per thread over a 1024-thread block.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t *warp_tot, uint32_t &total) {
    const unsigned lane = lane_id();
    const int warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= (unsigned)o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
        uint32_t t = warp_tot[lane];
        uint32_t s = t;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= (unsigned)o) s += y;
        }
        warp_tot[lane] = s - t;
        if (lane == 31) warp_tot[32] = s;
    }
    __syncthreads();
    uint32_t excl = x - v + warp_tot[warp];
    total = warp_tot[32];
    __syncthreads();
    return excl;
}

__global__ void __launch_bounds__(kScanThreads) scan_block_sums(const uint32_t *__restrict__ in, int64_t n,
                                                                 uint32_t *__restrict__ sums) {
    __shared__ uint32_t warp_tot[33];
    const int64_t base = (int64_t)blockIdx.x * kScanBlock + (int64_t)threadIdx.x * kScanItems;
    uint32_t s = 0;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j)
        if (base + j < n) s += in[base + j];
    uint32_t total;
    block_exclusive_scan(s, warp_tot, total);
    if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kScanThreads) scan_single(uint32_t *__restrict__ data, int64_t n) {
    __shared__ uint32_t warp_tot[33];
    const int64_t base = (int64_t)threadIdx.x * kScanItems;
    uint32_t v[kScanItems];
    uint32_t s = 0;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        v[j] = base + j < n ? data[base + j] : 0u;
        s += v[j];
    }
    uint32_t total;
    uint32_t run = block_exclusive_scan(s, warp_tot, total);
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        if (base + j < n) data[base + j] = run;
        run += v[j];
    }
}

__global__ void __launch_bounds__(kScanThreads) scan_apply(const uint32_t *__restrict__ in, uint32_t *__restrict__ out,
                                                            int64_t n, const uint32_t *__restrict__ sums) {
    __shared__ uint32_t warp_tot[33];
    const int64_t base = (int64_t)blockIdx.x * kScanBlock + (int64_t)threadIdx.x * kScanItems;
    uint32_t v[kScanItems];
    uint32_t s = 0;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        v[j] = base + j < n ? in[base + j] : 0u;
        s += v[j];
    }
    uint32_t total;
    uint32_t run = block_exclusive_scan(s, warp_tot, total) + sums[blockIdx.x];
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        if (base + j < n) out[base + j] = run;
        run += v[j];
    }
}

// Exclusive scan in place; `sums` holds ceil(n / 4096) entries.
int exclusive_scan(uint32_t *data, int64_t n, uint32_t *sums, cudaStream_t st) {
    if (n <= 0) return BDM_OK;
    if (n > kScanMax) return BDM_ERR_UNSUPPORTED;
    int64_t blocks = ceil_div(n, kScanBlock);
    if (blocks == 1) {
        scan_single<<<1, kScanThreads, 0, st>>>(data, n);
        return launch_status();
    }
    scan_block_sums<<<(unsigned)blocks, kScanThreads, 0, st>>>(data, n, sums);
    int rc = launch_status();
    if (rc) return rc;
    scan_single<<<1, kScanThreads, 0, st>>>(sums, blocks);
    rc = launch_status();
    if (rc) return rc;
    scan_apply<<<(unsigned)blocks, kScanThreads, 0, st>>>(data, data, n, sums);
    return launch_status();
}

// cu[x] = first position whose sequence id is >= x (x in [0, nseq]).
__global__ void seq_bounds(const uint32_t *__restrict__ keys, int64_t E, int64_t nseq, int64_t *__restrict__ cu) {
    for (int64_t x = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; x <= nseq; x += (int64_t)gridDim.x * blockDim.x) {
        int64_t lo = 0, hi = E;
        while (lo < hi) {
            int64_t mid = (lo + hi) >> 1;
            if ((int64_t)keys[mid] < x) lo = mid + 1;
            else hi = mid;
        }
        cu[x] = lo;
    }
}

struct Plan {
    int64_t E, nseq, tiles;
    int bits, passes, rb;
    int64_t table, sums;  // entries
    int64_t off_final, off_ak, off_av, off_bk, off_bv, off_table, off_sums, bytes;
};

inline int64_t align256(int64_t x) { return (x + 255) & ~(int64_t)255; }

// Workspace: final sorted sequence ids, two ping-pong (key, id) buffers for
// intermediate passes, the digit-major tile table and the scan block sums.
// With `sentinel` the sort also carries the id nseq (events of other ranks).
Plan make_plan(int64_t batch, int64_t time, int kw, int kr, int64_t J, bool sentinel = false) {
    Plan p{};
    p.E = batch * time * (int64_t)(kw + kr);
    p.nseq = batch * J;
    p.tiles = ceil_div(p.E > 0 ? p.E : 1, kTile);
    int bits = 0;
    while (bits < 32 && ((int64_t)1 << bits) < p.nseq + (sentinel ? 1 : 0)) ++bits;
    if (bits == 0) bits = 1;
    p.bits = bits;
    p.passes = (bits + kMaxRadixBits - 1) / kMaxRadixBits;
    p.rb = (bits + p.passes - 1) / p.passes;
    p.table = ((int64_t)1 << p.rb) * p.tiles;
    p.sums = ceil_div(p.table, kScanBlock);
    const int64_t e4 = align256((p.E > 0 ? p.E : 1) * 4);
    int64_t off = 0;
    p.off_final = off; off += e4;
    p.off_ak = off;    off += p.passes > 1 ? e4 : 0;
    p.off_av = off;    off += p.passes > 1 ? e4 : 0;
    p.off_bk = off;    off += p.passes > 2 ? e4 : 0;
    p.off_bv = off;    off += p.passes > 2 ? e4 : 0;
    p.off_table = off; off += align256(p.table * 4);
    p.off_sums = off;  off += align256(p.sums * 4);
    p.bytes = off;
    return p;
}

template <class Src, class Sink>
int set_down_smem(size_t bytes) {
    if (bytes <= 48 * 1024) return BDM_OK;
    return cuda_status(cudaFuncSetAttribute(radix_downsweep<Src, Sink>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)bytes));
}

template <class Src, class Sink>
int run_pass(const Src &src, const Sink &sink, const Plan &p, int shift, int rbits, bool first, uint32_t *table,
             uint32_t *sums, cudaStream_t st) {
    const int tiles = (int)p.tiles;
    const size_t up_smem = sizeof(uint32_t) << rbits;
    const size_t down_smem = (size_t)kSortWarps * (sizeof(uint32_t) << rbits);
    radix_upsweep<Src><<<tiles, kSortThreads, up_smem, st>>>(src, p.E, shift, rbits, tiles, table, first ? 1 : 0);
    int rc = launch_status();
    if (rc) return rc;
    rc = exclusive_scan(table, ((int64_t)1 << rbits) * tiles, sums, st);
    if (rc) return rc;
    rc = set_down_smem<Src, Sink>(down_smem);
    if (rc) return rc;
    radix_downsweep<Src, Sink><<<tiles, kSortThreads, down_smem, st>>>(src, sink, p.E, shift, rbits, tiles, table);
    return launch_status();
}

}  // namespace
}  // namespace bdm

extern "C" int64_t bdm_dispatch_workspace_bytes(int64_t batch, int64_t time, int kw, int kr, int64_t bank_count) {
    if (batch <= 0 || time <= 0 || kw <= 0 || kr <= 0 || bank_count <= 0) return -1;
    return bdm::make_plan(batch, time, kw, kr, bank_count).bytes;
}

namespace bdm {
namespace {

// owner == nullptr: plain dispatch over bank_count banks; otherwise only the
// events of banks with owner[bank] == rank, as local_banks sequences per batch row.
int dispatch_impl(const int64_t *write_idx, const int64_t *read_idx, int64_t batch, int64_t time, int kw, int kr,
                  int64_t bank_count, const int32_t *owner, const int32_t *slot, int rank, int64_t local_banks,
                  int64_t *order, int64_t *cu_seqlens, int64_t *inverse, int64_t *tokens, int32_t *error_word,
                  void *workspace, int64_t workspace_bytes, cudaStream_t st) {
    const bool owned = owner != nullptr;
    const int64_t seq_banks = owned ? local_banks : bank_count;
    Plan p = make_plan(batch, time, kw, kr, seq_banks, owned);
    if (p.E >= ((int64_t)1 << 32) - 1 || p.nseq >= ((int64_t)1 << 32) - 2) return BDM_ERR_UNSUPPORTED;
    if (p.table > kScanMax) return BDM_ERR_UNSUPPORTED;
    if (!workspace || workspace_bytes < p.bytes) return BDM_ERR_WORKSPACE;
    char *ws = static_cast<char *>(workspace);
    uint32_t *final_keys = reinterpret_cast<uint32_t *>(ws + p.off_final);
    uint32_t *buf_k[2] = {reinterpret_cast<uint32_t *>(ws + p.off_ak), reinterpret_cast<uint32_t *>(ws + p.off_bk)};
    uint32_t *buf_v[2] = {reinterpret_cast<uint32_t *>(ws + p.off_av), reinterpret_cast<uint32_t *>(ws + p.off_bv)};
    uint32_t *table = reinterpret_cast<uint32_t *>(ws + p.off_table);
    uint32_t *sums = reinterpret_cast<uint32_t *>(ws + p.off_sums);

    const int64_t nt = batch * time;
    EventSource src0{write_idx, read_idx, nt, time, bank_count, kw, kr, error_word,
                     owner, slot, rank, local_banks, p.nseq};
    FinalSink fin{final_keys, order, inverse, tokens, nt * kw, kw, kr};
    // Pass k (k < passes-1) writes buffer k%2; pass k > 0 reads buffer (k-1)%2;
    // the last pass writes the outputs.
    for (int pass = 0; pass < p.passes; ++pass) {
        const int shift = pass * p.rb;
        const int rbits = (p.bits - shift) < p.rb ? (p.bits - shift) : p.rb;
        const bool last = pass == p.passes - 1;
        BufferSink mid{buf_k[pass % 2], buf_v[pass % 2]};
        BufferSource prev{buf_k[(pass + 1) % 2], buf_v[(pass + 1) % 2]};
        int rc;
        if (pass == 0)
            rc = last ? run_pass(src0, fin, p, shift, rbits, true, table, sums, st)
                      : run_pass(src0, mid, p, shift, rbits, true, table, sums, st);
        else
            rc = last ? run_pass(prev, fin, p, shift, rbits, false, table, sums, st)
                      : run_pass(prev, mid, p, shift, rbits, false, table, sums, st);
        if (rc) return rc;
    }
    int64_t blocks = ceil_div(p.nseq + 1, 256);
    if (blocks > 64 * kNumSMs) blocks = 64 * kNumSMs;
    seq_bounds<<<(unsigned)blocks, 256, 0, st>>>(final_keys, p.E, p.nseq, cu_seqlens);
    return launch_status();
}

}  // namespace
}  // namespace bdm

extern "C" int bdm_dispatch(const int64_t *write_idx, const int64_t *read_idx, int64_t batch, int64_t time, int kw,
                            int kr, int64_t bank_count, int64_t *order, int64_t *cu_seqlens, int64_t *inverse,
                            int64_t *tokens, int32_t *error_word, void *workspace, int64_t workspace_bytes,
                            void *stream) {
    using namespace bdm;
    if (batch <= 0 || time <= 0 || kw <= 0 || kr <= 0 || bank_count <= 0) return BDM_ERR_INVALID;
    if (!write_idx || !read_idx || !order || !cu_seqlens) return BDM_ERR_INVALID;
    return dispatch_impl(write_idx, read_idx, batch, time, kw, kr, bank_count, nullptr, nullptr, 0, 0, order,
                         cu_seqlens, inverse, tokens, error_word, workspace, workspace_bytes, as_stream(stream));
}

extern "C" int64_t bdm_dispatch_owned_workspace_bytes(int64_t batch, int64_t time, int kw, int kr,
                                                      int64_t local_banks) {
    if (batch <= 0 || time <= 0 || kw <= 0 || kr <= 0 || local_banks <= 0) return -1;
    return bdm::make_plan(batch, time, kw, kr, local_banks, true).bytes;
}

extern "C" int bdm_dispatch_owned(const int64_t *write_idx, const int64_t *read_idx, int64_t batch, int64_t time,
                                  int kw, int kr, int64_t bank_count, const int32_t *owner, const int32_t *slot,
                                  int rank, int64_t local_banks, int64_t *order, int64_t *cu_seqlens,
                                  int64_t *inverse, int64_t *tokens, int32_t *error_word, void *workspace,
                                  int64_t workspace_bytes, void *stream) {
    using namespace bdm;
    if (batch <= 0 || time <= 0 || kw <= 0 || kr <= 0 || bank_count <= 0 || local_banks <= 0 || rank < 0)
        return BDM_ERR_INVALID;
    if (!write_idx || !read_idx || !owner || !slot || !order || !cu_seqlens) return BDM_ERR_INVALID;
    return dispatch_impl(write_idx, read_idx, batch, time, kw, kr, bank_count, owner, slot, rank, local_banks, order,
                         cu_seqlens, inverse, tokens, error_word, workspace, workspace_bytes, as_stream(stream));
}

// ---------------------------------------------------------------------------
// Dispatch without caller-provided scratch.
//
// Some callers cannot hand the library a workspace: code that runs while a
// CUDA graph is being captured (a cudaMalloc there breaks the capture),
// runtimes that plan every device allocation up front or own the only
// allocator in the process, and latency-critical servers that must not
// allocate on the request path.  This entry point sorts with a fixed scratch
// array that lives in the library itself, so it needs no allocation at all.
//
// The array is a file-scope __device__ variable of kNoAllocScratchBytes
// (32 MiB).  Every GPU that loads the library holds it until the process
// exits.  Host code cannot use the array's name as a device address; the
// first call on each device looks the address up with cudaGetSymbolAddress
// while that device is current and caches it with the id of the device's
// context, so make that first call before any stream capture.  A call after
// the context was re-created (cudaDeviceReset) looks the address up again.  All calls share the one array: calls whose kernels can
// overlap on the GPU (different streams, or different host threads on one
// device) race on it and must be ordered by the caller.  The sort writes every
// scratch byte it reads, so no clearing is needed between calls.
// ---------------------------------------------------------------------------
namespace bdm {
namespace {

constexpr int64_t kNoAllocScratchBytes = (int64_t)32 << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_dispatch_scratch[kNoAllocScratchBytes];

// The looked-up address per device, with the id of the context it belongs to: after
// cudaDeviceReset the device's primary context (and with it the array's address) is new, so
// a cached address is only used while the current context id matches.
struct ScratchSlot {
    unsigned long long context = 0;
    void *ptr = nullptr;
};
ScratchSlot g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

// Id of the calling thread's current context (driver entry points reached through the runtime,
// so the library needs no link against the driver library); 0 when unknown.
unsigned long long current_context_id() {
    using GetCurrentFn = int (*)(void **);
    using GetIdFn = int (*)(void *, unsigned long long *);
    static GetCurrentFn get_current = [] {
        void *f = nullptr;
        return cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault) == cudaSuccess
                   ? reinterpret_cast<GetCurrentFn>(f) : nullptr;
    }();
    static GetIdFn get_id = [] {
        void *f = nullptr;
        return cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault) == cudaSuccess
                   ? reinterpret_cast<GetIdFn>(f) : nullptr;
    }();
    void *ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != 0 || !ctx || get_id(ctx, &id) != 0) return 0;
    return id;
}

}  // namespace
}  // namespace bdm

extern "C" int bdm_dispatch_noalloc(const int64_t *write_idx, const int64_t *read_idx, int64_t batch, int64_t time,
                                    int kw, int kr, int64_t bank_count, int64_t *order, int64_t *cu_seqlens,
                                    int64_t *inverse, int64_t *tokens, int32_t *error_word, void *stream) {
    using namespace bdm;
    if (batch <= 0 || time <= 0 || kw <= 0 || kr <= 0 || bank_count <= 0) return BDM_ERR_INVALID;
    const int64_t need = make_plan(batch, time, kw, kr, bank_count).bytes;
    if (need > kNoAllocScratchBytes) return BDM_ERR_WORKSPACE;  // beyond the fixed 32 MiB scratch
    int dev = 0;
    int rc = cuda_status(cudaGetDevice(&dev));
    if (rc) return rc;
    if (dev < 0 || dev >= kMaxDevices) return BDM_ERR_UNSUPPORTED;
    void *ptr = nullptr;
    {
        const unsigned long long context = current_context_id();
        std::lock_guard<std::mutex> lock(g_scratch_mu);
        ScratchSlot &slot = g_scratch[dev];
        if (slot.ptr && context != 0 && slot.context == context) {
            ptr = slot.ptr;
        } else {  // first call on this device, or its context was re-created (or its id is unknown)
            rc = cuda_status(cudaGetSymbolAddress(&ptr, g_dispatch_scratch));
            if (rc) return rc;
            slot.ptr = ptr;
            slot.context = current_context_id();
        }
    }
    return bdm_dispatch(write_idx, read_idx, batch, time, kw, kr, bank_count, order, cu_seqlens, inverse, tokens,
                        error_word, ptr, kNoAllocScratchBytes, stream);
}
