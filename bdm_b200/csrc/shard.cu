// Bank partition for the bank-sharded forward (one rank per GPU).
//
// The reference runs the whole bank table on one device.  For tables too large
// or too busy for one GPU (J >= 16K banks), the table is partitioned over the
// ranks of one node: every rank owns J/world banks and their state, runs the
// recurrence of its own banks over all ranks' tokens, and returns FP32 read
// partials.  Which rank owns which bank is decided here.
//
// Contiguous index ranges are the simple choice, but routed traffic is skewed
// (a Zipf-popular bank can take several percent of all events), so the default
// partition is balanced by load, computed from the all-reduced per-bank event
// counts of the current call: banks sorted by (count desc, index asc), then
// dealt out in groups of `world`.  The first kGreedyGroups groups -- the heavy
// head of the distribution -- go greedily, the heaviest bank of a group to the
// least loaded rank so far; the light tail is dealt in one parallel step, in a
// serpentine over the ranks ordered by their load after the head.  Every rank
// gets exactly J/world banks, and the map is a pure function of the counts, so
// all ranks compute the same one.
#include "common.cuh"

namespace bdm {
namespace {

constexpr int kHistThreads = 256;
constexpr int kOwnThreads = 1024;
constexpr int kMaxBalancedBanks = 16384;  // keys of the whole table sorted in shared memory
constexpr int kMaxBalancedWorld = 32;     // one lane per rank
constexpr int kGreedyGroups = 128;        // groups dealt greedily (sequential); the rest in one serpentine

__global__ void __launch_bounds__(kHistThreads)
bank_histogram_kernel(const int64_t *__restrict__ wi, const int64_t *__restrict__ ri, int64_t ntok, int kw, int kr,
                      int64_t J, int32_t *__restrict__ counts, int private_hist) {
    extern __shared__ int32_t hist[];
    if (private_hist) {
        for (int64_t j = threadIdx.x; j < J; j += kHistThreads) hist[j] = 0;
        __syncthreads();
    }
    const int64_t ew = ntok * kw, e = ew + ntok * kr;
    for (int64_t i = (int64_t)blockIdx.x * kHistThreads + threadIdx.x; i < e; i += (int64_t)gridDim.x * kHistThreads) {
        int64_t bank = i < ew ? wi[i] : ri[i - ew];
        bank = bank < 0 ? 0 : (bank >= J ? J - 1 : bank);
        if (private_hist) atomicAdd(&hist[bank], 1);
        else atomicAdd(&counts[bank], 1);
    }
    if (private_hist) {
        __syncthreads();
        for (int64_t j = threadIdx.x; j < J; j += kHistThreads)
            if (hist[j]) atomicAdd(&counts[j], hist[j]);
    }
}

__global__ void contiguous_owners_kernel(int64_t J, int64_t per_rank, int32_t *__restrict__ owner,
                                         int32_t *__restrict__ slot, int32_t *__restrict__ members) {
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < J; j += (int64_t)gridDim.x * blockDim.x) {
        owner[j] = (int32_t)(j / per_rank);
        slot[j] = (int32_t)(j % per_rank);
        members[j] = (int32_t)j;
    }
}

// Exclusive scan of one value per thread over the 1024-thread block.
__device__ __forceinline__ int block_exclusive_scan(int v, int *warp_tot) {
    const unsigned lane = lane_id();
    const int warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= (unsigned)o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
        const int t = warp_tot[lane];
        int s = t;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= (unsigned)o) s += y;
        }
        warp_tot[lane] = s - t;
    }
    __syncthreads();
    const int excl = x - v + warp_tot[warp];
    __syncthreads();
    return excl;
}

// One CTA: sort (count desc, index asc), deal out by groups, then number each
// rank's banks in ascending index order.
__global__ void __launch_bounds__(kOwnThreads)
balanced_owners_kernel(const int32_t *__restrict__ counts, int J, int n_pow2, int world, int32_t *__restrict__ owner,
                       int32_t *__restrict__ slot, int32_t *__restrict__ members) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned long long *keys = reinterpret_cast<unsigned long long *>(smem_raw);
    unsigned char *own = smem_raw + (size_t)n_pow2 * sizeof(unsigned long long);
    __shared__ int warp_tot[32];
    const int tid = threadIdx.x;

    // key = (~count : index): ascending key order is (count desc, index asc).
    for (int i = tid; i < n_pow2; i += kOwnThreads) {
        unsigned long long key = ~0ull;
        if (i < J) {
            const int c = counts[i];
            const unsigned cu = c < 0 ? 0u : (unsigned)c;
            key = ((unsigned long long)(0xffffffffu - cu) << 32) | (unsigned)i;
        }
        keys[i] = key;
    }
    __syncthreads();
    // Bitonic sort, ascending.
    for (int k = 2; k <= n_pow2; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < n_pow2; i += kOwnThreads) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = keys[i], b = keys[ixj];
                    const bool up = (i & k) == 0;
                    if ((a > b) == up) {
                        keys[i] = b;
                        keys[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    // Deal out: group g holds sorted positions [g*world, (g+1)*world); in the
    // head, the rank with the p-th smallest load (ties: lower rank) takes
    // position g*world + p.
    __shared__ int rank_by_load[kMaxBalancedWorld];
    const int groups = J / world;
    const int head = min(groups, kGreedyGroups);
    if (tid < 32) {
        const int lane = tid;
        unsigned long long load = 0ull;
        int pos = 0;
        for (int g = 0; g <= head; ++g) {
            pos = 0;
            for (int l = 0; l < world; ++l) {
                const unsigned long long o = __shfl_sync(0xffffffffu, load, l);
                pos += (o < load) || (o == load && l < lane);
            }
            if (g < head && lane < world) {
                const unsigned long long key = keys[g * world + pos];
                own[(int)(key & 0xffffffffu)] = (unsigned char)lane;
                load += 0xffffffffu - (unsigned)(key >> 32);
            }
        }
        if (lane < world) rank_by_load[pos] = lane;  // rank order by load after the head
    }
    __syncthreads();
    // Tail: group head + k goes in serpentine order over rank_by_load.
    for (int i = head * world + tid; i < J; i += kOwnThreads) {
        const int k = i / world - head, p = i % world;
        const int r = rank_by_load[(k & 1) ? world - 1 - p : p];
        own[(int)(keys[i] & 0xffffffffu)] = (unsigned char)r;
    }
    __syncthreads();
    // Slots: each thread owns a contiguous run of bank indices.
    const int per = (J + kOwnThreads - 1) / kOwnThreads;
    const int lo = tid * per, hi = min(lo + per, J);
    const int per_rank = J / world;
    for (int i = lo; i < hi; ++i) owner[i] = own[i];
    for (int r = 0; r < world; ++r) {
        int c = 0;
        for (int i = lo; i < hi; ++i) c += own[i] == r;
        int s = block_exclusive_scan(c, warp_tot);
        for (int i = lo; i < hi; ++i) {
            if (own[i] == r) {
                slot[i] = s;
                members[(int64_t)r * per_rank + s] = i;
                ++s;
            }
        }
    }
}

}  // namespace
}  // namespace bdm

extern "C" int bdm_bank_histogram(const int64_t *write_idx, const int64_t *read_idx, int64_t ntok, int kw, int kr,
                                  int64_t bank_count, int32_t *counts, void *stream) {
    using namespace bdm;
    if (ntok < 0 || kw <= 0 || kr <= 0 || bank_count <= 0) return BDM_ERR_INVALID;
    if (ntok == 0) return BDM_OK;
    if (!write_idx || !read_idx || !counts) return BDM_ERR_INVALID;
    const int64_t e = ntok * (int64_t)(kw + kr);
    const bool private_hist = bank_count * 4 <= 96 * 1024;
    int64_t blocks = ceil_div(e, (int64_t)kHistThreads * 16);
    if (blocks > 2 * kNumSMs) blocks = 2 * kNumSMs;
    const size_t smem = private_hist ? (size_t)bank_count * 4 : 0;
    if (smem > 48 * 1024) {
        const int rc = cuda_status(
            cudaFuncSetAttribute(bank_histogram_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        if (rc) return rc;
    }
    bank_histogram_kernel<<<(unsigned)blocks, kHistThreads, smem, as_stream(stream)>>>(
        write_idx, read_idx, ntok, kw, kr, bank_count, counts, private_hist ? 1 : 0);
    return launch_status();
}

extern "C" int bdm_bank_owners(const int32_t *counts, int64_t bank_count, int world, int mode, int32_t *owner,
                               int32_t *slot, int32_t *members, void *stream) {
    using namespace bdm;
    if (bank_count <= 0 || world <= 0 || (mode != 0 && mode != 1)) return BDM_ERR_INVALID;
    if (!owner || !slot || !members || (mode == 1 && !counts)) return BDM_ERR_INVALID;
    if (bank_count % world) return BDM_ERR_UNSUPPORTED;
    if (bank_count >= ((int64_t)1 << 31)) return BDM_ERR_UNSUPPORTED;
    cudaStream_t st = as_stream(stream);
    if (mode == 0) {
        int64_t blocks = ceil_div(bank_count, 256);
        if (blocks > 8 * kNumSMs) blocks = 8 * kNumSMs;
        contiguous_owners_kernel<<<(unsigned)blocks, 256, 0, st>>>(bank_count, bank_count / world, owner, slot,
                                                                    members);
        return launch_status();
    }
    if (bank_count > kMaxBalancedBanks || world > kMaxBalancedWorld) return BDM_ERR_UNSUPPORTED;
    int n_pow2 = 1;
    while (n_pow2 < bank_count) n_pow2 <<= 1;
    const size_t smem = (size_t)n_pow2 * (sizeof(unsigned long long) + 1);
    int rc = cuda_status(
        cudaFuncSetAttribute(balanced_owners_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (rc) return rc;
    balanced_owners_kernel<<<1, kOwnThreads, smem, st>>>(counts, (int)bank_count, n_pow2, world, owner, slot,
                                                         members);
    return launch_status();
}
