// K4: onesweep LSD radix sort of (u64 key, u32 value) pairs, 8-bit digits.
//
// Replaces the reference's 12-pass 4-bit sort, whose prefix sum runs on one workgroup and
// whose scatter walks 128 elements per thread serially
// (shaders/gsplat/gsplat_radix_sort_{histogram,hist_prefix_sum,hist_scatter}.comp). Same
// result: a stable sort by key. One kernel per digit:
//   * a CTA takes the next 4096-key tile by ticket (so earlier tiles always have an owner),
//   * ranks its keys per warp with __match_any_sync (warp-level multisplit), stable in
//     position order,
//   * publishes its per-digit counts and looks back over earlier tiles' counts (decoupled
//     look-back, bounded waits) for its global digit offsets,
//   * stages the keys in shared memory in digit order and writes them out in coalesced runs.
// Digit histograms of all passes come from the emission kernel (render path) or
// k_key_histogram (standalone operator); a pass whose keys all share one digit is skipped.
//
// Roofline: HBM bound, 24 B moved per key per executed pass (read + write of 8 B key and
// 4 B value).
#include "kt_common.cuh"
#include "kt_kernels.h"

namespace kt {
namespace {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItems = kSortTile / kSortThreads;  // 16 keys per thread
constexpr int kWarpKeys = kSortItems * 32;            // 512 consecutive keys per warp

struct SortSmem {
    unsigned long long keys[kSortTile];
    uint32_t vals[kSortTile];
    uint32_t whist[kSortWarps][256];
    uint32_t lstart[256];
    unsigned long long gbase[256];
    uint32_t warp_tot[kSortWarps];
    uint32_t tile;
};

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

__global__ void __launch_bounds__(kSortThreads, 2)
k_sort_pass(SortIO io, FrameCtl* ctl, unsigned long long* status, uint32_t pass, uint32_t epoch) {
    if (!ctl->plan_ok || !ctl->pass_run[pass]) return;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SortSmem& sm = *reinterpret_cast<SortSmem*>(smem_raw);

    const uint64_t K = ctl->num_keys;
    const uint32_t ntiles = (uint32_t)((K + kSortTile - 1) / kSortTile);
    const uint32_t shift = 8 * pass;
    const uint32_t mask = ctl->pass_mask[pass];
    const unsigned long long* __restrict__ src_k = io_keys(io, ctl->pass_src[pass]);
    const uint32_t* __restrict__ src_v = io_vals(io, ctl->pass_src[pass]);
    unsigned long long* __restrict__ dst_k = io_keys(io, ctl->pass_dst[pass]);
    uint32_t* __restrict__ dst_v = io_vals(io, ctl->pass_dst[pass]);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t lt = lanemask_lt();
    const uint32_t bucket_base = ctl->base[pass][tid];

    for (;;) {
        if (tid == 0) sm.tile = atomicAdd(&ctl->pass_ticket[pass], 1u);
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) sm.whist[w][tid] = 0u;
        __syncthreads();
        const uint32_t tile = sm.tile;
        if (tile >= ntiles) break;
        const uint64_t tbase = (uint64_t)tile * kSortTile;

        // ---- load and rank within the warp (positions warp*512 + j*32 + lane)
        unsigned long long k[kSortItems];
        uint32_t v[kSortItems];
        uint32_t rank[kSortItems];
        const uint64_t wbase = tbase + (uint64_t)warp * kWarpKeys + lane;
#pragma unroll
        for (int j = 0; j < kSortItems; ++j) {
            const uint64_t idx = wbase + (uint64_t)j * 32;
            const bool valid = idx < K;
            k[j] = valid ? src_k[idx] : 0ull;
            v[j] = valid ? src_v[idx] : 0u;
        }
#pragma unroll
        for (int j = 0; j < kSortItems; ++j) {
            const uint64_t idx = wbase + (uint64_t)j * 32;
            const bool valid = idx < K;
            const uint32_t d = valid ? (uint32_t)(k[j] >> shift) & mask : 256u + lane;
            const uint32_t peers = __match_any_sync(0xFFFFFFFFu, d);
            const int leader = __ffs(peers) - 1;
            uint32_t b = 0;
            if (valid && lane == leader) {
                b = sm.whist[warp][d];
                sm.whist[warp][d] = b + __popc(peers);
            }
            b = __shfl_sync(0xFFFFFFFFu, b, leader);
            rank[j] = b + __popc(peers & lt);
            __syncwarp();
        }
        __syncthreads();

        // ---- per digit (thread tid = digit): prefix over warps, tile count
        uint32_t cnt = 0;
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) {
            const uint32_t t = sm.whist[w][tid];
            sm.whist[w][tid] = cnt;
            cnt += t;
        }

        // ---- decoupled look-back for this digit
        unsigned long long* st = status + (uint64_t)tile * 256 + tid;
        st_volatile_u64(st, pack_status(epoch, tile == 0 ? kFlagInclusive : kFlagAggregate, cnt));
        uint64_t excl = 0;
        if (tile > 0) {
            int64_t j = (int64_t)tile - 1;
            uint32_t spins = 0;
            while (j >= 0) {
                const uint64_t w = ld_volatile_u64(status + (uint64_t)j * 256 + tid);
                if (status_epoch(w) != epoch || status_flag(w) == 0) {
                    if (++spins > kSpinLimit) {
                        atomicOr(&ctl->error_flags, kErrTimeout);
                        break;
                    }
                    __nanosleep(32);
                    continue;
                }
                excl += status_value(w);
                if (status_flag(w) == kFlagInclusive) break;
                --j;
            }
            st_volatile_u64(st, pack_status(epoch, kFlagInclusive, excl + cnt));
        }
        sm.gbase[tid] = (unsigned long long)bucket_base + excl;

        // ---- tile-local digit starts: exclusive scan of cnt over digits
        {
            uint32_t x = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
                if (lane >= o) x += y;
            }
            if (lane == 31) sm.warp_tot[warp] = x;
            __syncthreads();
            uint32_t wex = 0;
#pragma unroll
            for (int w = 0; w < kSortWarps; ++w) wex += (w < warp) ? sm.warp_tot[w] : 0u;
            sm.lstart[tid] = wex + x - cnt;
        }
        __syncthreads();

        // ---- stage in digit order
#pragma unroll
        for (int j = 0; j < kSortItems; ++j) {
            const uint64_t idx = wbase + (uint64_t)j * 32;
            if (idx < K) {
                const uint32_t d = (uint32_t)(k[j] >> shift) & mask;
                const uint32_t pos = sm.lstart[d] + sm.whist[warp][d] + rank[j];
                sm.keys[pos] = k[j];
                sm.vals[pos] = v[j];
            }
        }
        __syncthreads();

        // ---- coalesced write-out
        const uint32_t tn = (uint32_t)min((uint64_t)kSortTile, K - tbase);
        for (uint32_t i = tid; i < tn; i += kSortThreads) {
            const unsigned long long key = sm.keys[i];
            const uint32_t d = (uint32_t)(key >> shift) & mask;
            const uint64_t g = sm.gbase[d] + (i - sm.lstart[d]);
            dst_k[g] = key;
            dst_v[g] = sm.vals[i];
        }
        __syncthreads();
    }
}

// Digit histograms of caller-supplied keys (standalone operator). Also records K and the
// key width for the plan.
__global__ void __launch_bounds__(256) k_key_histogram(const unsigned long long* __restrict__ keys,
                                                       uint64_t n, uint32_t key_bits, FrameCtl* ctl) {
    __shared__ uint32_t s_hist[kMaxPasses][256];
    for (int i = threadIdx.x; i < kMaxPasses * 256; i += blockDim.x) (&s_hist[0][0])[i] = 0u;
    __syncthreads();
    const uint32_t npasses = (key_bits + 7) / 8;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const unsigned long long key = keys[i];
        for (uint32_t p = 0; p < npasses; ++p) {
            const uint32_t lo = 8 * p;
            const uint32_t m = key_bits >= lo + 8 ? 255u : (1u << (key_bits - lo)) - 1u;
            atomicAdd(&s_hist[p][(uint32_t)(key >> lo) & m], 1u);
        }
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < npasses * 256; i += blockDim.x) {
        const uint32_t v = (&s_hist[0][0])[i];
        if (v) atomicAdd(&(&ctl->hist[0][0])[i], v);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        ctl->num_keys = n;
        ctl->key_bits = key_bits;
    }
}

}  // namespace

size_t sort_status_words(uint64_t max_keys) {
    return (size_t)((max_keys + kSortTile - 1) / kSortTile) * 256;
}

cudaError_t launch_key_histogram(const unsigned long long* keys, uint64_t n, uint32_t key_bits,
                                 FrameCtl* ctl, cudaStream_t stream) {
    unsigned blocks = (unsigned)((n + 4095) / 4096);
    const unsigned cap = (unsigned)device_sm_count() * 4;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    k_key_histogram<<<blocks, 256, 0, stream>>>(keys, n, key_bits, ctl);
    return cudaGetLastError();
}

cudaError_t launch_sort_pass(const SortIO& io, FrameCtl* ctl, unsigned long long* status,
                             uint32_t pass, uint32_t epoch, uint64_t max_keys,
                             cudaStream_t stream) {
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t smem = sizeof(SortSmem);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(k_sort_pass, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    const uint64_t tiles = (max_keys + kSortTile - 1) / kSortTile;
    uint64_t grid = (uint64_t)device_sm_count() * 2;  // persistent: every CTA resident
    if (tiles < grid) grid = tiles;
    if (grid < 1) grid = 1;
    k_sort_pass<<<(unsigned)grid, kSortThreads, smem, stream>>>(io, ctl, status, pass, epoch);
    return cudaGetLastError();
}

}  // namespace kt
