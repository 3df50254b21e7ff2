// K4: LSD radix sort, 8-bit digits, stable, one pass per digit.
//
// Replaces the reference's 12-pass 4-bit sort, whose prefix sum runs on one workgroup and whose
// scatter walks 128 elements per thread serially
// (shaders/gsplat/gsplat_radix_sort_{histogram,hist_prefix_sum,hist_scatter}.comp). Same result:
// a stable sort by key. Two forms of a pass share the tile code (4096 elements per tile, ranked
// per warp with one ballot per digit bit, staged in digit order in shared memory, written out in
// coalesced runs, the next tile bulk-copied into shared memory (cp.async.bulk, completion on an
// mbarrier, one destination CTA) while the current one is ranked):
//   * onesweep (k_sort_pass): one kernel; persistent CTAs take tiles by ticket, publish their
//     digit counts and look back over earlier tiles' epoch-tagged counts (16 predecessors per
//     round trip, bounded waits) for their global digit offsets. Used when all tiles fit in one
//     wave of resident CTAs, where the look-back chain is short.
//   * reduce-then-scan (k_rts_upsweep / k_rts_scan / k_rts_downsweep): each CTA owns a static
//     range of tiles; counts per range, a scan over ranges, then ranking and scatter with a
//     running offset. No inter-CTA waits; used for multi-wave sorts.
// Elements are either packed u64 words (key << idx_bits | index: 16 B moved per element per pass,
// ties already ordered by the index bits) or u64 keys with a separate u32 value array (24 B).
// Digit histograms of every pass come from k_depth_keys (the depth sort of the render path) or
// from k_key_histogram (standalone operator); passes whose keys share one digit are skipped.
#include "kt_common.cuh"
#include "kt_kernels.h"

namespace kt {
namespace {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItems = kSortTile / kSortThreads;  // 16 elements per thread
constexpr int kWarpKeys = kSortItems * 32;            // 512 consecutive elements per warp
constexpr uint32_t kBarSpinLimit = 1u << 22;

template <bool PACKED>
struct SortSmem {
    unsigned long long keys[2][kSortTile];                 // input tiles; the current one is
    uint32_t vals[PACKED ? 1 : 2][PACKED ? 4 : kSortTile];  //   reused as the staging buffer
    uint16_t whist[kSortWarps][256];                       // per-warp digit counts, then prefixes
    uint32_t tcount[256];                                  // the tile's digit counts (early)
    uint32_t lstart[256];                                  // tile-local digit starts
    unsigned long long gbase[256];                         // global start of each digit's run
    uint32_t warp_tot[kSortWarps];
    uint32_t tile[2];
    unsigned long long bar[2];                             // one mbarrier per input buffer
};

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// Stable ranks of this warp's 16 elements (positions base + j*32 + lane) among equal digits,
// counting per warp in whist. Lanes with the same digit are found with one ballot per digit bit
// (match.any runs at about half the rate of 8 ballots on this part). Returns the tile count
// part through whist only; rank[j] is the position among equal digits within the warp.
template <int DBITS, bool PACKED>
__device__ __forceinline__ void rank_warp(SortSmem<PACKED>& sm, int cur, uint32_t wpos, uint32_t valid_items,
                                          bool drop, uint32_t shift, uint32_t mask, uint32_t lane, uint32_t lt,
                                          uint16_t* whist, uint16_t (&rank)[kSortItems]) {
    const uint32_t kMask = mask & ((1u << DBITS) - 1u);  // the pass's digit bits
#pragma unroll
    for (int j = 0; j < kSortItems; ++j) {
        const unsigned long long key = sm.keys[cur][wpos + j * 32];
        const bool valid = (uint32_t)j < valid_items && !(drop && key == kDropKey);
        const uint32_t d = (uint32_t)(key >> shift) & kMask;
        uint32_t peers = __ballot_sync(0xFFFFFFFFu, valid);
#pragma unroll
        for (int b = 0; b < DBITS; ++b) {
            const uint32_t bal = __ballot_sync(0xFFFFFFFFu, (d >> b) & 1u);
            peers &= ((d >> b) & 1u) ? bal : ~bal;
        }
        const uint32_t before = __popc(peers & lt);
        const uint32_t base = valid ? whist[d] : 0u;
        __syncwarp();
        // the last lane of each group of equal digits advances the counter
        if (valid && (peers >> lane) == 1u) whist[d] = (uint16_t)(base + before + 1u);
        __syncwarp();
        rank[j] = (uint16_t)(base + before);
    }
}

// Issue the bulk copy of a full tile into buffer `b` (thread 0 only).
template <bool PACKED>
__device__ __forceinline__ void issue_tile(SortSmem<PACKED>& sm, int b, uint64_t tbase,
                                           const unsigned long long* src_k, const uint32_t* src_v) {
    fence_proxy_async_smem();
    const uint32_t kbytes = kSortTile * 8, vbytes = PACKED ? 0u : kSortTile * 4;
    mbar_arrive_expect_tx(&sm.bar[b], kbytes + vbytes);
    bulk_copy_g2s(sm.keys[b], src_k + tbase, kbytes, &sm.bar[b]);
    if (!PACKED) bulk_copy_g2s(sm.vals[b], src_v + tbase, vbytes, &sm.bar[b]);
}

constexpr int kLookbackWindow = 16;  // predecessors read per round trip

// Decoupled look-back for one digit: sum of this digit's counts over all earlier tiles.
// Gives up after `spin_limit` polls without progress: sets kErrTimeout and returns the partial sum,
// so the CTA finishes and publishes (the frame or sort is then reported as failed).
__device__ __forceinline__ uint64_t lookback_digit(const unsigned long long* status, uint32_t tile,
                                                   uint32_t digit, uint32_t epoch, FrameCtl* ctl,
                                                   uint32_t spin_limit = kSpinLimit) {
    uint64_t excl = 0;
    int64_t j = (int64_t)tile - 1;
    uint32_t spins = 0;
    while (j >= 0) {
        uint64_t w[kLookbackWindow];
#pragma unroll
        for (int q = 0; q < kLookbackWindow; ++q)
            w[q] = (j - q >= 0) ? ld_relaxed_u64(status + (uint64_t)(j - q) * 256 + digit) : 0ull;
        int used = 0;
        bool incl = false;
#pragma unroll
        for (int q = 0; q < kLookbackWindow; ++q) {
            if (incl || used != q || j - q < 0) continue;
            if (status_epoch(w[q]) != epoch || status_flag(w[q]) == 0) continue;
            excl += status_value(w[q]);
            incl = status_flag(w[q]) == kFlagInclusive;
            used = q + 1;
        }
        if (incl) break;
        if (used == 0) {
            if (++spins > spin_limit) {
                atomicOr(&ctl->error_flags, kErrTimeout);
                break;
            }
            if (spins > 64) __nanosleep(32);
        }
        j -= used;
    }
    return excl;
}

template <bool PACKED>
__global__ void __launch_bounds__(kSortThreads, PACKED ? 3 : 2)
k_sort_pass(SortIO io, FrameCtl* ctl, unsigned long long* status, uint32_t pass, uint32_t epoch) {
    if (!ctl->plan_ok || !ctl->pass_run[pass] || (ctl->packed != 0) != PACKED) return;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    SortSmem<PACKED>& sm = *reinterpret_cast<SortSmem<PACKED>*>(smem_raw);

    const uint64_t K = ctl->pass_in[pass];  // elements read; a dropping pass writes fewer
    const bool drop = PACKED && ctl->pass_drop[pass] != 0u;
    const uint32_t ntiles = (uint32_t)((K + kSortTile - 1) / kSortTile);
    const uint32_t shift = (PACKED ? ctl->idx_bits : 0u) + 8 * pass;
    const uint32_t mask = ctl->pass_mask[pass];
    const unsigned long long* __restrict__ src_k = io_keys(io, ctl->pass_src[pass]);
    const uint32_t* __restrict__ src_v = io_vals(io, ctl->pass_src[pass]);
    unsigned long long* __restrict__ dst_k = io_keys(io, ctl->pass_dst[pass]);
    uint32_t* __restrict__ dst_v = io_vals(io, ctl->pass_dst[pass]);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t lt = lanemask_lt();
    const uint32_t bucket_base = ctl->base[pass][tid];
    unsigned int* ticket = &ctl->pass_ticket[pass];
    // tiles that can be bulk-copied: whole 4096-element tiles of 16-B aligned arrays
    const bool aligned = ((reinterpret_cast<uintptr_t>(src_k) | (PACKED ? 0 : reinterpret_cast<uintptr_t>(src_v))) & 15u) == 0;
    const uint32_t full_tiles = aligned ? (uint32_t)(K / kSortTile) : 0u;

    if (tid == 0) {
        mbar_init(&sm.bar[0], 1);
        mbar_init(&sm.bar[1], 1);
        fence_mbar_init();
        const uint32_t t0 = atomicAdd(ticket, 1u);
        sm.tile[0] = t0;
        if (t0 < full_tiles) issue_tile<PACKED>(sm, 0, (uint64_t)t0 * kSortTile, src_k, src_v);
    }
    uint32_t phase = 0u;  // bit b: parity of buffer b's next mbarrier phase
    int cur = 0;
    bool failed = false;

    for (;;) {
        __syncthreads();  // previous tile fully written out; sm.tile[cur] visible
        const uint32_t tile = sm.tile[cur];
        if (tile >= ntiles || failed) {
            // after a timed-out wait, let the prefetch already issued land before leaving
            if (failed && tile < full_tiles) mbar_wait_bounded(&sm.bar[cur], (phase >> cur) & 1u, kBarSpinLimit);
            break;
        }
        const uint64_t tbase = (uint64_t)tile * kSortTile;
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) sm.whist[w][tid] = 0;
        sm.tcount[tid] = 0u;
        bool timed_out = false;
        if (tile < full_tiles) {
            const uint32_t par = (phase >> cur) & 1u;
            if (!mbar_wait_bounded(&sm.bar[cur], par, kBarSpinLimit)) {
                timed_out = true;
                if (!mbar_wait_bounded(&sm.bar[cur], par, kBarSpinLimit)) atomicOr(&ctl->error_flags, kErrTimeout);
            }
            phase ^= 1u << cur;
        } else {  // the partial last tile, or unaligned arrays: plain loads
            for (uint32_t i = tid; i < (uint32_t)min((uint64_t)kSortTile, K - tbase); i += kSortThreads) {
                sm.keys[cur][i] = src_k[tbase + i];
                if (!PACKED) sm.vals[cur][i] = src_v[tbase + i];
            }
        }
        if (__syncthreads_or(timed_out)) {
            if (tid == 0) atomicOr(&ctl->error_flags, kErrTimeout);
            failed = true;
        }

        const uint32_t wpos = warp * kWarpKeys + lane;
        const uint32_t rest = K > tbase + wpos ? (uint32_t)min((K - tbase - wpos + 31) / 32, (uint64_t)kSortItems) : 0u;
        const uint32_t valid_items = rest;  // this thread's elements that exist
        // ---- early counts: the tile's digit histogram, published before ranking so that later
        //      tiles' look-backs find it (and soon this tile's inclusive prefix) sooner
#pragma unroll
        for (int j = 0; j < kSortItems; ++j) {
            const unsigned long long key = sm.keys[cur][wpos + j * 32];
            if ((uint32_t)j < valid_items && !(drop && key == kDropKey))
                atomicAdd(&sm.tcount[(uint32_t)(key >> shift) & mask], 1u);
        }
        __syncthreads();
        const uint32_t cnt = sm.tcount[tid];
        unsigned long long* st = status + (uint64_t)tile * 256 + tid;
        st_relaxed_u64(st, pack_status(epoch, tile == 0 ? kFlagInclusive : kFlagAggregate, cnt));

        // ---- rank within the warp (positions warp*512 + j*32 + lane)
        uint16_t rank[kSortItems];
        // one ranking routine for every digit width: fewer instantiations keep the kernel's code
        // in the instruction cache (narrow digits only have zero high bits)
        rank_warp<8, PACKED>(sm, cur, wpos, valid_items, drop, shift, mask, lane, lt, sm.whist[warp], rank);
        __syncthreads();

        // ---- per digit (thread = digit): prefix over warps, then the look-back
        {
            uint32_t run = 0;
#pragma unroll
            for (int w = 0; w < kSortWarps; ++w) {
                const uint32_t t = sm.whist[w][tid];
                sm.whist[w][tid] = (uint16_t)run;
                run += t;
            }
        }
        uint64_t excl = 0;
        if (tile > 0) {
            excl = lookback_digit(status, tile, tid, epoch, ctl);
            st_relaxed_u64(st, pack_status(epoch, kFlagInclusive, excl + cnt));
        }
        sm.gbase[tid] = (unsigned long long)bucket_base + excl;
        // the next tile: taken only now (an earlier ticket would make later tiles wait for this
        // CTA to reach it), its bulk copy overlaps the staging and write-out below
        if (tid == 0) {
            const uint32_t tn = atomicAdd(ticket, 1u);
            sm.tile[cur ^ 1] = tn;
            if (tn < full_tiles) issue_tile<PACKED>(sm, cur ^ 1, (uint64_t)tn * kSortTile, src_k, src_v);
        }
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

        // ---- stage in digit order: read this thread's elements, then reuse the buffer
        unsigned long long k[kSortItems];
        uint32_t v[PACKED ? 1 : kSortItems];
#pragma unroll
        for (int j = 0; j < kSortItems; ++j) {
            k[j] = sm.keys[cur][wpos + j * 32];
            if (!PACKED) v[PACKED ? 0 : j] = sm.vals[cur][wpos + j * 32];
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kSortItems; ++j) {
            const uint32_t p = wpos + j * 32;
            if (tbase + p < K && !(drop && k[j] == kDropKey)) {
                const uint32_t d = (uint32_t)(k[j] >> shift) & mask;
                const uint32_t pos = sm.lstart[d] + sm.whist[warp][d] + rank[j];
                sm.keys[cur][pos] = k[j];
                if (!PACKED) sm.vals[cur][pos] = v[PACKED ? 0 : j];
            }
        }
        __syncthreads();

        // ---- coalesced write-out of the tile's kept elements
        uint32_t tn = 0;
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) tn += sm.warp_tot[w];
        for (uint32_t i = tid; i < tn; i += kSortThreads) {
            const unsigned long long key = sm.keys[cur][i];
            const uint32_t d = (uint32_t)(key >> shift) & mask;
            const uint64_t g = sm.gbase[d] + (i - sm.lstart[d]);
            dst_k[g] = key;
            if (!PACKED) dst_v[g] = sm.vals[cur][i];
        }
        fence_proxy_async_smem();  // this buffer is the target of a later bulk copy
        cur ^= 1;
    }
}

// ---------------------------------------------------------------- reduce-then-scan passes
// The same stable 8-bit pass without inter-CTA waits: G CTAs own G static ranges of whole tiles.
// k_rts_upsweep counts each range's digits, k_rts_scan turns the [G][256] counts into each
// range's global start per digit (bucket base + earlier ranges), and k_rts_downsweep ranks and
// scatters its range tile by tile with a running per-digit offset, bulk-prefetching the next
// tile while it works on the current one. One extra 8-B read per element against onesweep, but
// no decoupled look-back chain, whose L2 round trips set onesweep's pace on this GPU.

__device__ __forceinline__ void rts_range(uint32_t ntiles, uint32_t& t0, uint32_t& t1) {
    const uint32_t per = (ntiles + gridDim.x - 1) / gridDim.x;
    t0 = min(blockIdx.x * per, ntiles);
    t1 = min(t0 + per, ntiles);
}

template <bool PACKED>
__global__ void __launch_bounds__(256) k_rts_upsweep(SortIO io, FrameCtl* ctl, uint32_t* tab, uint32_t pass) {
    if (!ctl->plan_ok || !ctl->pass_run[pass] || (ctl->packed != 0) != PACKED) return;
    __shared__ uint32_t s_hist[8][256];
    const int tid = threadIdx.x, warp = tid >> 5;
#pragma unroll
    for (int w = 0; w < 8; ++w) s_hist[w][tid] = 0u;
    __syncthreads();
    const uint64_t K = ctl->pass_in[pass];
    const uint32_t ntiles = (uint32_t)((K + kSortTile - 1) / kSortTile);
    uint32_t t0, t1;
    rts_range(ntiles, t0, t1);
    const uint32_t shift = (PACKED ? ctl->idx_bits : 0u) + 8 * pass;
    const uint32_t mask = ctl->pass_mask[pass];
    const unsigned long long* __restrict__ src = io_keys(io, ctl->pass_src[pass]);
    const uint64_t e0 = (uint64_t)t0 * kSortTile, e1 = min((uint64_t)t1 * kSortTile, K);
    const bool drop = PACKED && ctl->pass_drop[pass] != 0u;
    for (uint64_t i = e0 + tid; i < e1; i += 256) {
        const unsigned long long key = __ldcs(src + i);
        if (!(drop && key == kDropKey)) atomicAdd(&s_hist[warp][(uint32_t)(key >> shift) & mask], 1u);
    }
    __syncthreads();
    uint32_t sum = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) sum += s_hist[w][tid];
    tab[(uint64_t)blockIdx.x * 256 + tid] = sum;
}

// One CTA per digit: the range starts of that digit, in place.
__global__ void __launch_bounds__(256) k_rts_scan(const FrameCtl* ctl, uint32_t* tab, uint32_t ranges,
                                                  uint32_t pass) {
    if (!ctl->plan_ok || !ctl->pass_run[pass]) return;
    __shared__ uint32_t s_warp[8];
    const uint32_t d = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t carry = ctl->base[pass][d];
    for (uint32_t r0 = 0; r0 < ranges; r0 += 256) {
        const uint32_t r = r0 + tid;
        const uint32_t v = r < ranges ? tab[(uint64_t)r * 256 + d] : 0u;
        uint32_t x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) s_warp[warp] = x;
        __syncthreads();
        uint32_t wex = 0, tot = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            wex += (w < warp) ? s_warp[w] : 0u;
            tot += s_warp[w];
        }
        if (r < ranges) tab[(uint64_t)r * 256 + d] = carry + wex + x - v;
        carry += tot;
        __syncthreads();
    }
}

template <bool PACKED>
__global__ void __launch_bounds__(kSortThreads, PACKED ? 3 : 2)
k_rts_downsweep(SortIO io, FrameCtl* ctl, const uint32_t* __restrict__ tab, uint32_t pass) {
    if (!ctl->plan_ok || !ctl->pass_run[pass] || (ctl->packed != 0) != PACKED) return;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    SortSmem<PACKED>& sm = *reinterpret_cast<SortSmem<PACKED>*>(smem_raw);

    const uint64_t K = ctl->pass_in[pass];  // elements read; a dropping pass writes fewer
    const bool drop = PACKED && ctl->pass_drop[pass] != 0u;
    const uint32_t ntiles = (uint32_t)((K + kSortTile - 1) / kSortTile);
    uint32_t t0, t1;
    rts_range(ntiles, t0, t1);
    if (t0 >= t1) return;
    const uint32_t shift = (PACKED ? ctl->idx_bits : 0u) + 8 * pass;
    const uint32_t mask = ctl->pass_mask[pass];
    const unsigned long long* __restrict__ src_k = io_keys(io, ctl->pass_src[pass]);
    const uint32_t* __restrict__ src_v = io_vals(io, ctl->pass_src[pass]);
    unsigned long long* __restrict__ dst_k = io_keys(io, ctl->pass_dst[pass]);
    uint32_t* __restrict__ dst_v = io_vals(io, ctl->pass_dst[pass]);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t lt = lanemask_lt();
    const bool aligned = ((reinterpret_cast<uintptr_t>(src_k) | (PACKED ? 0 : reinterpret_cast<uintptr_t>(src_v))) & 15u) == 0;
    const uint32_t full_tiles = aligned ? (uint32_t)(K / kSortTile) : 0u;
    unsigned long long running = tab[(uint64_t)blockIdx.x * 256 + tid];  // this digit's next slot

    if (tid == 0) {
        mbar_init(&sm.bar[0], 1);
        mbar_init(&sm.bar[1], 1);
        fence_mbar_init();
        if (t0 < full_tiles) issue_tile<PACKED>(sm, 0, (uint64_t)t0 * kSortTile, src_k, src_v);
    }
    uint32_t phase = 0u;
    int cur = 0;
    for (uint32_t tile = t0; tile < t1; ++tile) {
        __syncthreads();  // previous tile written out; its buffer may be refilled
        const uint64_t tbase = (uint64_t)tile * kSortTile;
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) sm.whist[w][tid] = 0;
        if (tid == 0 && tile + 1 < t1 && tile + 1 < full_tiles)
            issue_tile<PACKED>(sm, cur ^ 1, tbase + kSortTile, src_k, src_v);
        bool timed_out = false;
        if (tile < full_tiles) {
            const uint32_t par = (phase >> cur) & 1u;
            if (!mbar_wait_bounded(&sm.bar[cur], par, kBarSpinLimit)) {
                timed_out = true;
                if (!mbar_wait_bounded(&sm.bar[cur], par, kBarSpinLimit)) atomicOr(&ctl->error_flags, kErrTimeout);
            }
            phase ^= 1u << cur;
        } else {  // the partial last tile, or unaligned arrays: plain loads
            for (uint32_t i = tid; i < (uint32_t)min((uint64_t)kSortTile, K - tbase); i += kSortThreads) {
                sm.keys[cur][i] = src_k[tbase + i];
                if (!PACKED) sm.vals[cur][i] = src_v[tbase + i];
            }
        }
        if (__syncthreads_or(timed_out)) {
            if (tid == 0) atomicOr(&ctl->error_flags, kErrTimeout);
            // let the prefetch already issued land before leaving
            if (tile + 1 < t1 && tile + 1 < full_tiles)
                mbar_wait_bounded(&sm.bar[cur ^ 1], (phase >> (cur ^ 1)) & 1u, kBarSpinLimit);
            return;
        }
        const uint32_t wpos = warp * kWarpKeys + lane;
        const uint64_t rest = K > tbase + wpos ? (K - tbase - wpos + 31) / 32 : 0;
        const uint32_t valid_items = rest < (uint64_t)kSortItems ? (uint32_t)rest : (uint32_t)kSortItems;

        uint16_t rank[kSortItems];
        // one ranking routine for every digit width: fewer instantiations keep the kernel's code
        // in the instruction cache (narrow digits only have zero high bits)
        rank_warp<8, PACKED>(sm, cur, wpos, valid_items, drop, shift, mask, lane, lt, sm.whist[warp], rank);
        __syncthreads();

        // per digit (thread = digit): prefix over warps, the tile's count, its global start
        uint32_t cnt = 0;
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) {
            const uint32_t t = sm.whist[w][tid];
            sm.whist[w][tid] = (uint16_t)cnt;
            cnt += t;
        }
        sm.gbase[tid] = running;
        running += cnt;
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

        // stage in digit order: read this thread's elements, then reuse the buffer
        unsigned long long k[kSortItems];
        uint32_t v[PACKED ? 1 : kSortItems];
#pragma unroll
        for (int j = 0; j < kSortItems; ++j) {
            k[j] = sm.keys[cur][wpos + j * 32];
            if (!PACKED) v[PACKED ? 0 : j] = sm.vals[cur][wpos + j * 32];
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kSortItems; ++j) {
            if ((uint32_t)j < valid_items && !(drop && k[j] == kDropKey)) {
                const uint32_t d = (uint32_t)(k[j] >> shift) & mask;
                const uint32_t pos = sm.lstart[d] + sm.whist[warp][d] + rank[j];
                sm.keys[cur][pos] = k[j];
                if (!PACKED) sm.vals[cur][pos] = v[PACKED ? 0 : j];
            }
        }
        __syncthreads();

        // coalesced write-out of the tile's kept elements
        uint32_t tn = 0;
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) tn += sm.warp_tot[w];
        for (uint32_t i = tid; i < tn; i += kSortThreads) {
            const unsigned long long key = sm.keys[cur][i];
            const uint32_t d = (uint32_t)(key >> shift) & mask;
            const uint64_t g = sm.gbase[d] + (i - sm.lstart[d]);
            dst_k[g] = key;
            if (!PACKED) dst_v[g] = sm.vals[cur][i];
        }
        fence_proxy_async_smem();  // this buffer is the target of a later bulk copy
        cur ^= 1;
    }
}

template <bool PACKED>
int rts_grid(int dev) {
    static int per_sm[128] = {0};
    if (dev < 0 || dev >= 128) return 0;
    if (per_sm[dev] == 0) {
        const size_t smem = sizeof(SortSmem<PACKED>);
        if (cudaFuncSetAttribute(k_rts_downsweep<PACKED>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return 0;
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_rts_downsweep<PACKED>, kSortThreads, smem) !=
            cudaSuccess)
            return 0;
        per_sm[dev] = n > 0 ? n : 1;
    }
    return per_sm[dev] * device_sm_count();
}

template <bool PACKED>
cudaError_t launch_rts_pass(const SortIO& io, FrameCtl* ctl, uint32_t* tab, uint32_t pass, uint64_t max_keys,
                            cudaStream_t stream) {
    int dev = 0;
    cudaGetDevice(&dev);
    uint64_t grid = (uint64_t)rts_grid<PACKED>(dev);
    if (grid == 0) return cudaErrorInvalidConfiguration;
    const uint64_t tiles = (max_keys + kSortTile - 1) / kSortTile;
    if (tiles < grid) grid = tiles;
    if (grid < 1) grid = 1;
    k_rts_upsweep<PACKED><<<(unsigned)grid, 256, 0, stream>>>(io, ctl, tab, pass);
    k_rts_scan<<<256, 256, 0, stream>>>(ctl, tab, (uint32_t)grid, pass);
    k_rts_downsweep<PACKED><<<(unsigned)grid, kSortThreads, sizeof(SortSmem<PACKED>), stream>>>(io, ctl, tab, pass);
    return cudaGetLastError();
}

// Digit histograms of caller-supplied keys (standalone operator). Also records K and the key
// width for the plan.
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

template <bool PACKED>
cudaError_t launch_pass(const SortIO& io, FrameCtl* ctl, unsigned long long* status, uint32_t pass,
                        uint32_t epoch, uint64_t max_keys, cudaStream_t stream) {
    static int per_sm[128] = {0};  // resident CTAs per SM, per device
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t smem = sizeof(SortSmem<PACKED>);
    if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
    if (per_sm[dev] == 0) {
        cudaError_t e = cudaFuncSetAttribute(k_sort_pass<PACKED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        int n = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_sort_pass<PACKED>, kSortThreads, smem);
        if (e != cudaSuccess) return e;
        per_sm[dev] = n > 0 ? n : 1;
    }
    const uint64_t tiles = (max_keys + kSortTile - 1) / kSortTile;
    uint64_t grid = (uint64_t)device_sm_count() * per_sm[dev];  // persistent: all resident
    if (tiles < grid) grid = tiles;
    if (grid < 1) grid = 1;
    k_sort_pass<PACKED><<<(unsigned)grid, kSortThreads, smem, stream>>>(io, ctl, status, pass, epoch);
    return cudaGetLastError();
}

// The look-back wait of a sort pass, run by one CTA as tile 1 against tile 0's status words, which
// nothing publishes: every digit's wait runs out after `spin_limit` polls and records kErrTimeout
// in `ctl`, as a pass whose predecessor never finished would. Used to check the timeout path.
__global__ void __launch_bounds__(256) k_lookback_timeout_probe(const unsigned long long* status, FrameCtl* ctl,
                                                                uint32_t spin_limit) {
    (void)lookback_digit(status, 1u, threadIdx.x, 1u, ctl, spin_limit);
}

}  // namespace

size_t sort_status_words(uint64_t max_keys) {
    return (size_t)((max_keys + kSortTile - 1) / kSortTile) * 256;
}

size_t sort_table_words(uint64_t max_keys) {
    // at most one range per resident CTA: 2048 threads per SM / 256 per CTA
    uint64_t ranges = (max_keys + kSortTile - 1) / kSortTile;
    const uint64_t cap = (uint64_t)device_sm_count() * 8;
    if (ranges > cap) ranges = cap;
    if (ranges < 1) ranges = 1;
    return (size_t)ranges * 256;
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

// True when a sort of max_keys elements runs its passes as onesweep (see launch_sort_pass).
static bool sort_is_onesweep(uint64_t max_keys, bool packed) {
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t tiles = (max_keys + kSortTile - 1) / kSortTile;
    const uint64_t wave = packed ? (uint64_t)rts_grid<true>(dev) : (uint64_t)rts_grid<false>(dev);
    return tiles <= wave;
}

cudaError_t launch_lookback_timeout_probe(const unsigned long long* status, FrameCtl* ctl, uint32_t spin_limit,
                                          cudaStream_t stream) {
    k_lookback_timeout_probe<<<1, 256, 0, stream>>>(status, ctl, spin_limit);
    return cudaGetLastError();
}

uint32_t sort_pass_launches(uint64_t max_keys, bool packed) {
    return sort_is_onesweep(max_keys, packed) ? 1u : 3u;
}

cudaError_t launch_sort_pass(const SortIO& io, FrameCtl* ctl, unsigned long long* status, uint32_t* table,
                             uint32_t pass, uint32_t epoch, uint64_t max_keys, bool packed,
                             cudaStream_t stream) {
    // Sorts that fit in one wave of resident CTAs use onesweep (one kernel; its look-back chain is
    // one wave long). Larger ones use reduce-then-scan, whose passes never wait on other CTAs;
    // measured on the 16.9M-pair bin sort: 145 us per pass against 161 us for onesweep.
    if (sort_is_onesweep(max_keys, packed))
        return packed ? launch_pass<true>(io, ctl, status, pass, epoch, max_keys, stream)
                      : launch_pass<false>(io, ctl, status, pass, epoch, max_keys, stream);
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t wave = packed ? (uint64_t)rts_grid<true>(dev) : (uint64_t)rts_grid<false>(dev);
    if (!table || wave == 0 || wave > sort_table_words(max_keys) / 256) return cudaErrorInvalidValue;
    return packed ? launch_rts_pass<true>(io, ctl, table, pass, max_keys, stream)
                  : launch_rts_pass<false>(io, ctl, table, pass, max_keys, stream);
}

}  // namespace kt
