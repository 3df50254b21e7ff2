// The reference-structured binning path (KT_GS_FLAG_SORTED_KEYS): per-Gaussian bin counts are
// scanned in index order (decoupled look-back), one (key, value) pair is emitted per
// (bin, Gaussian) with the key laid out as the reference's, the pairs are radix-sorted by key
// (sort.cu, keys + values) and the bin ranges are found by a boundary search over the sorted keys.
//
//   reference                                          here
//   gsplat_binning.comp:112-159 (atomicAdd duplication)  k_key_scan_emit: exclusive scan of the
//                                                        counts + emission in (Gaussian, bin
//                                                        row, bin column) order
//   gsplat_radix_sort_include.glsl:51-63 (key)          key = bin << depth_bits | (depth - depth_min)
//                                                        with depth = floatBitsToUint(z) ^ 0x80000000;
//                                                        subtracting the frame's minimum is
//                                                        monotone, so the order is the reference's
//                                                        bin << 32 | depth order; value = index
//   gsplat_radix_sort_{histogram,hist_prefix_sum,       k_sort_pass / reduce-then-scan passes over
//     hist_scatter}.comp                                 8-bit digits (sort.cu), stable
//   gsplat_bin_bounds.comp:30-72                        k_key_ranges
//
// The default path (place.cu) reaches the same sorted order without materialising keys; this one
// produces the device-side offsets, keys and values of the reference's stage buffers.
#include "kt_common.cuh"
#include "kt_kernels.h"

namespace kt {
namespace {

constexpr int kScanThreads = 256;
constexpr int kScanItems = kScanChunk / kScanThreads;  // 8 consecutive Gaussians per thread

__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// Exclusive scan of one u32 per thread over a 256-thread CTA; *total receives the CTA sum.
__device__ __forceinline__ uint32_t cta_exclusive_scan(uint32_t v, uint32_t* s_warp, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < 8 ? s_warp[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < 8) s_warp[lane] = w;
    }
    __syncthreads();
    const uint32_t excl = warp == 0 ? 0u : s_warp[warp - 1];
    *total = s_warp[7];
    __syncthreads();
    return excl + x - v;
}

// Decoupled look-back over chunk aggregates by one full warp: publishes the chunk's aggregate,
// sums its predecessors' published values 32 at a time back to the nearest inclusive prefix,
// publishes its own inclusive prefix and returns the exclusive one. Polls are bounded: on
// timeout the error bit is set and a (wrong) inclusive value is published so successors finish.
__device__ uint64_t lookback_warp(unsigned long long* status, uint32_t idx, uint32_t epoch, uint64_t agg,
                                  FrameCtl* ctl) {
    const int lane = threadIdx.x & 31;
    if (lane == 0)
        st_volatile_u64(&status[idx], pack_status(epoch, idx == 0 ? kFlagInclusive : kFlagAggregate, agg));
    uint64_t excl = 0;
    if (idx > 0) {
        int64_t end = (int64_t)idx - 1;
        uint32_t spins = 0;
        for (;;) {
            const int64_t j = end - lane;
            const uint64_t w = j >= 0 ? ld_volatile_u64(&status[j]) : pack_status(epoch, kFlagInclusive, 0);
            const bool ready = status_epoch(w) == epoch && status_flag(w) != 0;
            const bool incl = ready && status_flag(w) == kFlagInclusive;
            const uint32_t ready_m = __ballot_sync(0xFFFFFFFFu, ready);
            const uint32_t incl_m = __ballot_sync(0xFFFFFFFFu, incl);
            // lanes up to and including the nearest inclusive one must be ready
            const uint32_t need = incl_m ? (((incl_m & (0u - incl_m)) << 1) - 1u) : 0xFFFFFFFFu;
            if ((ready_m & need) != need) {
                if (++spins > kSpinLimit) {
                    if (lane == 0) atomicOr(&ctl->error_flags, kErrTimeout);
                    break;
                }
                __nanosleep(32);
                continue;
            }
            excl += warp_sum_u64(((need >> lane) & 1u) ? status_value(w) : 0ull);
            if (incl_m) break;
            end -= 32;
        }
        if (lane == 0) st_volatile_u64(&status[idx], pack_status(epoch, kFlagInclusive, excl + agg));
    }
    return excl;
}

__global__ void __launch_bounds__(kScanThreads) k_key_scan_emit(FrameBufs fb, GridParams gp, uint64_t n,
                                                                uint32_t epoch, uint32_t max_passes) {
    __shared__ uint32_t s_off[kScanChunk + 1];
    __shared__ uint2 s_rect[kScanChunk];
    __shared__ uint32_t s_depth[kScanChunk];
    __shared__ uint32_t s_hist[kMaxPasses][256];
    __shared__ uint32_t s_warp[8];
    __shared__ uint32_t s_chunk;
    __shared__ unsigned long long s_base;

    FrameCtl* ctl = fb.ctl;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) s_chunk = atomicAdd(&ctl->scan_ticket, 1u);  // chunks start in ticket order
    for (int i = tid; i < kMaxPasses * 256; i += kScanThreads) (&s_hist[0][0])[i] = 0u;
    __syncthreads();
    const uint32_t chunk = s_chunk;
    const uint64_t nchunks = (n + kScanChunk - 1) / kScanChunk;
    const uint64_t c0 = (uint64_t)chunk * kScanChunk;

    uint32_t c[kScanItems];
    uint32_t sum = 0;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const uint64_t g = c0 + (uint64_t)tid * kScanItems + j;
        c[j] = g < n ? fb.counts[g] : 0u;
        sum += c[j];
    }
    uint32_t total;
    const uint32_t texcl = cta_exclusive_scan(sum, s_warp, &total);
    {
        uint32_t run = texcl;
#pragma unroll
        for (int j = 0; j < kScanItems; ++j) {
            const int l = tid * kScanItems + j;
            s_off[l] = run;
            if (c[j] != 0u) {
                s_rect[l] = fb.rect[c0 + l];
                s_depth[l] = fb.depth[c0 + l];
            }
            run += c[j];
        }
        if (tid == 0) s_off[kScanChunk] = total;
    }
    if (tid < 32) {
        const uint64_t b = lookback_warp(fb.scan_status, chunk, epoch, total, ctl);
        if (tid == 0) s_base = b;
    }
    __syncthreads();
    const uint64_t base = s_base;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const uint64_t g = c0 + (uint64_t)tid * kScanItems + j;
        if (g < n) fb.offsets[g] = base + s_off[tid * kScanItems + j];
    }

    // every CTA derives the same key layout from the frame's depth range
    const uint32_t dmin = ctl->depth_min, dmax = ctl->depth_max;
    const uint32_t dbits = dmax >= dmin ? bits_for((uint64_t)(dmax - dmin)) : 0u;
    const uint32_t key_bits = gp.tile_bits + dbits;
    uint32_t npasses = (key_bits + 7) / 8;
    if (npasses > max_passes) npasses = max_passes;
    const bool fits = base + total <= fb.key_capacity;
    unsigned long long* __restrict__ keys = fb.keys[0];
    uint32_t* __restrict__ vals = fb.vals[0];

    // Emission: warp w walks its 256 Gaussians in order; the lanes write one Gaussian's bins
    // (row-major over its rectangle) as one coalesced run.
    for (int q0 = warp * (kScanChunk / 8); q0 < (warp + 1) * (kScanChunk / 8); q0 += 32) {
        const int q = q0 + lane;
        uint32_t todo = __ballot_sync(0xFFFFFFFFu, s_off[q + 1] != s_off[q]);
        while (todo) {
            const int l = q0 + __ffs(todo) - 1;
            todo &= todo - 1u;
            const uint32_t off = s_off[l], cnt = s_off[l + 1] - off;
            const uint2 r = s_rect[l];
            const uint64_t dk = (uint64_t)(s_depth[l] - dmin);
            const uint32_t x0 = r.x & 0xFFFFu, w = (r.x >> 16) - x0, y0 = r.y & 0xFFFFu;
            const float inv_w = 1.0f / (float)w;
            for (uint32_t j0 = 0; j0 < cnt; j0 += 32) {
                const uint32_t j = j0 + lane;
                const bool on = j < cnt;
                uint32_t dy = (uint32_t)((float)j * inv_w);  // j / w, corrected exactly
                if (dy * w > j) --dy;
                if ((dy + 1) * w <= j) ++dy;
                const uint64_t tile = (uint64_t)(y0 + dy) * gp.tiles_x + x0 + (j - dy * w);
                const unsigned long long key = (tile << dbits) | dk;
                if (on && fits) {
                    keys[base + off + j] = key;
                    vals[base + off + j] = (uint32_t)(c0 + l);
                }
                // digit histograms; a digit shared by every active lane is added once
                const uint32_t act = __ballot_sync(0xFFFFFFFFu, on);
                const int leader = __ffs(act) - 1;
                for (uint32_t p = 0; p < npasses; ++p) {
                    const uint32_t d = (uint32_t)(key >> (8 * p)) & 255u;
                    const uint32_t d0 = __shfl_sync(0xFFFFFFFFu, d, leader);
                    if (__all_sync(0xFFFFFFFFu, !on || d == d0)) {
                        if (lane == leader) atomicAdd(&s_hist[p][d0], (uint32_t)__popc(act));
                    } else if (on) {
                        atomicAdd(&s_hist[p][d], 1u);
                    }
                }
            }
        }
    }
    __syncthreads();
    for (uint32_t i = tid; i < npasses * 256; i += kScanThreads) {
        const uint32_t v = (&s_hist[0][0])[i];
        if (v) atomicAdd(&(&ctl->hist[0][0])[i], v);
    }
    if (tid == 0 && (uint64_t)chunk == nchunks - 1) {  // the last chunk holds the total
        ctl->num_keys = base + total;
        ctl->depth_bits = dbits;
        ctl->key_bits = key_bits;
        ctl->packed = 0u;
        ctl->idx_bits = 0u;
    }
}

// gsplat_bin_bounds.comp:30-72: for sorted key i, a change of bin between i and i+1 ends the one
// and starts the other at i+1; the last key ends its bin. Empty bins keep {0, 0}.
__global__ void k_key_ranges(SortIO io, const FrameCtl* ctl, uint2* ranges) {
    if (!ctl->plan_ok) return;
    const uint64_t K = ctl->num_keys;
    const uint32_t dbits = ctl->depth_bits;
    const unsigned long long* __restrict__ keys = io_keys(io, ctl->final_buf);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < K; i += stride) {
        const uint32_t t = (uint32_t)(keys[i] >> dbits);
        if (i == K - 1) {
            ranges[t].y = (uint32_t)(i + 1);
        } else {
            const uint32_t tn = (uint32_t)(keys[i + 1] >> dbits);
            if (t != tn) {
                ranges[t].y = (uint32_t)(i + 1);
                ranges[tn].x = (uint32_t)(i + 1);
            }
        }
    }
}

}  // namespace

cudaError_t launch_key_scan_emit(const FrameBufs& fb, const GridParams& gp, uint64_t n, uint32_t epoch,
                                 uint32_t max_passes, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const unsigned chunks = (unsigned)((n + kScanChunk - 1) / kScanChunk);
    k_key_scan_emit<<<chunks, kScanThreads, 0, stream>>>(fb, gp, n, epoch, max_passes);
    return cudaGetLastError();
}

cudaError_t launch_key_ranges(const SortIO& io, const FrameCtl* ctl, uint2* ranges, uint64_t max_keys,
                              cudaStream_t stream) {
    uint64_t blocks = (max_keys + 255) / 256;
    const uint64_t cap = (uint64_t)device_sm_count() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    k_key_ranges<<<(unsigned)blocks, 256, 0, stream>>>(io, ctl, ranges);
    return cudaGetLastError();
}

}  // namespace kt
