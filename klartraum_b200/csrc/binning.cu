// K2+K3: exclusive scan of the per-Gaussian bin counts (decoupled look-back) fused with the
// emission of one (key, value) pair per overlapped bin; plus the per-frame reset, the sort
// plan and the bin-range search (K5).
//
// Replaces the atomicAdd duplication of shaders/gsplat/gsplat_binning.comp:112-159 (whose
// order is nondeterministic and capped at 2N) with count -> scan -> emit, which is exact and
// deterministic: Gaussians in index order, bins in ascending bin index per Gaussian.
//
// Keys are compact: (bin << depth_bits) | (depth - depth_min), where depth is
// floatBitsToUint(z) ^ 0x80000000 (gsplat_radix_sort_include.glsl:51-63) and depth_min /
// depth_bits come from the frame's range of depths. Subtracting the minimum is monotone, so
// the order is exactly the order of the reference key bin<<32 | depth, with fewer sort passes.
#include "kt_common.cuh"
#include "kt_kernels.h"

namespace kt {
namespace {

constexpr int kScanThreads = 256;
constexpr int kScanItems = kScanChunk / kScanThreads;  // 8

__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// Exclusive block scan of one u32 per thread (blockDim.x == 256). Returns the prefix; *total
// receives the block sum.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* s_warp,
                                                         uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < 8 ? s_warp[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            uint32_t y = __shfl_up_sync(0xFFFFFFFFu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < 8) s_warp[lane] = w;  // inclusive warp prefix
    }
    __syncthreads();
    const uint32_t warp_excl = warp == 0 ? 0u : s_warp[warp - 1];
    *total = s_warp[7];
    __syncthreads();
    return warp_excl + x - v;
}

// Decoupled look-back over chunk aggregates, run by one full warp. Publishes the chunk's
// aggregate, waits for its predecessors (32 at a time), publishes the inclusive prefix and
// returns the exclusive prefix. Waits are bounded: on timeout the error flag is set and the
// chunk publishes a (wrong) inclusive value so that its successors finish too.
__device__ uint64_t lookback_warp(unsigned long long* status, uint32_t idx, uint32_t epoch,
                                  uint64_t agg, FrameCtl* ctl) {
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

__global__ void k_frame_init(FrameCtl* ctl, uint2* ranges, uint32_t ntiles) {
    const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    if (blockIdx.x == 0) {
        uint32_t* w = reinterpret_cast<uint32_t*>(ctl);
        const uint32_t nw = sizeof(FrameCtl) / 4;
        for (uint32_t i = threadIdx.x; i < nw; i += blockDim.x) w[i] = 0u;
        __syncthreads();
        if (threadIdx.x == 0) ctl->depth_min = 0xFFFFFFFFu;
    }
    for (uint32_t t = tid; t < ntiles; t += gridDim.x * blockDim.x) ranges[t] = make_uint2(0u, 0u);
}

__global__ void __launch_bounds__(kScanThreads) k_scan_emit(FrameBufs fb, GridParams gp, uint64_t n,
                                                            uint32_t epoch, uint32_t max_passes) {
    __shared__ uint32_t s_off[kScanChunk + 1];
    __shared__ uint2 s_rect[kScanChunk];
    __shared__ uint32_t s_depth[kScanChunk];
    __shared__ uint32_t s_hist[kMaxPasses][256];
    __shared__ uint32_t s_warp[8];
    __shared__ uint32_t s_chunk;
    __shared__ unsigned long long s_base;

    FrameCtl* ctl = fb.ctl;
    const int tid = threadIdx.x;
    if (tid == 0) s_chunk = atomicAdd(&ctl->scan_ticket, 1u);
    for (int i = tid; i < kMaxPasses * 256; i += kScanThreads) (&s_hist[0][0])[i] = 0u;
    __syncthreads();
    const uint32_t chunk = s_chunk;
    const uint64_t nchunks = (n + kScanChunk - 1) / kScanChunk;
    const uint64_t c0 = (uint64_t)chunk * kScanChunk;

    // counts of this thread's 8 consecutive Gaussians
    uint32_t c[kScanItems];
    uint32_t sum = 0;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const uint64_t g = c0 + (uint64_t)tid * kScanItems + j;
        c[j] = g < n ? fb.counts[g] : 0u;
        sum += c[j];
    }
    uint32_t total;
    const uint32_t texcl = block_exclusive_scan(sum, s_warp, &total);
    {
        uint32_t run = texcl;
#pragma unroll
        for (int j = 0; j < kScanItems; ++j) {
            const int l = tid * kScanItems + j;
            const uint64_t g = c0 + l;
            s_off[l] = run;
            if (c[j] != 0u) {
                s_rect[l] = fb.rect[g];
                s_depth[l] = fb.depth[g];
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
        const int l = tid * kScanItems + j;
        const uint64_t g = c0 + l;
        if (g < n) fb.offsets[g] = base + s_off[l];
    }

    // every CTA derives the same key layout from the frame's depth range
    const uint32_t dmin = ctl->depth_min, dmax = ctl->depth_max;
    const uint32_t dbits = dmax >= dmin ? bits_for((uint64_t)(dmax - dmin)) : 0u;
    const uint32_t key_bits = gp.tile_bits + dbits;
    uint32_t npasses = (key_bits + 7) / 8;
    if (npasses > max_passes) npasses = max_passes;
    const bool fits = base + total <= fb.key_capacity;
    unsigned long long* keys = fb.keys[0];
    uint32_t* vals = fb.vals[0];

    for (uint32_t s = tid; s < total; s += kScanThreads) {
        // last Gaussian whose local offset is <= s (zero-count Gaussians share offsets)
        int lo = 0, hi = kScanChunk;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (s_off[mid] <= s) lo = mid; else hi = mid;
        }
        const uint32_t j = s - s_off[lo];
        const uint2 r = s_rect[lo];
        const uint32_t x0 = r.x & 0xFFFFu, x1 = r.x >> 16, y0 = r.y & 0xFFFFu;
        const uint32_t w = x1 - x0;
        const uint32_t dy = j / w;
        const uint32_t tx = x0 + (j - dy * w), ty = y0 + dy;
        const uint64_t tile = (uint64_t)ty * gp.tiles_x + tx;
        const unsigned long long key = (tile << dbits) | (uint64_t)(s_depth[lo] - dmin);
        if (fits) {
            keys[base + s] = key;
            vals[base + s] = (uint32_t)(c0 + lo);
        }
        for (uint32_t p = 0; p < npasses; ++p) atomicAdd(&s_hist[p][(key >> (8 * p)) & 255u], 1u);
    }
    __syncthreads();
    for (uint32_t i = tid; i < npasses * 256; i += kScanThreads) {
        const uint32_t v = (&s_hist[0][0])[i];
        if (v) atomicAdd(&(&ctl->hist[0][0])[i], v);
    }
    if (tid == 0 && (uint64_t)chunk == nchunks - 1) {
        ctl->num_keys = base + total;
        ctl->depth_bits = dbits;
        ctl->key_bits = key_bits;
    }
}

// One CTA of 256 threads: which passes move data, their bucket bases and buffer order.
__global__ void __launch_bounds__(256) k_plan(FrameCtl* ctl, uint64_t capacity, uint32_t max_passes,
                                              int mode) {
    __shared__ uint32_t s_warp[8];
    const int tid = threadIdx.x;
    const uint64_t K = ctl->num_keys;
    const bool ok = K <= capacity && (ctl->error_flags & kErrTimeout) == 0u;
    if (!ok) {
        if (tid == 0) {
            if (K > capacity) atomicOr(&ctl->error_flags, kErrCapacity);
            ctl->plan_ok = 0u;
        }
        return;
    }
    uint32_t npasses = (ctl->key_bits + 7) / 8;
    if (npasses > max_passes) npasses = max_passes;
    uint32_t run[kMaxPasses];
    uint32_t executed = 0;
    for (uint32_t p = 0; p < max_passes; ++p) {
        const uint32_t h = p < npasses ? ctl->hist[p][tid] : 0u;
        const int nz = __syncthreads_count(h != 0u);
        run[p] = nz > 1 ? 1u : 0u;
        uint32_t total;
        const uint32_t e = block_exclusive_scan(h, s_warp, &total);
        ctl->base[p][tid] = e;
        executed += run[p];
    }
    if (tid == 0) {
        if (mode == 1 && executed == 0 && K > 0) {
            run[0] = 1u;  // a single-bucket pass is a stable copy into the output
            executed = 1;
        }
        uint32_t cur = 0, e = 0;
        for (uint32_t p = 0; p < max_passes; ++p) {
            ctl->pass_run[p] = run[p];
            ctl->pass_ticket[p] = 0u;
            if (!run[p]) continue;
            uint32_t dst;
            if (mode == 0) {
                dst = cur ^ 1u;
            } else {
                dst = ((executed - 1 - e) % 2 == 0) ? 2u : 1u;
            }
            ctl->pass_src[p] = cur;
            ctl->pass_dst[p] = dst;
            cur = dst;
            ++e;
        }
        for (uint32_t p = 0; p < max_passes; ++p) {
            const uint32_t kb = ctl->key_bits, lo = 8 * p;
            ctl->pass_mask[p] = kb >= lo + 8 ? 255u : (kb > lo ? (1u << (kb - lo)) - 1u : 0u);
        }
        ctl->passes_run = executed;
        ctl->final_buf = (mode == 1 && executed == 0) ? 2u : cur;
        ctl->plan_ok = 1u;
    }
}

__global__ void k_ranges(SortIO io, const FrameCtl* ctl, uint2* ranges, FrameTotals* totals) {
    // every earlier kernel of the frame has finished: fold its error bits and sizes into the
    // running totals
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        if (ctl->error_flags) atomicOr(&totals->sticky_errors, ctl->error_flags);
        if (ctl->plan_ok) {
            totals->frames += 1ull;
            totals->keys += ctl->num_keys;
            totals->key_passes += ctl->num_keys * (unsigned long long)ctl->passes_run;
            totals->visible += ctl->num_visible;
        }
    }
    if (!ctl->plan_ok) return;
    const uint64_t K = ctl->num_keys;
    const uint32_t dbits = ctl->depth_bits;
    const unsigned long long* keys = io_keys(io, ctl->final_buf);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < K; i += stride) {
        const uint32_t t = (uint32_t)(keys[i] >> dbits);
        if (i == K - 1) {  // gsplat_bin_bounds.comp:44-52
            ranges[t].y = (uint32_t)(i + 1);
        } else {
            const uint32_t tn = (uint32_t)(keys[i + 1] >> dbits);
            if (t != tn) {  // comp:64-70
                ranges[t].y = (uint32_t)(i + 1);
                ranges[tn].x = (uint32_t)(i + 1);
            }
        }
    }
}

}  // namespace

cudaError_t launch_frame_init(FrameCtl* ctl, uint2* ranges, uint32_t ntiles, cudaStream_t stream) {
    unsigned blocks = (ntiles + 255) / 256;
    if (blocks < 1) blocks = 1;
    if (blocks > 1024) blocks = 1024;
    k_frame_init<<<blocks, 256, 0, stream>>>(ctl, ranges, ntiles);
    return cudaGetLastError();
}

cudaError_t launch_scan_emit(const FrameBufs& fb, const GridParams& gp, uint64_t n, uint32_t epoch,
                             uint32_t max_passes, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const unsigned chunks = (unsigned)((n + kScanChunk - 1) / kScanChunk);
    k_scan_emit<<<chunks, kScanThreads, 0, stream>>>(fb, gp, n, epoch, max_passes);
    return cudaGetLastError();
}

cudaError_t launch_plan(FrameCtl* ctl, uint64_t capacity, uint32_t max_passes, int mode,
                        cudaStream_t stream) {
    k_plan<<<1, 256, 0, stream>>>(ctl, capacity, max_passes, mode);
    return cudaGetLastError();
}

cudaError_t launch_ranges(const SortIO& io, const FrameCtl* ctl, uint2* ranges, FrameTotals* totals,
                          cudaStream_t stream) {
    k_ranges<<<device_sm_count() * 8, 256, 0, stream>>>(io, ctl, ranges, totals);
    return cudaGetLastError();
}

}  // namespace kt
