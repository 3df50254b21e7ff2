// Binning around the pair placement: the per-frame reset, the depth keys of the Gaussians with
// the digit histograms of their sort, the sort plan and the frame totals.
//
// The reference sorts one copy of each projected Gaussian per overlapped bin by the 48-bit key
// bin << 32 | depth, depth = floatBitsToUint(z) ^ 0x80000000
// (gsplat_radix_sort_include.glsl:51-63). Every copy carries its Gaussian's depth, so the same
// order is reached by sorting the N Gaussians by depth first (stable, ties by index) and then
// placing their pairs bin by bin in that order (place.cu). Depths enter as depth - depth_min of
// the frame (monotone, fewer bits).
#include "kt_common.cuh"
#include "kt_kernels.h"

namespace kt {
namespace {

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

__global__ void k_frame_init(FrameCtl* ctl, FrameCtl* ctl_depth, uint2* ranges, uint32_t ntiles) {
    const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    if (blockIdx.x == 0) {
        uint32_t* w = reinterpret_cast<uint32_t*>(ctl);
        uint32_t* wd = reinterpret_cast<uint32_t*>(ctl_depth);
        const uint32_t nw = sizeof(FrameCtl) / 4;
        for (uint32_t i = threadIdx.x; i < nw; i += blockDim.x) {
            w[i] = 0u;
            wd[i] = 0u;
        }
        __syncthreads();
        if (threadIdx.x == 0) ctl->depth_min = 0xFFFFFFFFu;
    }
    for (uint32_t t = tid; t < ntiles; t += gridDim.x * blockDim.x) ranges[t] = make_uint2(0u, 0u);
}

// Depth key of every Gaussian, (depth - depth_min) << idx_bits | index, with the digit
// histograms of the depth sort. A Gaussian that meets no bin is written as kDropKey and left out
// of the histograms: the sort's first executed pass drops it, so the sorted order holds the
// visible Gaussians only. The last CTA to finish plans the passes.
__device__ void plan_passes(FrameCtl* ctl, uint64_t capacity, uint32_t max_passes, int mode,
                            uint64_t keep);

__global__ void __launch_bounds__(256) k_depth_keys(FrameBufs fb, uint64_t n, uint32_t max_passes) {
    __shared__ uint32_t s_last;
    __shared__ uint32_t s_hist[8][4][256];  // per warp, per pass
    const FrameCtl* ctl = fb.ctl;
    FrameCtl* cd = fb.ctl_depth;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < 8 * 4 * 256; i += blockDim.x) (&s_hist[0][0][0])[i] = 0u;
    __syncthreads();
    const uint32_t dmin = ctl->depth_min, dmax = ctl->depth_max;
    const bool any = dmax >= dmin;
    const uint32_t dtop = any ? dmax - dmin : 0u;
    const uint32_t dbits = bits_for(dtop);
    const uint32_t ibits = bits_for(n - 1);
    const uint32_t npass = (dbits + 7) / 8;
    unsigned long long* out = fb.gsort[0];
    uint32_t (*hw)[256] = s_hist[warp];
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    constexpr int kItems = 4;  // elements per thread and round, loaded before they are used
    const uint64_t n_up = (n + 31) & ~31ull;  // whole warps iterate together
    for (uint64_t i0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n_up; i0 += stride * kItems) {
        uint32_t cnt[kItems], dep[kItems];
#pragma unroll
        for (int u = 0; u < kItems; ++u) {
            const uint64_t i = i0 + (uint64_t)u * stride;
            cnt[u] = i < n ? fb.counts[i] : 0u;
            dep[u] = i < n ? fb.depth[i] : 0u;
        }
#pragma unroll
        for (int u = 0; u < kItems; ++u) {
            const uint64_t i = i0 + (uint64_t)u * stride;
            if (i >= n_up) break;  // uniform over the warp
            const bool live = i < n;
            const bool vis = live && cnt[u] != 0u;
            const uint32_t dk = vis ? dep[u] - dmin : 0u;
            if (live) out[i] = vis ? (((unsigned long long)dk << ibits) | i) : kDropKey;
            const uint32_t act = __ballot_sync(0xFFFFFFFFu, vis);
            for (uint32_t p = 0; p < npass; ++p) {
                if (dbits - 8 * p == 1) {  // a one-bit digit (the top of a 25-bit range): two counts
                    const uint32_t ones = __ballot_sync(0xFFFFFFFFu, vis && ((dk >> (8 * p)) & 1u));
                    if (lane == 0) {
                        hw[p][0] += (uint32_t)__popc(act & ~ones);
                        hw[p][1] += (uint32_t)__popc(ones);
                    }
                } else if (vis) {  // warp-private counters: only lanes of this warp collide
                    atomicAdd(&hw[p][(dk >> (8 * p)) & 255u], 1u);
                }
            }
        }
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < npass * 256; i += blockDim.x) {
        uint32_t v = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) v += (&s_hist[w][0][0])[i];
        if (v) atomicAdd(&(&cd->hist[0][0])[i], v);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        cd->num_keys = n;
        cd->key_bits = dbits;
        cd->idx_bits = ibits;
        cd->packed = 1u;
    }
    __threadfence();  // this CTA's counts (and sizes) are visible before its ticket
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&cd->done_scan, 1u) == gridDim.x - 1u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    plan_passes(cd, n, max_passes, 0, __ldcg(&ctl->num_visible));
}

// One CTA of 256 threads: which passes move data, their bucket bases and buffer order. The
// histograms may come from other CTAs of the calling kernel (read at L2). keep < num_keys: only
// `keep` elements are not kDropKey; the first executed pass drops the others (a pass is forced
// if none would run) and the later passes read `keep` elements.
__device__ void plan_passes(FrameCtl* ctl, uint64_t capacity, uint32_t max_passes, int mode,
                            uint64_t keep) {
    __shared__ uint32_t s_warp[8];
    const int tid = threadIdx.x;
    const uint64_t K = __ldcg(&ctl->num_keys);
    const bool ok = K <= capacity && (__ldcg(&ctl->error_flags) & kErrTimeout) == 0u;
    if (!ok) {
        if (tid == 0) {
            if (K > capacity) atomicOr(&ctl->error_flags, kErrCapacity);
            ctl->plan_ok = 0u;
        }
        return;
    }
    const uint32_t key_bits = __ldcg(&ctl->key_bits);
    uint32_t npasses = (key_bits + 7) / 8;
    if (npasses > max_passes) npasses = max_passes;
    uint32_t run[kMaxPasses];
    uint32_t executed = 0;
    for (uint32_t p = 0; p < max_passes; ++p) {
        const uint32_t h = p < npasses ? __ldcg(&ctl->hist[p][tid]) : 0u;
        const int nz = __syncthreads_count(h != 0u);
        run[p] = nz > 1 ? 1u : 0u;
        uint32_t total;
        const uint32_t e = block_exclusive_scan(h, s_warp, &total);
        ctl->base[p][tid] = e;
        executed += run[p];
    }
    if (tid == 0) {
        const bool dropping = keep < K;
        if ((mode == 1 || dropping) && executed == 0 && K > 0) {
            run[0] = 1u;  // a single-bucket pass is a stable copy into the output (and drops)
            executed = 1;
        }
        uint32_t cur = 0, e = 0;
        bool dropped = false;
        for (uint32_t p = 0; p < max_passes; ++p) {
            ctl->pass_run[p] = run[p];
            ctl->pass_ticket[p] = 0u;
            ctl->pass_in[p] = dropped ? keep : K;
            ctl->pass_drop[p] = 0u;
            if (!run[p]) continue;
            if (dropping && !dropped) {
                ctl->pass_drop[p] = 1u;
                dropped = true;
            }
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
            const uint32_t kb = key_bits, lo = 8 * p;
            ctl->pass_mask[p] = kb >= lo + 8 ? 255u : (kb > lo ? (1u << (kb - lo)) - 1u : 0u);
        }
        ctl->passes_run = executed;
        ctl->final_buf = (mode == 1 && executed == 0) ? 2u : cur;
        ctl->plan_ok = 1u;
    }
}

__global__ void __launch_bounds__(256) k_plan(FrameCtl* ctl, uint64_t capacity, uint32_t max_passes,
                                              int mode) {
    plan_passes(ctl, capacity, max_passes, mode, ~0ull);
}

// After the pair placement: fold the frame's error bits and sizes into the running totals
// (kt_gs_counters, kt_gs_sync).
__global__ void k_frame_totals(const FrameCtl* ctl, const FrameCtl* ctl_depth, FrameTotals* totals) {
    const unsigned int err = ctl->error_flags | ctl_depth->error_flags;
    if (err) atomicOr(&totals->sticky_errors, err);
    if (ctl->plan_ok) {
        totals->frames += 1ull;
        totals->keys += ctl->num_keys;
        totals->key_passes += ctl->num_keys * (unsigned long long)ctl->passes_run;
        totals->visible += ctl->num_visible;
        // placement: (Gaussian, coarse bin) entries (8 B) and pairs (u32) written once; keys path:
        // the executed passes of the pair sort
        totals->sort_bytes += ctl->passes_run ? ctl->num_keys * (unsigned long long)ctl->passes_run *
                                                    (ctl->packed ? 16ull : 24ull)
                                              : ctl->num_keys * 4ull + ctl->num_entries * 8ull;
        unsigned long long moved = 0;
        for (int p = 0; p < kMaxPasses; ++p)
            if (ctl_depth->pass_run[p]) moved += ctl_depth->pass_in[p];
        totals->depth_sort_bytes += moved * 16ull;
    }
}

}  // namespace

cudaError_t launch_frame_init(FrameCtl* ctl, FrameCtl* ctl_depth, uint2* ranges, uint32_t ntiles,
                              cudaStream_t stream) {
    unsigned blocks = (ntiles + 255) / 256;
    if (blocks < 1) blocks = 1;
    if (blocks > 1024) blocks = 1024;
    k_frame_init<<<blocks, 256, 0, stream>>>(ctl, ctl_depth, ranges, ntiles);
    return cudaGetLastError();
}

cudaError_t launch_depth_keys(const FrameBufs& fb, uint64_t n, uint32_t max_passes, cudaStream_t stream) {
    if (n == 0) {  // nothing to sort: the plan alone
        k_plan<<<1, 256, 0, stream>>>(fb.ctl_depth, n, max_passes, 0);
        return cudaGetLastError();
    }
    // few CTAs with many Gaussians each: every CTA adds its histograms to the frame's once
    uint64_t blocks = (n + 2047) / 2048;
    const uint64_t cap = (uint64_t)device_sm_count() * 2;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    k_depth_keys<<<(unsigned)blocks, 256, 0, stream>>>(fb, n, max_passes);
    return cudaGetLastError();
}

cudaError_t launch_plan(FrameCtl* ctl, uint64_t capacity, uint32_t max_passes, int mode,
                        cudaStream_t stream) {
    k_plan<<<1, 256, 0, stream>>>(ctl, capacity, max_passes, mode);
    return cudaGetLastError();
}

cudaError_t launch_frame_totals(const FrameCtl* ctl, const FrameCtl* ctl_depth, FrameTotals* totals,
                                cudaStream_t stream) {
    k_frame_totals<<<1, 1, 0, stream>>>(ctl, ctl_depth, totals);
    return cudaGetLastError();
}

}  // namespace kt
