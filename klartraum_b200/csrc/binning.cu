// Binning: depth keys of the Gaussians, the exclusive scan of the per-Gaussian bin counts in
// depth order (decoupled look-back) fused with the emission of one element per (bin, Gaussian)
// pair; plus the per-frame reset, the sort plan and the bin-range search (K5).
//
// The reference duplicates each projected Gaussian once per overlapped bin with atomicAdd
// (shaders/gsplat/gsplat_binning.comp:112-159; order nondeterministic, capped at 2N) and then
// sorts the copies by the 48-bit key bin<<32 | depth, depth = floatBitsToUint(z) ^ 0x80000000
// (gsplat_radix_sort_include.glsl:51-63). Every copy carries its Gaussian's depth, so the same
// order is reached by sorting the N Gaussians by depth first (stable, ties by index), emitting
// the pairs in that order, and then sorting the pairs stably by bin alone: 2 passes over the
// pairs instead of 5. Depths enter as depth - depth_min of the frame (monotone, fewer bits).
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
// histograms of the depth sort. Gaussians that touch no bin take the largest depth; they
// emit nothing, so where they land does not matter.
__global__ void __launch_bounds__(256) k_depth_keys(FrameBufs fb, uint64_t n) {
    __shared__ uint32_t s_hist[4][256];
    const FrameCtl* ctl = fb.ctl;
    FrameCtl* cd = fb.ctl_depth;
    for (int i = threadIdx.x; i < 4 * 256; i += blockDim.x) (&s_hist[0][0])[i] = 0u;
    __syncthreads();
    const uint32_t dmin = ctl->depth_min, dmax = ctl->depth_max;
    const bool any = dmax >= dmin;
    const uint32_t dtop = any ? dmax - dmin : 0u;
    const uint32_t dbits = bits_for(dtop);
    const uint32_t ibits = bits_for(n - 1);
    const uint32_t npass = (dbits + 7) / 8;
    unsigned long long* out = fb.gsort[0];
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const int lane = threadIdx.x & 31;
    const uint64_t n_up = (n + 31) & ~31ull;  // whole warps iterate together
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_up; i += stride) {
        const bool live = i < n;
        const uint32_t dk = live ? (fb.counts[i] != 0u ? fb.depth[i] - dmin : dtop) : 0u;
        if (live) out[i] = ((unsigned long long)dk << ibits) | i;
        for (uint32_t p = 0; p < npass; ++p) {
            // lanes with the same digit add once (the top digits of nearby depths collide)
            const uint32_t d = live ? (dk >> (8 * p)) & 255u : 256u;
            const uint32_t peers = __match_any_sync(0xFFFFFFFFu, d);
            if (live && lane == __ffs(peers) - 1) atomicAdd(&s_hist[p][d], (uint32_t)__popc(peers));
        }
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < npass * 256; i += blockDim.x) {
        const uint32_t v = (&s_hist[0][0])[i];
        if (v) atomicAdd(&(&cd->hist[0][0])[i], v);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        cd->num_keys = n;
        cd->key_bits = dbits;
        cd->idx_bits = ibits;
        cd->packed = 1u;
    }
}

__global__ void __launch_bounds__(kScanThreads) k_scan_emit(FrameBufs fb, GridParams gp, uint64_t n,
                                                            uint32_t epoch, uint32_t max_passes) {
    __shared__ uint32_t s_off[kScanChunk + 1];
    __shared__ uint2 s_rect[kScanChunk];
    __shared__ uint32_t s_gid[kScanChunk];
    __shared__ uint32_t s_warp[8];
    __shared__ uint32_t s_chunk;
    __shared__ unsigned long long s_base;

    FrameCtl* ctl = fb.ctl;
    const FrameCtl* cd = fb.ctl_depth;
    const int tid = threadIdx.x;
    if (tid == 0) s_chunk = atomicAdd(&ctl->scan_ticket, 1u);
    __syncthreads();
    const uint32_t chunk = s_chunk;
    const uint64_t nchunks = (n + kScanChunk - 1) / kScanChunk;
    const uint64_t c0 = (uint64_t)chunk * kScanChunk;
    // Gaussians in depth order: the sorted depth keys carry the index in their low bits
    const unsigned long long* order = io_select(fb.gsort, cd->final_buf);
    const uint32_t ibits = cd->idx_bits;
    const unsigned long long imask = (1ull << ibits) - 1ull;

    // counts of this thread's 8 consecutive positions in depth order
    uint32_t c[kScanItems], gid[kScanItems];
    uint32_t sum = 0;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const uint64_t q = c0 + (uint64_t)tid * kScanItems + j;
        gid[j] = q < n ? (uint32_t)(order[q] & imask) : 0u;
        c[j] = q < n ? fb.counts[gid[j]] : 0u;
        sum += c[j];
    }
    uint32_t total;
    const uint32_t texcl = block_exclusive_scan(sum, s_warp, &total);
    {
        uint32_t run = texcl;
#pragma unroll
        for (int j = 0; j < kScanItems; ++j) {
            const int l = tid * kScanItems + j;
            s_off[l] = run;
            if (c[j] != 0u) {
                s_rect[l] = fb.rect[gid[j]];
                s_gid[l] = gid[j];
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

    // pairs: bin << idx_bits | index; the sort by bin is stable, so depth order survives
    // (the digit histograms of that sort come from k_bin_finalize)
    const uint32_t key_bits = gp.tile_bits;
    const bool fits = base + total <= fb.key_capacity;
    unsigned long long* keys = fb.keys[0];

    // Emission: warp w walks its 256 positions in order; the lanes write one Gaussian's bins
    // (row-major over its rectangle) as one coalesced run.
    const int lane = tid & 31, warp = tid >> 5;
    for (int q0 = warp * (kScanChunk / 8); q0 < (warp + 1) * (kScanChunk / 8); q0 += 32) {
        const int q = q0 + lane;
        uint32_t todo = __ballot_sync(0xFFFFFFFFu, s_off[q + 1] != s_off[q]);
        while (todo) {
            const int l = q0 + __ffs(todo) - 1;
            todo &= todo - 1u;
            const uint32_t off = s_off[l], cnt = s_off[l + 1] - off;
            const uint2 r = s_rect[l];
            const uint32_t gid = s_gid[l];
            const uint32_t x0 = r.x & 0xFFFFu, x1 = r.x >> 16, y0 = r.y & 0xFFFFu;
            const uint32_t w = x1 - x0;
            const float inv_w = 1.0f / (float)w;
            for (uint32_t j = lane; j < cnt; j += 32) {
                uint32_t dy = (uint32_t)((float)j * inv_w);  // j / w, then corrected exactly
                if (dy * w > j) --dy;
                if ((dy + 1) * w <= j) ++dy;
                const uint32_t tile = (y0 + dy) * gp.tiles_x + x0 + (j - dy * w);
                if (fits) keys[base + off + j] = ((unsigned long long)tile << ibits) | gid;
            }
        }
    }
    if (tid == 0 && (uint64_t)chunk == nchunks - 1) {
        const uint32_t dmin = ctl->depth_min, dmax = ctl->depth_max;
        ctl->num_keys = base + total;
        ctl->depth_bits = dmax >= dmin ? bits_for((uint64_t)(dmax - dmin)) : 0u;
        ctl->key_bits = key_bits;
        ctl->packed = 1u;
        ctl->idx_bits = ibits;
    }
}

// Per-bin pair counts from the Gaussians' bin rectangles: +1/-1 at the four corners of each
// rectangle in a (tiles_y + 1) x (tiles_x + 1) difference table, accumulated per CTA in shared
// memory when it fits (4 atomics per Gaussian instead of one per pair).
__global__ void __launch_bounds__(512) k_bin_diff(FrameBufs fb, GridParams gp, uint64_t n, int* gdiff,
                                                  int use_smem) {
    extern __shared__ int s_diff[];
    const uint32_t W1 = gp.tiles_x + 1;
    const uint32_t cells = W1 * (gp.tiles_y + 1);
    int* table = use_smem ? s_diff : gdiff;
    if (use_smem) {
        for (uint32_t i = threadIdx.x; i < cells; i += blockDim.x) s_diff[i] = 0;
        __syncthreads();
    }
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        if (fb.counts[i] == 0u) continue;
        const uint2 r = fb.rect[i];
        const uint32_t x0 = r.x & 0xFFFFu, x1 = r.x >> 16, y0 = r.y & 0xFFFFu, y1 = r.y >> 16;
        atomicAdd(&table[y0 * W1 + x0], 1);
        atomicAdd(&table[y0 * W1 + x1], -1);
        atomicAdd(&table[y1 * W1 + x0], -1);
        atomicAdd(&table[y1 * W1 + x1], 1);
    }
    if (use_smem) {
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < cells; i += blockDim.x)
            if (s_diff[i] != 0) atomicAdd(&gdiff[i], s_diff[i]);
    }
}

// One CTA of 1024 threads: 2D prefix sums of the difference table (in place) give the pairs per
// bin; their exclusive scan gives every bin's range {start, end} in the sorted pair list (empty
// bins stay {0, 0}, as the reference's zeroed StartAndEnd buffer), and their digits give the
// histograms of the bin sort. The table is left zeroed for the next frame.
__global__ void __launch_bounds__(1024) k_bin_finalize(FrameBufs fb, GridParams gp, int* gdiff,
                                                       uint32_t max_passes) {
    __shared__ uint32_t s_hist[kMaxPasses][256];
    __shared__ uint32_t s_warp[32];
    __shared__ unsigned long long s_carry;
    const uint32_t tx = gp.tiles_x, ty = gp.tiles_y, W1 = tx + 1;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < kMaxPasses * 256; i += blockDim.x) (&s_hist[0][0])[i] = 0u;
    // prefix along x, one warp per row
    for (uint32_t row = warp; row < ty; row += 32) {
        int carry = 0;
        for (uint32_t x0 = 0; x0 < tx; x0 += 32) {
            const uint32_t x = x0 + lane;
            int v = x < tx ? gdiff[row * W1 + x] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xFFFFFFFFu, v, o);
                if (lane >= o) v += y;
            }
            if (x < tx) gdiff[row * W1 + x] = v + carry;
            carry += __shfl_sync(0xFFFFFFFFu, v, 31);
        }
    }
    __syncthreads();
    // prefix along y, one warp per column: the pairs of bin (row, x)
    for (uint32_t x = warp; x < tx; x += 32) {
        int carry = 0;
        for (uint32_t y0 = 0; y0 < ty; y0 += 32) {
            const uint32_t y = y0 + lane;
            int v = y < ty ? gdiff[y * W1 + x] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xFFFFFFFFu, v, o);
                if (lane >= o) v += t;
            }
            if (y < ty) gdiff[y * W1 + x] = v + carry;
            carry += __shfl_sync(0xFFFFFFFFu, v, 31);
        }
    }
    __syncthreads();
    // exclusive scan over bins in row-major order, 1024 bins per round
    uint32_t npasses = (gp.tile_bits + 7) / 8;
    if (npasses > max_passes) npasses = max_passes;
    const uint32_t nbins = tx * ty;
    if (tid == 0) s_carry = 0ull;
    __syncthreads();
    for (uint32_t b0 = 0; b0 < nbins; b0 += 1024) {
        const uint32_t b = b0 + tid;
        const uint32_t by = b / tx, bx = b - by * tx;
        const uint32_t cnt = b < nbins ? (uint32_t)gdiff[by * W1 + bx] : 0u;
        uint32_t x = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, x, o);
            if (lane >= o) x += t;
        }
        if (lane == 31) s_warp[warp] = x;
        __syncthreads();
        if (warp == 0) {
            uint32_t w = s_warp[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, w, o);
                if (lane >= o) w += t;
            }
            s_warp[lane] = w;
        }
        __syncthreads();
        const unsigned long long start = s_carry + (warp ? s_warp[warp - 1] : 0u) + x - cnt;
        if (b < nbins) {
            fb.ranges[b] = cnt ? make_uint2((uint32_t)start, (uint32_t)(start + cnt)) : make_uint2(0u, 0u);
            for (uint32_t p = 0; p < npasses; ++p)
                if (cnt) atomicAdd(&s_hist[p][(b >> (8 * p)) & 255u], cnt);
        }
        __syncthreads();
        if (tid == 0) s_carry += s_warp[31];
        __syncthreads();
    }
    // clear the table for the next frame (every cell, including the padding row and column)
    const uint32_t cells = W1 * (ty + 1);
    for (uint32_t i = tid; i < cells; i += blockDim.x) gdiff[i] = 0;
    for (uint32_t i = tid; i < npasses * 256; i += blockDim.x) (&fb.ctl->hist[0][0])[i] = (&s_hist[0][0])[i];
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

// After the last sort pass: fold the frame's error bits and sizes into the running totals
// (kt_gs_counters, kt_gs_sync).
__global__ void k_frame_totals(const FrameCtl* ctl, const FrameCtl* ctl_depth, FrameTotals* totals) {
    if (ctl->error_flags) atomicOr(&totals->sticky_errors, ctl->error_flags);
    if (ctl->plan_ok) {
        totals->frames += 1ull;
        totals->keys += ctl->num_keys;
        totals->key_passes += ctl->num_keys * (unsigned long long)ctl->passes_run;
        totals->visible += ctl->num_visible;
        totals->sort_bytes += ctl->num_keys * (unsigned long long)ctl->passes_run * 16ull;
        totals->depth_sort_bytes += ctl_depth->num_keys * (unsigned long long)ctl_depth->passes_run * 16ull;
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

cudaError_t launch_bin_counts(const FrameBufs& fb, const GridParams& gp, uint64_t n, int* gdiff,
                              uint32_t max_passes, cudaStream_t stream) {
    const size_t cells = (size_t)(gp.tiles_x + 1) * (gp.tiles_y + 1);
    const size_t smem = cells * sizeof(int);
    const bool use_smem = smem <= 96 * 1024;
    static bool attr_set[128] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (use_smem && dev >= 0 && dev < 128 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(k_bin_diff, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    if (n > 0) {
        uint64_t blocks = (n + 511) / 512;
        const uint64_t cap = (uint64_t)device_sm_count() * (use_smem ? 2 : 8);
        if (blocks > cap) blocks = cap;
        k_bin_diff<<<(unsigned)blocks, 512, use_smem ? smem : 0, stream>>>(fb, gp, n, gdiff, use_smem ? 1 : 0);
    }
    k_bin_finalize<<<1, 1024, 0, stream>>>(fb, gp, gdiff, max_passes);
    return cudaGetLastError();
}

cudaError_t launch_depth_keys(const FrameBufs& fb, uint64_t n, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    uint64_t blocks = (n + 255) / 256;
    const uint64_t cap = (uint64_t)device_sm_count() * 8;
    if (blocks > cap) blocks = cap;
    k_depth_keys<<<(unsigned)blocks, 256, 0, stream>>>(fb, n);
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

cudaError_t launch_frame_totals(const FrameCtl* ctl, const FrameCtl* ctl_depth, FrameTotals* totals,
                                cudaStream_t stream) {
    k_frame_totals<<<1, 1, 0, stream>>>(ctl, ctl_depth, totals);
    return cudaGetLastError();
}

}  // namespace kt
