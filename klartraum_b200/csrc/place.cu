// Pairs by bin without a pair sort: a two-level stable counting sort of the (bin, Gaussian)
// pairs, fed with the Gaussians in depth order.
//
// The reference duplicates each projected Gaussian once per overlapped bin and sorts the copies
// by the 48-bit key bin << 32 | depth (shaders/gsplat/gsplat_binning.comp:112-159,
// gsplat_radix_sort_include.glsl:51-63). With the Gaussians already sorted by depth (stable,
// ties by index) that order is: by bin, then by the Gaussian's position in depth order. The
// pairs of one Gaussian cover a rectangle of bins, so they never need to exist unsorted.
//
// Level 1, coarse bins of 4x4 bins (a Gaussian meets 3.4 of them on average where it meets 20
// bins):
//   k_coarse_count   one CTA per group of 8 chunks (a chunk is a run of depth order): the
//                    Gaussians' rectangles are gathered into depth order (srect) and every
//                    coarse bin a rectangle meets is counted in shared memory per chunk:
//                    table[chunk][coarse bin] (prefix over the group's chunks) and
//                    gtable[group][coarse bin] (the group's total).
//   k_coarse_scan    per coarse bin, the exclusive prefix of gtable over groups (in place) and
//                    the bin's entry total; the last CTA to finish then computes K (the
//                    projection's pair total) and the capacity check, and the exclusive scans of
//                    the coarse totals (list starts) and of their segment counts (kSegLen entries
//                    per segment).
//   k_coarse_place   writes the segment -> coarse bin map (a warp per coarse bin), then
//                    persistent warps over (band, chunk) items: 32 Gaussians at a time, their
//                    (Gaussian, coarse bin) entries flattened in depth order and taken 32 at a
//                    time; lanes with equal coarse bins are ranked by lane (each sets its bit in the
//                    bin's word of a per-warp shared-memory array) and written at the bin's cursor
//                    as (Gaussian index, mask of the 4x4 bins met).
// Level 2, the bins of a coarse bin:
//   k_fine_count     a warp per segment of a coarse list: pairs per bin of the 4x4 (byte
//                    counters per lane, then warp sums), stored per segment and added to the
//                    bins' totals; the last CTA to finish scans the totals into ranges {start,
//                    end} (empty bins keep {0, 0}, as the reference's zeroed StartAndEnd buffer).
//   k_fine_place     a warp per segment: its bins' cursors are the bin starts plus the counts of
//                    the coarse list's earlier segments; then 32 entries at a time, for each bin
//                    of the 4x4 a ballot ranks the entries that meet it; each writes its Gaussian
//                    at the bin's cursor + rank (consecutive addresses per bin).
// Chunks take consecutive slices of every coarse list, segments consecutive slices of every bin
// and every step ranks by lane, so equal-bin pairs land in depth order: the stable sort of the
// pairs by bin. A pair is stored as its Gaussian's index (4 bytes); its bin is implied by the
// ranges.
#include "kt_common.cuh"
#include "kt_kernels.h"

namespace kt {
namespace {

constexpr uint32_t kCoarse = 4;                // bins per side of a coarse bin
constexpr uint32_t kChunkTarget = 256;         // Gaussians per chunk of depth order, about
constexpr uint32_t kMaxChunks = 8192;
constexpr uint32_t kCountThreads = 512;
constexpr uint32_t kCoarseMax = 16384;         // coarse bins x chunks of a count CTA (64 KB of counters)
constexpr uint32_t kGroupMax = 8;              // chunks of a count CTA
#ifndef KT_PLACE_BAND_MAX
#define KT_PLACE_BAND_MAX 1024
#endif
constexpr uint32_t kBandMax = KT_PLACE_BAND_MAX;  // coarse bins of a placement band (4 B of cursor per warp each)
constexpr uint32_t kPlaceWarps = 16;           // warps of a coarse-placement CTA
// Coarse bins of a placement band when the lists get long runs: every warp of the coarse placement
// writes each list of its band at its own cursor, so the partly written 32-B sectors in flight are
// about (warps in flight) x (bins of a band); when a (chunk, coarse bin) run holds several entries,
// a small band keeps those sectors in L2 until they are whole.
#ifndef KT_PLACE_LONG_RUN_BAND
#define KT_PLACE_LONG_RUN_BAND 64
#endif
constexpr uint32_t kLongRunBand = KT_PLACE_LONG_RUN_BAND;
constexpr uint32_t kLongRun = 4;               // entries per (chunk, coarse bin) that count as long runs
constexpr uint32_t kPlaceCtasPerSm = 2;
constexpr uint32_t kPlaceSmem = 2 * kPlaceWarps * kBandMax * 4;  // cursors and lane bits
constexpr uint32_t kSegLen = 256;              // entries of a segment of a coarse list
constexpr uint32_t kSegWarps = 8;              // warps of a pair-placement CTA
constexpr uint32_t kSegGroup = 8;              // consecutive segments a run of k_fine_place_runs holds, at most
constexpr uint32_t kCountWarps = 32;           // warps of a bin-count CTA (its last CTA scans 8192 bins a round)
constexpr int kRangesThreads = 1024;
constexpr int kRangesItems = 8;                // consecutive bins per thread and round

// (q, r) = (a / w, a % w) for a < 2^20, w >= 1: float quotient, then corrected exactly.
__device__ __forceinline__ void divmod_small(uint32_t a, uint32_t w, float inv_w, uint32_t& q, uint32_t& r) {
    q = (uint32_t)((float)a * inv_w);
    if (q * w > a) --q;
    if ((q + 1) * w <= a) ++q;
    r = a - q * w;
}

// Bits [lo, hi) of a 4-bit row or column set.
__device__ __forceinline__ uint32_t span4(uint32_t lo, uint32_t hi) {
    return ((1u << hi) - 1u) & ~((1u << lo) - 1u);
}

// Rectangle of a Gaussian in bins, clipped to the binned rows; rows relative to row_begin.
// Returns false for an empty rectangle.
__device__ __forceinline__ bool local_rect(uint2 r, const GridParams& gp, uint32_t& x0, uint32_t& x1, uint32_t& y0,
                                           uint32_t& y1) {
    x0 = r.x & 0xFFFFu;
    x1 = min(r.x >> 16, gp.tiles_x);
    y0 = max(r.y & 0xFFFFu, gp.row_begin);
    y1 = min(r.y >> 16, gp.row_end);
    if (x0 >= x1 || y0 >= y1) return false;
    y0 -= gp.row_begin;
    y1 -= gp.row_begin;
    return true;
}

// ------------------------------------------------------------------- level 1

// One CTA per group of chunks: the group's Gaussians counted per (chunk, coarse bin) in shared
// memory; table[chunk][bin] <- prefix over the group's earlier chunks, gtable[group][bin] <- the
// group's total.
__global__ void __launch_bounds__(kCountThreads) k_coarse_count(FrameBufs fb, GridParams gp, PlaceGeom pg,
                                                                uint64_t n) {
    // per chunk a (cty + 1) x (ctx + 1) difference array: a Gaussian adds its coarse rectangle's
    // four corners (+1, -1, -1, +1), and a 2D prefix sum turns the corners into the entry counts
    // of every coarse bin (four shared-memory atomics per Gaussian whatever its size)
    extern __shared__ uint32_t s_cnt[];  // [group][cty + 1][ctx + 1]
    const uint32_t cw = pg.ctx + 1u, ch = pg.cty + 1u, cells = cw * ch;
    const uint32_t c0 = blockIdx.x * pg.group, gk = min(pg.group, pg.nchunks - c0);
    const uint32_t words = gk * cells;
    for (uint32_t i = threadIdx.x; i < words; i += kCountThreads) s_cnt[i] = 0u;
    __syncthreads();
    const FrameCtl* cd = fb.ctl_depth;
    const unsigned long long* __restrict__ order = io_select(fb.gsort, cd->final_buf);
    const unsigned long long imask = (1ull << cd->idx_bits) - 1ull;
    // the depth order holds the Gaussians that meet a bin (the sort dropped the others)
    const uint64_t nsorted = min((uint64_t)fb.ctl->num_visible, n);
    const uint64_t q0 = (uint64_t)c0 * pg.chunk_len;
    const uint64_t q1 = min(q0 + (uint64_t)gk * pg.chunk_len, nsorted);
    constexpr int kU = 4;  // Gaussians in flight per thread
    for (uint64_t qb = q0 + threadIdx.x; qb < q1; qb += kU * kCountThreads) {
        uint32_t g[kU];
        uint2 r[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const uint64_t q = qb + (uint64_t)u * kCountThreads;
            g[u] = q < q1 ? (uint32_t)(order[q] & imask) : 0xFFFFFFFFu;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u)  // the projection stores an empty rectangle for a Gaussian without bins
            r[u] = g[u] != 0xFFFFFFFFu ? fb.rect[g[u]] : make_uint2(0u, 0u);
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const uint64_t q = qb + (uint64_t)u * kCountThreads;
            if (q >= q1) break;
            fb.srect[q] = r[u];
            uint32_t x0, x1, y0, y1;
            if (!local_rect(r[u], gp, x0, x1, y0, y1)) continue;
            uint32_t* cnt = s_cnt + ((uint32_t)(q - q0) / pg.chunk_len) * cells;
            const uint32_t cx0 = x0 / kCoarse, cx1 = (x1 + kCoarse - 1) / kCoarse;
            const uint32_t cy0 = y0 / kCoarse, cy1 = (y1 + kCoarse - 1) / kCoarse;
            atomicAdd(&cnt[cy0 * cw + cx0], 1u);
            atomicAdd(&cnt[cy0 * cw + cx1], 0xFFFFFFFFu);  // -1 (modulo 2^32: the sums stay exact)
            atomicAdd(&cnt[cy1 * cw + cx0], 0xFFFFFFFFu);
            atomicAdd(&cnt[cy1 * cw + cx1], 1u);
        }
    }
    __syncthreads();
    for (uint32_t t = threadIdx.x; t < gk * ch; t += kCountThreads) {  // along x, a thread per row
        uint32_t* row = s_cnt + (t / ch) * cells + (t % ch) * cw;
        uint32_t run = 0;
        for (uint32_t x = 0; x < cw; ++x) {
            run += row[x];
            row[x] = run;
        }
    }
    __syncthreads();
    for (uint32_t t = threadIdx.x; t < gk * cw; t += kCountThreads) {  // along y, a thread per column
        uint32_t* col = s_cnt + (t / cw) * cells + (t % cw);
        uint32_t run = 0;
        for (uint32_t y = 0; y < ch; ++y) {
            run += col[y * cw];
            col[y * cw] = run;
        }
    }
    __syncthreads();
    uint32_t* __restrict__ trow = fb.ctable + (uint64_t)c0 * pg.ncoarse;
    for (uint32_t b = threadIdx.x; b < pg.ncoarse; b += kCountThreads) {
        const uint32_t cell = (b / pg.ctx) * cw + (b % pg.ctx);
        uint32_t run = 0;
        for (uint32_t k = 0; k < gk; ++k) {
            const uint32_t v = s_cnt[k * cells + cell];
            trow[(uint64_t)k * pg.ncoarse + b] = run;
            run += v;
        }
        fb.gtable[(uint64_t)blockIdx.x * pg.ncoarse + b] = run;
    }
}

// 32 coarse bins per CTA (lanes), the groups split into 32 slices (warps): gtable becomes the
// exclusive prefix over groups, cinfo[bin].y the bin's entry total. The last CTA to finish then
// computes the coarse list starts and segments (coarse_ranges, below).
__device__ void coarse_ranges(const FrameBufs& fb, const GridParams& gp, const PlaceGeom& pg, uint32_t ncoarse);

__global__ void __launch_bounds__(1024) k_coarse_scan(FrameBufs fb, GridParams gp, PlaceGeom pg) {
    __shared__ uint32_t s_seg[32][33];
    __shared__ uint32_t s_last;
    const int lane = threadIdx.x & 31, seg = threadIdx.x >> 5;
    const uint64_t B = pg.ncoarse;
    const uint32_t b = blockIdx.x * 32 + lane;
    const bool live = b < pg.ncoarse;
    const uint32_t per = (pg.ngroups + 31) / 32;
    const uint32_t c0 = min(seg * per, pg.ngroups), c1 = min(c0 + per, pg.ngroups);
    uint32_t* __restrict__ col = fb.gtable + b;
    constexpr uint32_t kU = 8;      // rows in flight per thread
    constexpr uint32_t kHold = 16;  // rows a thread keeps in registers between the two passes
    const bool hold = per <= kHold;  // the same for the whole CTA
    uint32_t held[kHold];
    uint32_t sum = 0;
    if (hold) {
#pragma unroll
        for (uint32_t u = 0; u < kHold; ++u) {
            held[u] = live && c0 + u < c1 ? col[(uint64_t)(c0 + u) * B] : 0u;
            sum += held[u];
        }
    } else if (live) {
        for (uint32_t c = c0; c < c1; c += kU) {
            uint32_t v[kU];
#pragma unroll
            for (uint32_t u = 0; u < kU; ++u) v[u] = c + u < c1 ? col[(uint64_t)(c + u) * B] : 0u;
#pragma unroll
            for (uint32_t u = 0; u < kU; ++u) sum += v[u];
        }
    }
    s_seg[seg][lane] = sum;
    __syncthreads();
    uint32_t base = 0;
    for (int s = 0; s < seg; ++s) base += s_seg[s][lane];
    if (live) {
        if (seg == 31) fb.cinfo[b] = make_uint4(0u, base + sum, 0u, 0u);  // the bin's total
        if (hold) {
#pragma unroll
            for (uint32_t u = 0; u < kHold; ++u) {
                if (c0 + u < c1) col[(uint64_t)(c0 + u) * B] = base;
                base += held[u];
            }
        } else {
            for (uint32_t c = c0; c < c1; c += kU) {
                uint32_t v[kU];
#pragma unroll
                for (uint32_t u = 0; u < kU; ++u) v[u] = c + u < c1 ? col[(uint64_t)(c + u) * B] : 0u;
#pragma unroll
                for (uint32_t u = 0; u < kU; ++u) {
                    if (c + u < c1) col[(uint64_t)(c + u) * B] = base;
                    base += v[u];
                }
            }
        }
    }
    __threadfence();  // every thread's writes are visible before the CTA's ticket
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&fb.ctl->done_scan, 1u) == gridDim.x - 1u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    coarse_ranges(fb, gp, pg, pg.ncoarse);
}

// Exclusive block scan of two counters per thread; returns the prefixes, adds the block totals
// to the carries.
__device__ __forceinline__ uint2 block_scan2(uint32_t a, uint32_t b, uint32_t* s_a, uint32_t* s_b,
                                             unsigned long long& carry_a, unsigned long long& carry_b) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t xa = a, xb = b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t ta = __shfl_up_sync(0xFFFFFFFFu, xa, o);
        const uint32_t tb = __shfl_up_sync(0xFFFFFFFFu, xb, o);
        if (lane >= o) {
            xa += ta;
            xb += tb;
        }
    }
    if (lane == 31) {
        s_a[warp] = xa;
        s_b[warp] = xb;
    }
    __syncthreads();
    if (warp == 0) {
        uint32_t wa = s_a[lane], wb = s_b[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t ta = __shfl_up_sync(0xFFFFFFFFu, wa, o);
            const uint32_t tb = __shfl_up_sync(0xFFFFFFFFu, wb, o);
            if (lane >= o) {
                wa += ta;
                wb += tb;
            }
        }
        s_a[lane] = wa;
        s_b[lane] = wb;
    }
    __syncthreads();
    const uint2 out = make_uint2((uint32_t)carry_a + (warp ? s_a[warp - 1] : 0u) + xa - a,
                                 (uint32_t)carry_b + (warp ? s_b[warp - 1] : 0u) + xb - b);
    const uint32_t ta = s_a[31], tb = s_b[31];
    __syncthreads();
    carry_a += ta;
    carry_b += tb;
    return out;
}

// K and the capacity check; list starts and segments of the coarse bins (entry totals in
// cinfo[.].y, written by other CTAs of the same kernel or by an earlier one). One CTA.
__device__ void coarse_ranges(const FrameBufs& fb, const GridParams& gp, const PlaceGeom& pg, uint32_t ncoarse) {
    __shared__ uint32_t s_a[32], s_b[32];
    __shared__ uint32_t s_ok;
    FrameCtl* ctl = fb.ctl;
    const int tid = threadIdx.x;
    if (tid == 0) {
        const FrameCtl* cd = fb.ctl_depth;
        const unsigned long long K = ctl->pair_total;
        const uint32_t dmin = ctl->depth_min, dmax = ctl->depth_max;
        ctl->num_keys = K;
        ctl->depth_bits = dmax >= dmin ? bits_for((uint64_t)(dmax - dmin)) : 0u;
        ctl->key_bits = gp.tile_bits;
        ctl->packed = 0u;  // pairs are u32 Gaussian indices
        ctl->idx_bits = cd->idx_bits;
        ctl->final_buf = 0u;
        ctl->passes_run = 0u;
        const bool fits = K <= fb.key_capacity;
        if (!fits) atomicOr(&ctl->error_flags, kErrCapacity);
        if (cd->error_flags & kErrTimeout) atomicOr(&ctl->error_flags, kErrTimeout);
        // a timed-out depth sort leaves the depth order undefined: draw nothing
        ctl->plan_ok = (fits && (ctl->error_flags & kErrTimeout) == 0u) ? 1u : 0u;
        s_ok = ctl->plan_ok;
    }
    __syncthreads();
    if (!s_ok) return;  // the lists and segments below are sized by the capacity
    unsigned long long carry_e = 0, carry_s = 0;
    const uint32_t round = blockDim.x * kRangesItems;
    for (uint32_t r0 = 0; r0 < ncoarse; r0 += round) {
        const uint32_t first = r0 + (uint32_t)tid * kRangesItems;
        uint32_t cnt[kRangesItems];
        uint32_t ne = 0, ns = 0;
#pragma unroll
        for (int i = 0; i < kRangesItems; ++i) {
            cnt[i] = first + i < ncoarse ? __ldcg(&fb.cinfo[first + i].y) : 0u;
            ne += cnt[i];
            ns += (cnt[i] + kSegLen - 1) / kSegLen;
        }
        const uint2 st = block_scan2(ne, ns, s_a, s_b, carry_e, carry_s);
        uint32_t e = st.x, s = st.y;
#pragma unroll
        for (int i = 0; i < kRangesItems; ++i) {
            if (first + i >= ncoarse) break;
            const uint32_t k = (cnt[i] + kSegLen - 1) / kSegLen;
            fb.cinfo[first + i] = make_uint4(e, cnt[i], s, 0u);  // the segment map: k_coarse_place
            e += cnt[i];
            s += k;
        }
    }
    if (tid == 0) {
        ctl->num_entries = (uint32_t)carry_e;
        ctl->num_segments = (uint32_t)carry_s;
        // bands of the coarse placement: the widest the shared memory holds, or small ones when
        // the (chunk, coarse bin) runs are long (their partly written sectors then stay in L2)
        uint32_t rows = pg.band_rows, nb = pg.nbands;
        const unsigned long long cells = (unsigned long long)pg.nchunks * (ncoarse > 0u ? ncoarse : 1u);
        if (pg.ctx > 0u && carry_e >= (unsigned long long)kLongRun * cells) {
            const uint32_t r = kLongRunBand / pg.ctx > 0u ? kLongRunBand / pg.ctx : 1u;
            if (r < rows) {
                rows = r;
                nb = (pg.cty + rows - 1) / rows;
            }
        }
        ctl->place_band_rows = rows;
        ctl->place_nbands = nb;
    }
}

// Frames with nothing to bin: K, the flags and plan_ok.
__global__ void __launch_bounds__(kRangesThreads) k_coarse_ranges(FrameBufs fb, GridParams gp, PlaceGeom pg) {
    coarse_ranges(fb, gp, pg, 0u);
}

// Persistent: every warp takes (band, chunk) items from a ticket, band-major. For an item, the
// chunk's Gaussians 32 at a time (one per lane, in depth order): their entries (the coarse bins
// of the band their rectangles meet, row-major) are numbered in lane order, and the warp takes
// them 32 at a time. Entries of the same coarse bin in one step are ranked by lane; the last of
// them advances the bin's cursor.
__global__ void __launch_bounds__(kPlaceWarps * 32, kPlaceCtasPerSm) k_coarse_place(FrameBufs fb, GridParams gp, PlaceGeom pg,
                                                                      uint64_t n) {
    extern __shared__ uint32_t s_cur[];  // band_bins cursors, then band_bins lane-bit words, per warp
    __shared__ uint4 s_slots[kPlaceWarps][32];  // per warp: (first entry, x0|x1<<16, y0|y1<<16, index)
    FrameCtl* ctl = fb.ctl;
    if (!ctl->plan_ok) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t lt = (1u << lane) - 1u;
    uint32_t* cur = s_cur + (size_t)warp * pg.band_bins;
    uint32_t* mb = s_cur + (size_t)(kPlaceWarps + warp) * pg.band_bins;  // lane bits per coarse bin, kept zero
    for (uint32_t i = lane; i < pg.band_bins; i += 32) mb[i] = 0u;
    uint4* slots = s_slots[warp];
    const uint32_t gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nwarps = (gridDim.x * blockDim.x) >> 5;
    // the segment -> coarse bin map of the pair placement, a warp per coarse bin (coalesced); the
    // kernels that read it run after this one
    for (uint32_t c = gwarp; c < pg.ncoarse; c += nwarps) {
        const uint4 info = fb.cinfo[c];
        const uint32_t k = (info.y + kSegLen - 1) / kSegLen;
        for (uint32_t j = lane; j < k; j += 32) fb.seg_coarse[info.z + j] = c;
    }
    const FrameCtl* cd = fb.ctl_depth;
    const unsigned long long* __restrict__ order = io_select(fb.gsort, cd->final_buf);
    const unsigned long long imask = (1ull << cd->idx_bits) - 1ull;
    uint2* __restrict__ out = fb.clist;
    const uint64_t nsorted = min((uint64_t)ctl->num_visible, n);  // Gaussians in the depth order
    const uint32_t ctx = pg.ctx, band_rows = ctl->place_band_rows, items = ctl->place_nbands * pg.nchunks;
    for (;;) {
        uint32_t item = 0;
        if (lane == 0) item = atomicAdd(&ctl->scan_ticket, 1u);
        item = __shfl_sync(0xFFFFFFFFu, item, 0);
        if (item >= items) break;
        const uint32_t band = item / pg.nchunks, chunk = item - band * pg.nchunks;
        const uint32_t cb0 = band * band_rows, cb1 = min(cb0 + band_rows, pg.cty);
        const uint32_t nb = (cb1 - cb0) * ctx, bin0 = cb0 * ctx;
        const uint64_t q0 = (uint64_t)chunk * pg.chunk_len;
        const uint64_t q1 = min(q0 + (uint64_t)pg.chunk_len, nsorted);
        const uint32_t* __restrict__ trow = fb.ctable + (uint64_t)chunk * pg.ncoarse + bin0;
        const uint32_t* __restrict__ grow = fb.gtable + (uint64_t)(chunk / pg.group) * pg.ncoarse + bin0;
        __syncwarp();  // the previous item is done with the cursors
        for (uint32_t i = lane; i < nb; i += 32) cur[i] = trow[i] + grow[i] + fb.cinfo[bin0 + i].x;
        __syncwarp();
        // batch i is placed while batch i+1's rectangles and indices load
        uint64_t q = q0 + lane;
        uint2 r0 = q < q1 ? fb.srect[q] : make_uint2(0u, 0u);
        uint32_t g0 = q < q1 ? (uint32_t)(order[q] & imask) : 0u;
        for (uint64_t qb = q0; qb < q1; qb += 32) {
            q = qb + 32 + lane;
            const uint2 r1 = q < q1 ? fb.srect[q] : make_uint2(0u, 0u);
            const uint32_t g1 = q < q1 ? (uint32_t)(order[q] & imask) : 0u;
            // this lane's Gaussian: bins (x0..x1, y0..y1) and its number of coarse bins in the band
            uint32_t x0, x1, y0, y1, e = 0u;
            if (local_rect(r0, gp, x0, x1, y0, y1)) {
                const uint32_t cy0 = max(y0 / kCoarse, cb0), cy1 = min((y1 + kCoarse - 1) / kCoarse, cb1);
                if (cy0 < cy1) e = ((x1 + kCoarse - 1) / kCoarse - x0 / kCoarse) * (cy1 - cy0);
            }
            uint32_t incl = e;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                if (lane >= o) incl += t;
            }
            const uint32_t total = __shfl_sync(0xFFFFFFFFu, incl, 31);
            const uint32_t first = incl - e;  // this lane's first entry
            // the batch's Gaussians with entries, in lane order (first entries increasing)
            const uint32_t ne = __ballot_sync(0xFFFFFFFFu, e != 0u);
            __syncwarp();  // the previous batch's steps are done with the slots
            if (e != 0u) slots[__popc(ne & lt)] = make_uint4(first, x0 | (x1 << 16), y0 | (y1 << 16), g0);
            __syncwarp();
            for (uint32_t t0 = 0; t0 < total; t0 += 32) {
                const uint32_t t = t0 + lane;
                const bool valid = t < total;
                // the entry's slot: the last Gaussian whose first entry is <= t, i.e. the slots
                // starting at or before t0 (minus one) plus the slots starting in (t0, t]
                const uint32_t before = __popc(__ballot_sync(0xFFFFFFFFu, e != 0u && first <= t0)) - 1u;
                const uint32_t starts = __reduce_or_sync(
                    0xFFFFFFFFu, (e != 0u && first > t0 && first - t0 < 32u) ? 1u << (first - t0) : 0u);
                const uint4 sl = slots[before + __popc(starts & ((2u << lane) - 1u))];
                const uint32_t gx0 = sl.y & 0xFFFFu, gx1 = sl.y >> 16, gy0 = sl.z & 0xFFFFu, gy1 = sl.z >> 16;
                const uint32_t cx0 = gx0 / kCoarse, cw = (gx1 + kCoarse - 1) / kCoarse - cx0;
                uint32_t dy = 0, dx = 0;
                if (valid) divmod_small(t - sl.x, cw, __frcp_rn((float)cw), dy, dx);
                const uint32_t ccx = cx0 + dx, ccy = max(gy0 / kCoarse, cb0) + dy;
                const uint32_t cl = (ccy - cb0) * ctx + ccx;  // band-local coarse bin
                // the bins of the coarse bin's 4x4 that the rectangle meets
                const uint32_t bx = ccx * kCoarse, by = ccy * kCoarse;
                const uint32_t cols = span4(max(gx0, bx) - bx, min(gx1, bx + kCoarse) - bx);
                const uint32_t rows = span4(max(gy0, by) - by, min(gy1, by + kCoarse) - by);
                const uint32_t spread = (rows & 1u) | ((rows & 2u) << 3) | ((rows & 4u) << 6) | ((rows & 8u) << 9);
                const uint32_t mask = cols * spread;
                // lanes of this step with the same coarse bin: every entry sets its lane's bit in
                // the bin's word; the bin's last entry of the step advances the cursor and clears it
                if (valid) atomicOr(&mb[cl], 1u << lane);
                __syncwarp();
                uint32_t peers = 0, pos = 0;
                if (valid) {
                    peers = mb[cl];
                    pos = cur[cl] + __popc(peers & lt);
                }
                __syncwarp();
                if (valid && (peers >> lane) == 1u) {
                    cur[cl] = pos + 1u;
                    mb[cl] = 0u;
                }
                __syncwarp();
                if (valid) out[pos] = make_uint2(sl.w, mask);
            }
            r0 = r1;
            g0 = g1;
        }
    }
}

// ------------------------------------------------------------------- level 2

struct Segment {
    uint32_t coarse, e0, e1, nseg, seg0;
};

__device__ __forceinline__ Segment segment_of(const FrameBufs& fb, uint32_t s) {
    const uint32_t c = fb.seg_coarse[s];
    const uint4 info = fb.cinfo[c];
    const uint32_t e0 = info.x + (s - info.z) * kSegLen;
    return Segment{c, e0, min(e0 + kSegLen, info.x + info.y), (info.y + kSegLen - 1) / kSegLen, info.z};
}

constexpr int kSegWaves = kSegLen / 32;

// One CTA: exclusive scan of the per-bin totals (ranges[.].y, written by other CTAs) over the
// binned rows in row-major order -> ranges {start, end}; empty bins {0, 0}.
__device__ void fine_ranges(const FrameBufs& fb, const GridParams& gp) {
    __shared__ uint32_t s_warp[32];
    __shared__ unsigned long long s_carry;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    const uint32_t b0 = gp.row_begin * gp.tiles_x, b1 = gp.row_end * gp.tiles_x;
    if (tid == 0) s_carry = 0ull;
    __syncthreads();
    const uint32_t round = blockDim.x * kRangesItems;
    for (uint32_t r0 = b0; r0 < b1; r0 += round) {
        const uint32_t first = r0 + (uint32_t)tid * kRangesItems;
        uint32_t cnt[kRangesItems];
        uint32_t sum = 0;
#pragma unroll
        for (int i = 0; i < kRangesItems; ++i) {
            cnt[i] = first + i < b1 ? __ldcg(&fb.ranges[first + i].y) : 0u;
            sum += cnt[i];
        }
        uint32_t x = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, x, o);
            if (lane >= o) x += t;
        }
        if (lane == 31) s_warp[warp] = x;
        __syncthreads();
        if (warp == 0) {
            uint32_t w = lane < nwarps ? s_warp[lane] : 0u;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, w, o);
                if (lane >= o) w += t;
            }
            s_warp[lane] = w;
        }
        __syncthreads();
        unsigned long long start = s_carry + (warp ? s_warp[warp - 1] : 0u) + x - sum;
#pragma unroll
        for (int i = 0; i < kRangesItems; ++i) {
            if (first + i < b1)
                fb.ranges[first + i] =
                    cnt[i] ? make_uint2((uint32_t)start, (uint32_t)(start + cnt[i])) : make_uint2(0u, 0u);
            start += cnt[i];
        }
        __syncthreads();
        if (tid == 0) s_carry += s_warp[nwarps - 1];
        __syncthreads();
    }
}

// A warp per segment: pairs per bin of the 4x4, stored per segment and added to the bins' totals
// (ranges[.].y); the last CTA to finish scans the totals into the bin ranges.
// Two resident CTAs of 32 warps per SM (32 registers instead of 40, no spills), as the grid assumes.
#ifndef KT_FINE_COUNT_MIN_CTAS
#define KT_FINE_COUNT_MIN_CTAS 2
#endif
__global__ void __launch_bounds__(kCountWarps * 32, KT_FINE_COUNT_MIN_CTAS) k_fine_count(FrameBufs fb, GridParams gp, PlaceGeom pg) {
    __shared__ uint32_t s_last;
    FrameCtl* ctl = fb.ctl;
    if (!ctl->plan_ok) return;  // the same for every CTA
    const uint32_t ns = ctl->num_segments;
    const int lane = threadIdx.x & 31;
    const uint32_t nw = (gridDim.x * blockDim.x) >> 5;
    for (uint32_t s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < ns; s += nw) {
        const Segment sg = segment_of(fb, s);
        uint32_t m[kSegWaves];  // the whole segment in flight
#pragma unroll
        for (int i = 0; i < kSegWaves; ++i) {
            const uint32_t e = sg.e0 + i * 32 + lane;
            m[i] = e < sg.e1 ? fb.clist[e].y : 0u;
        }
        // per lane, bit 4r+k of the masks counted in byte k of acc[r] (at most kSegWaves = 16)
        uint32_t acc[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int i = 0; i < kSegWaves; ++i)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[r] += (((m[i] >> (4 * r)) & 0xFu) * 0x00204081u) & 0x01010101u;
        // warp sums, two 16-bit fields per reduction (at most 32 * 16 each)
        uint32_t mine = 0;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const uint32_t lo = __reduce_add_sync(0xFFFFFFFFu, acc[r] & 0x00FF00FFu);         // bits 4r, 4r+2
            const uint32_t hi = __reduce_add_sync(0xFFFFFFFFu, (acc[r] >> 8) & 0x00FF00FFu);  // bits 4r+1, 4r+3
            if (lane == 4 * r) mine = lo & 0xFFFFu;
            if (lane == 4 * r + 1) mine = hi & 0xFFFFu;
            if (lane == 4 * r + 2) mine = lo >> 16;
            if (lane == 4 * r + 3) mine = hi >> 16;
        }
        if (lane < 16) {
            fb.seg_cnt[(uint64_t)s * 16 + lane] = mine;
            const uint32_t cy = sg.coarse / pg.ctx, cx = sg.coarse - cy * pg.ctx;
            const uint32_t bx = cx * kCoarse + (lane & 3), by = gp.row_begin + cy * kCoarse + (lane >> 2);
            if (mine && bx < gp.tiles_x && by < gp.row_end)  // the bin's total, over the segments
                atomicAdd(&fb.ranges[(uint64_t)by * gp.tiles_x + bx].y, mine);
        }
    }
    __threadfence();  // every thread's writes are visible before the CTA's ticket
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&ctl->done_count, 1u) == gridDim.x - 1u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    fine_ranges(fb, gp);
}

// Every pair of a segment's entries at its bin's cursor (off[] advances past them): per step of 32
// entries and bin of the 4x4, a ballot ranks the entries that meet the bin.
__device__ __forceinline__ void place_segment(const uint2 (&v)[kSegWaves], int lane, uint32_t lt, uint32_t (&off)[16],
                                              uint32_t* __restrict__ out) {
#pragma unroll
    for (int i = 0; i < kSegWaves; ++i) {
        // the step's pairs per bin, bit 4r+k of the masks summed in byte k of tot[r] (at most 32):
        // warp sums on the integer pipe instead of a population count per bin
        uint32_t tot[4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
            tot[r] = __reduce_add_sync(0xFFFFFFFFu, (((v[i].y >> (4 * r)) & 0xFu) * 0x00204081u) & 0x01010101u);
#pragma unroll
        for (int f = 0; f < 16; ++f) {
            const bool bit = (v[i].y >> f) & 1u;
            const uint32_t b = __ballot_sync(0xFFFFFFFFu, bit);
            if (bit) out[off[f] + __popc(b & lt)] = v[i].x;
            off[f] += (tot[f >> 2] >> (8 * (f & 3))) & 0xFFu;
        }
    }
}

// The bins' write cursors at segment s of coarse list `sg`: the bin starts plus the pairs of each
// bin in the list's earlier segments (lanes take every 32nd segment). Lane f < 16 returns bin f's.
__device__ __forceinline__ uint32_t segment_cursor(const FrameBufs& fb, const GridParams& gp, const PlaceGeom& pg,
                                                   const Segment& sg, uint32_t s, int lane) {
    const uint32_t cy = sg.coarse / pg.ctx, cx = sg.coarse - cy * pg.ctx;
    uint32_t part[16];
#pragma unroll
    for (int f = 0; f < 16; ++f) part[f] = 0u;
    for (uint32_t k = lane; k < s - sg.seg0; k += 32) {
        const uint4* q = reinterpret_cast<const uint4*>(fb.seg_cnt + (uint64_t)(sg.seg0 + k) * 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 c = q[i];
            part[4 * i] += c.x;
            part[4 * i + 1] += c.y;
            part[4 * i + 2] += c.z;
            part[4 * i + 3] += c.w;
        }
    }
    uint32_t mine = 0;
#pragma unroll
    for (int f = 0; f < 16; ++f) {
        const uint32_t before = __reduce_add_sync(0xFFFFFFFFu, part[f]);
        if (lane == f) mine = before;
    }
    if (lane < 16) {
        const uint32_t bx = cx * kCoarse + (lane & 3), by = gp.row_begin + cy * kCoarse + (lane >> 2);
        if (bx < gp.tiles_x && by < gp.row_end) mine += fb.ranges[(uint64_t)by * gp.tiles_x + bx].x;
    }
    return mine;
}

__device__ __forceinline__ void load_segment(const FrameBufs& fb, const Segment& sg, int lane,
                                             uint2 (&v)[kSegWaves]) {
#pragma unroll
    for (int i = 0; i < kSegWaves; ++i) {
        const uint32_t e = sg.e0 + i * 32 + lane;
        v[i] = e < sg.e1 ? fb.clist[e] : make_uint2(0u, 0u);
    }
}

// A warp per segment: the bins' cursors, then 32 entries at a time, for each bin of the 4x4, a
// ballot ranks the entries that meet it and they write consecutive addresses. For frames with
// fewer segments than about two per warp (the whole segment is loaded at once; few registers, four
// CTAs per SM).
// Three resident CTAs per SM (80 registers instead of 106, no spills): the grid is sized for full
// occupancy, and with two CTAs per SM it ran in four waves. Measured with the bin count below: the
// pair-placement stage 68.8 -> 64.5 us on the 1M frame (frame rate +3 %); four CTAs (64 registers,
// a few spilled bytes) were no better.
#ifndef KT_FINE_PLACE_MIN_CTAS
#define KT_FINE_PLACE_MIN_CTAS 3
#endif
__global__ void __launch_bounds__(kSegWarps * 32, KT_FINE_PLACE_MIN_CTAS) k_fine_place(FrameBufs fb, GridParams gp, PlaceGeom pg) {
    const FrameCtl* ctl = fb.ctl;
    if (!ctl->plan_ok) return;
    const uint32_t ns = ctl->num_segments;
    const int lane = threadIdx.x & 31;
    const uint32_t lt = (1u << lane) - 1u;
    uint32_t* __restrict__ out = fb.pairs;
    const uint32_t nw = (gridDim.x * blockDim.x) >> 5;
    for (uint32_t s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < ns; s += nw) {
        const Segment sg = segment_of(fb, s);
        const uint32_t mine = segment_cursor(fb, gp, pg, sg, s, lane);
        uint2 v[kSegWaves];  // the whole segment in flight
        load_segment(fb, sg, lane, v);
        uint32_t off[16];  // write cursor of each bin of the 4x4
#pragma unroll
        for (int f = 0; f < 16; ++f) off[f] = __shfl_sync(0xFFFFFFFFu, mine, f);
        place_segment(v, lane, lt, off, out);
    }
}

// A warp per run of up to kSegGroup consecutive segments, for frames with many segments per warp
// (long coarse lists): the next segment's entries load while the current one is placed, and within
// one coarse list the bins' cursors carry over from segment to segment (the sum over the list's
// earlier segments is taken once per run). About 100 registers (two CTAs per SM); measured on the
// 2M stress frame against precomputed per-list prefixes, longer runs and a 128-register build: this
// one is the fastest (3.9 against 4.7-4.9 ms for the stage).
#ifndef KT_FINE_RUNS_MIN_CTAS
#define KT_FINE_RUNS_MIN_CTAS 1
#endif
__global__ void __launch_bounds__(kSegWarps * 32, KT_FINE_RUNS_MIN_CTAS) k_fine_place_runs(FrameBufs fb, GridParams gp,
                                                                                         PlaceGeom pg) {
    const FrameCtl* ctl = fb.ctl;
    if (!ctl->plan_ok) return;
    const uint32_t ns = ctl->num_segments;
    const int lane = threadIdx.x & 31;
    const uint32_t lt = (1u << lane) - 1u;
    uint32_t* __restrict__ out = fb.pairs;
    const uint32_t nw = (gridDim.x * blockDim.x) >> 5;
    uint32_t G = ns / (2u * nw);
    G = G < 1u ? 1u : (G > kSegGroup ? kSegGroup : G);
    const uint32_t nruns = (ns + G - 1) / G;
    for (uint32_t run = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; run < nruns; run += nw) {
        const uint32_t s0 = run * G, s1 = min(s0 + G, ns);
        Segment sg = segment_of(fb, s0);
        uint2 v[kSegWaves];  // the whole segment in flight
        load_segment(fb, sg, lane, v);
        uint32_t off[16];    // write cursor of each bin of the 4x4
        uint32_t list = 0xFFFFFFFFu;
        for (uint32_t s = s0; s < s1; ++s) {
            Segment sn = sg;
            uint2 vn[kSegWaves];
            const bool next = s + 1 < s1;
            if (next) {
                sn = segment_of(fb, s + 1);
                load_segment(fb, sn, lane, vn);
            }
            if (sg.coarse != list) {  // the bin starts plus the list's earlier segments
                const uint32_t mine = segment_cursor(fb, gp, pg, sg, s, lane);
#pragma unroll
                for (int f = 0; f < 16; ++f) off[f] = __shfl_sync(0xFFFFFFFFu, mine, f);
                list = sg.coarse;
            }
            place_segment(v, lane, lt, off, out);
            if (next) {
                sg = sn;
#pragma unroll
                for (int i = 0; i < kSegWaves; ++i) v[i] = vn[i];
            }
        }
    }
}

}  // namespace

cudaError_t place_geometry(const GridParams& gp, uint64_t n, uint64_t capacity, PlaceGeom* out) {
    PlaceGeom g{};
    const uint32_t rows = gp.row_end - gp.row_begin;
    g.ctx = (gp.tiles_x + kCoarse - 1) / kCoarse;
    g.cty = (rows + kCoarse - 1) / kCoarse;
    g.ncoarse = g.ctx * g.cty;
    if (g.ctx > kBandMax || g.ncoarse > kCoarseMax) return cudaErrorInvalidValue;  // too many bins
    // placement bands: whole coarse rows, at most kBandMax coarse bins
    const uint32_t br = g.ctx ? kBandMax / g.ctx : 1u;
    g.nbands = g.cty == 0 ? 1u : (g.cty + br - 1) / br;
    g.band_rows = g.cty == 0 ? 0u : (g.cty + g.nbands - 1) / g.nbands;
    // chunks of depth order
    uint64_t chunks = (n + kChunkTarget - 1) / kChunkTarget;
    if (chunks > kMaxChunks) chunks = kMaxChunks;
    if (chunks < 1) chunks = 1;
    const uint64_t len = n == 0 ? 1 : (n + chunks - 1) / chunks;
    chunks = n == 0 ? 1 : (n + len - 1) / len;
    g.nchunks = (uint32_t)chunks;
    g.chunk_len = (uint32_t)len;
    // groups of chunks: one count CTA's difference arrays, (chunks of the group) x (cty + 1) x
    // (ctx + 1) counters, fit
    const uint32_t nc = g.ncoarse > 0u ? g.ncoarse : 1u;
    const uint32_t cells = (g.ctx + 1u) * (g.cty + 1u);
    if (cells > kCoarseMax) return cudaErrorInvalidValue;
    g.group = kCoarseMax / cells < kGroupMax ? kCoarseMax / cells : kGroupMax;
    g.ngroups = (g.nchunks + g.group - 1) / g.group;
    g.count_smem = g.group * cells * 4u;
    const uint32_t sms = (uint32_t)device_sm_count();
    g.place_ctas = sms * kPlaceCtasPerSm;
    g.band_bins = g.band_rows * g.ctx > 0u ? g.band_rows * g.ctx : 1u;
    g.place_smem = 2u * kPlaceWarps * g.band_bins * 4u;
    g.seg_ctas = sms * (2048u / (kSegWarps * 32u));
    g.run_ctas = g.seg_ctas;  // two resident per SM; the rest start as CTAs finish
    g.count_ctas = sms * (2048u / (kCountWarps * 32u));
    g.table_words = chunks * nc;
    g.gtable_words = (uint64_t)g.ngroups * nc;
    // entries <= pairs <= capacity; a coarse list of c entries has ceil(c / kSegLen) segments
    g.max_segments = capacity / kSegLen + g.ncoarse + 1;

    static int attr_set[128] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(k_coarse_count, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kCoarseMax * 4));
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(k_coarse_place, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPlaceSmem);
        if (e != cudaSuccess) return e;
        attr_set[dev] = 1;
    }
    *out = g;
    return cudaSuccess;
}

cudaError_t launch_coarse_count(const FrameBufs& fb, const GridParams& gp, const PlaceGeom& pg, uint64_t n,
                                cudaStream_t stream) {
    if (n == 0 || gp.row_end <= gp.row_begin) {  // nothing to bin: K, the flags and plan_ok
        k_coarse_ranges<<<1, kRangesThreads, 0, stream>>>(fb, gp, pg);
        return cudaGetLastError();
    }
    k_coarse_count<<<pg.ngroups, kCountThreads, pg.count_smem, stream>>>(fb, gp, pg, n);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    k_coarse_scan<<<(pg.ncoarse + 31) / 32, 1024, 0, stream>>>(fb, gp, pg);
    return cudaGetLastError();
}

cudaError_t launch_coarse_place(const FrameBufs& fb, const GridParams& gp, const PlaceGeom& pg, uint64_t n,
                                cudaStream_t stream) {
    if (n == 0 || gp.row_end <= gp.row_begin) return cudaSuccess;
    k_coarse_place<<<pg.place_ctas, kPlaceWarps * 32, pg.place_smem, stream>>>(fb, gp, pg, n);
    return cudaGetLastError();
}

cudaError_t launch_fine_place(const FrameBufs& fb, const GridParams& gp, const PlaceGeom& pg, uint64_t n,
                              bool runs, cudaStream_t stream) {
    if (n == 0 || gp.row_end <= gp.row_begin) return cudaSuccess;
    k_fine_count<<<pg.count_ctas, kCountWarps * 32, 0, stream>>>(fb, gp, pg);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (runs)
        k_fine_place_runs<<<pg.run_ctas, kSegWarps * 32, 0, stream>>>(fb, gp, pg);
    else
        k_fine_place<<<pg.seg_ctas, kSegWarps * 32, 0, stream>>>(fb, gp, pg);
    return cudaGetLastError();
}

uint32_t fine_place_warps(const PlaceGeom& pg) { return pg.seg_ctas * kSegWarps; }

}  // namespace kt
