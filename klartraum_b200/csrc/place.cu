// Pairs by bin without a sort: a stable counting sort of the (bin, Gaussian) pairs, fed with the
// Gaussians in depth order.
//
// The reference duplicates each projected Gaussian once per overlapped bin and sorts the copies
// by the 48-bit key bin << 32 | depth (shaders/gsplat/gsplat_binning.comp:112-159,
// gsplat_radix_sort_include.glsl:51-63). With the Gaussians already sorted by depth (stable,
// ties by index) that order is: by bin, then by the Gaussian's position in depth order. The
// pairs of one Gaussian cover a rectangle of bins, so they never need to exist unsorted:
//   k_depth_rects  the Gaussians' bin rectangles gathered into depth order (empty rectangle for
//                  Gaussians without bins), so that everything after reads them coalesced.
//   k_pair_count   one CTA per (chunk, count band). A chunk is a contiguous run of depth order;
//                  its Gaussians add +1/-1 at the corners of their rectangles in a shared-memory
//                  difference table of the band's bin rows; the table's 2D prefix sums are the
//                  chunk's pairs per bin, stored as table[chunk][bin].
//   k_pair_scan    per bin, the exclusive prefix of table[.][bin] over chunks (in place) and the
//                  bin's total.
//   k_bin_ranges   exclusive scan of the totals over bins: ranges {start, end} (empty bins keep
//                  {0, 0}, as the reference's zeroed StartAndEnd buffer), K, the capacity check.
//   k_pair_place   persistent warps take (band, chunk) items in band-major order. A band is a
//                  few bin rows; the warp keeps one write cursor per bin of the band in shared
//                  memory (bin start + the chunk's prefix), walks the chunk's Gaussians in depth
//                  order and, for each one meeting the band, lets its lanes write the pairs at
//                  their bins' cursors, which then advance.
// A warp visits its Gaussians in order and chunks take consecutive slices of every bin, so
// equal-bin pairs land in depth order: the stable sort of the pairs by bin, with no pass over
// unsorted pairs. A pair is stored as its Gaussian's index (4 bytes); its bin is implied by the
// bin ranges. Band-major order keeps the output sectors being filled at any moment (items in
// flight x bins per band) within L2, so partial sectors merge there instead of in DRAM.
#include "kt_common.cuh"
#include "kt_kernels.h"

namespace kt {
namespace {

constexpr uint32_t kPlaceWarps = 16;           // warps of a placement CTA (one CTA per SM)
constexpr uint32_t kBandTargetBins = 768;      // bins of a placement band, about
constexpr uint32_t kBandMaxBins = 1024;        // cursors of one warp (4 KB)
constexpr uint32_t kPlaceSmem = kPlaceWarps * kBandMaxBins * 4;
constexpr uint32_t kCountThreads = 512;
constexpr uint32_t kCountMaxCells = 16384;     // difference table of a count CTA (64 KB)
constexpr uint32_t kChunkTarget = 1024;        // Gaussians per chunk, about (the length of a warp's serial walk)
constexpr uint32_t kMaxChunks = 1024;
constexpr uint32_t kNone = 0xFFFFFFFFu;
constexpr int kRangesThreads = 1024;
constexpr int kRangesItems = 8;                // consecutive bins per thread and round

// (q, r) = (a / w, a % w) for a < 2^20, w >= 1: float quotient, then corrected exactly.
__device__ __forceinline__ void divmod_small(uint32_t a, uint32_t w, float inv_w, uint32_t& q, uint32_t& r) {
    q = (uint32_t)((float)a * inv_w);
    if (q * w > a) --q;
    if ((q + 1) * w <= a) ++q;
    r = a - q * w;
}

__global__ void __launch_bounds__(256) k_depth_rects(FrameBufs fb, uint64_t n) {
    const FrameCtl* cd = fb.ctl_depth;
    const unsigned long long* __restrict__ order = io_select(fb.gsort, cd->final_buf);
    const unsigned long long imask = (1ull << cd->idx_bits) - 1ull;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t p = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n; p += stride) {
        const uint32_t g = (uint32_t)(order[p] & imask);
        fb.srect[p] = fb.counts[g] != 0u ? fb.rect[g] : make_uint2(0u, 0u);
    }
}

__global__ void __launch_bounds__(kCountThreads) k_pair_count(FrameBufs fb, GridParams gp, PlaceGeom pg, uint64_t n,
                                                              uint32_t* __restrict__ table) {
    extern __shared__ int s_tab[];
    const uint32_t chunk = blockIdx.x / pg.ncbands, cband = blockIdx.x - chunk * pg.ncbands;
    const uint32_t by0 = gp.row_begin + cband * pg.cband_rows;
    const uint32_t by1 = min(by0 + pg.cband_rows, gp.row_end);
    if (by0 >= by1) return;  // uniform over the CTA
    const uint32_t rows = by1 - by0, tx = gp.tiles_x, W1 = tx + 1;
    const uint32_t cells = W1 * (rows + 1);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (uint32_t i = tid; i < cells; i += kCountThreads) s_tab[i] = 0;
    __syncthreads();
    const uint64_t q0 = (uint64_t)chunk * pg.chunk_len;
    const uint64_t q1 = min(q0 + (uint64_t)pg.chunk_len, n);
    for (uint64_t q = q0 + tid; q < q1; q += kCountThreads) {
        const uint2 r = fb.srect[q];
        const uint32_t y0 = max(r.y & 0xFFFFu, by0), y1 = min(r.y >> 16, by1);
        const uint32_t x0 = r.x & 0xFFFFu, x1 = r.x >> 16;
        if (x0 >= x1 || y0 >= y1) continue;
        const uint32_t a = (y0 - by0) * W1, b = (y1 - by0) * W1;
        atomicAdd(&s_tab[a + x0], 1);
        atomicAdd(&s_tab[a + x1], -1);
        atomicAdd(&s_tab[b + x0], -1);
        atomicAdd(&s_tab[b + x1], 1);
    }
    __syncthreads();
    // 2D prefix sums: along x (a warp per row, 32 columns per step), then along y (a thread
    // per column, 8 loads in flight)
    constexpr uint32_t kWarps = kCountThreads / 32;
    for (uint32_t y = warp; y < rows; y += kWarps) {
        int carry = 0;
        for (uint32_t x0 = 0; x0 < tx; x0 += 32) {
            const uint32_t x = x0 + lane;
            int v = x < tx ? s_tab[y * W1 + x] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xFFFFFFFFu, v, o);
                if (lane >= o) v += t;
            }
            if (x < tx) s_tab[y * W1 + x] = v + carry;
            carry += __shfl_sync(0xFFFFFFFFu, v, 31);
        }
    }
    __syncthreads();
    for (uint32_t x = tid; x < tx; x += kCountThreads) {
        int run = 0;
        uint32_t y = 0;
        for (; y + 8 <= rows; y += 8) {
            int v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = s_tab[(y + u) * W1 + x];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                run += v[u];
                s_tab[(y + u) * W1 + x] = run;
            }
        }
        for (; y < rows; ++y) {
            run += s_tab[y * W1 + x];
            s_tab[y * W1 + x] = run;
        }
    }
    __syncthreads();
    uint32_t* __restrict__ trow = table + (uint64_t)chunk * tx * gp.tiles_y + (uint64_t)by0 * tx;
    for (uint32_t i = tid; i < rows * tx; i += kCountThreads) {
        const uint32_t y = i / tx, x = i - y * tx;
        trow[i] = (uint32_t)s_tab[y * W1 + x];
    }
}

// 32 bins per CTA (lanes), the chunks split into 32 segments (warps). Bins outside the binned
// rows are not touched (their ranges stay {0, 0} from k_frame_init).
__global__ void __launch_bounds__(1024) k_pair_scan(GridParams gp, PlaceGeom pg, uint32_t* __restrict__ table,
                                                    uint2* __restrict__ ranges) {
    __shared__ uint32_t s_seg[32][33];
    const int lane = threadIdx.x & 31, seg = threadIdx.x >> 5;
    const uint64_t B = (uint64_t)gp.tiles_x * gp.tiles_y;
    const uint32_t b_end = gp.row_end * gp.tiles_x;
    const uint32_t b = gp.row_begin * gp.tiles_x + blockIdx.x * 32 + lane;
    const bool live = b < b_end;
    const uint32_t per = (pg.nchunks + 31) / 32;
    const uint32_t c0 = min(seg * per, pg.nchunks), c1 = min(c0 + per, pg.nchunks);
    uint32_t* __restrict__ col = table + b;
    uint32_t sum = 0;
    if (live) {
        uint32_t c = c0;
        for (; c + 4 <= c1; c += 4)
            sum += col[(uint64_t)c * B] + col[(uint64_t)(c + 1) * B] + col[(uint64_t)(c + 2) * B] +
                   col[(uint64_t)(c + 3) * B];
        for (; c < c1; ++c) sum += col[(uint64_t)c * B];
    }
    s_seg[seg][lane] = sum;
    __syncthreads();
    uint32_t base = 0;
    for (int s = 0; s < seg; ++s) base += s_seg[s][lane];
    if (!live) return;
    if (seg == 31) ranges[b] = make_uint2(0u, base + sum);  // the bin's total, for k_bin_ranges
    for (uint32_t c = c0; c < c1; ++c) {
        const uint32_t v = col[(uint64_t)c * B];
        col[(uint64_t)c * B] = base;
        base += v;
    }
}

// One CTA: exclusive scan of the per-bin totals over the binned rows in row-major order.
__global__ void __launch_bounds__(kRangesThreads) k_bin_ranges(FrameBufs fb, GridParams gp) {
    __shared__ uint32_t s_warp[32];
    __shared__ unsigned long long s_carry;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t b0 = gp.row_begin * gp.tiles_x, b1 = gp.row_end * gp.tiles_x;
    if (tid == 0) s_carry = 0ull;
    __syncthreads();
    constexpr uint32_t kRound = kRangesThreads * kRangesItems;
    for (uint32_t r0 = b0; r0 < b1; r0 += kRound) {
        const uint32_t first = r0 + (uint32_t)tid * kRangesItems;
        uint32_t cnt[kRangesItems];
        uint32_t sum = 0;
#pragma unroll
        for (int i = 0; i < kRangesItems; ++i) {
            cnt[i] = first + i < b1 ? fb.ranges[first + i].y : 0u;
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
            uint32_t w = s_warp[lane];
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
        if (tid == 0) s_carry += s_warp[31];
        __syncthreads();
    }
    if (tid == 0) {
        FrameCtl* ctl = fb.ctl;
        const FrameCtl* cd = fb.ctl_depth;
        const unsigned long long K = s_carry;
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
    }
}

// One lane's Gaussian of a batch, clipped to the band, with what the placement loop needs.
struct BatchGauss {
    uint32_t idx;   // Gaussian index
    uint32_t xw;    // x0 | w << 16 (0: nothing in this band)
    uint32_t yc;    // band-local y0 | pair count in the band << 16 (count <= kBandMaxBins)
    uint32_t step;  // (32 / w) | (32 % w) << 16
    float inv_w;    // 1 / w
};

// (o / w) | (o % w) << 8 for w in 1..32, o in 0..31, in shared memory
struct DivTable {
    uint16_t qr[33][32];
};

__device__ __forceinline__ BatchGauss batch_gauss(uint32_t g, uint2 r, uint32_t by0, uint32_t by1,
                                                  const DivTable& dt) {
    BatchGauss b{g, 0u, 0u, 0u, 0.0f};
    const uint32_t y0 = max(r.y & 0xFFFFu, by0), y1 = min(r.y >> 16, by1);
    const uint32_t x0 = r.x & 0xFFFFu, x1 = r.x >> 16;
    if (x0 >= x1 || y0 >= y1) return b;
    const uint32_t w = x1 - x0;
    b.xw = x0 | (w << 16);
    b.yc = (y0 - by0) | ((w * (y1 - y0)) << 16);
    uint32_t sy, sx;
    if (w <= 32u) {  // 32 = 31 + 1
        const uint32_t d = dt.qr[w][31];
        sy = d & 0xFFu;
        sx = (d >> 8) + 1u;
        if (sx == w) {
            ++sy;
            sx = 0u;
        }
    } else {
        b.inv_w = 1.0f / (float)w;
        divmod_small(32u, w, b.inv_w, sy, sx);
    }
    b.step = sy | (sx << 16);
    return b;
}

// Persistent: every warp takes (band, chunk) items from a ticket, band-major. For an item, the
// chunk's Gaussians in depth order, one at a time: the lanes take the Gaussian's bins in the
// band (row-major), write each pair at its bin's cursor and advance the cursor. The rectangle
// arithmetic of a batch of 32 Gaussians is done by their own lanes beforehand.
__global__ void __launch_bounds__(kPlaceWarps * 32, 1) k_pair_place(FrameBufs fb, GridParams gp, PlaceGeom pg,
                                                                    uint64_t n, const uint32_t* __restrict__ table) {
    extern __shared__ uint32_t s_cur[];  // kBandMaxBins cursors per warp
    __shared__ DivTable s_div;
    FrameCtl* ctl = fb.ctl;
    if (!ctl->plan_ok) return;
    for (uint32_t i = threadIdx.x; i < 33 * 32; i += blockDim.x) {
        const uint32_t w = i >> 5, o = i & 31u;
        s_div.qr[w][o] = w ? (uint16_t)((o / w) | ((o % w) << 8)) : (uint16_t)0;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t* cur = s_cur + (size_t)warp * kBandMaxBins;
    const FrameCtl* cd = fb.ctl_depth;
    const unsigned long long* __restrict__ order = io_select(fb.gsort, cd->final_buf);
    const unsigned long long imask = (1ull << cd->idx_bits) - 1ull;
    uint32_t* __restrict__ out = fb.pairs;
    const uint32_t tx = gp.tiles_x, items = pg.nbands * pg.nchunks;
    for (;;) {
        uint32_t item = 0;
        if (lane == 0) item = atomicAdd(&ctl->scan_ticket, 1u);
        item = __shfl_sync(0xFFFFFFFFu, item, 0);
        if (item >= items) break;
        const uint32_t band = item / pg.nchunks, chunk = item - band * pg.nchunks;
        const uint32_t by0 = gp.row_begin + band * pg.band_rows;
        const uint32_t by1 = min(by0 + pg.band_rows, gp.row_end);
        const uint64_t q0 = (uint64_t)chunk * pg.chunk_len;
        const uint64_t q1 = min(q0 + (uint64_t)pg.chunk_len, n);
        const uint32_t nb = (by1 - by0) * tx, bin0 = by0 * tx;
        const uint32_t* __restrict__ trow = table + (uint64_t)chunk * tx * gp.tiles_y + bin0;
        __syncwarp();  // the previous item is done with the cursors
        for (uint32_t i = lane; i < nb; i += 32) cur[i] = trow[i] + fb.ranges[bin0 + i].x;
        __syncwarp();
        // batch i is placed while batch i+1's rectangles and indices load
        uint64_t q = q0 + lane;
        uint2 r0 = q < q1 ? fb.srect[q] : make_uint2(0u, 0u);
        uint32_t g0 = q < q1 ? (uint32_t)(order[q] & imask) : kNone;
        for (uint64_t qb = q0; qb < q1; qb += 32) {
            q = qb + 32 + lane;
            const uint2 r1 = q < q1 ? fb.srect[q] : make_uint2(0u, 0u);
            const uint32_t g1 = q < q1 ? (uint32_t)(order[q] & imask) : kNone;
            const BatchGauss mine = batch_gauss(g0, r0, by0, by1, s_div);
            uint32_t todo = __ballot_sync(0xFFFFFFFFu, mine.xw != 0u);
            while (todo) {  // this batch's Gaussians in depth order
                const int src = __ffs(todo) - 1;
                todo &= todo - 1u;
                const uint32_t gg = __shfl_sync(0xFFFFFFFFu, mine.idx, src);
                const uint32_t xw = __shfl_sync(0xFFFFFFFFu, mine.xw, src);
                const uint32_t yc = __shfl_sync(0xFFFFFFFFu, mine.yc, src);
                const uint32_t st = __shfl_sync(0xFFFFFFFFu, mine.step, src);
                const float inv_w = __shfl_sync(0xFFFFFFFFu, mine.inv_w, src);
                const uint32_t x0 = xw & 0xFFFFu, w = xw >> 16, ly0 = yc & 0xFFFFu, cnt = yc >> 16;
                const uint32_t sy = st & 0xFFFFu, sx = st >> 16;
                uint32_t dy, dx;  // this lane's first bin
                if (w <= 32u) {
                    const uint32_t d = s_div.qr[w][lane];
                    dy = d & 0xFFu;
                    dx = d >> 8;
                } else {
                    divmod_small((uint32_t)lane, w, inv_w, dy, dx);
                }
                for (uint32_t j = lane; j < cnt; j += 32) {
                    const uint32_t li = (ly0 + dy) * tx + x0 + dx;
                    const uint32_t pos = cur[li];
                    cur[li] = pos + 1u;
                    out[pos] = gg;
                    dx += sx;
                    dy += sy;
                    if (dx >= w) {
                        dx -= w;
                        ++dy;
                    }
                }
                __syncwarp();  // cursor updates visible to every lane before the next Gaussian
            }
            r0 = r1;
            g0 = g1;
        }
    }
}

}  // namespace

cudaError_t place_geometry(const GridParams& gp, uint64_t n, PlaceGeom* out) {
    PlaceGeom g{};
    const uint32_t tx = gp.tiles_x, rows = gp.row_end - gp.row_begin;
    if (tx > kBandMaxBins || tx + 1 > kCountMaxCells / 2) return cudaErrorInvalidValue;  // too many bins per row
    // placement bands: about kBandTargetBins bins each
    uint32_t br = kBandTargetBins / tx;
    if (br < 1) br = 1;
    if (br * tx > kBandMaxBins) br = kBandMaxBins / tx;
    g.nbands = rows == 0 ? 1u : (rows + br - 1) / br;
    g.band_rows = rows == 0 ? 0u : (rows + g.nbands - 1) / g.nbands;
    // count bands: the largest row ranges whose difference table fits
    const uint32_t cmax = kCountMaxCells / (tx + 1) - 1;
    g.ncbands = rows == 0 ? 1u : (rows + cmax - 1) / cmax;
    g.cband_rows = rows == 0 ? 0u : (rows + g.ncbands - 1) / g.ncbands;
    g.count_smem = (tx + 1) * (g.cband_rows + 1) * 4u;
    // chunks of depth order
    uint64_t chunks = (n + kChunkTarget - 1) / kChunkTarget;
    if (chunks > kMaxChunks) chunks = kMaxChunks;
    if (chunks < 1) chunks = 1;
    const uint64_t len = n == 0 ? 1 : (n + chunks - 1) / chunks;
    chunks = n == 0 ? 1 : (n + len - 1) / len;
    g.nchunks = (uint32_t)chunks;
    g.chunk_len = (uint32_t)len;
    g.place_ctas = (uint32_t)device_sm_count();
    g.table_words = chunks * tx * gp.tiles_y;

    static int attr_set[128] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(k_pair_count, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kCountMaxCells * 4));
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(k_pair_place, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPlaceSmem);
        if (e != cudaSuccess) return e;
        attr_set[dev] = 1;
    }
    *out = g;
    return cudaSuccess;
}

cudaError_t launch_pair_count(const FrameBufs& fb, const GridParams& gp, const PlaceGeom& pg, uint64_t n,
                              uint32_t* table, cudaStream_t stream) {
    if (n == 0 || gp.row_end <= gp.row_begin) return cudaSuccess;
    unsigned blocks = (unsigned)((n + 255) / 256);
    const unsigned cap = (unsigned)device_sm_count() * 8;
    if (blocks > cap) blocks = cap;
    k_depth_rects<<<blocks, 256, 0, stream>>>(fb, n);
    k_pair_count<<<pg.nchunks * pg.ncbands, kCountThreads, pg.count_smem, stream>>>(fb, gp, pg, n, table);
    return cudaGetLastError();
}

cudaError_t launch_pair_ranges(const FrameBufs& fb, const GridParams& gp, const PlaceGeom& pg, uint64_t n,
                               uint32_t* table, cudaStream_t stream) {
    const uint32_t nbins = (gp.row_end - gp.row_begin) * gp.tiles_x;
    if (n > 0 && nbins > 0) {
        k_pair_scan<<<(nbins + 31) / 32, 1024, 0, stream>>>(gp, pg, table, fb.ranges);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    k_bin_ranges<<<1, kRangesThreads, 0, stream>>>(fb, gp);
    return cudaGetLastError();
}

cudaError_t launch_pair_place(const FrameBufs& fb, const GridParams& gp, const PlaceGeom& pg, uint64_t n,
                              const uint32_t* table, cudaStream_t stream) {
    if (n == 0 || gp.row_end <= gp.row_begin) return cudaSuccess;
    k_pair_place<<<pg.place_ctas, kPlaceWarps * 32, kPlaceSmem, stream>>>(fb, gp, pg, n, table);
    return cudaGetLastError();
}

}  // namespace kt
