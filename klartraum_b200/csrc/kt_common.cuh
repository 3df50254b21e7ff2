// Internal types shared by the renderer's kernels and its host code.
//
// Device data layout (per context):
//   scene planes   pos   float4[N]  (x, y, z, alpha)
//                  rot   float4[N]  (x, y, z, w)
//                  scale float4[N]  (sx, sy, sz, 0)
//                  sh    float4[P][N], P = ceil(3 (d+1)^2 / 4): the SH coefficients of
//                        degree d interleaved per coefficient (R,G,B), DC first
//   per path       rec   float4[3N] (px, py, alpha, z) (covInv 00,01,10,11) (r, g, b, 0)
//                  counts u32[N], rect u32x2[N] (x0|x1<<16, y0|y1<<16), depth u32[N],
//                  srect u32x2[N] (rect in depth order),
//                  gsort u64[2][N] (Gaussians by depth), pairs u32[cap] (the Gaussian of
//                  every (bin, Gaussian) pair, in bin order; the bin is implied by the ranges),
//                  ranges u32x2[tiles], coarse table u32[chunks][coarse bins], coarse info
//                  u32x4[coarse bins], coarse lists u32x2[cap] (Gaussian, 4x4 bin mask),
//                  segment map u32[segments], segment counts u32[segments][16], look-back
//                  status words of the depth sort, two FrameCtl blocks.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace kt {

constexpr int kMaxPasses = 8;          // 8-bit digits over at most 64 key bits
constexpr uint32_t kErrCapacity = 1u;  // key count above the key buffers' capacity
constexpr uint32_t kErrTimeout = 2u;   // a look-back wait ran out of iterations
constexpr uint32_t kSpinLimit = 1u << 22;  // look-back polls before giving up (~seconds)
// Element of the depth sort for a Gaussian that meets no bin: the first executed pass drops it.
constexpr unsigned long long kDropKey = ~0ull;

// Look-back status word: [epoch:24][flag:2][value:38].
constexpr uint64_t kFlagAggregate = 1ull;
constexpr uint64_t kFlagInclusive = 2ull;
constexpr int kValueBits = 38;
constexpr uint64_t kValueMask = (1ull << kValueBits) - 1ull;
constexpr uint32_t kEpochMax = (1u << 24) - 1u;

__host__ __device__ inline uint64_t pack_status(uint32_t epoch, uint64_t flag, uint64_t value) {
    return ((uint64_t)epoch << 40) | (flag << kValueBits) | (value & kValueMask);
}
__host__ __device__ inline uint32_t status_epoch(uint64_t w) { return (uint32_t)(w >> 40); }
__host__ __device__ inline uint64_t status_flag(uint64_t w) { return (w >> kValueBits) & 3ull; }
__host__ __device__ inline uint64_t status_value(uint64_t w) { return w & kValueMask; }

// Per-frame control block in device memory, reset by k_frame_init.
struct FrameCtl {
    unsigned long long num_keys;      // K: pairs (render path) or keys (sorts)
    unsigned long long pair_total;    // sum of the Gaussians' bin counts (projection)
    unsigned int depth_min;           // min / max of floatBitsToUint(z) ^ 0x80000000
    unsigned int depth_max;           //   over Gaussians with a non-zero tile count
    unsigned int num_visible;         // Gaussians with a non-zero tile count
    unsigned int error_flags;         // kErr*
    unsigned int scan_ticket;         // work ticket of the pair placement
    unsigned int plan_ok;             // the keys fit and the stages after may run
    unsigned int depth_bits;          // bits of depth_max - depth_min
    unsigned int key_bits;
    unsigned int passes_run;
    unsigned int final_buf;           // which key/value buffer holds the sorted data
    unsigned int packed;              // 1: elements are (key << idx_bits) | index, no value array
    unsigned int idx_bits;            // bits of the index field of a packed element (0 unpacked)
    unsigned int num_entries;         // (Gaussian, coarse bin) entries of the pair placement
    unsigned int num_segments;        // segments of the coarse lists (second placement level)
    unsigned int done_scan;           // CTAs of the coarse scan that finished
    unsigned int done_count;          // CTAs of the bin count that finished
    unsigned int place_band_rows;     // coarse rows per band of the coarse placement, this frame
    unsigned int place_nbands;        // bands of the coarse placement, this frame
    unsigned int pass_ticket[kMaxPasses];
    unsigned int pass_run[kMaxPasses];
    unsigned int pass_src[kMaxPasses];
    unsigned int pass_dst[kMaxPasses];
    unsigned int pass_mask[kMaxPasses];  // digit mask: 255, or fewer bits in the last pass
    unsigned int pass_drop[kMaxPasses];  // 1: the pass drops elements equal to kDropKey (packed sorts)
    unsigned long long pass_in[kMaxPasses];  // elements the pass reads
    unsigned int hist[kMaxPasses][256];   // digit histograms of the keys
    unsigned int base[kMaxPasses][256];   // exclusive scans of hist
};

// Device-side totals over frames (kt_gs_counters), accumulated by the ranges kernel.
struct FrameTotals {
    unsigned long long frames;
    unsigned long long keys;
    unsigned long long key_passes;
    unsigned long long visible;
    unsigned long long sort_bytes;
    unsigned long long depth_sort_bytes;
    unsigned int sticky_errors;  // error bits of every frame since the last sync
    unsigned int pad;
};

// Camera values derived once per frame on the host (same formulas as the shader).
struct CamParams {
    float pvm[16];   // ubo.proj * ubo.view * ubo.model
    float mv[16];    // ubo.model * ubo.view
    float focal_x;   // ubo.proj[0][0]
    float focal_y;   // ubo.proj[1][1]
    float lim_x;     // 1.3 * (1 / focal_x) (gsplat_projection.comp:76-77, 86-87)
    float lim_y;     // 1.3 * (1 / focal_y)
};

// Screen / binning geometry.
struct GridParams {
    float half_w, half_h;        // W/2, H/2 (256 at 512: gsplat_projection.comp:202)
    float sxx, syy, sxy;         // covariance scale (512*512 at 512: comp:208)
    float cell_w, cell_h;        // bin size in px, as float
    float inv_cell_w, inv_cell_h; // 1 / cell (rounded; seeds the exact overlap search)
    float cull_z;
    uint32_t tiles_x, tiles_y;
    uint32_t row_begin, row_end; // binned bin rows [begin, end)
    uint32_t width, height;
    uint32_t bin_w, bin_h;       // bin size in px
    uint32_t tile_bits;          // bits of (tiles_x * tiles_y - 1)
};

struct SceneDev {
    const float4* pos;
    const float4* rot;
    const float4* scale;
    const float4* sh;   // planes of n float4
    uint32_t nplanes;
    int deg;
    uint64_t n;
};

// Work split of the pair placement (place.cu).
struct PlaceGeom {
    uint32_t ctx, cty;        // coarse grid (4x4 bins per coarse bin) over the binned rows
    uint32_t ncoarse;         // ctx * cty
    uint32_t nchunks;         // chunks of consecutive Gaussians in depth order
    uint32_t chunk_len;       // Gaussians per chunk (the last may be shorter)
    uint32_t group;           // chunks per count CTA (a group)
    uint32_t ngroups;
    uint32_t nbands;          // placement bands of coarse rows (one warp's cursors each)
    uint32_t band_rows;       // coarse rows per placement band (the last may be shorter)
    uint32_t count_smem;      // dynamic shared memory of a count CTA
    uint32_t place_ctas;      // persistent coarse-placement CTAs
    uint32_t band_bins;       // coarse bins of the largest placement band (cursor stride)
    uint32_t place_smem;      // dynamic shared memory of a coarse-placement CTA
    uint32_t seg_ctas;        // CTAs of the pair placement (a warp per segment)
    uint32_t run_ctas;        // CTAs of the pair placement by runs of segments
    uint32_t count_ctas;      // CTAs of the bin count
    uint64_t table_words;     // u32 words of table[chunk][coarse bin]
    uint64_t gtable_words;    // u32 words of gtable[group][coarse bin]
    uint64_t max_segments;    // segments the key capacity can produce, at most
};

struct FrameBufs {
    float4* rec;
    uint32_t* counts;
    uint2* rect;
    uint2* srect;                  // rect in depth order (empty for Gaussians without bins)
    uint32_t* depth;
    unsigned long long* gsort[2];  // Gaussians by depth: (depth - min) << idx_bits | index
    uint32_t* pairs;               // Gaussian index of every (bin, Gaussian) pair, in bin order
    // pair placement: (chunk, coarse bin) table, coarse lists and their segments
    uint32_t* ctable;              // per (chunk, coarse bin): prefix of the entries over the group's chunks
    uint32_t* gtable;              // per (group, coarse bin): entries, then their prefix over groups
    uint4* cinfo;                  // per coarse bin: list start, entries, first segment, 0
    uint2* clist;                  // (Gaussian index, 4x4 bin mask) by coarse bin, depth order
    uint32_t* seg_coarse;          // coarse bin of every segment
    uint32_t* seg_cnt;             // pairs per (segment, bin of the 4x4)
    // reference-structured path (KT_GS_FLAG_SORTED_KEYS): offsets, keys and values
    unsigned long long* offsets;   // exclusive scan of the counts, index order
    unsigned long long* keys[2];   // bin << depth_bits | (depth - depth_min), ping-pong
    uint32_t* vals[2];             // Gaussian index, ping-pong
    unsigned long long* scan_status;
    uint2* ranges;
    unsigned long long* sort_status;
    FrameCtl* ctl;                 // the frame, and the sort of the pairs by bin
    FrameCtl* ctl_depth;           // the sort of the Gaussians by depth
    uint64_t key_capacity;
};

__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_volatile_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Look-back status words: relaxed, device-scope (coherent at L2) loads and stores.
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// SM count of the current device (cached per device).
int device_sm_count();

// ---- mbarrier / bulk-copy helpers (sm_90+ PTX; every copy has a single destination CTA)
#ifdef __CUDACC__

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(unsigned long long* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before later async-proxy
// (bulk copy) accesses to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

// Global -> shared bulk copy (16-B aligned addresses, size a multiple of 16), completing on `bar`.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              unsigned long long* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for phase `parity` of `bar`; false if it did not complete within `limit` polls.
__device__ __forceinline__ bool mbar_wait_bounded(unsigned long long* bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

#endif  // __CUDACC__

__host__ __device__ inline uint32_t bits_for(uint64_t v) {
    uint32_t b = 0;
    while (b < 64 && (v >> b) != 0) ++b;
    return b;
}

}  // namespace kt
