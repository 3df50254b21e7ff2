// Host-side launchers of the renderer's kernels (one .cu file per stage).
#pragma once

#include "kt_common.cuh"

namespace kt {

// Key/value buffers of the sort: render path uses [0]/[1] ping-pong; the standalone
// operator uses [0] = input, [1] = scratch, [2] = output.
struct SortIO {
    unsigned long long* keys[3];
    uint32_t* vals[3];
};

// Buffer i of a SortIO without dynamic indexing of the kernel-parameter array (which would
// force a local-memory copy).
__device__ __forceinline__ unsigned long long* io_keys(const SortIO& io, uint32_t i) {
    return i == 0 ? io.keys[0] : (i == 1 ? io.keys[1] : io.keys[2]);
}
__device__ __forceinline__ uint32_t* io_vals(const SortIO& io, uint32_t i) {
    return i == 0 ? io.vals[0] : (i == 1 ? io.vals[1] : io.vals[2]);
}
__device__ __forceinline__ const unsigned long long* io_select(unsigned long long* const (&b)[2], uint32_t i) {
    return i == 0 ? b[0] : b[1];
}

#ifndef KT_SORT_TILE
#define KT_SORT_TILE 4096
#endif
constexpr int kSortTile = KT_SORT_TILE;  // keys per sort tile
constexpr int kScanChunk = 2048;  // Gaussians per scan/emit CTA (keys path)

// project.cu (compiled with -fmad=false)
// The camera is a kernel parameter; a captured frame graph gets each frame's camera by an update of
// that parameter (project_count_kernel identifies the kernel node among the graph's nodes).
cudaError_t launch_project_count(const SceneDev& sc, const CamParams& cam, const GridParams& gp, const FrameBufs& fb,
                                 cudaStream_t stream);
const void* project_count_kernel(int deg);
cudaError_t launch_load_projected(const float* d_g2d, uint64_t n, const GridParams& gp,
                                  const FrameBufs& fb, cudaStream_t stream);
cudaError_t launch_pack_scene(const float* d_aos, uint64_t n, float4* pos, float4* rot,
                              float4* scale, float4* sh, int deg, uint32_t nplanes,
                              cudaStream_t stream);

// binning.cu
cudaError_t launch_frame_init(FrameCtl* ctl, FrameCtl* ctl_depth, uint2* ranges, uint32_t ntiles,
                              cudaStream_t stream);
// depth keys, their digit histograms and (last CTA) the pass plan of the depth sort
cudaError_t launch_depth_keys(const FrameBufs& fb, uint64_t n, uint32_t max_passes, cudaStream_t stream);
// mode 0: ping-pong between io.keys[0] and [1]; mode 1: [0] -> ... -> [2] via [1]
cudaError_t launch_plan(FrameCtl* ctl, uint64_t capacity, uint32_t max_passes, int mode,
                        cudaStream_t stream);
cudaError_t launch_frame_totals(const FrameCtl* ctl, const FrameCtl* ctl_depth, FrameTotals* totals,
                                cudaStream_t stream);

// place.cu: pairs by bin from the Gaussians in depth order (two-level counting sort, no pair sort)
cudaError_t place_geometry(const GridParams& gp, uint64_t n, uint64_t capacity, PlaceGeom* out);
// rectangles in depth order; coarse entries per (chunk, coarse bin) and their prefix; K and the
// capacity check (FrameCtl::plan_ok); coarse list starts and segments
cudaError_t launch_coarse_count(const FrameBufs& fb, const GridParams& gp, const PlaceGeom& pg, uint64_t n,
                                cudaStream_t stream);
// every (Gaussian, coarse bin) entry at its place in its coarse list
cudaError_t launch_coarse_place(const FrameBufs& fb, const GridParams& gp, const PlaceGeom& pg, uint64_t n,
                                cudaStream_t stream);
// bin counts, bin ranges, and every pair at its place in bin order; runs: a warp per run of
// consecutive segments with the next one prefetched (frames with many segments per warp)
cudaError_t launch_fine_place(const FrameBufs& fb, const GridParams& gp, const PlaceGeom& pg, uint64_t n,
                              bool runs, cudaStream_t stream);
uint32_t fine_place_warps(const PlaceGeom& pg);  // warps of the per-segment pair placement

// keys.cu: the reference-structured path (scan, key emission, boundary search)
cudaError_t launch_key_scan_emit(const FrameBufs& fb, const GridParams& gp, uint64_t n, uint32_t epoch,
                                 uint32_t max_passes, cudaStream_t stream);
cudaError_t launch_key_ranges(const SortIO& io, const FrameCtl* ctl, uint2* ranges, uint64_t max_keys,
                              cudaStream_t stream);

// sort.cu
cudaError_t launch_key_histogram(const unsigned long long* keys, uint64_t n, uint32_t key_bits,
                                 FrameCtl* ctl, cudaStream_t stream);
// One stable 8-bit pass. Sorts of at most one wave of resident tiles run onesweep on the
// epoch-tagged look-back words in `status`; larger ones run reduce-then-scan with its per-range
// digit table in `table` (sort_table_words(max_keys) u32). The two must not overlap when other
// sorts share `status`: a table value read as a look-back word could carry a live epoch tag.
// packed: launch the variant for (key << idx_bits | index) elements; the variant that does not
// match the frame's layout (FrameCtl::packed) returns at once.
cudaError_t launch_sort_pass(const SortIO& io, FrameCtl* ctl, unsigned long long* status, uint32_t* table,
                             uint32_t pass, uint32_t epoch, uint64_t max_keys, bool packed,
                             cudaStream_t stream);
size_t sort_status_words(uint64_t max_keys);
// One CTA runs the sort's look-back wait as tile 1 against tile 0's 256 status words (which must
// hold no live entry): it gives up after spin_limit polls and sets kErrTimeout in ctl.
cudaError_t launch_lookback_timeout_probe(const unsigned long long* status, FrameCtl* ctl, uint32_t spin_limit,
                                          cudaStream_t stream);
size_t sort_table_words(uint64_t max_keys);
uint32_t sort_pass_launches(uint64_t max_keys, bool packed);  // kernels one pass launches

// raster.cu
// every pixel of an RGBA8 image set to `value` (the render pass's clear before the splatting)
cudaError_t launch_fill_image(uchar4* img, uint64_t pixels, uchar4 value, cudaStream_t stream);
// 16-pixel rows of blocks of the rasterised band, and the rasteriser over block rows
// [first_block_row, first_block_row + block_rows) of it (all of them by default)
uint32_t raster_block_rows(const GridParams& gp);
cudaError_t launch_rasterize(const float4* rec, const SortIO& io, const uint2* ranges,
                             const FrameCtl* ctl, const GridParams& gp, uchar4* img,
                             bool per_element_exit, cudaStream_t stream, uint32_t first_block_row = 0,
                             uint32_t block_rows = 0xFFFFFFFFu);

}  // namespace kt
