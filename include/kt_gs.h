/*
 * kt_gs.h - C ABI of the B200 Gaussian-splatting renderer.
 *
 * This library replaces the Vulkan compute pipeline that klartraum's
 * VulkanGaussianSplatting graph node records (projection -> binning ->
 * radix sort -> bin bounds -> binned splatting). Every entry point takes
 * plain pointers and sizes; CUDA streams are passed as opaque `void*`
 * (a cudaStream_t, NULL = the legacy default stream).
 *
 * Every call returns a kt_status. On failure kt_gs_last_error() gives a
 * message for the context; the C++ node shim turns a non-OK status into
 * std::runtime_error, the reference's error convention
 * (src/vulkan_gaussian_splatting.cpp:33,37,223,227,230).
 *
 * Threading: a context is used by one host thread at a time. Contexts on
 * different devices may be driven concurrently from different threads.
 */
#ifndef KT_GS_H
#define KT_GS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KT_GS_ABI_VERSION 3

typedef enum kt_status {
    KT_OK = 0,
    KT_ERR_ARG = 1,      /* invalid argument or configuration */
    KT_ERR_CUDA = 2,     /* a CUDA runtime call failed */
    KT_ERR_CAPACITY = 3, /* key buffer too small; kt_gs_frame_stats().num_keys holds the need */
    KT_ERR_TIMEOUT = 4,  /* a bounded device-side wait (decoupled look-back) ran out */
    KT_ERR_NCCL = 5,     /* reserved for the multi-GPU strip gather */
    KT_ERR_IO = 6,       /* file could not be read or parsed */
    KT_ERR_STATE = 7,    /* call out of order (e.g. render before any Gaussians were set) */
    KT_ERR_NOMEM = 8     /* a device or pinned-host allocation failed */
} kt_status;

/*
 * One 3D Gaussian, 236 bytes, field order of klartraum::Gaussian3D
 * (include/klartraum/vulkan_gaussian_splatting_types.hpp:24-33) and of the
 * GLSL `Gaussian` (shaders/gsplat/gsplat_types.glsl:1-10). scale is already
 * exp()'d and alpha already sigmoid()'ed, as loadSPZModel leaves them
 * (src/vulkan_gaussian_splatting.cpp:348,356-358). color is the raw SH DC
 * coefficient per channel; shR/shG/shB are bands 1..3 (15 each).
 */
typedef struct kt_gaussian3d {
    float position[3];
    float rotation[4]; /* x, y, z, w */
    float scale[3];
    float color[3];
    float alpha;
    float shR[15];
    float shG[15];
    float shB[15];
} kt_gaussian3d;

/*
 * Camera uniform block, 192 bytes: three column-major 4x4 matrices, element
 * (col c, row r) at index 4*c + r. Layout of klartraum::CameraMVP
 * (include/klartraum/camera.hpp:44-48) and of the projection shader's UBO
 * (shaders/gsplat/gsplat_projection.comp:14-18).
 */
typedef struct kt_camera_mvp {
    float model[16];
    float view[16];
    float proj[16];
} kt_camera_mvp;

/*
 * Projected Gaussian, 48 bytes, the GLSL scalar layout of `Gaussian2D`
 * (shaders/gsplat/gsplat_types.glsl:12-19): pixel position, clip-space z,
 * bin mask, inverse covariance (column-major c00,c01,c10,c11), colour,
 * alpha. Used for stage dumps and for kt_gs_render_projected().
 */
typedef struct kt_gaussian2d {
    float position[2];
    float z;
    uint32_t binMask;
    float covInv[4];
    float color[3];
    float alpha;
} kt_gaussian2d;

/* Flags for kt_gs_config.flags. */
#define KT_GS_FLAG_EXIT_PER_ELEMENT 0x1u /* stop a pixel after any Gaussian once T <= 1-0.9999,
                                            instead of only at 64-Gaussian batch ends
                                            (gsplat_binned_splatting.comp:98,114) */
#define KT_GS_FLAG_NO_AUTOGROW 0x2u      /* on key overflow return KT_ERR_CAPACITY instead of
                                            growing the key buffers and rendering again */
#define KT_GS_FLAG_ASYNC 0x4u            /* do not wait for the frame status after a render;
                                            kt_gs_sync() reports overflow/timeouts later */
#define KT_GS_FLAG_KEEP_UNSORTED 0x8u    /* accepted for compatibility; the unsorted dumps are always
                                            available (rebuilt from the device's bin rectangles) */
#define KT_GS_FLAG_TIMING 0x10u          /* record CUDA events around every stage */
#define KT_GS_FLAG_GRAPH 0x40u          /* replay each path's frame as a captured CUDA graph: the
                                            kernels of a frame are captured once (again when the image
                                            pointer, scene, buffers, Gaussian count or flags change)
                                            and launched with one call; the camera is copied into
                                            device memory before each replay. Stage timers are not
                                            recorded in this mode */
#define KT_GS_FLAG_SORTED_KEYS 0x20u     /* bin through the reference's stage structure: scan of the
                                            counts in index order, one (bin << depth_bits | depth, index)
                                            pair per bin and Gaussian, radix sort of the pairs, boundary
                                            search for the bin ranges (same image and dumps; slower) */

typedef struct kt_gs_config {
    uint32_t width;          /* screen width in pixels (reference: 512, vulkan_gaussian_splatting.cpp:20) */
    uint32_t height;         /* screen height in pixels (reference: 512, :21) */
    uint32_t bin_width;      /* binning cell in pixels; 16 = 16x16 tiles. 128 at 512x512 is the
                                reference's 4x4 grid (:23, gsplat_binning.comp:55-56). Multiple of 16. */
    uint32_t bin_height;
    int32_t sh_degree;       /* 0..3 bands kept on the device; -1 = detect from the data */
    float cull_z;            /* Gaussians with clip-space z below this are dropped (1.0,
                                gsplat_binning.comp:113) */
    uint32_t flags;          /* KT_GS_FLAG_* */
    uint32_t num_paths;      /* frames in flight, each with its own device workspace (reference
                                numberPaths, src/klartraum_engine.cpp:71) */
    uint64_t key_capacity;   /* initial (tile, Gaussian) key capacity per path; 0 = size on demand */
    uint32_t tile_row_begin; /* screen band: only bin rows [begin, end) are binned and drawn; */
    uint32_t tile_row_end;   /* end = 0 means all rows (used by the banded multi-GPU split) */
} kt_gs_config;

/* Per-frame statistics of the last render on a path. */
typedef struct kt_gs_stats {
    uint64_t num_gaussians;  /* N */
    uint64_t num_keys;       /* K = sum of tile counts = (bin, Gaussian) pairs */
    uint64_t key_capacity;   /* current key capacity of the path */
    uint64_t num_visible;    /* Gaussians with a non-zero tile count */
    uint32_t tiles_x;
    uint32_t tiles_y;
    uint32_t key_bits;       /* significant bits of the compact sort key (bin bits + depth bits) */
    uint32_t depth_bits;     /* bits of the depth field after subtracting the frame's minimum */
    uint32_t sort_passes;    /* passes over the pairs: 0, they are placed in bin order directly */
    uint32_t error_flags;    /* device error bits: 1 = capacity, 2 = look-back timeout */
    uint32_t depth_min_bits; /* smallest (floatBitsToUint(z) ^ 0x80000000) over binned Gaussians */
    uint32_t depth_max_bits;
    uint32_t status_bytes;   /* bytes of frame status copied device->host after every frame */
    uint32_t launches;       /* kernels launched per frame */
    uint32_t packed;         /* 1: pairs are (bin << idx_bits | index) words */
    uint32_t idx_bits;       /* index bits of a packed element */
    uint32_t place_chunks;   /* chunks of depth order the pair placement split the Gaussians into */
    uint32_t place_bands;    /* bands of coarse-bin rows (4x4 bins each) of the pair placement */
    uint32_t place_runs;     /* 1: pairs placed by runs of segments (long coarse lists), 0: a warp
                                per segment */
} kt_gs_stats;

/* Totals accumulated on the device over every frame rendered on a path since the last
 * kt_gs_counters_take(); used to turn stage times into bandwidth without per-frame syncs. */
typedef struct kt_gs_counters {
    uint64_t frames;      /* frames whose sort plan ran */
    uint64_t keys;        /* sum of K */
    uint64_t key_passes;  /* sum of K * (passes over the pairs; 0 with direct placement) */
    uint64_t visible;     /* sum of Gaussians with a non-zero tile count */
    uint64_t sort_bytes;  /* sum of bytes written by the binning: 4 per pair + 8 per (Gaussian,
                             coarse bin) entry of the placement; 24 or 16 per pair and pass of
                             the pair sort with KT_GS_FLAG_SORTED_KEYS */
    uint64_t depth_sort_bytes; /* same for the depth sort of the Gaussians */
} kt_gs_counters;

/* Buffers that kt_gs_debug_dump() can copy out after a render.
 *
 * Device buffers on both binning paths: PROJECTED, TILE_COUNTS, VALUES_SORTED, TILE_RANGES.
 * KT_GS_FLAG_SORTED_KEYS also keeps OFFSETS and KEYS_SORTED in device buffers. The default path
 * (pairs placed in bin order) has no such buffers: there OFFSETS, KEYS_UNSORTED and
 * VALUES_UNSORTED are REBUILT ON THE HOST from the device's counts, bin rectangles and depths,
 * and KEYS_SORTED is assembled on the host from the device's pairs, bin ranges and depths; they
 * exist to compare against the reference's stage layout and are no evidence of a kernel. The
 * placement's own device products are DEPTH_ORDER, COARSE_INFO, COARSE_LISTS and
 * SEGMENT_COUNTS (default path only). */
typedef enum kt_gs_stage {
    KT_GS_STAGE_PROJECTED = 0,       /* kt_gaussian2d[N], binMask = 0xFFFFFFFF as projected
                                        (gsplat_projection.comp:228); the colour of a Gaussian that
                                        meets no bin is 0 (no later stage reads it) */
    KT_GS_STAGE_TILE_COUNTS = 1,     /* uint32[N] bins overlapped by each Gaussian (0 if culled) */
    KT_GS_STAGE_OFFSETS = 2,         /* uint64[N] exclusive scan of the tile counts in Gaussian index
                                        order (default path: host-rebuilt from the counts) */
    KT_GS_STAGE_KEYS_UNSORTED = 3,   /* uint64[K] bin<<32 | (floatBitsToUint(z) ^ 0x80000000), Gaussians
                                        in index order, bins ascending (both paths: host-rebuilt from
                                        the device's per-Gaussian bin rectangles and depths) */
    KT_GS_STAGE_VALUES_UNSORTED = 4, /* uint32[K] Gaussian index, same order (host-rebuilt) */
    KT_GS_STAGE_KEYS_SORTED = 5,     /* uint64[K], same key layout, stably sorted (default path:
                                        host-assembled from the device's pairs, ranges and depths) */
    KT_GS_STAGE_VALUES_SORTED = 6,   /* uint32[K] Gaussian index of every pair in sorted order */
    KT_GS_STAGE_TILE_RANGES = 7,     /* uint32[2 * tiles] {start, end} per bin (StartAndEnd,
                                        gsplat_types.glsl:21-24); empty bins {0, 0} */
    KT_GS_STAGE_DEPTH_ORDER = 8,     /* uint32[num_visible] Gaussian index at each position of the depth
                                        sort's output: the Gaussians that meet a bin, stably by depth
                                        (the sort drops the others) */
    KT_GS_STAGE_COARSE_INFO = 9,     /* uint32[4 * coarse bins] per coarse bin (4x4 bins, over the binned
                                        rows): list start, entries, first segment, 0 */
    KT_GS_STAGE_COARSE_LISTS = 10,   /* uint32[2 * entries] (Gaussian index, mask of the 4x4 bins met:
                                        bit 4*row + col) by coarse bin, depth order within a list */
    KT_GS_STAGE_SEGMENT_COUNTS = 11, /* uint32[16 * segments] pairs per bin of the 4x4 in each segment
                                        (256 consecutive entries of one coarse list) */
    KT_GS_STAGE_COUNT = 12
} kt_gs_stage;

/* Stage timers (KT_GS_FLAG_TIMING), in the order the stages run. */
#define KT_GS_NSTAGES 7
/* Default binning: 0 projection + count, 1 depth keys + depth sort of the Gaussians, 2 coarse
 * counts + their prefix over chunks + coarse list starts and K, 3 coarse placement, 4 bin counts +
 * bin ranges + pair placement (+ frame counters), 5 rasterise, 6 whole frame.
 * KT_GS_FLAG_SORTED_KEYS: 0 projection + count, 1 scan + key emission, 2 sort of the pairs by
 * key, 3 bin ranges (boundary search), 4 frame counters, 5 rasterise, 6 whole frame. */

typedef struct kt_gs_ctx kt_gs_ctx;

/* Fill a config with the reference's defaults: 512x512, 128-px bins (4x4 grid), SH3, cull 1.0. */
void kt_gs_config_default(kt_gs_config* cfg);

/* Library ABI version (KT_GS_ABI_VERSION). */
int kt_gs_abi_version(void);

/* Human-readable name of a status code. */
const char* kt_gs_status_string(kt_status status);

/*
 * Create a renderer on CUDA device `device`.
 * Replaces the constructor VulkanGaussianSplatting(ctx, imageViewSrc, cameraUBO, path)
 * (include/klartraum/vulkan_gaussian_splatting.hpp:44-48, src/vulkan_gaussian_splatting.cpp:13-213)
 * minus the scene load, which is kt_gs_set_gaussians() / kt_gs_load_spz().
 */
kt_status kt_gs_create(const kt_gs_config* cfg, int device, kt_gs_ctx** out);

/* Release every device buffer of the context (reference destructor, .cpp:215-218). */
kt_status kt_gs_destroy(kt_gs_ctx* ctx);

/* Message of the last failed call on this context ("" if none). Valid until the next call. */
const char* kt_gs_last_error(const kt_gs_ctx* ctx);

/* Replace the context's KT_GS_FLAG_* bits (e.g. switch to KT_GS_FLAG_ASYNC after warm-up). */
kt_status kt_gs_set_flags(kt_gs_ctx* ctx, uint32_t flags);

/* Copy of the context's configuration (with sh_degree resolved once Gaussians are set). */
kt_status kt_gs_get_config(const kt_gs_ctx* ctx, kt_gs_config* cfg);

/*
 * Upload n Gaussians from host memory (array of structs, 236 B each) and keep them on the
 * device as planes of float4. Replaces the Gaussians3D buffer upload
 * (src/vulkan_gaussian_splatting.cpp:40-43). Synchronous.
 */
kt_status kt_gs_set_gaussians(kt_gs_ctx* ctx, const kt_gaussian3d* host, uint64_t n);

/* Same from device memory (e.g. a buffer filled by a collective broadcast), on `stream`. */
kt_status kt_gs_set_gaussians_device(kt_gs_ctx* ctx, const kt_gaussian3d* dev, uint64_t n,
                                     void* stream);

/*
 * Load an .spz file (gzip-compressed packed Gaussians) and upload it with the activations of
 * loadSPZModel (src/vulkan_gaussian_splatting.cpp:322-365): alpha = sigmoid, scale = exp.
 */
kt_status kt_gs_load_spz(kt_gs_ctx* ctx, const char* path);

/*
 * Decode an .spz file on the host into Gaussian3D records with loadSPZModel's activations
 * (the records kt_gs_load_spz uploads). With out == NULL only *count (and *sh_degree) are set;
 * otherwise capacity must be >= *count. KT_ERR_IO for unreadable or malformed files.
 * No counterpart in the reference (its loader decodes straight into the node's buffer).
 */
kt_status kt_gs_spz_decode(const char* path, kt_gaussian3d* out, uint64_t capacity, uint64_t* count,
                           uint32_t* sh_degree);

/*
 * Load a 3D Gaussian Splatting .ply file (binary little endian or ASCII; x y z, f_dc_0..2,
 * opacity, scale_0..2, rot_0..3 with rot_0 = w) as loadPLYModel does
 * (src/vulkan_gaussian_splatting.cpp:367-417): only Gaussians inside [-1.5, 1.5]^3, alpha =
 * sigmoid(opacity), scale = exp, colour pre-baked as 0.5 + 0.282095 f_dc, higher SH zero.
 */
kt_status kt_gs_load_ply(kt_gs_ctx* ctx, const char* path);

/* The same decode into host records; with out == NULL only *count (Gaussians kept) is set. */
kt_status kt_gs_ply_decode(const char* path, kt_gaussian3d* out, uint64_t capacity, uint64_t* count);

/*
 * Render one frame. `cam` is host memory (the per-path camera UBO, uniformbufferobject.hpp:67-70).
 * `d_rgba8` is a device image of width*height RGBA8 pixels, row-major, row 0 at the top, 4-byte
 * aligned (KT_ERR_ARG otherwise); it is read-modify-written:
 * out = clamp(in + vec4(C,1)*(1-T)) (gsplat_binned_splatting.comp:119-121).
 * Work is enqueued on `stream`; unless KT_GS_FLAG_ASYNC is set the call waits for the frame
 * status and, on key overflow, grows the key buffers and renders again.
 * Replaces ComputeGraph::submitTo of the node's sub-graph (computegraph.hpp:122-139).
 */
kt_status kt_gs_render(kt_gs_ctx* ctx, const kt_camera_mvp* cam, void* d_rgba8, uint32_t path,
                       void* stream);

/*
 * Render one frame into a host image: copies the host image to the device, renders, and
 * copies it back, all on `stream`, and waits. `h_rgba8` should be pinned for full speed.
 * With KT_GS_FLAG_ASYNC nothing is waited for: the image is ready (and errors are reported)
 * after kt_gs_sync(path), so frames on different paths and streams overlap their copies with
 * each other's kernels.
 */
kt_status kt_gs_render_host(kt_gs_ctx* ctx, const kt_camera_mvp* cam, void* h_rgba8,
                            uint32_t path, void* stream);

/*
 * The same with the image cleared on the device to `clear_rgba` before the splatting, as the
 * reference's render pass clears the swap-chain image to (0, 0, 0, 1) before the compute pass
 * blends into it (include/klartraum/renderpass.hpp:170, gsplat_binned_splatting.comp:119-124):
 * nothing is copied to the device but the camera; the rendered image is copied out.
 */
kt_status kt_gs_render_host_clear(kt_gs_ctx* ctx, const kt_camera_mvp* cam, const uint8_t clear_rgba[4],
                                  void* h_rgba8, uint32_t path, void* stream);

/* Render n_views cameras, view v into d_rgba8[v] (device pointers), on `stream`. */
kt_status kt_gs_render_batch(kt_gs_ctx* ctx, const kt_camera_mvp* cams, uint32_t n_views,
                             void* const* d_rgba8, void* stream);

/*
 * Run binning -> sort -> bin bounds -> splatting on n already projected Gaussians given in
 * host memory (the input the reference's binning test feeds, tests/test_gaussian_splatting.cpp:247-320).
 * The records' binMask fields are ignored.
 */
kt_status kt_gs_render_projected(kt_gs_ctx* ctx, const kt_gaussian2d* host, uint64_t n,
                                 void* d_rgba8, uint32_t path, void* stream);

/* Wait for all work of `path` and report any device error of the frames rendered on it since
 * the previous sync (key overflow: those frames drew nothing; look-back timeout). */
kt_status kt_gs_sync(kt_gs_ctx* ctx, uint32_t path);

/* Statistics of the last frame rendered on `path` (waits for it). */
kt_status kt_gs_frame_stats(kt_gs_ctx* ctx, uint32_t path, kt_gs_stats* out);

/* Copy a stage buffer of the last frame on `path` to host memory (waits for it).
 * `bytes` is the size of host_dst; *written receives the bytes copied. */
kt_status kt_gs_debug_dump(kt_gs_ctx* ctx, uint32_t path, kt_gs_stage stage, void* host_dst,
                           uint64_t bytes, uint64_t* written);

/* Elements [first, first + count) of a stage buffer (count is clipped to the stage's length;
 * the element is one record, word or range as listed in kt_gs_stage). For slices of stages too
 * large to copy whole, e.g. the sorted pairs of one band of bin rows (their positions are given
 * by TILE_RANGES). With host_dst == NULL only *written (the bytes needed) is set. */
kt_status kt_gs_debug_dump_range(kt_gs_ctx* ctx, uint32_t path, kt_gs_stage stage, uint64_t first,
                                 uint64_t count, void* host_dst, uint64_t bytes, uint64_t* written);

/* Per-stage milliseconds of the last frame on `path` (needs KT_GS_FLAG_TIMING). */
kt_status kt_gs_stage_times(kt_gs_ctx* ctx, uint32_t path, float ms[KT_GS_NSTAGES]);

/* Read and reset the device-side frame counters of `path` (waits for its work). */
kt_status kt_gs_counters_take(kt_gs_ctx* ctx, uint32_t path, kt_gs_counters* out);

/*
 * Sums of the per-stage milliseconds of every frame rendered on `path` with
 * KT_GS_FLAG_TIMING since the previous call (waits for them), and their number; resets.
 */
kt_status kt_gs_stage_times_total(kt_gs_ctx* ctx, uint32_t path, double ms_total[KT_GS_NSTAGES],
                                  uint64_t* frames);

/*
 * Stable LSD radix sort of (uint64 key, uint32 value) pairs by key bits [0, key_bits), on the
 * device. The operator behind the GaussianSort BufferTransformation
 * (src/vulkan_gaussian_splatting.cpp:95-143, shaders/gsplat/gsplat_radix_sort_*.comp).
 * Two-phase scratch protocol: call with d_temp == NULL to get *temp_bytes, allocate, call again.
 * keys_in/vals_in are not modified; keys_out/vals_out must not alias them.
 */
kt_status kt_gs_radix_sort_pairs(const uint64_t* d_keys_in, const uint32_t* d_vals_in,
                                 uint64_t* d_keys_out, uint32_t* d_vals_out, uint64_t n,
                                 uint32_t key_bits, void* d_temp, size_t* temp_bytes,
                                 void* stream);

/*
 * The same stable pair sort as kt_gs_radix_sort_pairs, for callers that cannot allocate device
 * memory: a render loop with a fixed frame budget (cudaMalloc/cudaFree may synchronise the
 * device), a plugin inside a host engine whose allocator owns all device memory, a process whose
 * memory pool already holds the device's free memory. No counterpart in the reference.
 *
 * The caller passes inputs and outputs only; the scratch is one fixed array of
 * KT_GS_STATIC_SORT_SCRATCH_BYTES (13,127,680 bytes, 12.52 MiB) in the library, kept on every
 * device that loads it until the process exits. n above KT_GS_STATIC_SORT_MAX_PAIRS returns
 * KT_ERR_CAPACITY without doing anything. keys_out/vals_out must not alias keys_in/vals_in
 * (KT_ERR_ARG). Every call looks up the array's device address on the current device; the first
 * call on a device also loads the module there, so make that first call before any stream
 * capture. All calls share the array: calls that overlap on the GPU race and must be ordered by
 * the caller (e.g. issued on one stream). Asynchronous on `stream`; no allocation of any kind.
 * A look-back wait that runs out is reported by kt_gs_radix_sort_status(NULL, stream).
 */
#define KT_GS_STATIC_SORT_MAX_PAIRS 1048576u
#define KT_GS_STATIC_SORT_SCRATCH_BYTES 13127680u
kt_status kt_gs_radix_sort_pairs_static(const uint64_t* d_keys_in, const uint32_t* d_vals_in,
                                        uint64_t* d_keys_out, uint32_t* d_vals_out, uint64_t n,
                                        uint32_t key_bits, void* stream);

/*
 * Wait for `stream` and report the device error bits of the last sort that used a scratch:
 * d_temp of kt_gs_radix_sort_pairs, or NULL for kt_gs_radix_sort_pairs_static's fixed array.
 * KT_ERR_TIMEOUT when a bounded look-back wait ran out (that sort's output is not sorted).
 * No counterpart in the reference (its sort reports nothing).
 */
kt_status kt_gs_radix_sort_status(const void* d_temp, void* stream);

/*
 * Check of the timeout path: runs the sort's look-back wait against status words of the fixed
 * scratch that nothing publishes, giving up after spin_limit polls (1 .. 2^22); the timeout is
 * recorded in the scratch's control block as a sort would record it, so the next
 * kt_gs_radix_sort_status(NULL, stream) returns KT_ERR_TIMEOUT, until the next
 * kt_gs_radix_sort_pairs_static clears it. No fault, no hang: the wait is bounded. Shares the
 * fixed scratch (order it with the static sorts). No counterpart in the reference.
 */
kt_status kt_gs_radix_sort_static_timeout_probe(uint32_t spin_limit, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KT_GS_H */
