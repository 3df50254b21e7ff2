/*
 * kt_oracle.h - CPU restatement of klartraum's Gaussian-splatting compute shaders.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the CUDA renderer is compared against;
 * it is never linked into, loaded by, or called from the product library. Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.
 *
 * Every stage follows one shader of the reference (paths relative to the klartraum
 * repository), in float32 with the shader's operation order, compiled with
 * -ffp-contract=off so that no multiply-add is fused:
 *   ko_project        shaders/gsplat/gsplat_projection.comp:37-237
 *   ko_tile_counts    shaders/gsplat/gsplat_binning.comp:53-81,85-147
 *   ko_emit_keys      shaders/gsplat/gsplat_binning.comp:112-147 + radix_sort_include.glsl:51-63
 *   ko_sort_pairs     shaders/gsplat/gsplat_radix_sort_{histogram,hist_prefix_sum,hist_scatter}.comp
 *   ko_tile_ranges    shaders/gsplat/gsplat_bin_bounds.comp:30-72
 *   ko_rasterize      shaders/gsplat/gsplat_binned_splatting.comp:41-125
 * ko_project_f64 / ko_render_frame_f64 repeat the same stages in double precision, the
 * reference's algorithm without float32 rounding, to log how far float32 images drift.
 * The reference's screen (512x512), 4x4 bin grid and 2N key cap are generalised to a
 * W x H screen with bin_width x bin_height cells and an exactly sized key list; with
 * W = H = 512 and 128-px bins the geometry is the reference's.
 */
#ifndef KT_ORACLE_H
#define KT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* klartraum::Gaussian3D / GLSL Gaussian, 236 B (gsplat_types.glsl:1-10). */
typedef struct ko_gaussian3d {
    float position[3];
    float rotation[4];
    float scale[3];
    float color[3];
    float alpha;
    float shR[15];
    float shG[15];
    float shB[15];
} ko_gaussian3d;

/* GLSL Gaussian2D in scalar layout, 48 B (gsplat_types.glsl:12-19). */
typedef struct ko_gaussian2d {
    float position[2];
    float z;
    uint32_t binMask;
    float covInv[4]; /* column-major: [0][0], [0][1], [1][0], [1][1] */
    float color[3];
    float alpha;
} ko_gaussian2d;

/* CameraMVP: model, view, proj, column-major (camera.hpp:44-48). */
typedef struct ko_camera {
    float model[16];
    float view[16];
    float proj[16];
} ko_camera;

typedef struct ko_config {
    uint32_t width, height;         /* screen, px */
    uint32_t bin_width, bin_height; /* binning cell, px */
    int32_t sh_degree;              /* SH bands evaluated: coefficients 0..(d+1)^2-2 of shX[] */
    float cull_z;                   /* gsplat_binning.comp:113 threshold (1.0) */
    uint32_t exit_per_element;      /* 0: early exit only at 64-batch ends (reference) */
    uint32_t row_begin, row_end;    /* bin rows binned/drawn; row_end = 0 -> all */
} ko_config;

uint32_t ko_tiles_x(const ko_config* cfg);
uint32_t ko_tiles_y(const ko_config* cfg);

/* Number of OpenMP threads the oracle uses (0 = all). */
void ko_set_threads(int n);
int ko_get_threads(void);

/* Stage 1: 3D -> 2D projection, colour and alpha; binMask = 0xFFFFFFFF. */
void ko_project(const ko_config* cfg, const ko_camera* cam, const ko_gaussian3d* in, uint64_t n,
                ko_gaussian2d* out);

/* Stage 2: number of bins each projected Gaussian overlaps (0 when z < cull_z). */
void ko_tile_counts(const ko_config* cfg, const ko_gaussian2d* g, uint64_t n, uint32_t* counts);

/* Exclusive scan of the counts; returns the total. */
uint64_t ko_exclusive_scan(const uint32_t* counts, uint64_t n, uint64_t* offsets);

/* Stage 3: one (bin<<32 | (floatBitsToUint(z) ^ 0x80000000), index) pair per overlapped bin,
 * Gaussians in index order and bins in ascending bin index per Gaussian. */
void ko_emit_keys(const ko_config* cfg, const ko_gaussian2d* g, uint64_t n, const uint64_t* offsets,
                  uint64_t* keys, uint32_t* vals);

/* Stage 4: stable sort by key (LSD radix over bits [0, key_bits)), in place. */
void ko_sort_pairs(uint64_t* keys, uint32_t* vals, uint64_t k, uint32_t key_bits);

/* Stage 5: {start, end} per bin from the sorted keys (bin = key >> 32); others {0, 0}. */
void ko_tile_ranges(const uint64_t* keys, uint64_t k, uint32_t ntiles, uint32_t* ranges);

/* Stage 6: front-to-back splatting into an RGBA8 image, read-modify-write. */
void ko_rasterize(const ko_config* cfg, const ko_gaussian2d* g, const uint32_t* vals,
                  const uint32_t* ranges, uint8_t* rgba);

/* Bin rectangle of every projected Gaussian: rects[4i..4i+3] = x0, x1, y0, y1 (half-open, bins;
 * rows clipped to the binned rows), all zero when culled (gsplat_binning.comp:53-81,113). */
void ko_tile_rects(const ko_config* cfg, const ko_gaussian2d* g, uint64_t n, uint32_t* rects);

/* A projected Gaussian in double precision (same fields as ko_gaussian2d, no bin mask). */
typedef struct ko_gaussian2d_f64 {
    double position[2];
    double z;
    double covInv[4];
    double color[3];
    double alpha;
} ko_gaussian2d_f64;

/* Projection in double precision: the same operations as ko_project, every one in double. */
void ko_project_f64(const ko_config* cfg, const ko_camera* cam, const ko_gaussian3d* in, uint64_t n,
                    ko_gaussian2d_f64* out);

/* Whole frame in double precision: projection, bin rectangles, pairs by (bin, depth, index),
 * splatting with the reference's exit rules; rgba_out = unquantised RGBA in [0, 1] (rows outside
 * the binned rows keep rgba_in / 255). Returns the pair count, UINT64_MAX on allocation failure.
 * Used to measure how far float32 images (the GPU's and ko_render_frame's) drift. */
uint64_t ko_render_frame_f64(const ko_config* cfg, const ko_camera* cam, const ko_gaussian3d* in,
                             uint64_t n, const uint8_t* rgba_in, double* rgba_out);

/*
 * Whole frame from 3D Gaussians. Scratch is allocated inside. Returns the key count, or
 * UINT64_MAX on allocation failure. Any of the optional outputs may be NULL:
 * g2d[n], counts[n], offsets[n], keys/vals (sorted; need k_cap >= K), ranges[2*tiles].
 */
uint64_t ko_render_frame(const ko_config* cfg, const ko_camera* cam, const ko_gaussian3d* in,
                         uint64_t n, uint8_t* rgba, ko_gaussian2d* g2d, uint32_t* counts,
                         uint64_t* offsets, uint64_t* keys, uint32_t* vals, uint64_t k_cap,
                         uint32_t* ranges);

/* Same from projected Gaussians (binning onwards). */
uint64_t ko_render_projected(const ko_config* cfg, const ko_gaussian2d* g2d, uint64_t n,
                             uint8_t* rgba, uint64_t* keys, uint32_t* vals, uint64_t k_cap,
                             uint32_t* ranges);

#ifdef __cplusplus
}
#endif

#endif
