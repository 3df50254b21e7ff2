/*
 * kt_oracle.c - CPU restatement of klartraum's gsplat compute shaders (test infrastructure).
 *
 * The checker for the CUDA renderer: nothing in the product links or loads this file.
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fno-fast-math -fopenmp).
 *
 * GLSL semantics restated here:
 *  - matrices are column-major, m[c][r]; the constructor mat3(a,b,c, d,e,f, g,h,i) fills
 *    column 0 with (a,b,c);
 *  - A*B and M*v sum the products in ascending k, left to right;
 *  - `a * b * c` is (a * b) * c;
 *  - inverse(mat2) is the adjugate times 1/det (the driver's choice is not specified by
 *    GLSL; this is the form glm uses on the CPU);
 *  - normalize(v) = v / length(v) (GLSL spec's definition);
 *  - float32 throughout, no fused multiply-add.
 */
#include "kt_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ helpers */

typedef struct { float m[3][3]; } mat3;
typedef struct { float m[4][4]; } mat4;
typedef struct { float m[2][2]; } mat2;

static int g_threads = 0;

void ko_set_threads(int n) { g_threads = n; }

int ko_get_threads(void) {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

static mat4 mat4_load(const float* p) {
    mat4 r;
    for (int c = 0; c < 4; ++c)
        for (int k = 0; k < 4; ++k) r.m[c][k] = p[4 * c + k];
    return r;
}

static mat4 mat4_mul(mat4 a, mat4 b) {
    mat4 r;
    for (int c = 0; c < 4; ++c)
        for (int k = 0; k < 4; ++k)
            r.m[c][k] = a.m[0][k] * b.m[c][0] + a.m[1][k] * b.m[c][1] + a.m[2][k] * b.m[c][2] +
                        a.m[3][k] * b.m[c][3];
    return r;
}

static void mat4_vec(mat4 a, const float v[4], float out[4]) {
    for (int k = 0; k < 4; ++k)
        out[k] = a.m[0][k] * v[0] + a.m[1][k] * v[1] + a.m[2][k] * v[2] + a.m[3][k] * v[3];
}

static mat3 mat3_mul(mat3 a, mat3 b) {
    mat3 r;
    for (int c = 0; c < 3; ++c)
        for (int k = 0; k < 3; ++k)
            r.m[c][k] = a.m[0][k] * b.m[c][0] + a.m[1][k] * b.m[c][1] + a.m[2][k] * b.m[c][2];
    return r;
}

static mat3 mat3_transpose(mat3 a) {
    mat3 r;
    for (int c = 0; c < 3; ++c)
        for (int k = 0; k < 3; ++k) r.m[c][k] = a.m[k][c];
    return r;
}

static mat3 mat3_cols(float a, float b, float c, float d, float e, float f, float g, float h,
                      float i) {
    mat3 r;
    r.m[0][0] = a; r.m[0][1] = b; r.m[0][2] = c;
    r.m[1][0] = d; r.m[1][1] = e; r.m[1][2] = f;
    r.m[2][0] = g; r.m[2][1] = h; r.m[2][2] = i;
    return r;
}

static mat2 mat2_inverse(mat2 a) {
    float det = a.m[0][0] * a.m[1][1] - a.m[1][0] * a.m[0][1];
    float inv = 1.0f / det;
    mat2 r;
    r.m[0][0] = a.m[1][1] * inv;
    r.m[0][1] = -a.m[0][1] * inv;
    r.m[1][0] = -a.m[1][0] * inv;
    r.m[1][1] = a.m[0][0] * inv;
    return r;
}

static uint32_t f2u(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

uint32_t ko_tiles_x(const ko_config* cfg) { return (cfg->width + cfg->bin_width - 1) / cfg->bin_width; }
uint32_t ko_tiles_y(const ko_config* cfg) { return (cfg->height + cfg->bin_height - 1) / cfg->bin_height; }

static void row_span(const ko_config* cfg, uint32_t* rb, uint32_t* re) {
    uint32_t ty = ko_tiles_y(cfg);
    *rb = cfg->row_begin;
    *re = cfg->row_end == 0 ? ty : cfg->row_end;
    if (*re > ty) *re = ty;
    if (*rb > *re) *rb = *re;
}

/* ------------------------------------------------------------ projection */

/* gsplat_projection.comp:37-51 (quatToMat3) */
static mat3 quat_to_mat3(const float q[4]) {
    float x = q[0], y = q[1], z = q[2], w = q[3];
    float xx = x * x, yy = y * y, zz = z * z;
    float xy = x * y, xz = x * z, yz = y * z;
    float wx = w * x, wy = w * y, wz = w * z;
    return mat3_cols(1.0f - 2.0f * (yy + zz), 2.0f * (xy - wz), 2.0f * (xz + wy),
                     2.0f * (xy + wz), 1.0f - 2.0f * (xx + zz), 2.0f * (yz - wx),
                     2.0f * (xz - wy), 2.0f * (yz + wx), 1.0f - 2.0f * (xx + yy));
}

/* gsplat_projection.comp:53-118 (calculateCovarianceMatrix2D); mv = ubo.model * ubo.view */
static mat2 covariance_2d(const ko_gaussian3d* g, mat4 mv, const mat4* proj) {
    mat3 S = mat3_cols(g->scale[0], 0.0f, 0.0f, 0.0f, g->scale[1], 0.0f, 0.0f, 0.0f, g->scale[2]);
    mat3 R = quat_to_mat3(g->rotation);
    mat3 M = mat3_mul(S, R);
    mat3 cov3d = mat3_mul(mat3_transpose(M), M);

    float p4[4] = {g->position[0], g->position[1], g->position[2], 1.0f};
    float t4[4];
    mat4_vec(mv, p4, t4);
    float tx = t4[0], ty = t4[1], tz = t4[2];

    float focalX = proj->m[0][0];
    float focalY = proj->m[1][1];
    float tanFovX = 1.0f / focalX;
    float tanFovY = 1.0f / focalY;
    const float limx = 1.3f * tanFovX;
    const float limy = 1.3f * tanFovY;
    const float txtz = tx / tz;
    const float tytz = ty / tz;
    tx = fminf(limx, fmaxf(-limx, txtz)) * tz;
    ty = fmaxf(limy, fminf(-limy, tytz)) * tz;

    mat3 J = mat3_cols(focalX / tz, 0.0f, -(focalX * tx) / (tz * tz),
                       0.0f, focalY / tz, -(focalY * ty) / (tz * tz),
                       0.0f, 0.0f, 0.0f);
    mat3 W = mat3_cols(mv.m[0][0], mv.m[1][0], mv.m[2][0],
                       mv.m[0][1], mv.m[1][1], mv.m[2][1],
                       mv.m[0][2], mv.m[1][2], mv.m[2][2]);
    mat3 T = mat3_mul(W, J);
    mat3 cov = mat3_mul(mat3_mul(mat3_transpose(T), mat3_transpose(cov3d)), T);
    mat2 c2;
    c2.m[0][0] = cov.m[0][0];
    c2.m[0][1] = cov.m[0][1];
    c2.m[1][0] = cov.m[1][0];
    c2.m[1][1] = cov.m[1][1];
    return c2;
}

/* gsplat_projection.comp:120-161 (computeSphericalHarmonicsColor), bands up to `deg` */
static float sh_color(float base, const float coeffs[15], const float dir[3], int deg) {
    float x = dir[0], y = dir[1], z = dir[2];
    float x2 = x * x, y2 = y * y, z2 = z * z;
    float sh[16];
    sh[0] = 0.282095f;
    sh[1] = -0.488603f * y;
    sh[2] = -0.488603f * z;
    sh[3] = -0.488603f * x;
    sh[4] = 1.092548f * x * y;
    sh[5] = -1.092548f * y * z;
    sh[6] = 0.315392f * (2.0f * z2 - x2 - y2);
    sh[7] = -1.092548f * x * z;
    sh[8] = 0.546274f * (x2 - y2);
    sh[9] = -0.590044f * y * (3.0f * x2 - y2);
    sh[10] = 2.890611f * x * y * z;
    sh[11] = -0.457046f * y * (4.0f * z2 - x2 - y2);
    sh[12] = 0.373176f * z * (2.0f * z2 - 3.0f * x2 - 3.0f * y2);
    sh[13] = -0.457046f * x * (4.0f * z2 - x2 - y2);
    sh[14] = 1.445306f * z * (x2 - y2);
    sh[15] = -0.590044f * x * (x2 - 3.0f * y2);
    int ncoef = (deg + 1) * (deg + 1) - 1; /* the shader always runs 15; zero terms add nothing */
    float value = 0.5f + base * sh[0];
    for (int i = 0; i < ncoef; i++) value += coeffs[i] * sh[i + 1];
    return value;
}

void ko_project(const ko_config* cfg, const ko_camera* cam, const ko_gaussian3d* in, uint64_t n,
                ko_gaussian2d* out) {
    mat4 model = mat4_load(cam->model), view = mat4_load(cam->view), proj = mat4_load(cam->proj);
    mat4 pvm = mat4_mul(mat4_mul(proj, view), model); /* ubo.proj * ubo.view * ubo.model */
    mat4 mv = mat4_mul(model, view);                  /* ubo.model * ubo.view */
    const float half_w = (float)cfg->width * 0.5f;    /* 256.0 at 512 (comp:202) */
    const float half_h = (float)cfg->height * 0.5f;
    const float sxx = (float)cfg->width * (float)cfg->width; /* 512*512 at 512 (comp:208) */
    const float syy = (float)cfg->height * (float)cfg->height;
    const float sxy = (float)cfg->width * (float)cfg->height;
    int deg = cfg->sh_degree < 0 ? 3 : cfg->sh_degree;

#pragma omp parallel for schedule(static) num_threads(ko_get_threads())
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        const ko_gaussian3d* g = &in[i];
        float p4[4] = {g->position[0], g->position[1], g->position[2], 1.0f};
        float pos[4];
        mat4_vec(pvm, p4, pos);
        ko_gaussian2d o;
        float nx = pos[0] / pos[3];
        float ny = pos[1] / pos[3];
        o.position[0] = (nx + 1.0f) * half_w;
        o.position[1] = (ny + 1.0f) * half_h;
        o.z = pos[2];

        mat2 cov = covariance_2d(g, mv, &proj);
        cov.m[0][0] *= sxx;
        cov.m[0][1] *= sxy;
        cov.m[1][0] *= sxy;
        cov.m[1][1] *= syy;
        cov.m[0][0] += 0.3f;
        cov.m[1][1] += 0.3f;
        mat2 ci = mat2_inverse(cov);
        o.covInv[0] = ci.m[0][0];
        o.covInv[1] = ci.m[0][1];
        o.covInv[2] = ci.m[1][0];
        o.covInv[3] = ci.m[1][1];

        float t4[4];
        mat4_vec(mv, p4, t4);
        float len = sqrtf(t4[0] * t4[0] + t4[1] * t4[1] + t4[2] * t4[2]);
        float dir[3] = {t4[0] / len, t4[1] / len, t4[2] / len};
        o.color[0] = sh_color(g->color[0], g->shR, dir, deg);
        o.color[1] = sh_color(g->color[1], g->shG, dir, deg);
        o.color[2] = sh_color(g->color[2], g->shB, dir, deg);
        o.alpha = g->alpha;
        o.binMask = 0xFFFFFFFFu;
        out[i] = o;
    }
}

/* ------------------------------------------------------------- binning */

/* Half extents from gsplat_binning.comp:69-76: sqrt of the diagonal of inverse(covInv), x2.5 */
static void gauss_bounds(const ko_gaussian2d* g, float mn[2], float mx[2]) {
    mat2 ci;
    ci.m[0][0] = g->covInv[0];
    ci.m[0][1] = g->covInv[1];
    ci.m[1][0] = g->covInv[2];
    ci.m[1][1] = g->covInv[3];
    mat2 cov = mat2_inverse(ci);
    float stdDevX = sqrtf(cov.m[0][0]);
    float stdDevY = sqrtf(cov.m[1][1]);
    float spreadX = stdDevX * 2.5f;
    float spreadY = stdDevY * 2.5f;
    mn[0] = g->position[0] - spreadX;
    mn[1] = g->position[1] - spreadY;
    mx[0] = g->position[0] + spreadX;
    mx[1] = g->position[1] + spreadY;
}

/* The overlap test of gsplat_binning.comp:78-80 is an AND of an x part and a y part:
 * !(gmax.x < binMin.x || gmin.x > binMax.x) && !(gmax.y < binMin.y || gmin.y > binMax.y),
 * binMin = cell index * cell size and binMax = (index + 1) * cell size, both float.
 * This evaluates the x part for every column and the y part for every row. */
static int x_overlaps(float mn, float mx, uint32_t gx, float cw) {
    float bmin = (float)gx * cw;
    float bmax = (float)(gx + 1) * cw;
    return !(mx < bmin || mn > bmax);
}

static void overlap_spans(const ko_config* cfg, const ko_gaussian2d* g, uint32_t* x0, uint32_t* x1,
                          uint32_t* y0, uint32_t* y1) {
    float mn[2], mx[2];
    gauss_bounds(g, mn, mx);
    uint32_t tx = ko_tiles_x(cfg), rb, re;
    row_span(cfg, &rb, &re);
    float cw = (float)cfg->bin_width, ch = (float)cfg->bin_height;
    /* the overlapping columns/rows form one contiguous run: find first and last */
    uint32_t a = tx, b = 0;
    for (uint32_t gx = 0; gx < tx; ++gx)
        if (x_overlaps(mn[0], mx[0], gx, cw)) {
            if (a == tx) a = gx;
            b = gx + 1;
        }
    uint32_t c = re, d = rb;
    for (uint32_t gy = rb; gy < re; ++gy)
        if (x_overlaps(mn[1], mx[1], gy, ch)) {
            if (c == re) c = gy;
            d = gy + 1;
        }
    if (a >= b || c >= d) { a = b = 0; c = d = 0; }
    *x0 = a; *x1 = b; *y0 = c; *y1 = d;
}

void ko_tile_counts(const ko_config* cfg, const ko_gaussian2d* g, uint64_t n, uint32_t* counts) {
#pragma omp parallel for schedule(static) num_threads(ko_get_threads())
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        if (g[i].z < cfg->cull_z) { /* gsplat_binning.comp:113 */
            counts[i] = 0;
            continue;
        }
        uint32_t x0, x1, y0, y1;
        overlap_spans(cfg, &g[i], &x0, &x1, &y0, &y1);
        counts[i] = (x1 - x0) * (y1 - y0);
    }
}

uint64_t ko_exclusive_scan(const uint32_t* counts, uint64_t n, uint64_t* offsets) {
    uint64_t s = 0;
    for (uint64_t i = 0; i < n; ++i) {
        offsets[i] = s;
        s += counts[i];
    }
    return s;
}

void ko_emit_keys(const ko_config* cfg, const ko_gaussian2d* g, uint64_t n, const uint64_t* offsets,
                  uint64_t* keys, uint32_t* vals) {
    uint32_t tx = ko_tiles_x(cfg);
#pragma omp parallel for schedule(dynamic, 1024) num_threads(ko_get_threads())
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        if (g[i].z < cfg->cull_z) continue;
        uint32_t x0, x1, y0, y1;
        overlap_spans(cfg, &g[i], &x0, &x1, &y0, &y1);
        /* radix_sort_include.glsl:51-63: the depth digits are floatBitsToUint(z) ^ 0x80000000 */
        uint64_t depth = (uint64_t)(f2u(g[i].z) ^ 0x80000000u);
        uint64_t o = offsets[i];
        for (uint32_t gy = y0; gy < y1; ++gy)
            for (uint32_t gx = x0; gx < x1; ++gx) {
                uint64_t bin = (uint64_t)gy * tx + gx;
                keys[o] = (bin << 32) | depth;
                vals[o] = (uint32_t)i;
                ++o;
            }
    }
}

/* ---------------------------------------------------------------- sort */

void ko_sort_pairs(uint64_t* keys, uint32_t* vals, uint64_t k, uint32_t key_bits) {
    if (k <= 1) return;
    uint64_t* kb = (uint64_t*)malloc(k * sizeof(uint64_t));
    uint32_t* vb = (uint32_t*)malloc(k * sizeof(uint32_t));
    if (!kb || !vb) { free(kb); free(vb); abort(); }
    int nt = ko_get_threads();
    if ((uint64_t)nt > k / 4096 + 1) nt = (int)(k / 4096 + 1);
    uint64_t* hist = (uint64_t*)calloc((size_t)nt * 256, sizeof(uint64_t));
    uint64_t *src_k = keys, *dst_k = kb;
    uint32_t *src_v = vals, *dst_v = vb;
    for (uint32_t shift = 0; shift < key_bits; shift += 8) {
        memset(hist, 0, (size_t)nt * 256 * sizeof(uint64_t));
#pragma omp parallel num_threads(nt)
        {
#ifdef _OPENMP
            int t = omp_get_thread_num();
#else
            int t = 0;
#endif
            uint64_t lo = k * t / nt, hi = k * (t + 1) / nt;
            uint64_t* h = hist + (size_t)t * 256;
            for (uint64_t i = lo; i < hi; ++i) h[(src_k[i] >> shift) & 255]++;
        }
        /* digit-major, chunk-minor exclusive scan keeps the scatter stable */
        uint64_t s = 0;
        int single = 0;
        for (int d = 0; d < 256; ++d) {
            uint64_t dsum = 0;
            for (int t = 0; t < nt; ++t) {
                uint64_t c = hist[(size_t)t * 256 + d];
                hist[(size_t)t * 256 + d] = s;
                s += c;
                dsum += c;
            }
            if (dsum == k) single = 1;
        }
        if (single) continue; /* every key has the same digit: the pass would not move anything */
#pragma omp parallel num_threads(nt)
        {
#ifdef _OPENMP
            int t = omp_get_thread_num();
#else
            int t = 0;
#endif
            uint64_t lo = k * t / nt, hi = k * (t + 1) / nt;
            uint64_t* h = hist + (size_t)t * 256;
            for (uint64_t i = lo; i < hi; ++i) {
                uint64_t p = h[(src_k[i] >> shift) & 255]++;
                dst_k[p] = src_k[i];
                dst_v[p] = src_v[i];
            }
        }
        uint64_t* tk = src_k; src_k = dst_k; dst_k = tk;
        uint32_t* tv = src_v; src_v = dst_v; dst_v = tv;
    }
    if (src_k != keys) {
        memcpy(keys, src_k, k * sizeof(uint64_t));
        memcpy(vals, src_v, k * sizeof(uint32_t));
    }
    free(hist);
    free(kb);
    free(vb);
}

/* ---------------------------------------------------------- bin bounds */

void ko_tile_ranges(const uint64_t* keys, uint64_t k, uint32_t ntiles, uint32_t* ranges) {
    memset(ranges, 0, (size_t)ntiles * 2 * sizeof(uint32_t)); /* zeroed each frame (.cpp:149) */
#pragma omp parallel for schedule(static) num_threads(ko_get_threads())
    for (int64_t i = 0; i < (int64_t)k; ++i) {
        uint32_t b = (uint32_t)(keys[i] >> 32);
        if (i == (int64_t)k - 1) { /* gsplat_bin_bounds.comp:44-52 */
            ranges[2 * b + 1] = (uint32_t)(i + 1);
        } else {
            uint32_t bn = (uint32_t)(keys[i + 1] >> 32);
            if (b != bn) { /* :64-70 */
                ranges[2 * b + 1] = (uint32_t)(i + 1);
                ranges[2 * bn] = (uint32_t)(i + 1);
            }
        }
    }
}

/* ------------------------------------------------------------- splatting */

/* 1.0 - 0.9999 as a constant expression folded in double and stored as float */
#define KO_T_MIN ((float)(1.0 - 0.9999))

/* gsplat_binned_splatting.comp:41-45 */
static float eval_gaussian(float px, float py, const ko_gaussian2d* g) {
    float dx = px - g->position[0];
    float dy = py - g->position[1];
    float sx = g->covInv[0] * dx + g->covInv[2] * dy;
    float sy = g->covInv[1] * dx + g->covInv[3] * dy;
    float distance = dx * sx + dy * sy;
    return expf(-0.5f * distance);
}

static inline float clamp01(float v) { return v < 0.0f ? 0.0f : (v > 1.0f ? 1.0f : v); }

void ko_rasterize(const ko_config* cfg, const ko_gaussian2d* g, const uint32_t* vals,
                  const uint32_t* ranges, uint8_t* rgba) {
    uint32_t tx = ko_tiles_x(cfg), rb, re;
    row_span(cfg, &rb, &re);
    uint32_t ypix0 = rb * cfg->bin_height, ypix1 = re * cfg->bin_height;
    if (ypix1 > cfg->height) ypix1 = cfg->height;
    const int per_elem = cfg->exit_per_element != 0;
#pragma omp parallel for schedule(dynamic, 1) num_threads(ko_get_threads())
    for (int64_t y = ypix0; y < (int64_t)ypix1; ++y) {
        for (uint32_t x = 0; x < cfg->width; ++x) {
            uint32_t bin = (uint32_t)(y / cfg->bin_height) * tx + x / cfg->bin_width;
            uint32_t start = ranges[2 * bin], end = ranges[2 * bin + 1];
            uint32_t preend = start + ((end - start) / 64) * 64;
            float px = (float)x, py = (float)y; /* integer pixel coordinates (comp:56,61) */
            float C[3] = {0.0f, 0.0f, 0.0f};
            float T = 1.0f;
            int done = 0;
            for (uint32_t i = start; i < preend && !done; i += 64) {
                for (uint32_t j = 0; j < 64; ++j) {
                    const ko_gaussian2d* gg = &g[vals[i + j]];
                    float a = eval_gaussian(px, py, gg) * gg->alpha;
                    C[0] += gg->color[0] * a * T;
                    C[1] += gg->color[1] * a * T;
                    C[2] += gg->color[2] * a * T;
                    T *= (1.0f - a);
                    if (per_elem && T <= KO_T_MIN) { done = 1; break; }
                }
                if (T <= KO_T_MIN) break; /* comp:98: checked once per 64-batch */
            }
            /* comp:104-117: the tail loop runs even after an early exit above */
            if (!done)
                for (uint32_t i = preend; i < end; ++i) {
                    const ko_gaussian2d* gg = &g[vals[i]];
                    float a = eval_gaussian(px, py, gg) * gg->alpha;
                    C[0] += gg->color[0] * a * T;
                    C[1] += gg->color[1] * a * T;
                    C[2] += gg->color[2] * a * T;
                    T *= (1.0f - a);
                    if (T <= KO_T_MIN) break;
                }
            uint8_t* p = &rgba[((size_t)y * cfg->width + x) * 4];
            float w = 1.0f - T;
            float o[4];
            o[0] = (float)p[0] / 255.0f + C[0] * w;
            o[1] = (float)p[1] / 255.0f + C[1] * w;
            o[2] = (float)p[2] / 255.0f + C[2] * w;
            o[3] = (float)p[3] / 255.0f + 1.0f * w;
            for (int c = 0; c < 4; ++c) p[c] = (uint8_t)rintf(clamp01(o[c]) * 255.0f);
        }
    }
}

/* ------------------------------------------------------------ whole frame */

static uint32_t bits_for(uint64_t v) {
    uint32_t b = 0;
    while (b < 64 && (v >> b) != 0) ++b;
    return b;
}

uint64_t ko_render_projected(const ko_config* cfg, const ko_gaussian2d* g2d, uint64_t n,
                             uint8_t* rgba, uint64_t* keys_out, uint32_t* vals_out, uint64_t k_cap,
                             uint32_t* ranges_out) {
    uint32_t ntiles = ko_tiles_x(cfg) * ko_tiles_y(cfg);
    uint32_t* counts = (uint32_t*)malloc((n ? n : 1) * sizeof(uint32_t));
    uint64_t* offsets = (uint64_t*)malloc((n ? n : 1) * sizeof(uint64_t));
    if (!counts || !offsets) { free(counts); free(offsets); return UINT64_MAX; }
    ko_tile_counts(cfg, g2d, n, counts);
    uint64_t k = ko_exclusive_scan(counts, n, offsets);
    uint64_t* keys = (uint64_t*)malloc((k ? k : 1) * sizeof(uint64_t));
    uint32_t* vals = (uint32_t*)malloc((k ? k : 1) * sizeof(uint32_t));
    uint32_t* ranges = (uint32_t*)malloc((size_t)ntiles * 2 * sizeof(uint32_t));
    if (!keys || !vals || !ranges) {
        free(counts); free(offsets); free(keys); free(vals); free(ranges);
        return UINT64_MAX;
    }
    ko_emit_keys(cfg, g2d, n, offsets, keys, vals);
    ko_sort_pairs(keys, vals, k, 32 + bits_for(ntiles ? ntiles - 1 : 0));
    ko_tile_ranges(keys, k, ntiles, ranges);
    if (rgba) ko_rasterize(cfg, g2d, vals, ranges, rgba);
    if (keys_out && k <= k_cap) memcpy(keys_out, keys, k * sizeof(uint64_t));
    if (vals_out && k <= k_cap) memcpy(vals_out, vals, k * sizeof(uint32_t));
    if (ranges_out) memcpy(ranges_out, ranges, (size_t)ntiles * 2 * sizeof(uint32_t));
    free(counts); free(offsets); free(keys); free(vals); free(ranges);
    return k;
}

uint64_t ko_render_frame(const ko_config* cfg, const ko_camera* cam, const ko_gaussian3d* in,
                         uint64_t n, uint8_t* rgba, ko_gaussian2d* g2d_out, uint32_t* counts_out,
                         uint64_t* offsets_out, uint64_t* keys, uint32_t* vals, uint64_t k_cap,
                         uint32_t* ranges) {
    ko_gaussian2d* g2d = g2d_out ? g2d_out : (ko_gaussian2d*)malloc((n ? n : 1) * sizeof(ko_gaussian2d));
    if (!g2d) return UINT64_MAX;
    ko_project(cfg, cam, in, n, g2d);
    if (counts_out || offsets_out) {
        uint32_t* c = counts_out ? counts_out : (uint32_t*)malloc((n ? n : 1) * 4);
        uint64_t* o = offsets_out ? offsets_out : (uint64_t*)malloc((n ? n : 1) * 8);
        if (c && o) {
            ko_tile_counts(cfg, g2d, n, c);
            ko_exclusive_scan(c, n, o);
        }
        if (!counts_out) free(c);
        if (!offsets_out) free(o);
    }
    uint64_t k = ko_render_projected(cfg, g2d, n, rgba, keys, vals, k_cap, ranges);
    if (!g2d_out) free(g2d);
    return k;
}

/* -------------------------------------------------------- bin rectangles */

void ko_tile_rects(const ko_config* cfg, const ko_gaussian2d* g, uint64_t n, uint32_t* rects) {
#pragma omp parallel for schedule(static) num_threads(ko_get_threads())
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        uint32_t x0 = 0, x1 = 0, y0 = 0, y1 = 0;
        if (!(g[i].z < cfg->cull_z)) overlap_spans(cfg, &g[i], &x0, &x1, &y0, &y1);
        rects[4 * i] = x0;
        rects[4 * i + 1] = x1;
        rects[4 * i + 2] = y0;
        rects[4 * i + 3] = y1;
    }
}

/* ======================================================= double precision
 *
 * The same five stages with every float operation done in double: projection
 * (gsplat_projection.comp:37-237), bin rectangles (gsplat_binning.comp:53-81),
 * the order of the (bin, Gaussian) pairs (bin, then depth, ties by index:
 * gsplat_radix_sort_include.glsl:51-63 with the stable sort), and splatting with
 * the reference's exit rules (gsplat_binned_splatting.comp:41-125). The image
 * stays in double, unquantised, so that a float32 image's distance from it can
 * be measured. */

typedef struct { double m[3][3]; } dmat3;
typedef struct { double m[4][4]; } dmat4;

static dmat4 dmat4_load(const float* p) {
    dmat4 r;
    for (int c = 0; c < 4; ++c)
        for (int k = 0; k < 4; ++k) r.m[c][k] = (double)p[4 * c + k];
    return r;
}

static dmat4 dmat4_mul(dmat4 a, dmat4 b) {
    dmat4 r;
    for (int c = 0; c < 4; ++c)
        for (int k = 0; k < 4; ++k)
            r.m[c][k] = a.m[0][k] * b.m[c][0] + a.m[1][k] * b.m[c][1] + a.m[2][k] * b.m[c][2] +
                        a.m[3][k] * b.m[c][3];
    return r;
}

static void dmat4_vec(dmat4 a, const double v[4], double out[4]) {
    for (int k = 0; k < 4; ++k)
        out[k] = a.m[0][k] * v[0] + a.m[1][k] * v[1] + a.m[2][k] * v[2] + a.m[3][k] * v[3];
}

static dmat3 dmat3_mul(dmat3 a, dmat3 b) {
    dmat3 r;
    for (int c = 0; c < 3; ++c)
        for (int k = 0; k < 3; ++k)
            r.m[c][k] = a.m[0][k] * b.m[c][0] + a.m[1][k] * b.m[c][1] + a.m[2][k] * b.m[c][2];
    return r;
}

static dmat3 dmat3_transpose(dmat3 a) {
    dmat3 r;
    for (int c = 0; c < 3; ++c)
        for (int k = 0; k < 3; ++k) r.m[c][k] = a.m[k][c];
    return r;
}

static dmat3 dmat3_cols(double a, double b, double c, double d, double e, double f, double g, double h,
                        double i) {
    dmat3 r;
    r.m[0][0] = a; r.m[0][1] = b; r.m[0][2] = c;
    r.m[1][0] = d; r.m[1][1] = e; r.m[1][2] = f;
    r.m[2][0] = g; r.m[2][1] = h; r.m[2][2] = i;
    return r;
}

/* inverse of a column-major 2x2 given as (c00, c01, c10, c11) */
static void dmat2_inverse(const double a[4], double r[4]) {
    double det = a[0] * a[3] - a[2] * a[1];
    double inv = 1.0 / det;
    r[0] = a[3] * inv;
    r[1] = -a[1] * inv;
    r[2] = -a[2] * inv;
    r[3] = a[0] * inv;
}

static double dsh_color(double base, const float coeffs[15], const double dir[3], int deg) {
    double x = dir[0], y = dir[1], z = dir[2];
    double x2 = x * x, y2 = y * y, z2 = z * z;
    double sh[16];
    sh[0] = 0.282095;
    sh[1] = -0.488603 * y;
    sh[2] = -0.488603 * z;
    sh[3] = -0.488603 * x;
    sh[4] = 1.092548 * x * y;
    sh[5] = -1.092548 * y * z;
    sh[6] = 0.315392 * (2.0 * z2 - x2 - y2);
    sh[7] = -1.092548 * x * z;
    sh[8] = 0.546274 * (x2 - y2);
    sh[9] = -0.590044 * y * (3.0 * x2 - y2);
    sh[10] = 2.890611 * x * y * z;
    sh[11] = -0.457046 * y * (4.0 * z2 - x2 - y2);
    sh[12] = 0.373176 * z * (2.0 * z2 - 3.0 * x2 - 3.0 * y2);
    sh[13] = -0.457046 * x * (4.0 * z2 - x2 - y2);
    sh[14] = 1.445306 * z * (x2 - y2);
    sh[15] = -0.590044 * x * (x2 - 3.0 * y2);
    int ncoef = (deg + 1) * (deg + 1) - 1;
    double value = 0.5 + base * sh[0];
    for (int i = 0; i < ncoef; i++) value += (double)coeffs[i] * sh[i + 1];
    return value;
}

void ko_project_f64(const ko_config* cfg, const ko_camera* cam, const ko_gaussian3d* in, uint64_t n,
                    ko_gaussian2d_f64* out) {
    dmat4 model = dmat4_load(cam->model), view = dmat4_load(cam->view), proj = dmat4_load(cam->proj);
    dmat4 pvm = dmat4_mul(dmat4_mul(proj, view), model);
    dmat4 mv = dmat4_mul(model, view);
    const double half_w = (double)cfg->width * 0.5, half_h = (double)cfg->height * 0.5;
    const double sxx = (double)cfg->width * cfg->width, syy = (double)cfg->height * cfg->height;
    const double sxy = (double)cfg->width * cfg->height;
    const int deg = cfg->sh_degree < 0 ? 3 : cfg->sh_degree;
    const double focalX = proj.m[0][0], focalY = proj.m[1][1];
    const double limx = 1.3 * (1.0 / focalX), limy = 1.3 * (1.0 / focalY);
#pragma omp parallel for schedule(static) num_threads(ko_get_threads())
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        const ko_gaussian3d* g = &in[i];
        double p4[4] = {g->position[0], g->position[1], g->position[2], 1.0};
        double pos[4], t4[4];
        dmat4_vec(pvm, p4, pos);
        dmat4_vec(mv, p4, t4);
        ko_gaussian2d_f64 o;
        o.position[0] = (pos[0] / pos[3] + 1.0) * half_w;
        o.position[1] = (pos[1] / pos[3] + 1.0) * half_h;
        o.z = pos[2];
        /* calculateCovarianceMatrix2D (comp:53-118) */
        double qx = g->rotation[0], qy = g->rotation[1], qz = g->rotation[2], qw = g->rotation[3];
        dmat3 R = dmat3_cols(1.0 - 2.0 * (qy * qy + qz * qz), 2.0 * (qx * qy - qw * qz), 2.0 * (qx * qz + qw * qy),
                             2.0 * (qx * qy + qw * qz), 1.0 - 2.0 * (qx * qx + qz * qz), 2.0 * (qy * qz - qw * qx),
                             2.0 * (qx * qz - qw * qy), 2.0 * (qy * qz + qw * qx), 1.0 - 2.0 * (qx * qx + qy * qy));
        dmat3 S = dmat3_cols(g->scale[0], 0, 0, 0, g->scale[1], 0, 0, 0, g->scale[2]);
        dmat3 M = dmat3_mul(S, R);
        dmat3 cov3d = dmat3_mul(dmat3_transpose(M), M);
        double tx = t4[0], ty = t4[1], tz = t4[2];
        double txtz = tx / tz, tytz = ty / tz;
        tx = fmin(limx, fmax(-limx, txtz)) * tz;
        ty = fmax(limy, fmin(-limy, tytz)) * tz; /* the shader's clamp of t.y, kept as written */
        dmat3 J = dmat3_cols(focalX / tz, 0.0, -(focalX * tx) / (tz * tz),
                             0.0, focalY / tz, -(focalY * ty) / (tz * tz),
                             0.0, 0.0, 0.0);
        dmat3 W = dmat3_cols(mv.m[0][0], mv.m[1][0], mv.m[2][0],
                             mv.m[0][1], mv.m[1][1], mv.m[2][1],
                             mv.m[0][2], mv.m[1][2], mv.m[2][2]);
        dmat3 T = dmat3_mul(W, J);
        dmat3 cov = dmat3_mul(dmat3_mul(dmat3_transpose(T), dmat3_transpose(cov3d)), T);
        double c2[4] = {cov.m[0][0] * sxx + 0.3, cov.m[0][1] * sxy, cov.m[1][0] * sxy, cov.m[1][1] * syy + 0.3};
        dmat2_inverse(c2, o.covInv);
        double len = sqrt(t4[0] * t4[0] + t4[1] * t4[1] + t4[2] * t4[2]);
        double dir[3] = {t4[0] / len, t4[1] / len, t4[2] / len};
        o.color[0] = dsh_color(g->color[0], g->shR, dir, deg);
        o.color[1] = dsh_color(g->color[1], g->shG, dir, deg);
        o.color[2] = dsh_color(g->color[2], g->shB, dir, deg);
        o.alpha = g->alpha;
        out[i] = o;
    }
}

/* bins met by a double record, as overlap_spans: a closed-interval test per column and row */
static void overlap_spans_f64(const ko_config* cfg, const ko_gaussian2d_f64* g, uint32_t r[4]) {
    double cov[4];
    dmat2_inverse(g->covInv, cov);
    double sx = sqrt(cov[0]) * 2.5, sy = sqrt(cov[3]) * 2.5;
    double mn[2] = {g->position[0] - sx, g->position[1] - sy};
    double mx[2] = {g->position[0] + sx, g->position[1] + sy};
    uint32_t tx = ko_tiles_x(cfg), rb, re;
    row_span(cfg, &rb, &re);
    double cw = cfg->bin_width, ch = cfg->bin_height;
    uint32_t a = tx, b = 0, c = re, d = rb;
    for (uint32_t gx = 0; gx < tx; ++gx)
        if (!(mx[0] < gx * cw || mn[0] > (gx + 1) * cw)) {
            if (a == tx) a = gx;
            b = gx + 1;
        }
    for (uint32_t gy = rb; gy < re; ++gy)
        if (!(mx[1] < gy * ch || mn[1] > (gy + 1) * ch)) {
            if (c == re) c = gy;
            d = gy + 1;
        }
    if (a >= b || c >= d) a = b = c = d = 0;
    r[0] = a; r[1] = b; r[2] = c; r[3] = d;
}

typedef struct { double z; uint32_t idx; } ko_depth_item;

static int cmp_depth(const void* pa, const void* pb) {
    const ko_depth_item* a = (const ko_depth_item*)pa;
    const ko_depth_item* b = (const ko_depth_item*)pb;
    if (a->z < b->z) return -1;
    if (a->z > b->z) return 1;
    return a->idx < b->idx ? -1 : (a->idx > b->idx);
}

uint64_t ko_render_frame_f64(const ko_config* cfg, const ko_camera* cam, const ko_gaussian3d* in,
                             uint64_t n, const uint8_t* rgba_in, double* rgba_out) {
    uint32_t tx = ko_tiles_x(cfg), ntiles = tx * ko_tiles_y(cfg), rb, re;
    row_span(cfg, &rb, &re);
    ko_gaussian2d_f64* g = (ko_gaussian2d_f64*)malloc((n ? n : 1) * sizeof(ko_gaussian2d_f64));
    uint32_t* rect = (uint32_t*)malloc((n ? n : 1) * 4 * sizeof(uint32_t));
    ko_depth_item* order = (ko_depth_item*)malloc((n ? n : 1) * sizeof(ko_depth_item));
    uint64_t* start = (uint64_t*)calloc((size_t)ntiles + 1, sizeof(uint64_t));
    if (!g || !rect || !order || !start) {
        free(g); free(rect); free(order); free(start);
        return UINT64_MAX;
    }
    ko_project_f64(cfg, cam, in, n, g);
#pragma omp parallel for schedule(static) num_threads(ko_get_threads())
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        uint32_t* r = &rect[4 * i];
        r[0] = r[1] = r[2] = r[3] = 0;
        if (!(g[i].z < (double)cfg->cull_z)) overlap_spans_f64(cfg, &g[i], r);
    }
    /* pairs by bin, then depth (ties by index): a stable counting sort of the Gaussians in
     * depth order */
    uint64_t nv = 0;
    for (uint64_t i = 0; i < n; ++i) {
        const uint32_t* r = &rect[4 * i];
        if (r[1] <= r[0] || r[3] <= r[2]) continue;
        order[nv].z = g[i].z;
        order[nv].idx = (uint32_t)i;
        ++nv;
        for (uint32_t y = r[2]; y < r[3]; ++y)
            for (uint32_t x = r[0]; x < r[1]; ++x) start[(uint64_t)y * tx + x + 1]++;
    }
    qsort(order, nv, sizeof(ko_depth_item), cmp_depth);
    for (uint32_t b = 0; b < ntiles; ++b) start[b + 1] += start[b];
    uint64_t k = start[ntiles];
    uint32_t* vals = (uint32_t*)malloc((k ? k : 1) * sizeof(uint32_t));
    uint64_t* cur = (uint64_t*)malloc((size_t)ntiles * sizeof(uint64_t));
    if (!vals || !cur) {
        free(g); free(rect); free(order); free(start); free(vals); free(cur);
        return UINT64_MAX;
    }
    memcpy(cur, start, (size_t)ntiles * sizeof(uint64_t));
    for (uint64_t q = 0; q < nv; ++q) {
        const uint32_t* r = &rect[4 * order[q].idx];
        for (uint32_t y = r[2]; y < r[3]; ++y)
            for (uint32_t x = r[0]; x < r[1]; ++x) vals[cur[(uint64_t)y * tx + x]++] = order[q].idx;
    }
    const double tmin = 1.0 - 0.9999;
    const int per_elem = cfg->exit_per_element != 0;
    uint32_t ypix0 = rb * cfg->bin_height, ypix1 = re * cfg->bin_height;
    if (ypix1 > cfg->height) ypix1 = cfg->height;
#pragma omp parallel for schedule(dynamic, 1) num_threads(ko_get_threads())
    for (int64_t y = 0; y < (int64_t)cfg->height; ++y) {
        for (uint32_t x = 0; x < cfg->width; ++x) {
            const uint8_t* p = &rgba_in[((size_t)y * cfg->width + x) * 4];
            double* o = &rgba_out[((size_t)y * cfg->width + x) * 4];
            if (y < (int64_t)ypix0 || y >= (int64_t)ypix1) { /* rows outside the band: untouched */
                for (int c = 0; c < 4; ++c) o[c] = p[c] / 255.0;
                continue;
            }
            uint32_t bin = (uint32_t)(y / cfg->bin_height) * tx + x / cfg->bin_width;
            uint64_t s0 = start[bin], s1 = start[bin + 1];
            uint64_t preend = s0 + ((s1 - s0) / 64) * 64;
            double C[3] = {0, 0, 0}, T = 1.0;
            int done = 0;
            for (uint64_t i = s0; i < s1; ++i) {
                const ko_gaussian2d_f64* gg = &g[vals[i]];
                double dx = (double)x - gg->position[0], dy = (double)y - gg->position[1];
                double sx = gg->covInv[0] * dx + gg->covInv[2] * dy;
                double sy = gg->covInv[1] * dx + gg->covInv[3] * dy;
                double a = exp(-0.5 * (dx * sx + dy * sy)) * gg->alpha;
                for (int c = 0; c < 3; ++c) C[c] += gg->color[c] * a * T;
                T *= (1.0 - a);
                if (per_elem || i >= preend) {
                    if (T <= tmin) { done = 1; break; }
                } else if ((i + 1 - s0) % 64 == 0 && T <= tmin) {
                    /* batch-end exit (comp:98); the tail loop (comp:104-117) still runs */
                    i = preend - 1;
                    if (preend == s1) { done = 1; break; }
                }
            }
            (void)done;
            double w = 1.0 - T;
            for (int c = 0; c < 3; ++c) {
                double v = p[c] / 255.0 + C[c] * w;
                o[c] = v < 0 ? 0 : (v > 1 ? 1 : v);
            }
            double v = p[3] / 255.0 + w;
            o[3] = v < 0 ? 0 : (v > 1 ? 1 : v);
        }
    }
    free(g); free(rect); free(order); free(start); free(vals); free(cur);
    return k;
}
