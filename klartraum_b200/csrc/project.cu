// K1: projection + SH colour + bin-overlap count, one thread per Gaussian.
//
// Restates shaders/gsplat/gsplat_projection.comp:37-237 (projection) and the overlap test of
// shaders/gsplat/gsplat_binning.comp:53-81,112-147 (counted here instead of duplicated with
// atomics). This file is compiled with -fmad=false and IEEE division / square root, so every
// float result is the correctly rounded value of the shader's own operation sequence.
//
// Roofline: HBM bound. Per Gaussian it reads the geometry planes (48 B) and its SH planes (16 B
// per float4 plane: 192 B at SH3), loaded together up front; it writes 48 B record + 4 B count +
// 8 B rect + 4 B depth. The colour of a Gaussian that meets no bin is stored as 0 (the reference
// computes it but no later stage reads it).
#include "kt_common.cuh"
#include "kt_kernels.h"

namespace kt {
namespace {

// ---------------------------------------------------------------- matrix helpers
// Column-major m[4*c + r] (mat4) and m[3*c + r] (mat3); products sum k = 0.. in order.

__device__ __forceinline__ void mat4_vec(const float* m, float x, float y, float z, float w,
                                         float out[4]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) out[k] = m[k] * x + m[4 + k] * y + m[8 + k] * z + m[12 + k] * w;
}

__device__ __forceinline__ void mat3_mul(const float* a, const float* b, float* r) {
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int k = 0; k < 3; ++k)
            r[3 * c + k] = a[k] * b[3 * c] + a[3 + k] * b[3 * c + 1] + a[6 + k] * b[3 * c + 2];
}

__device__ __forceinline__ void mat3_transpose(const float* a, float* r) {
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int k = 0; k < 3; ++k) r[3 * c + k] = a[3 * k + c];
}

// inverse(mat2) as adjugate * (1/det); a = {[0][0], [0][1], [1][0], [1][1]}
__device__ __forceinline__ void mat2_inverse(const float a[4], float r[4]) {
    float det = a[0] * a[3] - a[2] * a[1];
    float inv = 1.0f / det;
    r[0] = a[3] * inv;
    r[1] = -a[1] * inv;
    r[2] = -a[2] * inv;
    r[3] = a[0] * inv;
}

// --------------------------------------------------------------- bin overlap spans
// gsplat_binning.comp:78-80: a bin overlaps iff !(gmax < binMin || gmin > binMax) on both
// axes, binMin = float(i) * cell, binMax = float(i + 1) * cell. Along one axis the bins that
// pass form one run [lo, hi); it is found from a floor() estimate and corrected with the exact
// comparisons, so it equals testing every bin.

__device__ __forceinline__ bool right_of_min(float mn, int i, float cell) {
    return !(mn > (float)(i + 1) * cell);
}
__device__ __forceinline__ bool left_of_max(float mx, int i, float cell) {
    return !(mx < (float)i * cell);
}

// `inv_cell` (1 / cell, rounded) only seeds the search: the exact comparisons that follow move the
// run's ends to the bins that pass whatever the estimate, so no division is needed.
__device__ __forceinline__ void axis_span(float mn, float mx, float cell, float inv_cell, int n, int& lo,
                                          int& hi) {
    float e = floorf(mn * inv_cell) - 1.0f;
    int l = !(e > 0.0f) ? 0 : (e > (float)n ? n : (int)e);
    while (l > 0 && right_of_min(mn, l - 1, cell)) --l;
    while (l < n && !right_of_min(mn, l, cell)) ++l;
    float f = floorf(mx * inv_cell);
    int h = (mx != mx) ? n - 1 : (!(f > -1.0f) ? -1 : (f > (float)(n - 1) ? n - 1 : (int)f));
    while (h < n - 1 && left_of_max(mx, h + 1, cell)) ++h;
    while (h >= 0 && !left_of_max(mx, h, cell)) --h;
    lo = l;
    hi = h + 1;
}

// Count and rectangle of bins overlapped by a projected Gaussian (0 if culled by z).
__device__ __forceinline__ uint32_t bin_span(float px, float py, float z, const float ci[4],
                                             const GridParams& gp, uint2& rect) {
    rect = make_uint2(0u, 0u);
    if (z < gp.cull_z) return 0u;  // gsplat_binning.comp:113
    float cov[4];
    mat2_inverse(ci, cov);  // comp:69
    float spreadX = sqrtf(cov[0]) * 2.5f;
    float spreadY = sqrtf(cov[3]) * 2.5f;
    float mnx = px - spreadX, mny = py - spreadY;
    float mxx = px + spreadX, mxy = py + spreadY;
    int x0, x1, y0, y1;
    axis_span(mnx, mxx, gp.cell_w, gp.inv_cell_w, (int)gp.tiles_x, x0, x1);
    axis_span(mny, mxy, gp.cell_h, gp.inv_cell_h, (int)gp.tiles_y, y0, y1);
    y0 = max(y0, (int)gp.row_begin);
    y1 = min(y1, (int)gp.row_end);
    if (x1 <= x0 || y1 <= y0) return 0u;
    rect = make_uint2((uint32_t)x0 | ((uint32_t)x1 << 16), (uint32_t)y0 | ((uint32_t)y1 << 16));
    return (uint32_t)(x1 - x0) * (uint32_t)(y1 - y0);
}

// Block-wide min/max of the depth bits of counted Gaussians, their number and their bin count.
__device__ __forceinline__ void reduce_depth(uint32_t count, uint32_t flip, FrameCtl* ctl) {
    __shared__ uint32_t s_min[32], s_max[32];
    __shared__ unsigned long long s_sum[32];
    const bool counted = count > 0u;
    uint32_t dmin = counted ? flip : 0xFFFFFFFFu;
    uint32_t dmax = counted ? flip : 0u;
    dmin = __reduce_min_sync(0xFFFFFFFFu, dmin);
    dmax = __reduce_max_sync(0xFFFFFFFFu, dmax);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned long long sum = count;
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    if (lane == 0) {
        s_min[warp] = dmin;
        s_max[warp] = dmax;
        s_sum[warp] = sum;
    }
    int vis = __syncthreads_count(counted);
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        dmin = lane < nw ? s_min[lane] : 0xFFFFFFFFu;
        dmax = lane < nw ? s_max[lane] : 0u;
        dmin = __reduce_min_sync(0xFFFFFFFFu, dmin);
        dmax = __reduce_max_sync(0xFFFFFFFFu, dmax);
        sum = lane < nw ? s_sum[lane] : 0ull;
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
        if (lane == 0 && vis > 0) {
            atomicMin(&ctl->depth_min, dmin);
            atomicMax(&ctl->depth_max, dmax);
            atomicAdd(&ctl->num_visible, (unsigned)vis);
            atomicAdd(&ctl->pair_total, sum);
        }
    }
}

__device__ __forceinline__ void store_outputs(uint64_t i, float px, float py, float z,
                                              const float ci[4], float r, float g, float b,
                                              float alpha, uint32_t count, uint2 rect,
                                              const FrameBufs& fb) {
    fb.rec[3 * i + 0] = make_float4(px, py, alpha, z);
    fb.rec[3 * i + 1] = make_float4(ci[0], ci[1], ci[2], ci[3]);
    fb.rec[3 * i + 2] = make_float4(r, g, b, 0.0f);
    fb.counts[i] = count;
    fb.rect[i] = rect;
    fb.depth[i] = __float_as_uint(z) ^ 0x80000000u;
}

// --------------------------------------------------------------------- K1

template <int DEG>
__global__ void __launch_bounds__(256, 3) k_project_count(SceneDev sc, CamParams cam, GridParams gp, FrameBufs fb) {
    constexpr int kCoef = (DEG + 1) * (DEG + 1);
    constexpr int kPlanes = (3 * kCoef + 3) / 4;
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = i < sc.n;
    uint32_t count = 0, flip = 0;
    if (live) {
        const float4 P = __ldg(&sc.pos[i]);
        const float4 Q = __ldg(&sc.rot[i]);
        const float4 S = __ldg(&sc.scale[i]);
        float f[4 * kPlanes];
#pragma unroll
        for (int p = 0; p < kPlanes; ++p) {
            const float4 v = __ldg(&sc.sh[(uint64_t)p * sc.n + i]);
            f[4 * p + 0] = v.x;
            f[4 * p + 1] = v.y;
            f[4 * p + 2] = v.z;
            f[4 * p + 3] = v.w;
        }

        // comp:198-203: clip position, pixel position, depth
        float pos[4];
        mat4_vec(cam.pvm, P.x, P.y, P.z, 1.0f, pos);
        const float nx = pos[0] / pos[3];
        const float ny = pos[1] / pos[3];
        const float px = (nx + 1.0f) * gp.half_w;
        const float py = (ny + 1.0f) * gp.half_h;
        const float z = pos[2];

        // comp:53-118: 2D covariance
        float Sm[9] = {S.x, 0.0f, 0.0f, 0.0f, S.y, 0.0f, 0.0f, 0.0f, S.z};
        float R[9];
        {
            const float x = Q.x, y = Q.y, zq = Q.z, w = Q.w;
            const float xx = x * x, yy = y * y, zz = zq * zq;
            const float xy = x * y, xz = x * zq, yz = y * zq;
            const float wx = w * x, wy = w * y, wz = w * zq;
            R[0] = 1.0f - 2.0f * (yy + zz);
            R[1] = 2.0f * (xy - wz);
            R[2] = 2.0f * (xz + wy);
            R[3] = 2.0f * (xy + wz);
            R[4] = 1.0f - 2.0f * (xx + zz);
            R[5] = 2.0f * (yz - wx);
            R[6] = 2.0f * (xz - wy);
            R[7] = 2.0f * (yz + wx);
            R[8] = 1.0f - 2.0f * (xx + yy);
        }
        float M[9], Mt[9], cov3[9];
        mat3_mul(Sm, R, M);
        mat3_transpose(M, Mt);
        mat3_mul(Mt, M, cov3);

        float t4[4];
        mat4_vec(cam.mv, P.x, P.y, P.z, 1.0f, t4);
        float tx = t4[0], ty = t4[1];
        const float tz = t4[2];
        const float focalX = cam.focal_x, focalY = cam.focal_y;
        // tanFov = 1 / focal and lim = 1.3 * tanFov are the same for every Gaussian: the host
        // computes them once with the same float operations
        const float limx = cam.lim_x;
        const float limy = cam.lim_y;
        const float txtz = tx / tz;
        const float tytz = ty / tz;
        tx = fminf(limx, fmaxf(-limx, txtz)) * tz;
        ty = fmaxf(limy, fminf(-limy, tytz)) * tz;

        const float J[9] = {focalX / tz, 0.0f, -(focalX * tx) / (tz * tz),
                            0.0f, focalY / tz, -(focalY * ty) / (tz * tz),
                            0.0f, 0.0f, 0.0f};
        const float* mv = cam.mv;
        const float W[9] = {mv[0], mv[4], mv[8], mv[1], mv[5], mv[9], mv[2], mv[6], mv[10]};
        float T[9], Tt[9], cov3t[9], A[9], C[9];
        mat3_mul(W, J, T);
        mat3_transpose(T, Tt);
        mat3_transpose(cov3, cov3t);
        mat3_mul(Tt, cov3t, A);
        mat3_mul(A, T, C);
        float cov[4] = {C[0], C[1], C[3], C[4]};
        cov[0] *= gp.sxx;
        cov[1] *= gp.sxy;
        cov[2] *= gp.sxy;
        cov[3] *= gp.syy;
        cov[0] += 0.3f;
        cov[3] += 0.3f;
        float ci[4];
        mat2_inverse(cov, ci);

        uint2 rect;
        count = bin_span(px, py, z, ci, gp, rect);
        flip = __float_as_uint(z) ^ 0x80000000u;
        // comp:218-224: view direction and SH colour, for Gaussians that meet a bin: no later
        // stage reads the colour of the others (stored as 0)
        float rgb[3] = {0.0f, 0.0f, 0.0f};
        if (count != 0u) {
        const float len = sqrtf(t4[0] * t4[0] + t4[1] * t4[1] + t4[2] * t4[2]);
        const float dx = t4[0] / len, dy = t4[1] / len, dz = t4[2] / len;
        float sh[16];
        {
            const float x = dx, y = dy, zz = dz;
            const float x2 = x * x, y2 = y * y, z2 = zz * zz;
            sh[0] = 0.282095f;
            sh[1] = -0.488603f * y;
            sh[2] = -0.488603f * zz;
            sh[3] = -0.488603f * x;
            sh[4] = 1.092548f * x * y;
            sh[5] = -1.092548f * y * zz;
            sh[6] = 0.315392f * (2.0f * z2 - x2 - y2);
            sh[7] = -1.092548f * x * zz;
            sh[8] = 0.546274f * (x2 - y2);
            sh[9] = -0.590044f * y * (3.0f * x2 - y2);
            sh[10] = 2.890611f * x * y * zz;
            sh[11] = -0.457046f * y * (4.0f * z2 - x2 - y2);
            sh[12] = 0.373176f * zz * (2.0f * z2 - 3.0f * x2 - 3.0f * y2);
            sh[13] = -0.457046f * x * (4.0f * z2 - x2 - y2);
            sh[14] = 1.445306f * zz * (x2 - y2);
            sh[15] = -0.590044f * x * (x2 - 3.0f * y2);
        }
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) {
            float value = 0.5f + f[ch] * sh[0];
#pragma unroll
            for (int k = 1; k < kCoef; ++k) value += f[3 * k + ch] * sh[k];
            rgb[ch] = value;
        }
        }
        // Every record is written, also for a Gaussian that meets no bin of the binned rows: leaving
        // those out (a band of a banded frame) made the warps' interleaved 48-B record stores partial
        // and the kernel slower (290 against 277 us on a half-screen band of the 6M frame).
        store_outputs(i, px, py, z, ci, rgb[0], rgb[1], rgb[2], P.w, count, rect, fb);
    }
    reduce_depth(count, flip, fb.ctl);
}

// Projected records supplied by the caller (kt_gaussian2d layout) -> internal buffers.
__global__ void __launch_bounds__(256) k_load_projected(const float* __restrict__ g2d, uint64_t n,
                                                         GridParams gp, FrameBufs fb) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    uint32_t count = 0, flip = 0;
    if (i < n) {
        const float* g = g2d + 12 * i;
        const float px = g[0], py = g[1], z = g[2];
        const float ci[4] = {g[4], g[5], g[6], g[7]};
        uint2 rect;
        count = bin_span(px, py, z, ci, gp, rect);
        flip = __float_as_uint(z) ^ 0x80000000u;
        store_outputs(i, px, py, z, ci, g[8], g[9], g[10], g[11], count, rect, fb);
    }
    reduce_depth(count, flip, fb.ctl);
}

// Array-of-structs Gaussian3D (59 floats) -> device planes.
__global__ void __launch_bounds__(256) k_pack_scene(const float* __restrict__ aos, uint64_t n,
                                                     float4* pos, float4* rot, float4* scale,
                                                     float4* sh, int deg, uint32_t nplanes) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* g = aos + 59 * i;
    pos[i] = make_float4(g[0], g[1], g[2], g[13]);
    rot[i] = make_float4(g[3], g[4], g[5], g[6]);
    scale[i] = make_float4(g[7], g[8], g[9], 0.0f);
    const int ncoef = (deg + 1) * (deg + 1);
    for (uint32_t p = 0; p < nplanes; ++p) {
        float v[4];
        for (int q = 0; q < 4; ++q) {
            const int idx = 4 * (int)p + q;  // interleaved coefficient index 3k + ch
            const int k = idx / 3, ch = idx % 3;
            float x = 0.0f;
            if (k < ncoef) x = (k == 0) ? g[10 + ch] : g[14 + 15 * ch + (k - 1)];
            v[q] = x;
        }
        sh[(uint64_t)p * n + i] = make_float4(v[0], v[1], v[2], v[3]);
    }
}

}  // namespace

// ------------------------------------------------------------------ launchers

cudaError_t launch_project_count(const SceneDev& sc, const CamParams& cam, const GridParams& gp, const FrameBufs& fb,
                                 cudaStream_t stream) {
    if (sc.n == 0) return cudaSuccess;
    const dim3 grid((unsigned)((sc.n + 255) / 256));
    switch (sc.deg) {
        case 0: k_project_count<0><<<grid, 256, 0, stream>>>(sc, cam, gp, fb); break;
        case 1: k_project_count<1><<<grid, 256, 0, stream>>>(sc, cam, gp, fb); break;
        case 2: k_project_count<2><<<grid, 256, 0, stream>>>(sc, cam, gp, fb); break;
        default: k_project_count<3><<<grid, 256, 0, stream>>>(sc, cam, gp, fb); break;
    }
    return cudaGetLastError();
}

const void* project_count_kernel(int deg) {
    switch (deg) {
        case 0: return reinterpret_cast<const void*>(&k_project_count<0>);
        case 1: return reinterpret_cast<const void*>(&k_project_count<1>);
        case 2: return reinterpret_cast<const void*>(&k_project_count<2>);
        default: return reinterpret_cast<const void*>(&k_project_count<3>);
    }
}

cudaError_t launch_load_projected(const float* d_g2d, uint64_t n, const GridParams& gp,
                                  const FrameBufs& fb, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_load_projected<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(d_g2d, n, gp, fb);
    return cudaGetLastError();
}

cudaError_t launch_pack_scene(const float* d_aos, uint64_t n, float4* pos, float4* rot,
                              float4* scale, float4* sh, int deg, uint32_t nplanes,
                              cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    k_pack_scene<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(d_aos, n, pos, rot, scale, sh,
                                                                   deg, nplanes);
    return cudaGetLastError();
}

}  // namespace kt
