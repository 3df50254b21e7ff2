// K6: front-to-back splatting, one CTA per 16x16 pixel block, two pixels per thread.
//
// Restates shaders/gsplat/gsplat_binned_splatting.comp:41-125 per pixel:
//   a = exp(-0.5 * dot(d, covInv * d)) * alpha, d = pixel - mean (integer pixel coordinates)
//   C += color * a * T;  T *= 1 - a
//   out = clamp(in + vec4(C, 1) * (1 - T), 0, 1) stored as RGBA8 (read-modify-write).
// A pixel stops once T <= 1 - 0.9999, tested (reference mode) only at the end of each
// 64-Gaussian batch counted from the bin's start; after such a stop the reference's tail
// loop still blends the first element past the last full batch (comp:104-117). With
// KT_GS_FLAG_EXIT_PER_ELEMENT the test runs after every Gaussian.
//
// The CTA stages 128 sorted Gaussians at a time in shared memory (each thread gathers one
// 48-B record by index) and leaves the list as soon as every pixel of the block is done or
// only owes the reference's one tail element, which it then blends from global memory.
#include "kt_common.cuh"
#include "kt_kernels.h"

namespace kt {
namespace {

constexpr int kRasterThreads = 128;  // two pixels per thread
constexpr int kBatch = 128;

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// One blend step: a = exp(-0.5 * dot(d, covInv d)) * alpha; C += color * a * T; T *= 1 - a.
// `q` = (A, B, C, alpha) with A = covInv[0][0] * k, B = (covInv[0][1] + covInv[1][0]) * k,
// C = covInv[1][1] * k and k = -0.5 * log2(e), so the exponent is one quadratic form and the
// exponential one exp2: power = (A dx) dx + (C dy + B dx) dy. The dx terms (`Xterms`) depend on
// the pixel column only and are shared by the two pixels of a thread. `cola` is color * alpha;
// with u = exp2(power) * T the step is C += cola * u, T -= alpha * u.
struct Xterms {
    float adx2, bdx;
};

__device__ __forceinline__ Xterms xterms(float fx, float2 mean, const float4& q) {
    const float dx = fx - mean.x;
    return Xterms{(q.x * dx) * dx, q.y * dx};
}

__device__ __forceinline__ void blend_y(const Xterms& xt, float fy, float2 mean, const float4& q, const float4& cola,
                                        float& C0, float& C1, float& C2, float& T) {
    const float dy = fy - mean.y;
    const float power = fmaf(fmaf(q.z, dy, xt.bdx), dy, xt.adx2);
    const float u = ex2_approx(power) * T;
    C0 = fmaf(cola.x, u, C0);
    C1 = fmaf(cola.y, u, C1);
    C2 = fmaf(cola.z, u, C2);
    T = fmaf(-q.w, u, T);
}

__device__ __forceinline__ void blend(float fx, float fy, float2 mean, const float4& q, const float4& cola,
                                      float& C0, float& C1, float& C2, float& T) {
    blend_y(xterms(fx, mean, q), fy, mean, q, cola, C0, C1, C2, T);
}

// A record's colour times its alpha.
__device__ __forceinline__ float4 color_alpha(float4 col, float alpha) {
    return make_float4(col.x * alpha, col.y * alpha, col.z * alpha, 0.0f);
}

__device__ __forceinline__ float4 quad_form(float4 cov, float alpha) {
    const float k = -0.5f * 1.44269504088896340736f;  // -0.5 * log2(e)
    return make_float4(cov.x * k, (cov.y + cov.z) * k, cov.w * k, alpha);
}

// One pixel's blend state.
struct Pix {
    float C0, C1, C2, T;
    bool done;       // finished (T below the threshold, or outside the image)
    bool wait_tail;  // stopped at a 64-batch end; owes the reference's one tail element
};

__device__ __forceinline__ void write_pixel(uchar4* img, const GridParams& gp, uint32_t px, uint32_t py,
                                            const Pix& p) {
    uchar4* pix = &img[(uint64_t)py * gp.width + px];
    const uchar4 in = *pix;
    const float w = 1.0f - p.T;
    float o0 = (float)in.x / 255.0f + p.C0 * w;
    float o1 = (float)in.y / 255.0f + p.C1 * w;
    float o2 = (float)in.z / 255.0f + p.C2 * w;
    float o3 = (float)in.w / 255.0f + 1.0f * w;
    o0 = fminf(fmaxf(o0, 0.0f), 1.0f);
    o1 = fminf(fmaxf(o1, 0.0f), 1.0f);
    o2 = fminf(fmaxf(o2, 0.0f), 1.0f);
    o3 = fminf(fmaxf(o3, 0.0f), 1.0f);
    *pix = make_uchar4((unsigned char)__float2uint_rn(o0 * 255.0f), (unsigned char)__float2uint_rn(o1 * 255.0f),
                       (unsigned char)__float2uint_rn(o2 * 255.0f), (unsigned char)__float2uint_rn(o3 * 255.0f));
}

// The reference's tail loop from `preend` for a pixel that stopped at a 64-batch end: one element
// unless that element raised T again.
template <typename IndexAt>
__device__ __forceinline__ void blend_tail(const float4* __restrict__ rec, IndexAt index_at, uint32_t preend,
                                           uint32_t end, float fx, float fy, float tmin, Pix& p) {
    for (uint32_t i = preend; i < end; ++i) {
        const uint32_t idx = index_at(i);
        const float4 g = rec[3 * (uint64_t)idx + 0];
        blend(fx, fy, make_float2(g.x, g.y), quad_form(rec[3 * (uint64_t)idx + 1], g.z),
              color_alpha(rec[3 * (uint64_t)idx + 2], g.z),
              p.C0, p.C1, p.C2, p.T);
        if (p.T <= tmin) break;
    }
}

// Each thread shades two pixels of the 16x16 block, rows y and y + 8 of one column, so every
// staged Gaussian read from shared memory serves both.
// Ten resident CTAs (40 warps) per SM: the register budget drops from 61 to 48 per thread (a few
// spilled bytes outside the blend loop) and more warps hide the staging batches' gathers. Measured on
// one B200: 134 against 143 us on the 1M frame, 437 against 507 us on the 6M frame; twelve CTAs
// (40 registers) were no better.
#ifndef KT_RASTER_MIN_CTAS
#define KT_RASTER_MIN_CTAS 10
#endif

template <bool PER_ELEM>
__global__ void __launch_bounds__(kRasterThreads, KT_RASTER_MIN_CTAS)
k_rasterize(const float4* __restrict__ rec, SortIO io, const uint2* __restrict__ ranges,
            const FrameCtl* __restrict__ ctl, GridParams gp, uchar4* __restrict__ img,
            uint32_t ypix0) {
    __shared__ float2 s_mean[kBatch];  // px, py
    __shared__ float4 s_q[kBatch];     // quadratic form, alpha
    __shared__ float4 s_col[kBatch];   // r, g, b times alpha
    if (!ctl->plan_ok) return;

    const int tid = threadIdx.x;
    const uint32_t bx0 = blockIdx.x * 16, by0 = ypix0 + blockIdx.y * 16;
    const uint32_t px = bx0 + (tid & 15), py0 = by0 + (tid >> 4), py1 = py0 + 8;
    const uint32_t bin = (by0 / gp.bin_h) * gp.tiles_x + bx0 / gp.bin_w;
    const uint2 r = ranges[bin];
    const uint32_t start = r.x, end = r.y;
    const uint32_t preend = start + ((end - start) / 64) * 64;
    // sorted Gaussian indices: the low idx_bits of packed elements, or the value array
    const bool packed = ctl->packed != 0;
    const unsigned long long* __restrict__ elems = io_keys(io, ctl->final_buf);
    const uint32_t* __restrict__ vals = io_vals(io, ctl->final_buf);
    const unsigned long long imask = (1ull << ctl->idx_bits) - 1ull;
    auto index_at = [&](uint32_t i) -> uint32_t {
        return packed ? (uint32_t)(elems[i] & imask) : vals[i];
    };
    const float tmin = (float)(1.0 - 0.9999);
    const float fx = (float)px, fy0 = (float)py0, fy1 = (float)py1;

    // Reference exit rule: a pixel whose T <= 1-0.9999 at the end of a 64-batch leaves the batch
    // loop, but the tail loop (comp:104-117) still blends the element at `preend` before it
    // stops. Such a pixel waits and takes that one element after the staged loop.
    Pix p0{0.0f, 0.0f, 0.0f, 1.0f, !(px < gp.width && py0 < gp.height), false};
    Pix p1{0.0f, 0.0f, 0.0f, 1.0f, !(px < gp.width && py1 < gp.height), false};

    for (uint32_t b = start; b < end; b += kBatch) {
        const bool idle = (p0.done || p0.wait_tail) && (p1.done || p1.wait_tail);
        if (__syncthreads_and(idle)) break;
        const uint32_t nb = min((uint32_t)kBatch, end - b);
        for (uint32_t k = (uint32_t)tid; k < nb; k += kRasterThreads) {
            const uint32_t idx = index_at(b + k);
            const float4 g = rec[3 * (uint64_t)idx + 0];
            s_mean[k] = make_float2(g.x, g.y);
            s_q[k] = quad_form(rec[3 * (uint64_t)idx + 1], g.z);
            s_col[k] = color_alpha(rec[3 * (uint64_t)idx + 2], g.z);
        }
        __syncthreads();
        bool a0 = !(p0.done || p0.wait_tail), a1 = !(p1.done || p1.wait_tail);
        if (!a0 && !a1) continue;
        if (PER_ELEM) {
            for (uint32_t jj = 0; jj < nb && (a0 || a1); ++jj) {
                const float2 m = s_mean[jj];
                const float4 q = s_q[jj], c = s_col[jj];
                if (a0) {
                    blend(fx, fy0, m, q, c, p0.C0, p0.C1, p0.C2, p0.T);
                    if (p0.T <= tmin) p0.done = true, a0 = false;
                }
                if (a1) {
                    blend(fx, fy1, m, q, c, p1.C0, p1.C1, p1.C2, p1.T);
                    if (p1.T <= tmin) p1.done = true, a1 = false;
                }
            }
            continue;
        }
        // 64-element blocks counted from `start` (batches start kBatch apart, a multiple of 64, so blocks align)
        for (uint32_t j0 = 0; j0 < nb; j0 += 64) {
            if (b + j0 < preend) {  // a whole 64-batch of the reference: test once at its end
                if (a0 && a1) {
#pragma unroll 4
                    for (uint32_t jj = j0; jj < j0 + 64; ++jj) {
                        const float2 m = s_mean[jj];
                        const float4 q = s_q[jj], c = s_col[jj];
                        const Xterms xt = xterms(fx, m, q);
                        blend_y(xt, fy0, m, q, c, p0.C0, p0.C1, p0.C2, p0.T);
                        blend_y(xt, fy1, m, q, c, p1.C0, p1.C1, p1.C2, p1.T);
                    }
                } else if (a0) {
#pragma unroll 8
                    for (uint32_t jj = j0; jj < j0 + 64; ++jj)
                        blend(fx, fy0, s_mean[jj], s_q[jj], s_col[jj], p0.C0, p0.C1, p0.C2, p0.T);
                } else {
#pragma unroll 8
                    for (uint32_t jj = j0; jj < j0 + 64; ++jj)
                        blend(fx, fy1, s_mean[jj], s_q[jj], s_col[jj], p1.C0, p1.C1, p1.C2, p1.T);
                }
                if (a0 && p0.T <= tmin) {
                    p0.wait_tail = preend < end;
                    p0.done = !p0.wait_tail;
                    a0 = false;
                }
                if (a1 && p1.T <= tmin) {
                    p1.wait_tail = preend < end;
                    p1.done = !p1.wait_tail;
                    a1 = false;
                }
                if (!a0 && !a1) break;
            } else {  // the tail: test after every element
                for (uint32_t jj = j0; jj < nb && (a0 || a1); ++jj) {
                    const float2 m = s_mean[jj];
                    const float4 q = s_q[jj], c = s_col[jj];
                    if (a0) {
                        blend(fx, fy0, m, q, c, p0.C0, p0.C1, p0.C2, p0.T);
                        if (p0.T <= tmin) p0.done = true, a0 = false;
                    }
                    if (a1) {
                        blend(fx, fy1, m, q, c, p1.C0, p1.C1, p1.C2, p1.T);
                        if (p1.T <= tmin) p1.done = true, a1 = false;
                    }
                }
                break;
            }
        }
    }
    if (p0.wait_tail) blend_tail(rec, index_at, preend, end, fx, fy0, tmin, p0);
    if (p1.wait_tail) blend_tail(rec, index_at, preend, end, fx, fy1, tmin, p1);
    if (px < gp.width && py0 < gp.height) write_pixel(img, gp, px, py0, p0);
    if (px < gp.width && py1 < gp.height) write_pixel(img, gp, px, py1, p1);
}

// Every pixel of an RGBA8 image set to one colour, 16 bytes per store where the image allows.
__global__ void __launch_bounds__(256) k_fill_image(uchar4* __restrict__ img, uint64_t n, uchar4 v) {
    const uint32_t w = (uint32_t)v.x | (uint32_t)v.y << 8 | (uint32_t)v.z << 16 | (uint32_t)v.w << 24;
    const uint4 q = make_uint4(w, w, w, w);
    const uint64_t nq = ((reinterpret_cast<uintptr_t>(img) & 15u) == 0) ? n / 4 : 0;
    uint4* __restrict__ img4 = reinterpret_cast<uint4*>(img);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nq; i += stride) img4[i] = q;
    for (uint64_t i = nq * 4 + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) img[i] = v;
}

}  // namespace

cudaError_t launch_fill_image(uchar4* img, uint64_t pixels, uchar4 value, cudaStream_t stream) {
    if (pixels == 0) return cudaSuccess;
    uint64_t blocks = (pixels / 4 + 255) / 256;
    const uint64_t cap = (uint64_t)device_sm_count() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    k_fill_image<<<(unsigned)blocks, 256, 0, stream>>>(img, pixels, value);
    return cudaGetLastError();
}

uint32_t raster_block_rows(const GridParams& gp) {
    const uint32_t y0 = gp.row_begin * gp.bin_h;
    uint32_t y1 = gp.row_end * gp.bin_h;
    if (y1 > gp.height) y1 = gp.height;
    return y1 > y0 ? (y1 - y0 + 15) / 16 : 0u;
}

cudaError_t launch_rasterize(const float4* rec, const SortIO& io, const uint2* ranges,
                             const FrameCtl* ctl, const GridParams& gp, uchar4* img,
                             bool per_element_exit, cudaStream_t stream, uint32_t first_block_row,
                             uint32_t block_rows) {
    const uint32_t total = raster_block_rows(gp);
    if (first_block_row >= total) return cudaSuccess;
    const uint32_t rows = block_rows < total - first_block_row ? block_rows : total - first_block_row;
    const uint32_t y0 = gp.row_begin * gp.bin_h + 16u * first_block_row;
    const dim3 grid((gp.width + 15) / 16, rows);
    if (per_element_exit)
        k_rasterize<true><<<grid, kRasterThreads, 0, stream>>>(rec, io, ranges, ctl, gp, img, y0);
    else
        k_rasterize<false><<<grid, kRasterThreads, 0, stream>>>(rec, io, ranges, ctl, gp, img, y0);
    return cudaGetLastError();
}

}  // namespace kt
