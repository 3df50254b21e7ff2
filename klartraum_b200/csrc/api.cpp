// C ABI of the renderer (include/kt_gs.h): context, device workspaces and the frame driver.
//
// Host-side counterpart of klartraum's VulkanGaussianSplatting node
// (src/vulkan_gaussian_splatting.cpp:13-316): where the node builds a five-element compute
// sub-graph with Vulkan buffers, this context owns the device buffers of each path (frame in
// flight) and enqueues the kernels of one frame on a CUDA stream:
//   init -> K1 project+count -> depth keys + plan -> depth sort passes (Gaussians)
//   -> coarse-bin counts per (chunk of depth order, coarse bin) -> prefix, K, coarse list starts
//   -> coarse placement -> bin counts + bin ranges (K5) -> pair placement by bin (K2-K4 without
//   a pair sort) -> totals -> K6.
// No host synchronisation happens inside a frame: the key count, the capacity check and the
// depth-sort plan live in device memory. After the frame a 2.6 KB control block is copied back;
// unless KT_GS_FLAG_ASYNC is set the call waits for it and, if the keys did not fit, grows
// the key buffers and renders again (nothing was drawn in that case).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstddef>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "kt_common.cuh"
#include "kt_gs.h"
#include "kt_kernels.h"

namespace kt {

int device_sm_count() {
    static int cache[128] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 148;
    if (cache[dev] == 0) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = v > 0 ? v : 148;
    }
    return cache[dev];
}

}  // namespace kt

using namespace kt;

namespace {

constexpr uint64_t kMaxKeyCapacity = 0xFFFFF000ull;  // values and ranges are 32-bit
constexpr uint32_t kDepthPasses = 4;                  // 8-bit passes over <= 31 depth bits

// What a captured frame graph bakes in (kernel arguments and buffer addresses).
struct GraphKey {
    const void* img = nullptr;
    uint64_t n = 0;
    uint64_t cap = 0;
    uint32_t flags = 0;
    int src = 0;
    uint64_t scene_gen = 0;
    uint64_t buf_gen = 0;
    bool place_runs = false;
    bool operator==(const GraphKey& o) const {
        return img == o.img && n == o.n && cap == o.cap && flags == o.flags && src == o.src &&
               scene_gen == o.scene_gen && buf_gen == o.buf_gen && place_runs == o.place_runs;
    }
};

struct PathWs {
    uint64_t n_alloc = 0;
    uint64_t cap = 0;
    float4* rec = nullptr;
    uint32_t* counts = nullptr;
    uint2* rect = nullptr;
    uint2* srect = nullptr;  // rect in depth order
    uint32_t* depth = nullptr;
    unsigned long long* gsort[2] = {nullptr, nullptr};  // Gaussians by depth
    uint32_t* pairs = nullptr;  // Gaussian of every (bin, Gaussian) pair, in bin order
    unsigned long long* sort_status = nullptr;
    uint32_t* sort_table = nullptr;  // per-range digit table of reduce-then-scan passes
    uint64_t status_words = 0;
    // pair placement (default path), allocated on first use
    uint32_t* ctable = nullptr;  // entries per (chunk, coarse bin), then their prefix over chunks
    uint64_t ctable_words = 0;
    uint32_t* gtable = nullptr;  // entries per (group of chunks, coarse bin), then their prefix over groups
    uint64_t gtable_words = 0;
    uint4* cinfo = nullptr;      // per coarse bin: list start, entries, first segment
    uint64_t cinfo_n = 0;
    uint2* clist = nullptr;      // (Gaussian, 4x4 bin mask) by coarse bin
    uint64_t clist_n = 0;
    uint32_t* seg_coarse = nullptr;  // coarse bin of every segment
    uint32_t* seg_cnt = nullptr;     // pairs per (segment, bin of the 4x4)
    uint64_t seg_n = 0;
    uint2* ranges = nullptr;
    // reference-structured path (KT_GS_FLAG_SORTED_KEYS), allocated on first use
    unsigned long long* keys[2] = {nullptr, nullptr};  // bin << depth_bits | depth, ping-pong
    uint32_t* vals[2] = {nullptr, nullptr};            // Gaussian index, ping-pong
    uint64_t key_cap = 0;
    unsigned long long* key_status = nullptr;  // look-back words of the pair sort
    uint32_t* key_table = nullptr;             // reduce-then-scan table of the pair sort
    uint32_t key_epoch = 0;
    unsigned long long* offsets = nullptr;      // scan of the counts, index order
    unsigned long long* scan_status = nullptr;  // look-back words of that scan
    uint64_t key_n = 0;
    uint32_t scan_epoch = 0;
    bool keys_frame = false;  // the path's last frame took the keys path
    // frame graph (KT_GS_FLAG_GRAPH)
    cudaGraphExec_t gexec = nullptr;
    cudaGraph_t graph = nullptr;        // the captured graph gexec was made from (owns k1_node)
    GraphKey gkey{};
    // the projection's kernel node and its arguments: each replay sets its camera argument
    cudaGraphNode_t k1_node = nullptr;
    cudaKernelNodeParams k1_params{};
    SceneDev k1_sc{};
    CamParams k1_cam{};
    GridParams k1_gp{};
    FrameBufs k1_fb{};
    void* k1_args[4] = {};
    cudaStream_t cap_stream = nullptr;  // capture stream
    uint64_t buf_gen = 0;               // bumped whenever a buffer of the path is reallocated
    FrameCtl* ctl = nullptr;
    FrameCtl* ctl_depth = nullptr;
    FrameCtl* host_ctl = nullptr;  // pinned copy of the last frame's control block
    uint32_t sort_epoch = 0;
    cudaEvent_t done_ev = nullptr;
    // stage timers: a ring of event sets, one set per timed frame, drained into sums
    static constexpr int kRing = 16;
    cudaEvent_t ring[kRing][KT_GS_NSTAGES] = {};
    bool ring_used[kRing] = {};
    int ring_next = 0;
    int ring_last = -1;
    double stage_sum[KT_GS_NSTAGES] = {};
    uint64_t timed_frames = 0;
    FrameTotals* totals = nullptr;  // device: counters and sticky error bits across frames
    bool timed = false;
    bool have_frame = false;
    uint64_t frame_n = 0;
    uint32_t last_ncoarse = 0;  // coarse bins of the last frame's pair placement
    // pair placement by runs of segments while the path's frames have many segments per warp
    bool place_runs = false;
    // device image for kt_gs_render_host
    uchar4* img = nullptr;
    // device copy of caller-supplied projected records
    float* g2d = nullptr;
    uint64_t g2d_n = 0;
};

template <class T>
void dfree(T*& p) {
    if (p) cudaFree((void*)p);
    p = nullptr;
}

}  // namespace

struct kt_gs_ctx {
    kt_gs_config cfg{};
    int device = 0;
    std::string err;
    float4* pos = nullptr;
    float4* rot = nullptr;
    float4* scale = nullptr;
    float4* sh = nullptr;
    uint32_t nplanes = 0;
    int deg = 0;
    uint64_t n = 0;
    bool has_scene = false;
    GridParams gp{};
    uint64_t scene_gen = 0;  // bumped by every scene upload (frame graphs bake the scene's address)
    std::vector<PathWs> paths;
};

namespace {

kt_status fail(kt_gs_ctx* c, kt_status s, const std::string& msg) {
    if (c) c->err = msg;
    return s;
}

#define KT_TRY_CUDA(ctx, call)                                                              \
    do {                                                                                    \
        cudaError_t e_ = (call);                                                            \
        if (e_ != cudaSuccess)                                                              \
            return fail((ctx), e_ == cudaErrorMemoryAllocation ? KT_ERR_NOMEM : KT_ERR_CUDA, \
                        std::string(#call) + ": " + cudaGetErrorString(e_));                \
    } while (0)

// GLSL mat4 * mat4, column-major, products summed in ascending k (matches the shader).
void mat4_mul(const float* a, const float* b, float* r) {
    for (int c = 0; c < 4; ++c)
        for (int k = 0; k < 4; ++k)
            r[4 * c + k] = a[k] * b[4 * c] + a[4 + k] * b[4 * c + 1] + a[8 + k] * b[4 * c + 2] +
                           a[12 + k] * b[4 * c + 3];
}

CamParams make_cam(const kt_camera_mvp* cam) {
    CamParams p;
    float pv[16];
    mat4_mul(cam->proj, cam->view, pv);
    mat4_mul(pv, cam->model, p.pvm);     // ubo.proj * ubo.view * ubo.model
    mat4_mul(cam->model, cam->view, p.mv);  // ubo.model * ubo.view
    p.focal_x = cam->proj[0];
    p.focal_y = cam->proj[5];
    // tanFov = 1 / focal, lim = 1.3 * tanFov (gsplat_projection.comp:76-77, 86-87): IEEE float
    // division and product, the values the shader's own operations give
    const float tan_fov_x = 1.0f / p.focal_x;
    const float tan_fov_y = 1.0f / p.focal_y;
    p.lim_x = 1.3f * tan_fov_x;
    p.lim_y = 1.3f * tan_fov_y;
    return p;
}

GridParams make_grid(const kt_gs_config& c) {
    GridParams g;
    g.width = c.width;
    g.height = c.height;
    g.bin_w = c.bin_width;
    g.bin_h = c.bin_height;
    g.half_w = (float)c.width * 0.5f;
    g.half_h = (float)c.height * 0.5f;
    g.sxx = (float)c.width * (float)c.width;
    g.syy = (float)c.height * (float)c.height;
    g.sxy = (float)c.width * (float)c.height;
    g.cell_w = (float)c.bin_width;
    g.cell_h = (float)c.bin_height;
    g.inv_cell_w = 1.0f / g.cell_w;
    g.inv_cell_h = 1.0f / g.cell_h;
    g.cull_z = c.cull_z;
    g.tiles_x = (c.width + c.bin_width - 1) / c.bin_width;
    g.tiles_y = (c.height + c.bin_height - 1) / c.bin_height;
    g.row_end = c.tile_row_end == 0 ? g.tiles_y : std::min(c.tile_row_end, g.tiles_y);
    g.row_begin = std::min(c.tile_row_begin, g.row_end);
    g.tile_bits = bits_for((uint64_t)g.tiles_x * g.tiles_y - 1);
    return g;
}

uint32_t ntiles(const kt_gs_ctx* c) { return c->gp.tiles_x * c->gp.tiles_y; }

void free_path(PathWs& w) {
    dfree(w.rec); dfree(w.counts); dfree(w.rect); dfree(w.srect); dfree(w.depth); dfree(w.gsort[0]);
    dfree(w.gsort[1]);
    dfree(w.pairs); dfree(w.ctable); dfree(w.gtable); dfree(w.cinfo); dfree(w.clist); dfree(w.seg_coarse); dfree(w.seg_cnt);
    w.ctable_words = w.gtable_words = w.cinfo_n = w.clist_n = w.seg_n = 0;
    dfree(w.sort_status); dfree(w.sort_table); dfree(w.ranges); dfree(w.ctl); dfree(w.ctl_depth);
    dfree(w.keys[0]); dfree(w.keys[1]); dfree(w.vals[0]); dfree(w.vals[1]); dfree(w.key_status);
    dfree(w.key_table); dfree(w.offsets); dfree(w.scan_status);
    w.key_cap = w.key_n = 0;
    if (w.gexec) cudaGraphExecDestroy(w.gexec);
    w.gexec = nullptr;
    if (w.graph) cudaGraphDestroy(w.graph);
    w.graph = nullptr;
    w.k1_node = nullptr;
    if (w.cap_stream) cudaStreamDestroy(w.cap_stream);
    w.cap_stream = nullptr;
    dfree(w.img); dfree(w.g2d);
    if (w.host_ctl) cudaFreeHost(w.host_ctl);
    w.host_ctl = nullptr;
    if (w.done_ev) cudaEventDestroy(w.done_ev);
    w.done_ev = nullptr;
    for (auto& set : w.ring)
        for (auto& e : set) {
            if (e) cudaEventDestroy(e);
            e = nullptr;
        }
    dfree(w.totals);
    w.n_alloc = w.cap = 0;
}

kt_status ensure_path_base(kt_gs_ctx* c, PathWs& w) {
    if (!w.ctl) {
        KT_TRY_CUDA(c, cudaMalloc(&w.ctl, sizeof(FrameCtl)));
        KT_TRY_CUDA(c, cudaMemset(w.ctl, 0, sizeof(FrameCtl)));
        KT_TRY_CUDA(c, cudaMalloc(&w.ctl_depth, sizeof(FrameCtl)));
        KT_TRY_CUDA(c, cudaMemset(w.ctl_depth, 0, sizeof(FrameCtl)));
        KT_TRY_CUDA(c, cudaMallocHost(&w.host_ctl, sizeof(FrameCtl)));
        std::memset(w.host_ctl, 0, sizeof(FrameCtl));
        KT_TRY_CUDA(c, cudaMalloc(&w.ranges, sizeof(uint2) * std::max(1u, ntiles(c))));
        KT_TRY_CUDA(c, cudaEventCreateWithFlags(&w.done_ev, cudaEventDisableTiming));
        for (auto& set : w.ring)
            for (auto& e : set) KT_TRY_CUDA(c, cudaEventCreate(&e));
        KT_TRY_CUDA(c, cudaMalloc(&w.totals, sizeof(FrameTotals)));
        KT_TRY_CUDA(c, cudaMemset(w.totals, 0, sizeof(FrameTotals)));
    }
    return KT_OK;
}

// Look-back status words of the depth sort (n elements), and its reduce-then-scan table when it
// spans more than one wave of CTAs.
kt_status ensure_status(kt_gs_ctx* c, PathWs& w) {
    const uint64_t need = sort_status_words(w.n_alloc);
    if (need <= w.status_words) return KT_OK;
    dfree(w.sort_status);
    dfree(w.sort_table);
    ++w.buf_gen;
    w.status_words = 0;
    const size_t table = sort_table_words(w.n_alloc);
    KT_TRY_CUDA(c, cudaMalloc(&w.sort_table, sizeof(uint32_t) * table));
    KT_TRY_CUDA(c, cudaMalloc(&w.sort_status, sizeof(unsigned long long) * need));
    KT_TRY_CUDA(c, cudaMemset(w.sort_status, 0, sizeof(unsigned long long) * need));
    w.sort_epoch = 0;
    w.status_words = need;
    return KT_OK;
}

kt_status ensure_n(kt_gs_ctx* c, PathWs& w, uint64_t n) {
    if (n <= w.n_alloc) return KT_OK;
    dfree(w.rec); dfree(w.counts); dfree(w.rect); dfree(w.srect); dfree(w.depth); dfree(w.gsort[0]);
    dfree(w.gsort[1]);
    ++w.buf_gen;
    w.n_alloc = 0;
    const uint64_t m = std::max<uint64_t>(n, 1);
    KT_TRY_CUDA(c, cudaMalloc(&w.rec, sizeof(float4) * 3 * m));
    KT_TRY_CUDA(c, cudaMalloc(&w.counts, sizeof(uint32_t) * m));
    KT_TRY_CUDA(c, cudaMalloc(&w.rect, sizeof(uint2) * m));
    KT_TRY_CUDA(c, cudaMalloc(&w.srect, sizeof(uint2) * m));
    KT_TRY_CUDA(c, cudaMalloc(&w.depth, sizeof(uint32_t) * m));
    KT_TRY_CUDA(c, cudaMalloc(&w.gsort[0], sizeof(unsigned long long) * m));
    KT_TRY_CUDA(c, cudaMalloc(&w.gsort[1], sizeof(unsigned long long) * m));
    w.n_alloc = m;
    return ensure_status(c, w);
}

kt_status ensure_cap(kt_gs_ctx* c, PathWs& w, uint64_t cap) {
    if (cap <= w.cap) return KT_OK;
    if (cap > kMaxKeyCapacity)
        return fail(c, KT_ERR_CAPACITY, "key count " + std::to_string(cap) +
                                            " exceeds the 32-bit index range of the key buffers");
    cap = std::min<uint64_t>(((cap + kSortTile - 1) / kSortTile) * kSortTile, kMaxKeyCapacity);
    dfree(w.pairs);
    ++w.buf_gen;
    w.cap = 0;
    KT_TRY_CUDA(c, cudaMalloc(&w.pairs, sizeof(uint32_t) * cap));
    w.cap = cap;
    return KT_OK;
}

// Buffers of the reference-structured path, sized for the path's capacity and n Gaussians.
kt_status ensure_keys(kt_gs_ctx* c, PathWs& w, uint64_t n) {
    if (w.key_cap < w.cap) {
        ++w.buf_gen;
        dfree(w.keys[0]); dfree(w.keys[1]); dfree(w.vals[0]); dfree(w.vals[1]);
        dfree(w.key_status); dfree(w.key_table);
        w.key_cap = 0;
        for (int b = 0; b < 2; ++b) {
            KT_TRY_CUDA(c, cudaMalloc(&w.keys[b], sizeof(unsigned long long) * w.cap));
            KT_TRY_CUDA(c, cudaMalloc(&w.vals[b], sizeof(uint32_t) * w.cap));
        }
        const size_t words = sort_status_words(w.cap);
        KT_TRY_CUDA(c, cudaMalloc(&w.key_status, sizeof(unsigned long long) * words));
        KT_TRY_CUDA(c, cudaMemset(w.key_status, 0, sizeof(unsigned long long) * words));
        KT_TRY_CUDA(c, cudaMalloc(&w.key_table, sizeof(uint32_t) * sort_table_words(w.cap)));
        w.key_epoch = 0;
        w.key_cap = w.cap;
    }
    if (w.key_n < n) {
        ++w.buf_gen;
        dfree(w.offsets); dfree(w.scan_status);
        w.key_n = 0;
        const uint64_t chunks = (n + kScanChunk - 1) / kScanChunk;
        KT_TRY_CUDA(c, cudaMalloc(&w.offsets, sizeof(unsigned long long) * n));
        KT_TRY_CUDA(c, cudaMalloc(&w.scan_status, sizeof(unsigned long long) * chunks));
        KT_TRY_CUDA(c, cudaMemset(w.scan_status, 0, sizeof(unsigned long long) * chunks));
        w.scan_epoch = 0;
        w.key_n = n;
    }
    return KT_OK;
}

// 8-bit passes the keys path's sort may need: bin bits + up to 32 depth bits
uint32_t key_passes(const kt_gs_ctx* c) { return (c->gp.tile_bits + 32 + 7) / 8; }

FrameBufs frame_bufs(const PathWs& w) {
    FrameBufs fb;
    fb.rec = w.rec;
    fb.counts = w.counts;
    fb.rect = w.rect;
    fb.srect = w.srect;
    fb.depth = w.depth;
    fb.gsort[0] = w.gsort[0];
    fb.gsort[1] = w.gsort[1];
    fb.pairs = w.pairs;
    fb.ctable = w.ctable;
    fb.gtable = w.gtable;
    fb.cinfo = w.cinfo;
    fb.clist = w.clist;
    fb.seg_coarse = w.seg_coarse;
    fb.seg_cnt = w.seg_cnt;
    fb.offsets = w.offsets;
    fb.keys[0] = w.keys[0];
    fb.keys[1] = w.keys[1];
    fb.vals[0] = w.vals[0];
    fb.vals[1] = w.vals[1];
    fb.scan_status = w.scan_status;
    fb.ranges = w.ranges;
    fb.sort_status = w.sort_status;
    fb.ctl = w.ctl;
    fb.ctl_depth = w.ctl_depth;
    fb.key_capacity = w.cap;
    return fb;
}

enum class Source { Scene, Projected };

// bytes of FrameCtl copied back after every frame (everything before the histograms)
constexpr size_t kCtlHeaderBytes = offsetof(FrameCtl, hist);

// Wait for a timed frame's events and add its stage times to the running sums.
kt_status drain_slot(kt_gs_ctx* c, PathWs& w, int slot) {
    if (!w.ring_used[slot]) return KT_OK;
    cudaEvent_t* ev = w.ring[slot];
    constexpr int L = KT_GS_NSTAGES - 1;  // events 0..L bracket the stages
    KT_TRY_CUDA(c, cudaEventSynchronize(ev[L]));
    float ms = 0.0f;
    for (int i = 0; i < L; ++i) {
        KT_TRY_CUDA(c, cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
        w.stage_sum[i] += ms;
    }
    KT_TRY_CUDA(c, cudaEventElapsedTime(&ms, ev[0], ev[L]));
    w.stage_sum[L] += ms;
    w.timed_frames += 1;
    w.ring_used[slot] = false;
    return KT_OK;
}

// What one frame needs besides its buffers: the placement split and the look-back epochs.
struct FramePlan {
    bool keys = false;          // reference-structured binning (KT_GS_FLAG_SORTED_KEYS)
    PlaceGeom pg{};             // placement split (default path)
    uint32_t sort_epoch0 = 1;   // depth-sort passes (default path)
    uint32_t scan_epoch = 1;    // keys path: scan
    uint32_t key_epoch0 = 1;    // keys path: sort passes
    bool clear_status = false;  // graph replays clear the look-back words at the frame's start
    bool place_runs = false;    // pair placement by runs of segments (k_fine_place_runs)
};

// Allocations and look-back epochs of a frame. Never called inside a stream capture.
// The pair-placement kernel for the next frame of a path: a warp per segment while the segments
// are at most a few per warp (few registers, full occupancy), runs of segments with the next one
// prefetched when each warp would take many (long coarse lists). From the segment count of the
// path's last completed frame, switching above 6 and back below 4 segments per warp.
bool choose_place_runs(const PathWs& w, const PlaceGeom& pg) {
    if (!w.have_frame || !w.host_ctl || w.keys_frame) return w.place_runs;
    const double per_warp = (double)w.host_ctl->num_segments / (double)std::max<uint32_t>(1u, fine_place_warps(pg));
    if (w.place_runs) return per_warp > 4.0;
    return per_warp > 6.0;
}

kt_status prepare_frame(kt_gs_ctx* c, PathWs& w, uint64_t n, bool graph, FramePlan& fp, cudaStream_t stream) {
    fp.keys = (c->cfg.flags & KT_GS_FLAG_SORTED_KEYS) != 0;
    fp.clear_status = graph;
    if (fp.keys) {
        kt_status st = ensure_keys(c, w, std::max<uint64_t>(n, 1));
        if (st != KT_OK) return st;
        if (graph) return KT_OK;  // fixed epochs, words cleared by the graph
        const uint32_t passes = key_passes(c);
        if (++w.scan_epoch > kEpochMax) {
            KT_TRY_CUDA(c, cudaMemsetAsync(w.scan_status, 0,
                                           sizeof(unsigned long long) * ((w.key_n + kScanChunk - 1) / kScanChunk),
                                           stream));
            w.scan_epoch = 1;
        }
        if (w.key_epoch + passes + 1 > kEpochMax) {
            KT_TRY_CUDA(c, cudaMemsetAsync(w.key_status, 0,
                                           sizeof(unsigned long long) * sort_status_words(w.key_cap), stream));
            w.key_epoch = 0;
        }
        fp.scan_epoch = w.scan_epoch;
        fp.key_epoch0 = w.key_epoch + 1;
        w.key_epoch += passes;
        return KT_OK;
    }
    KT_TRY_CUDA(c, place_geometry(c->gp, n, w.cap, &fp.pg));
    w.place_runs = choose_place_runs(w, fp.pg);
    fp.place_runs = w.place_runs;
    if (fp.pg.table_words > w.ctable_words) {
        dfree(w.ctable);
        w.ctable_words = 0;
        KT_TRY_CUDA(c, cudaMalloc(&w.ctable, sizeof(uint32_t) * fp.pg.table_words));
        w.ctable_words = fp.pg.table_words;
        ++w.buf_gen;
    }
    if (fp.pg.gtable_words > w.gtable_words) {
        dfree(w.gtable);
        w.gtable_words = 0;
        KT_TRY_CUDA(c, cudaMalloc(&w.gtable, sizeof(uint32_t) * fp.pg.gtable_words));
        w.gtable_words = fp.pg.gtable_words;
        ++w.buf_gen;
    }
    if (fp.pg.ncoarse > w.cinfo_n) {
        dfree(w.cinfo);
        w.cinfo_n = 0;
        KT_TRY_CUDA(c, cudaMalloc(&w.cinfo, sizeof(uint4) * fp.pg.ncoarse));
        w.cinfo_n = fp.pg.ncoarse;
        ++w.buf_gen;
    }
    if (w.cap > w.clist_n) {  // entries <= pairs <= capacity
        dfree(w.clist);
        w.clist_n = 0;
        KT_TRY_CUDA(c, cudaMalloc(&w.clist, sizeof(uint2) * w.cap));
        w.clist_n = w.cap;
        ++w.buf_gen;
    }
    if (fp.pg.max_segments > w.seg_n) {
        dfree(w.seg_coarse);
        dfree(w.seg_cnt);
        w.seg_n = 0;
        KT_TRY_CUDA(c, cudaMalloc(&w.seg_coarse, sizeof(uint32_t) * fp.pg.max_segments));
        KT_TRY_CUDA(c, cudaMalloc(&w.seg_cnt, sizeof(uint32_t) * 16 * fp.pg.max_segments));
        w.seg_n = fp.pg.max_segments;
        ++w.buf_gen;
    }
    if (graph) return KT_OK;
    if (w.sort_epoch + kDepthPasses + 1 > kEpochMax) {
        KT_TRY_CUDA(c, cudaMemsetAsync(w.sort_status, 0, sizeof(unsigned long long) * w.status_words, stream));
        w.sort_epoch = 0;
    }
    fp.sort_epoch0 = w.sort_epoch + 1;
    w.sort_epoch += kDepthPasses;
    return KT_OK;
}

// The kernels and copies of one frame on `stream`: no allocation and no host wait, so the
// sequence can be captured into a CUDA graph. `ev` (may be null) receives the stage events.
//   default: init -> K1 -> depth keys + plan -> depth passes -> rectangles in depth order +
//            coarse counts -> prefix over chunks + coarse ranges -> coarse placement -> bin
//            counts + bin ranges + pair placement -> totals -> K6
//   keys:    init -> K1 -> scan + key emission -> plan + key sort passes -> boundary search ->
//            totals -> K6
kt_status record_frame(kt_gs_ctx* c, PathWs& w, Source src, uint64_t n, const CamParams* cam, uchar4* img,
                       cudaStream_t stream, cudaEvent_t* ev, const FramePlan& fp) {
    const bool timed = ev != nullptr;
    FrameBufs fb = frame_bufs(w);
    if (fp.clear_status) {
        if (fp.keys) {
            KT_TRY_CUDA(c, cudaMemsetAsync(w.scan_status, 0,
                                           sizeof(unsigned long long) * ((w.key_n + kScanChunk - 1) / kScanChunk),
                                           stream));
            KT_TRY_CUDA(c, cudaMemsetAsync(w.key_status, 0,
                                           sizeof(unsigned long long) * sort_status_words(w.key_cap), stream));
        } else {
            KT_TRY_CUDA(c, cudaMemsetAsync(w.sort_status, 0, sizeof(unsigned long long) * w.status_words, stream));
        }
    }
    if (timed) KT_TRY_CUDA(c, cudaEventRecord(ev[0], stream));
    KT_TRY_CUDA(c, launch_frame_init(w.ctl, w.ctl_depth, w.ranges, ntiles(c), stream));
    if (src == Source::Scene) {
        SceneDev sc{c->pos, c->rot, c->scale, c->sh, c->nplanes, c->deg, c->n};
        const CamParams none{};
        KT_TRY_CUDA(c, launch_project_count(sc, cam ? *cam : none, c->gp, fb, stream));
    } else {
        KT_TRY_CUDA(c, launch_load_projected(w.g2d, n, c->gp, fb, stream));
    }
    if (timed) KT_TRY_CUDA(c, cudaEventRecord(ev[1], stream));
    SortIO io{};
    if (fp.keys) {
        const uint32_t passes = key_passes(c);
        io.keys[0] = w.keys[0];
        io.keys[1] = w.keys[1];
        io.vals[0] = w.vals[0];
        io.vals[1] = w.vals[1];
        KT_TRY_CUDA(c, launch_key_scan_emit(fb, c->gp, n, fp.scan_epoch, passes, stream));
        if (timed) KT_TRY_CUDA(c, cudaEventRecord(ev[2], stream));
        KT_TRY_CUDA(c, launch_plan(w.ctl, w.cap, passes, 0, stream));
        for (uint32_t p = 0; p < passes; ++p)
            KT_TRY_CUDA(c, launch_sort_pass(io, w.ctl, w.key_status, w.key_table, p, fp.key_epoch0 + p, w.cap,
                                            false, stream));
        if (timed) KT_TRY_CUDA(c, cudaEventRecord(ev[3], stream));
        KT_TRY_CUDA(c, launch_key_ranges(io, w.ctl, w.ranges, w.cap, stream));
        if (timed) KT_TRY_CUDA(c, cudaEventRecord(ev[4], stream));
    } else {
        io.vals[0] = w.pairs;  // the rasteriser reads Gaussian indices
        SortIO io_depth{};
        io_depth.keys[0] = w.gsort[0];
        io_depth.keys[1] = w.gsort[1];
        // Gaussians by depth (stable: ties keep index order)
        KT_TRY_CUDA(c, launch_depth_keys(fb, n, kDepthPasses, stream));  // and the plan of the passes
        for (uint32_t p = 0; p < kDepthPasses; ++p)
            KT_TRY_CUDA(c, launch_sort_pass(io_depth, w.ctl_depth, w.sort_status, w.sort_table, p,
                                            fp.sort_epoch0 + p, n, true, stream));
        if (timed) KT_TRY_CUDA(c, cudaEventRecord(ev[2], stream));
        // entries per (chunk of depth order, coarse bin), their prefix over chunks, K, the coarse
        // list starts and segments
        KT_TRY_CUDA(c, launch_coarse_count(fb, c->gp, fp.pg, n, stream));
        if (timed) KT_TRY_CUDA(c, cudaEventRecord(ev[3], stream));
        // coarse lists in depth order
        KT_TRY_CUDA(c, launch_coarse_place(fb, c->gp, fp.pg, n, stream));
        if (timed) KT_TRY_CUDA(c, cudaEventRecord(ev[4], stream));
        // bin counts and ranges; every pair at its place in bin order (depth order within a bin)
        KT_TRY_CUDA(c, launch_fine_place(fb, c->gp, fp.pg, n, fp.place_runs, stream));
    }
    KT_TRY_CUDA(c, launch_frame_totals(w.ctl, w.ctl_depth, w.totals, stream));
    if (timed) KT_TRY_CUDA(c, cudaEventRecord(ev[5], stream));
    KT_TRY_CUDA(c, launch_rasterize(w.rec, io, w.ranges, w.ctl, c->gp, img,
                                    (c->cfg.flags & KT_GS_FLAG_EXIT_PER_ELEMENT) != 0, stream));
    if (timed) KT_TRY_CUDA(c, cudaEventRecord(ev[6], stream));
    KT_TRY_CUDA(c, cudaMemcpyAsync(w.host_ctl, w.ctl, kCtlHeaderBytes, cudaMemcpyDeviceToHost, stream));
    return KT_OK;
}

// Enqueue one frame on `stream`. Does not wait.
kt_status enqueue_frame(kt_gs_ctx* c, PathWs& w, Source src, const CamParams* cam, uchar4* img,
                        cudaStream_t stream) {
    const uint64_t n = src == Source::Scene ? c->n : w.g2d_n;
    const bool timed = (c->cfg.flags & KT_GS_FLAG_TIMING) != 0;
    w.timed = timed;
    cudaEvent_t* ev = nullptr;
    if (timed) {
        const int slot = w.ring_next;
        if (w.ring_used[slot]) {
            kt_status s = drain_slot(c, w, slot);
            if (s != KT_OK) return s;
        }
        ev = w.ring[slot];
        w.ring_used[slot] = true;
        w.ring_last = slot;
        w.ring_next = (slot + 1) % PathWs::kRing;
    }
    FramePlan fp;
    kt_status s = prepare_frame(c, w, n, false, fp, stream);
    if (s != KT_OK) return s;
    w.keys_frame = fp.keys;
    w.last_ncoarse = fp.keys ? 0u : fp.pg.ncoarse;
    if ((s = record_frame(c, w, src, n, cam, img, stream, ev, fp)) != KT_OK) return s;
    KT_TRY_CUDA(c, cudaEventRecord(w.done_ev, stream));
    w.have_frame = true;
    w.frame_n = n;
    return KT_OK;
}

// The projection's kernel node of a captured frame graph and a copy of its arguments, so that a
// replay can be given a new camera (cudaGraphExecKernelNodeSetParams). Leaves k1_node null when the
// graph has no projection (caller-supplied projected records).
cudaError_t find_k1_node(kt_gs_ctx* c, PathWs& w, cudaGraph_t g) {
    w.k1_node = nullptr;
    size_t count = 0;
    cudaError_t e = cudaGraphGetNodes(g, nullptr, &count);
    if (e != cudaSuccess || count == 0) return e;
    std::vector<cudaGraphNode_t> nodes(count);
    if ((e = cudaGraphGetNodes(g, nodes.data(), &count)) != cudaSuccess) return e;
    const void* fn = project_count_kernel(c->deg);
    for (cudaGraphNode_t nd : nodes) {
        cudaGraphNodeType t;
        if ((e = cudaGraphNodeGetType(nd, &t)) != cudaSuccess) return e;
        if (t != cudaGraphNodeTypeKernel) continue;
        cudaKernelNodeParams p{};
        if ((e = cudaGraphKernelNodeGetParams(nd, &p)) != cudaSuccess) return e;
        if (p.func != fn) continue;
        // k_project_count(SceneDev, CamParams, GridParams, FrameBufs)
        std::memcpy(&w.k1_sc, p.kernelParams[0], sizeof(SceneDev));
        std::memcpy(&w.k1_cam, p.kernelParams[1], sizeof(CamParams));
        std::memcpy(&w.k1_gp, p.kernelParams[2], sizeof(GridParams));
        std::memcpy(&w.k1_fb, p.kernelParams[3], sizeof(FrameBufs));
        w.k1_args[0] = &w.k1_sc;
        w.k1_args[1] = &w.k1_cam;
        w.k1_args[2] = &w.k1_gp;
        w.k1_args[3] = &w.k1_fb;
        w.k1_params = p;
        w.k1_params.kernelParams = w.k1_args;
        w.k1_params.extra = nullptr;
        w.k1_node = nd;
        break;
    }
    return cudaSuccess;
}

// Enqueue one frame as a replay of the path's captured frame graph (KT_GS_FLAG_GRAPH). The graph
// is captured again when anything baked into it changed: the image pointer, the scene or any
// buffer of the path, the Gaussian count, the flags or the source. Only the camera changes
// between replays: it is the projection kernel's argument, set in the executable graph before the
// launch (launches already enqueued keep the camera they were launched with).
kt_status enqueue_graph_frame(kt_gs_ctx* c, PathWs& w, Source src, const CamParams* cam, uchar4* img,
                              cudaStream_t stream) {
    const uint64_t n = src == Source::Scene ? c->n : w.g2d_n;
    FramePlan fp;
    kt_status s = prepare_frame(c, w, n, true, fp, stream);
    if (s != KT_OK) return s;
    if (!w.cap_stream) KT_TRY_CUDA(c, cudaStreamCreateWithFlags(&w.cap_stream, cudaStreamNonBlocking));
    const uint32_t kFlagsBaked = ~(KT_GS_FLAG_ASYNC | KT_GS_FLAG_TIMING | KT_GS_FLAG_NO_AUTOGROW);
    const GraphKey key{img, n, w.cap, c->cfg.flags & kFlagsBaked, (int)src, c->scene_gen, w.buf_gen, fp.place_runs};
    bool captured = false;
    if (!w.gexec || !(key == w.gkey)) {
        if (w.gexec) cudaGraphExecDestroy(w.gexec);
        w.gexec = nullptr;
        if (w.graph) cudaGraphDestroy(w.graph);
        w.graph = nullptr;
        w.k1_node = nullptr;
        KT_TRY_CUDA(c, cudaStreamBeginCapture(w.cap_stream, cudaStreamCaptureModeThreadLocal));
        const kt_status rs = record_frame(c, w, src, n, cam, img, w.cap_stream, nullptr, fp);
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(w.cap_stream, &g);  // ends the capture in every case
        if (rs != KT_OK) {
            if (g) cudaGraphDestroy(g);
            return rs;
        }
        KT_TRY_CUDA(c, e);
        const cudaError_t ei = cudaGraphInstantiate(&w.gexec, g, 0);
        if (ei != cudaSuccess) cudaGraphDestroy(g);
        KT_TRY_CUDA(c, ei);
        w.graph = g;
        KT_TRY_CUDA(c, find_k1_node(c, w, g));
        if (src == Source::Scene && !w.k1_node) return fail(c, KT_ERR_STATE, "frame graph without its projection node");
        w.gkey = key;
        captured = true;  // the capture holds this frame's camera
    }
    if (cam && w.k1_node && !captured) {
        w.k1_cam = *cam;
        KT_TRY_CUDA(c, cudaGraphExecKernelNodeSetParams(w.gexec, w.k1_node, &w.k1_params));
    }
    KT_TRY_CUDA(c, cudaGraphLaunch(w.gexec, stream));
    KT_TRY_CUDA(c, cudaEventRecord(w.done_ev, stream));
    w.keys_frame = fp.keys;
    w.last_ncoarse = fp.keys ? 0u : fp.pg.ncoarse;
    w.timed = false;
    w.have_frame = true;
    w.frame_n = n;
    return KT_OK;
}

// Wait for the path's last frame and translate its device error flags.
kt_status check_frame(kt_gs_ctx* c, PathWs& w) {
    if (!w.have_frame) return KT_OK;
    KT_TRY_CUDA(c, cudaEventSynchronize(w.done_ev));
    const uint32_t e = w.host_ctl->error_flags;
    if (e & kErrTimeout) return fail(c, KT_ERR_TIMEOUT, "a bounded device wait of the depth sort timed out");
    if (e & kErrCapacity)
        return fail(c, KT_ERR_CAPACITY, "frame needs " + std::to_string(w.host_ctl->num_keys) +
                                            " keys, capacity is " + std::to_string(w.cap));
    return KT_OK;
}

kt_status render_impl(kt_gs_ctx* c, uint32_t path, Source src, const kt_camera_mvp* cam,
                      uchar4* img, cudaStream_t stream) {
    if (path >= c->paths.size()) return fail(c, KT_ERR_ARG, "path index out of range");
    if (src == Source::Scene && !c->has_scene)
        return fail(c, KT_ERR_STATE, "no Gaussians set on this context");
    if (!img) return fail(c, KT_ERR_ARG, "output image is NULL");
    if (reinterpret_cast<uintptr_t>(img) & 3u) return fail(c, KT_ERR_ARG, "output image is not 4-byte aligned");
    KT_TRY_CUDA(c, cudaSetDevice(c->device));
    PathWs& w = c->paths[path];
    kt_status s = ensure_path_base(c, w);
    if (s != KT_OK) return s;
    const uint64_t n = src == Source::Scene ? c->n : w.g2d_n;
    if ((s = ensure_n(c, w, n)) != KT_OK) return s;
    if (w.cap == 0) {
        uint64_t guess = c->cfg.key_capacity ? c->cfg.key_capacity : std::max<uint64_t>(16 * n, 1u << 20);
        guess = std::min(guess, kMaxKeyCapacity);
        if ((s = ensure_cap(c, w, guess)) != KT_OK) return s;
    }
    CamParams cp{};
    if (cam) cp = make_cam(cam);
    const bool async = (c->cfg.flags & KT_GS_FLAG_ASYNC) != 0;
    for (int attempt = 0; attempt < 4; ++attempt) {
        s = (c->cfg.flags & KT_GS_FLAG_GRAPH) ? enqueue_graph_frame(c, w, src, cam ? &cp : nullptr, img, stream)
                                              : enqueue_frame(c, w, src, cam ? &cp : nullptr, img, stream);
        if (s != KT_OK) return s;
        if (async) return KT_OK;
        s = check_frame(c, w);
        if (s != KT_OK) {
            // this frame's error is reported (or handled) here, not by a later kt_gs_sync
            KT_TRY_CUDA(c, cudaMemsetAsync(&w.totals->sticky_errors, 0, sizeof(unsigned int), stream));
        }
        if (s != KT_ERR_CAPACITY || (c->cfg.flags & KT_GS_FLAG_NO_AUTOGROW)) return s;
        const uint64_t need = w.host_ctl->num_keys;
        const uint64_t grow = need + need / 4 + kSortTile;
        if ((s = ensure_cap(c, w, std::min(grow, kMaxKeyCapacity))) != KT_OK) return s;
        if (need > w.cap) return fail(c, KT_ERR_CAPACITY, "key count exceeds the maximum capacity");
    }
    return fail(c, KT_ERR_CAPACITY, "key buffers kept overflowing");
}

int detect_degree(const kt_gaussian3d* g, uint64_t n) {
    int deg = 0;
    for (uint64_t i = 0; i < n && deg < 3; ++i) {
        const float* bands[3] = {g[i].shR, g[i].shG, g[i].shB};
        for (int ch = 0; ch < 3; ++ch)
            for (int k = 0; k < 15; ++k)
                if (bands[ch][k] != 0.0f) {
                    const int d = k < 3 ? 1 : (k < 8 ? 2 : 3);
                    deg = std::max(deg, d);
                }
    }
    return deg;
}

kt_status upload_scene(kt_gs_ctx* c, const kt_gaussian3d* src, bool src_on_device, uint64_t n,
                       int deg, cudaStream_t stream) {
    KT_TRY_CUDA(c, cudaSetDevice(c->device));
    dfree(c->pos); dfree(c->rot); dfree(c->scale); dfree(c->sh);
    c->has_scene = false;
    ++c->scene_gen;
    c->n = n;
    c->deg = deg;
    c->nplanes = (uint32_t)((3 * (deg + 1) * (deg + 1) + 3) / 4);
    const uint64_t m = std::max<uint64_t>(n, 1);
    KT_TRY_CUDA(c, cudaMalloc(&c->pos, sizeof(float4) * m));
    KT_TRY_CUDA(c, cudaMalloc(&c->rot, sizeof(float4) * m));
    KT_TRY_CUDA(c, cudaMalloc(&c->scale, sizeof(float4) * m));
    KT_TRY_CUDA(c, cudaMalloc(&c->sh, sizeof(float4) * m * c->nplanes));
    if (n > 0) {
        const float* aos = reinterpret_cast<const float*>(src);
        float* tmp = nullptr;
        if (!src_on_device) {
            KT_TRY_CUDA(c, cudaMalloc(&tmp, sizeof(kt_gaussian3d) * n));
            KT_TRY_CUDA(c, cudaMemcpyAsync(tmp, src, sizeof(kt_gaussian3d) * n, cudaMemcpyHostToDevice, stream));
            aos = tmp;
        }
        cudaError_t e = launch_pack_scene(aos, n, c->pos, c->rot, c->scale, c->sh, deg, c->nplanes, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (tmp) cudaFree(tmp);
        KT_TRY_CUDA(c, e);
    }
    c->has_scene = true;
    return KT_OK;
}

// A frame rendered into a host image. With `clear` the device image is first set to that colour
// (the render pass's clear, renderpass.hpp:170) instead of being copied in from the host image.
kt_status render_host_impl(kt_gs_ctx* c, const kt_camera_mvp* cam, const uint8_t* clear, void* h_rgba8,
                           uint32_t path, void* stream) {
    if (!c) return KT_ERR_ARG;
    if (!cam || !h_rgba8) return fail(c, KT_ERR_ARG, "NULL camera or image");
    if (path >= c->paths.size()) return fail(c, KT_ERR_ARG, "path index out of range");
    KT_TRY_CUDA(c, cudaSetDevice(c->device));
    PathWs& w = c->paths[path];
    const uint64_t pixels = (uint64_t)c->cfg.width * c->cfg.height;
    const size_t bytes = pixels * 4;
    if (!w.img) KT_TRY_CUDA(c, cudaMalloc(&w.img, bytes));
    cudaStream_t s = (cudaStream_t)stream;
    if (clear)
        KT_TRY_CUDA(c, launch_fill_image(w.img, pixels, make_uchar4(clear[0], clear[1], clear[2], clear[3]), s));
    else
        KT_TRY_CUDA(c, cudaMemcpyAsync(w.img, h_rgba8, bytes, cudaMemcpyHostToDevice, s));
    if (c->cfg.flags & KT_GS_FLAG_ASYNC) {
        // frames in flight: everything is enqueued; kt_gs_sync(path) waits for the image copy too
        kt_status st = render_impl(c, path, Source::Scene, cam, w.img, s);
        if (st != KT_OK) return st;
        KT_TRY_CUDA(c, cudaMemcpyAsync(h_rgba8, w.img, bytes, cudaMemcpyDeviceToHost, s));
        KT_TRY_CUDA(c, cudaEventRecord(w.done_ev, s));
        return KT_OK;
    }
    const uint32_t saved = c->cfg.flags;
    c->cfg.flags &= ~KT_GS_FLAG_ASYNC;
    kt_status st = render_impl(c, path, Source::Scene, cam, w.img, s);
    c->cfg.flags = saved;
    if (st != KT_OK) return st;
    KT_TRY_CUDA(c, cudaMemcpyAsync(h_rgba8, w.img, bytes, cudaMemcpyDeviceToHost, s));
    KT_TRY_CUDA(c, cudaStreamSynchronize(s));
    return KT_OK;
}

// Elements [first, first + count) of a stage buffer of the path's last frame, copied to host
// memory (count is clipped to the stage's length). The default binning path has no device
// buffer for OFFSETS, KEYS_UNSORTED and VALUES_UNSORTED: those dumps are rebuilt here on the
// host from the device's counts, rectangles and depths (the reference's stage layout, for
// comparisons), and KEYS_SORTED is assembled from the device's pairs, bin ranges and depths.
kt_status dump_window(kt_gs_ctx* c, uint32_t path, kt_gs_stage stage, uint64_t first, uint64_t count, void* dst,
                      uint64_t bytes, uint64_t* written) {
    if (!c) return KT_ERR_ARG;
    if (written) *written = 0;
    if (path >= c->paths.size()) return fail(c, KT_ERR_ARG, "path index out of range");
    KT_TRY_CUDA(c, cudaSetDevice(c->device));
    PathWs& w = c->paths[path];
    if (!w.have_frame) return fail(c, KT_ERR_STATE, "no frame rendered on this path");
    KT_TRY_CUDA(c, cudaEventSynchronize(w.done_ev));
    const FrameCtl& h = *w.host_ctl;
    const uint64_t n = w.frame_n;
    const uint64_t K = h.num_keys;
    const bool sorted_ok = h.plan_ok != 0;
    const uint32_t tx = c->gp.tiles_x;
    const bool placed = !w.keys_frame;
    uint64_t len = 0, esize = 0;  // elements of the stage, bytes per element
    switch (stage) {
        case KT_GS_STAGE_PROJECTED: len = n; esize = sizeof(kt_gaussian2d); break;
        case KT_GS_STAGE_TILE_COUNTS: len = n; esize = 4; break;
        case KT_GS_STAGE_OFFSETS: len = n; esize = 8; break;
        case KT_GS_STAGE_KEYS_UNSORTED: len = K; esize = 8; break;
        case KT_GS_STAGE_VALUES_UNSORTED: len = K; esize = 4; break;
        case KT_GS_STAGE_KEYS_SORTED: len = K; esize = 8; break;
        case KT_GS_STAGE_VALUES_SORTED: len = K; esize = 4; break;
        case KT_GS_STAGE_TILE_RANGES: len = ntiles(c); esize = 8; break;
        case KT_GS_STAGE_DEPTH_ORDER: len = std::min<uint64_t>(h.num_visible, n); esize = 4; break;
        case KT_GS_STAGE_COARSE_INFO: len = w.last_ncoarse; esize = 16; break;
        case KT_GS_STAGE_COARSE_LISTS: len = h.num_entries; esize = 8; break;
        case KT_GS_STAGE_SEGMENT_COUNTS: len = h.num_segments; esize = 64; break;
        default: return fail(c, KT_ERR_ARG, "unknown stage");
    }
    const bool placement_stage = stage == KT_GS_STAGE_DEPTH_ORDER || stage == KT_GS_STAGE_COARSE_INFO ||
                                 stage == KT_GS_STAGE_COARSE_LISTS || stage == KT_GS_STAGE_SEGMENT_COUNTS;
    if (placement_stage && !placed)
        return fail(c, KT_ERR_STATE, "placement buffers exist only on the default binning path");
    if ((stage == KT_GS_STAGE_KEYS_SORTED || stage == KT_GS_STAGE_VALUES_SORTED ||
         stage == KT_GS_STAGE_COARSE_LISTS || stage == KT_GS_STAGE_SEGMENT_COUNTS) && !sorted_ok)
        return fail(c, KT_ERR_STATE, "the last frame was not sorted");
    if (first > len) return fail(c, KT_ERR_ARG, "first element beyond the stage's length");
    const uint64_t cnt = std::min(count, len - first);
    const uint64_t need = cnt * esize;
    if (!dst) {
        if (written) *written = need;
        return KT_OK;
    }
    if (bytes < need) return fail(c, KT_ERR_ARG, "buffer too small: need " + std::to_string(need) + " bytes");
    auto fetch = [&](const void* d, size_t nbytes, void* out) -> kt_status {
        if (nbytes) KT_TRY_CUDA(c, cudaMemcpy(out, d, nbytes, cudaMemcpyDeviceToHost));
        return KT_OK;
    };
    const uint64_t last = first + cnt;
    kt_status st = KT_OK;
    if (stage == KT_GS_STAGE_PROJECTED) {
        std::vector<float4> rec(3 * cnt);
        if ((st = fetch(w.rec + 3 * first, sizeof(float4) * 3 * cnt, rec.data())) != KT_OK) return st;
        kt_gaussian2d* o = (kt_gaussian2d*)dst;
        for (uint64_t i = 0; i < cnt; ++i) {
            const float4 a = rec[3 * i], b = rec[3 * i + 1], cc = rec[3 * i + 2];
            o[i].position[0] = a.x;
            o[i].position[1] = a.y;
            o[i].z = a.w;
            o[i].binMask = 0xFFFFFFFFu;
            o[i].covInv[0] = b.x;
            o[i].covInv[1] = b.y;
            o[i].covInv[2] = b.z;
            o[i].covInv[3] = b.w;
            o[i].color[0] = cc.x;
            o[i].color[1] = cc.y;
            o[i].color[2] = cc.z;
            o[i].alpha = a.z;
        }
    } else if (stage == KT_GS_STAGE_TILE_COUNTS) {
        if ((st = fetch(w.counts + first, need, dst)) != KT_OK) return st;
    } else if (stage == KT_GS_STAGE_TILE_RANGES) {
        if ((st = fetch(w.ranges + first, need, dst)) != KT_OK) return st;
    } else if (stage == KT_GS_STAGE_COARSE_INFO) {
        if ((st = fetch(w.cinfo + first, need, dst)) != KT_OK) return st;
    } else if (stage == KT_GS_STAGE_COARSE_LISTS) {
        if ((st = fetch(w.clist + first, need, dst)) != KT_OK) return st;
    } else if (stage == KT_GS_STAGE_SEGMENT_COUNTS) {
        if ((st = fetch(w.seg_cnt + 16 * first, need, dst)) != KT_OK) return st;
    } else if (stage == KT_GS_STAGE_DEPTH_ORDER) {
        // the depth sort's result: (depth - min) << idx_bits | index words in its final buffer
        FrameCtl cd;
        if ((st = fetch(w.ctl_depth, offsetof(FrameCtl, hist), &cd)) != KT_OK) return st;
        std::vector<unsigned long long> words(cnt);
        if ((st = fetch(w.gsort[cd.final_buf & 1u] + first, cnt * 8, words.data())) != KT_OK) return st;
        const unsigned long long imask = cd.idx_bits >= 64 ? ~0ull : (1ull << cd.idx_bits) - 1ull;
        for (uint64_t i = 0; i < cnt; ++i) ((uint32_t*)dst)[i] = (uint32_t)(words[i] & imask);
    } else if (stage == KT_GS_STAGE_OFFSETS && !placed) {
        if ((st = fetch(w.offsets + first, need, dst)) != KT_OK) return st;
    } else if (stage == KT_GS_STAGE_OFFSETS) {
        // host-rebuilt: the index-order exclusive scan of the device's counts
        std::vector<uint32_t> cn(last);
        if ((st = fetch(w.counts, last * 4, cn.data())) != KT_OK) return st;
        uint64_t run = 0;
        for (uint64_t i = 0; i < last; ++i) {
            if (i >= first) ((uint64_t*)dst)[i - first] = run;
            run += cn[i];
        }
    } else if ((stage == KT_GS_STAGE_KEYS_SORTED || stage == KT_GS_STAGE_VALUES_SORTED) && !placed) {
        if (stage == KT_GS_STAGE_VALUES_SORTED) {
            if ((st = fetch(w.vals[h.final_buf] + first, need, dst)) != KT_OK) return st;
        } else {
            // bin << depth_bits | (depth - depth_min)  ->  bin << 32 | depth, the reference's key
            if ((st = fetch(w.keys[h.final_buf] + first, need, dst)) != KT_OK) return st;
            unsigned long long* k = (unsigned long long*)dst;
            const uint32_t db = h.depth_bits;
            const unsigned long long dm = db ? ((1ull << db) - 1ull) : 0ull;
            for (uint64_t i = 0; i < cnt; ++i)
                k[i] = ((k[i] >> db) << 32) | (unsigned long long)((uint32_t)(k[i] & dm) + h.depth_min);
        }
    } else if (stage == KT_GS_STAGE_VALUES_SORTED) {
        if ((st = fetch(w.pairs + first, need, dst)) != KT_OK) return st;
    } else if (stage == KT_GS_STAGE_KEYS_SORTED) {
        // host-assembled: bin << 32 | depth bits, the bin of each pair read off the device's ranges
        std::vector<uint32_t> g(cnt), depth(n);
        std::vector<uint2> rng(ntiles(c));
        if ((st = fetch(w.pairs + first, cnt * 4, g.data())) != KT_OK) return st;
        if ((st = fetch(w.depth, n * 4, depth.data())) != KT_OK) return st;
        if ((st = fetch(w.ranges, rng.size() * 8, rng.data())) != KT_OK) return st;
        unsigned long long* k = (unsigned long long*)dst;
        for (uint64_t b = 0; b < rng.size(); ++b) {
            const uint64_t a = std::max<uint64_t>(rng[b].x, first), e = std::min<uint64_t>(rng[b].y, last);
            for (uint64_t i = a; i < e; ++i) {
                const uint32_t gi = g[i - first];
                k[i - first] = ((unsigned long long)b << 32) | (gi < n ? depth[gi] : 0u);
            }
        }
    } else {
        // host-rebuilt: pairs as the reference's binning would list them without its atomic
        // reordering (Gaussians in index order, bins ascending), from the device's rectangles
        std::vector<uint32_t> cn(n), depth(n);
        std::vector<uint2> rect(n);
        const bool is_keys = stage == KT_GS_STAGE_KEYS_UNSORTED;
        if ((st = fetch(w.counts, n * 4, cn.data())) != KT_OK) return st;
        if ((st = fetch(w.rect, n * 8, rect.data())) != KT_OK) return st;
        if ((st = fetch(w.depth, n * 4, depth.data())) != KT_OK) return st;
        uint64_t o = 0;
        for (uint64_t g = 0; g < n && o < last; ++g) {
            if (!cn[g]) continue;
            if (o + cn[g] <= first) {
                o += cn[g];
                continue;
            }
            const uint32_t x0 = rect[g].x & 0xFFFFu, x1 = rect[g].x >> 16;
            const uint32_t y0 = rect[g].y & 0xFFFFu, y1 = rect[g].y >> 16;
            for (uint32_t y = y0; y < y1; ++y)
                for (uint32_t x = x0; x < x1 && o < last; ++x, ++o) {
                    if (o < first) continue;
                    if (is_keys)
                        ((unsigned long long*)dst)[o - first] = ((unsigned long long)(y * tx + x) << 32) | depth[g];
                    else
                        ((uint32_t*)dst)[o - first] = (uint32_t)g;
                }
        }
    }
    if (written) *written = need;
    return KT_OK;
}

}  // namespace

// ======================================================================= C ABI

extern "C" {

void kt_gs_config_default(kt_gs_config* cfg) {
    if (!cfg) return;
    std::memset(cfg, 0, sizeof(*cfg));
    cfg->width = 512;
    cfg->height = 512;
    cfg->bin_width = 128;
    cfg->bin_height = 128;
    cfg->sh_degree = 3;
    cfg->cull_z = 1.0f;
    cfg->flags = 0;
    cfg->num_paths = 1;
    cfg->key_capacity = 0;
    cfg->tile_row_begin = 0;
    cfg->tile_row_end = 0;
}

int kt_gs_abi_version(void) { return KT_GS_ABI_VERSION; }

const char* kt_gs_status_string(kt_status s) {
    switch (s) {
        case KT_OK: return "KT_OK";
        case KT_ERR_ARG: return "KT_ERR_ARG";
        case KT_ERR_CUDA: return "KT_ERR_CUDA";
        case KT_ERR_CAPACITY: return "KT_ERR_CAPACITY";
        case KT_ERR_TIMEOUT: return "KT_ERR_TIMEOUT";
        case KT_ERR_NCCL: return "KT_ERR_NCCL";
        case KT_ERR_IO: return "KT_ERR_IO";
        case KT_ERR_STATE: return "KT_ERR_STATE";
        case KT_ERR_NOMEM: return "KT_ERR_NOMEM";
    }
    return "KT_ERR_UNKNOWN";
}

kt_status kt_gs_create(const kt_gs_config* cfg, int device, kt_gs_ctx** out) {
    if (!cfg || !out) return KT_ERR_ARG;
    *out = nullptr;
    if (cfg->width == 0 || cfg->height == 0 || cfg->width > 65535 * 16 || cfg->height > 65535 * 16)
        return KT_ERR_ARG;
    if (cfg->bin_width == 0 || cfg->bin_height == 0 || cfg->bin_width % 16 != 0 ||
        cfg->bin_height % 16 != 0)
        return KT_ERR_ARG;
    if (cfg->sh_degree < -1 || cfg->sh_degree > 3) return KT_ERR_ARG;
    if (cfg->num_paths == 0 || cfg->num_paths > 16) return KT_ERR_ARG;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return KT_ERR_CUDA;
    if (cudaSetDevice(device) != cudaSuccess) return KT_ERR_CUDA;
    kt_gs_ctx* c = new (std::nothrow) kt_gs_ctx();
    if (!c) return KT_ERR_NOMEM;
    c->cfg = *cfg;
    c->device = device;
    c->gp = make_grid(*cfg);
    c->paths.resize(cfg->num_paths);
    *out = c;
    return KT_OK;
}

kt_status kt_gs_destroy(kt_gs_ctx* c) {
    if (!c) return KT_OK;
    cudaSetDevice(c->device);
    for (auto& w : c->paths) {
        if (w.have_frame && w.done_ev) cudaEventSynchronize(w.done_ev);
        free_path(w);
    }
    dfree(c->pos); dfree(c->rot); dfree(c->scale); dfree(c->sh);
    delete c;
    return KT_OK;
}

const char* kt_gs_last_error(const kt_gs_ctx* c) { return c ? c->err.c_str() : "null context"; }

kt_status kt_gs_get_config(const kt_gs_ctx* c, kt_gs_config* cfg) {
    if (!c || !cfg) return KT_ERR_ARG;
    *cfg = c->cfg;
    if (c->has_scene) cfg->sh_degree = c->deg;
    return KT_OK;
}

kt_status kt_gs_set_gaussians(kt_gs_ctx* c, const kt_gaussian3d* host, uint64_t n) {
    if (!c) return KT_ERR_ARG;
    if (n > 0 && !host) return fail(c, KT_ERR_ARG, "NULL Gaussian array");
    if (n > 0xFFFFFFFFull) return fail(c, KT_ERR_ARG, "more than 2^32-1 Gaussians");
    const int deg = c->cfg.sh_degree >= 0 ? c->cfg.sh_degree : detect_degree(host, n);
    return upload_scene(c, host, false, n, deg, nullptr);
}

kt_status kt_gs_set_gaussians_device(kt_gs_ctx* c, const kt_gaussian3d* dev, uint64_t n,
                                     void* stream) {
    if (!c) return KT_ERR_ARG;
    if (n > 0 && !dev) return fail(c, KT_ERR_ARG, "NULL Gaussian array");
    if (n > 0xFFFFFFFFull) return fail(c, KT_ERR_ARG, "more than 2^32-1 Gaussians");
    const int deg = c->cfg.sh_degree >= 0 ? c->cfg.sh_degree : 3;
    return upload_scene(c, dev, true, n, deg, (cudaStream_t)stream);
}

kt_status kt_gs_render(kt_gs_ctx* c, const kt_camera_mvp* cam, void* d_rgba8, uint32_t path,
                       void* stream) {
    if (!c) return KT_ERR_ARG;
    if (!cam) return fail(c, KT_ERR_ARG, "camera is NULL");
    return render_impl(c, path, Source::Scene, cam, (uchar4*)d_rgba8, (cudaStream_t)stream);
}

kt_status kt_gs_render_host(kt_gs_ctx* c, const kt_camera_mvp* cam, void* h_rgba8, uint32_t path,
                            void* stream) {
    return render_host_impl(c, cam, nullptr, h_rgba8, path, stream);
}

kt_status kt_gs_render_host_clear(kt_gs_ctx* c, const kt_camera_mvp* cam, const uint8_t clear_rgba[4],
                                  void* h_rgba8, uint32_t path, void* stream) {
    if (!clear_rgba) return c ? fail(c, KT_ERR_ARG, "NULL clear colour") : KT_ERR_ARG;
    return render_host_impl(c, cam, clear_rgba, h_rgba8, path, stream);
}

kt_status kt_gs_render_batch(kt_gs_ctx* c, const kt_camera_mvp* cams, uint32_t n_views,
                             void* const* d_rgba8, void* stream) {
    if (!c) return KT_ERR_ARG;
    if (n_views > 0 && (!cams || !d_rgba8)) return fail(c, KT_ERR_ARG, "NULL cameras or images");
    for (uint32_t v = 0; v < n_views; ++v) {
        kt_status s = render_impl(c, 0, Source::Scene, &cams[v], (uchar4*)d_rgba8[v], (cudaStream_t)stream);
        if (s != KT_OK) return s;
    }
    return KT_OK;
}

kt_status kt_gs_render_projected(kt_gs_ctx* c, const kt_gaussian2d* host, uint64_t n,
                                 void* d_rgba8, uint32_t path, void* stream) {
    if (!c) return KT_ERR_ARG;
    if (n > 0 && !host) return fail(c, KT_ERR_ARG, "NULL record array");
    if (n > 0xFFFFFFFFull) return fail(c, KT_ERR_ARG, "more than 2^32-1 records");
    if (path >= c->paths.size()) return fail(c, KT_ERR_ARG, "path index out of range");
    KT_TRY_CUDA(c, cudaSetDevice(c->device));
    PathWs& w = c->paths[path];
    if (n > w.g2d_n || !w.g2d) {
        ++w.buf_gen;
        dfree(w.g2d);
        KT_TRY_CUDA(c, cudaMalloc(&w.g2d, sizeof(kt_gaussian2d) * std::max<uint64_t>(n, 1)));
    }
    w.g2d_n = n;
    cudaStream_t s = (cudaStream_t)stream;
    if (n) KT_TRY_CUDA(c, cudaMemcpyAsync(w.g2d, host, sizeof(kt_gaussian2d) * n, cudaMemcpyHostToDevice, s));
    return render_impl(c, path, Source::Projected, nullptr, (uchar4*)d_rgba8, s);
}

kt_status kt_gs_sync(kt_gs_ctx* c, uint32_t path) {
    if (!c) return KT_ERR_ARG;
    if (path >= c->paths.size()) return fail(c, KT_ERR_ARG, "path index out of range");
    KT_TRY_CUDA(c, cudaSetDevice(c->device));
    PathWs& w = c->paths[path];
    if (!w.have_frame || !w.totals) return KT_OK;
    KT_TRY_CUDA(c, cudaEventSynchronize(w.done_ev));
    // every frame folds its error bits into the sticky word; checked frames clear what they
    // already reported, so each error is reported once
    unsigned int sticky = 0;
    KT_TRY_CUDA(c, cudaMemcpy(&sticky, &w.totals->sticky_errors, sizeof(sticky), cudaMemcpyDeviceToHost));
    KT_TRY_CUDA(c, cudaMemset(&w.totals->sticky_errors, 0, sizeof(sticky)));
    if (sticky & kErrTimeout) return fail(c, KT_ERR_TIMEOUT, "a frame since the last sync timed out in a look-back wait");
    if (sticky & kErrCapacity)
        return fail(c, KT_ERR_CAPACITY, "a frame since the last sync overflowed the key buffers (nothing drawn)");
    return KT_OK;
}

kt_status kt_gs_frame_stats(kt_gs_ctx* c, uint32_t path, kt_gs_stats* out) {
    if (!c || !out) return KT_ERR_ARG;
    if (path >= c->paths.size()) return fail(c, KT_ERR_ARG, "path index out of range");
    KT_TRY_CUDA(c, cudaSetDevice(c->device));
    PathWs& w = c->paths[path];
    std::memset(out, 0, sizeof(*out));
    out->tiles_x = c->gp.tiles_x;
    out->tiles_y = c->gp.tiles_y;
    out->key_capacity = w.cap;
    if (!w.have_frame) return KT_OK;
    KT_TRY_CUDA(c, cudaEventSynchronize(w.done_ev));
    const FrameCtl& h = *w.host_ctl;
    out->num_gaussians = w.frame_n;
    out->num_keys = h.num_keys;
    out->num_visible = h.num_visible;
    out->key_bits = h.key_bits;
    out->depth_bits = h.depth_bits;
    out->sort_passes = h.passes_run;
    out->error_flags = h.error_flags;
    out->depth_min_bits = h.depth_min;
    out->depth_max_bits = h.depth_max;
    out->status_bytes = (uint32_t)kCtlHeaderBytes;
    // init, project, depth keys (+ plan), the depth passes, coarse count, coarse scan (+ list
    // starts), coarse placement, bin count (+ bin ranges), pair placement, totals, rasterise; or
    // init, project, scan/emit, plan, the key passes, ranges, totals, rasterise
    out->launches = w.keys_frame ? 7 + key_passes(c) * sort_pass_launches(w.cap, false)
                                 : 10 + kDepthPasses * sort_pass_launches(w.frame_n, true);
    out->packed = h.packed;
    out->idx_bits = h.idx_bits;
    PlaceGeom pg{};
    if (place_geometry(c->gp, w.frame_n, w.cap, &pg) == cudaSuccess) {
        out->place_chunks = pg.nchunks;
        out->place_bands = h.place_nbands ? h.place_nbands : pg.nbands;  // the device's choice for the frame
    }
    out->place_runs = (!w.keys_frame && w.place_runs) ? 1u : 0u;
    return KT_OK;
}

kt_status kt_gs_counters_take(kt_gs_ctx* c, uint32_t path, kt_gs_counters* out) {
    if (!c || !out) return KT_ERR_ARG;
    if (path >= c->paths.size()) return fail(c, KT_ERR_ARG, "path index out of range");
    KT_TRY_CUDA(c, cudaSetDevice(c->device));
    PathWs& w = c->paths[path];
    std::memset(out, 0, sizeof(*out));
    if (!w.totals) return KT_OK;
    if (w.have_frame) KT_TRY_CUDA(c, cudaEventSynchronize(w.done_ev));
    FrameTotals t;
    KT_TRY_CUDA(c, cudaMemcpy(&t, w.totals, sizeof(t), cudaMemcpyDeviceToHost));
    out->frames = t.frames;
    out->keys = t.keys;
    out->key_passes = t.key_passes;
    out->visible = t.visible;
    out->sort_bytes = t.sort_bytes;
    out->depth_sort_bytes = t.depth_sort_bytes;
    // reset the counters; the sticky error bits stay until kt_gs_sync reports them
    KT_TRY_CUDA(c, cudaMemset(w.totals, 0, offsetof(FrameTotals, sticky_errors)));
    return KT_OK;
}

kt_status kt_gs_set_flags(kt_gs_ctx* c, uint32_t flags) {
    if (!c) return KT_ERR_ARG;
    c->cfg.flags = flags;
    return KT_OK;
}

kt_status kt_gs_debug_dump(kt_gs_ctx* c, uint32_t path, kt_gs_stage stage, void* dst,
                           uint64_t bytes, uint64_t* written) {
    return dump_window(c, path, stage, 0, UINT64_MAX, dst, bytes, written);
}

kt_status kt_gs_debug_dump_range(kt_gs_ctx* c, uint32_t path, kt_gs_stage stage, uint64_t first,
                                 uint64_t count, void* dst, uint64_t bytes, uint64_t* written) {
    return dump_window(c, path, stage, first, count, dst, bytes, written);
}

kt_status kt_gs_stage_times(kt_gs_ctx* c, uint32_t path, float ms[KT_GS_NSTAGES]) {
    if (!c || !ms) return KT_ERR_ARG;
    if (path >= c->paths.size()) return fail(c, KT_ERR_ARG, "path index out of range");
    PathWs& w = c->paths[path];
    if (!w.have_frame || !w.timed) return fail(c, KT_ERR_STATE, "no timed frame (KT_GS_FLAG_TIMING)");
    KT_TRY_CUDA(c, cudaSetDevice(c->device));
    KT_TRY_CUDA(c, cudaEventSynchronize(w.done_ev));
    cudaEvent_t* ev = w.ring[w.ring_last];
    constexpr int L = KT_GS_NSTAGES - 1;
    KT_TRY_CUDA(c, cudaEventSynchronize(ev[L]));
    for (int i = 0; i < L; ++i) KT_TRY_CUDA(c, cudaEventElapsedTime(&ms[i], ev[i], ev[i + 1]));
    KT_TRY_CUDA(c, cudaEventElapsedTime(&ms[L], ev[0], ev[L]));
    return KT_OK;
}

kt_status kt_gs_stage_times_total(kt_gs_ctx* c, uint32_t path, double ms_total[KT_GS_NSTAGES],
                                  uint64_t* frames) {
    if (!c || !ms_total) return KT_ERR_ARG;
    if (path >= c->paths.size()) return fail(c, KT_ERR_ARG, "path index out of range");
    KT_TRY_CUDA(c, cudaSetDevice(c->device));
    PathWs& w = c->paths[path];
    for (int k = 0; k < PathWs::kRing; ++k) {
        const int slot = (w.ring_next + k) % PathWs::kRing;  // oldest first
        kt_status s = drain_slot(c, w, slot);
        if (s != KT_OK) return s;
    }
    for (int i = 0; i < KT_GS_NSTAGES; ++i) {
        ms_total[i] = w.stage_sum[i];
        w.stage_sum[i] = 0.0;
    }
    if (frames) *frames = w.timed_frames;
    w.timed_frames = 0;
    return KT_OK;
}

kt_status kt_gs_load_spz(kt_gs_ctx* c, const char* path) {
    if (!c || !path) return KT_ERR_ARG;
    uint64_t n = 0;
    uint32_t deg = 0;
    kt_status s = kt_gs_spz_decode(path, nullptr, 0, &n, &deg);
    if (s != KT_OK) return fail(c, s, std::string("cannot read spz file ") + path);
    std::vector<kt_gaussian3d> g;
    try {
        g.resize(n);
    } catch (const std::bad_alloc&) {
        return fail(c, KT_ERR_NOMEM, "no host memory for the spz records");
    }
    s = kt_gs_spz_decode(path, g.data(), n, &n, &deg);
    if (s != KT_OK) return fail(c, s, std::string("cannot decode spz file ") + path);
    return kt_gs_set_gaussians(c, g.data(), n);
}

kt_status kt_gs_load_ply(kt_gs_ctx* c, const char* path) {
    if (!c || !path) return KT_ERR_ARG;
    uint64_t n = 0;
    kt_status s = kt_gs_ply_decode(path, nullptr, 0, &n);
    if (s != KT_OK) return fail(c, s, std::string("cannot read ply file ") + path);
    std::vector<kt_gaussian3d> g;
    try {
        g.resize(n);
    } catch (const std::bad_alloc&) {
        return fail(c, KT_ERR_NOMEM, "no host memory for the ply records");
    }
    s = kt_gs_ply_decode(path, g.data(), n, &n);
    if (s != KT_OK) return fail(c, s, std::string("cannot decode ply file ") + path);
    return kt_gs_set_gaussians(c, g.data(), n);
}

kt_status kt_gs_radix_sort_pairs(const uint64_t* keys_in, const uint32_t* vals_in,
                                 uint64_t* keys_out, uint32_t* vals_out, uint64_t n,
                                 uint32_t key_bits, void* d_temp, size_t* temp_bytes,
                                 void* stream) {
    if (!temp_bytes || key_bits > 64) return KT_ERR_ARG;
    const size_t ctl_bytes = (sizeof(FrameCtl) + 255) & ~size_t(255);
    const size_t kbytes = ((size_t)n * 8 + 255) & ~size_t(255);
    const size_t vbytes = ((size_t)n * 4 + 255) & ~size_t(255);
    const size_t sbytes = sort_status_words(n) * 8;
    const size_t total = ctl_bytes + kbytes + vbytes + sbytes;
    if (!d_temp) {
        *temp_bytes = total;
        return KT_OK;
    }
    if (*temp_bytes < total) return KT_ERR_ARG;
    if (n == 0) return KT_OK;
    if (n > kMaxKeyCapacity || !keys_in || !vals_in || !keys_out || !vals_out) return KT_ERR_ARG;
    if ((const void*)keys_out == (const void*)keys_in || (const void*)vals_out == (const void*)vals_in)
        return KT_ERR_ARG;  // in place would race between the CTAs of a single-pass sort
    cudaStream_t s = (cudaStream_t)stream;
    unsigned char* t = (unsigned char*)d_temp;
    FrameCtl* ctl = (FrameCtl*)t;
    unsigned long long* alt_k = (unsigned long long*)(t + ctl_bytes);
    uint32_t* alt_v = (uint32_t*)(t + ctl_bytes + kbytes);
    unsigned long long* status = (unsigned long long*)(t + ctl_bytes + kbytes + vbytes);
    const uint32_t max_passes = std::max<uint32_t>(1, (key_bits + 7) / 8);
    if (cudaMemsetAsync(ctl, 0, sizeof(FrameCtl), s) != cudaSuccess) return KT_ERR_CUDA;
    if (cudaMemsetAsync(status, 0, sbytes, s) != cudaSuccess) return KT_ERR_CUDA;
    if (launch_key_histogram((const unsigned long long*)keys_in, n, key_bits, ctl, s) != cudaSuccess)
        return KT_ERR_CUDA;
    if (launch_plan(ctl, n, max_passes, 1, s) != cudaSuccess) return KT_ERR_CUDA;
    SortIO io{};
    io.keys[0] = (unsigned long long*)keys_in;
    io.keys[1] = alt_k;
    io.keys[2] = (unsigned long long*)keys_out;
    io.vals[0] = (uint32_t*)vals_in;
    io.vals[1] = alt_v;
    io.vals[2] = vals_out;
    // Every pass of one call takes the same algorithm (it depends on n only) and the status words
    // were cleared above, so they can also hold the reduce-then-scan table of a large call.
    for (uint32_t p = 0; p < max_passes; ++p)
        if (launch_sort_pass(io, ctl, status, (uint32_t*)status, p, p + 1, n, false, s) != cudaSuccess)
            return KT_ERR_CUDA;
    return KT_OK;
}

}  // extern "C"
