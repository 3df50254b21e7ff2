// kt_gs_radix_sort_pairs_static: the pair sort of kt_gs_radix_sort_pairs for callers that
// cannot allocate device memory, with its scratch in a fixed array of this module.
//
// Some callers cannot call cudaMalloc: a render loop with a fixed frame budget (an allocation
// or free may synchronise the whole device), a plugin inside a host engine whose own allocator
// owns all device memory, or a process whose memory pool already holds the device's free
// memory. They pass their inputs and outputs; the scratch (control block, the second key and
// value buffers, look-back status words) lives in g_sort_scratch below.
//
// The array is KT_GS_STATIC_SORT_SCRATCH_BYTES (13,127,680 bytes, 12.52 MiB) and every device that
// loads this module keeps it until the process exits. In host code the name g_sort_scratch is
// only a host-side stand-in for the symbol, not a device address: every call looks the device
// address up with cudaGetSymbolAddress on the current device (the first call on a device also
// loads the module there, which is why that first call should come before any stream capture;
// looking it up each time keeps it right after a cudaDeviceReset reloads the module elsewhere).
// All calls share the one array: calls whose work overlaps on the GPU race on it and must be
// ordered by the caller (e.g. one stream). Each call clears what must start at zero (the
// control block and the status words it uses); the rest keeps the previous call's contents
// and is overwritten before it is read.
//
// kt_gs_radix_sort_status reports a sort's device error bits (a look-back wait that ran out)
// from the control block of either entry point's scratch; kt_gs_radix_sort_static_timeout_probe
// makes that wait run out on purpose (a status word that nothing publishes), so that the
// reporting path can be checked without a faulty sort.
#include "kt_common.cuh"
#include "kt_gs.h"
#include "kt_kernels.h"

namespace kt {
namespace {

constexpr uint64_t kStaticMaxPairs = KT_GS_STATIC_SORT_MAX_PAIRS;
constexpr size_t kCtlBytes = 20480;  // control block region, fixed so the array's size is stable
static_assert(sizeof(FrameCtl) <= kCtlBytes, "control block outgrew its region");
constexpr size_t kKeyBytes = kStaticMaxPairs * 8;
constexpr size_t kValBytes = kStaticMaxPairs * 4;
constexpr size_t kStatusBytes = (kStaticMaxPairs / kSortTile) * 256 * 8;
constexpr size_t kScratchBytes = kCtlBytes + kKeyBytes + kValBytes + kStatusBytes;
static_assert(kScratchBytes == KT_GS_STATIC_SORT_SCRATCH_BYTES, "scratch size in kt_gs.h is stale");
static_assert(kStaticMaxPairs % kSortTile == 0, "maximum must be a whole number of sort tiles");

static __device__ __align__(256) unsigned char g_sort_scratch[kScratchBytes];

// Device address of the scratch on the current device. Looked up on every call: the lookup is a
// host-side table read once the module is loaded, and a cached address would go stale when
// cudaDeviceReset unloads the module.
cudaError_t scratch_address(unsigned char** out) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_sort_scratch);
    if (e != cudaSuccess) return e;
    *out = (unsigned char*)p;
    return cudaSuccess;
}

}  // namespace
}  // namespace kt

using namespace kt;

extern "C" kt_status kt_gs_radix_sort_pairs_static(const uint64_t* keys_in, const uint32_t* vals_in,
                                                   uint64_t* keys_out, uint32_t* vals_out, uint64_t n,
                                                   uint32_t key_bits, void* stream) {
    if (key_bits > 64) return KT_ERR_ARG;
    if (n > kStaticMaxPairs) return KT_ERR_CAPACITY;  // more pairs than the fixed scratch holds
    if (n == 0) return KT_OK;
    if (!keys_in || !vals_in || !keys_out || !vals_out) return KT_ERR_ARG;
    if ((const void*)keys_out == (const void*)keys_in || (const void*)vals_out == (const void*)vals_in)
        return KT_ERR_ARG;  // in place would race between the CTAs of a single-pass sort
    unsigned char* t = nullptr;
    if (scratch_address(&t) != cudaSuccess) return KT_ERR_CUDA;
    cudaStream_t s = (cudaStream_t)stream;
    FrameCtl* ctl = (FrameCtl*)t;
    unsigned long long* alt_k = (unsigned long long*)(t + kCtlBytes);
    uint32_t* alt_v = (uint32_t*)(t + kCtlBytes + kKeyBytes);
    unsigned long long* status = (unsigned long long*)(t + kCtlBytes + kKeyBytes + kValBytes);
    const uint32_t max_passes = key_bits == 0 ? 1u : (key_bits + 7) / 8;
    if (cudaMemsetAsync(ctl, 0, sizeof(FrameCtl), s) != cudaSuccess) return KT_ERR_CUDA;
    if (cudaMemsetAsync(status, 0, sort_status_words(n) * 8, s) != cudaSuccess) return KT_ERR_CUDA;
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

extern "C" kt_status kt_gs_radix_sort_status(const void* d_temp, void* stream) {
    const unsigned char* base = (const unsigned char*)d_temp;
    if (!base) {
        unsigned char* t = nullptr;
        if (scratch_address(&t) != cudaSuccess) return KT_ERR_CUDA;
        base = t;
    }
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return KT_ERR_CUDA;
    unsigned int flags = 0;
    if (cudaMemcpy(&flags, base + offsetof(FrameCtl, error_flags), sizeof(flags), cudaMemcpyDeviceToHost) !=
        cudaSuccess)
        return KT_ERR_CUDA;
    if (flags & kErrTimeout) return KT_ERR_TIMEOUT;
    return KT_OK;
}

extern "C" kt_status kt_gs_radix_sort_static_timeout_probe(uint32_t spin_limit, void* stream) {
    if (spin_limit == 0 || spin_limit > kSpinLimit) return KT_ERR_ARG;
    unsigned char* t = nullptr;
    if (scratch_address(&t) != cudaSuccess) return KT_ERR_CUDA;
    cudaStream_t s = (cudaStream_t)stream;
    FrameCtl* ctl = (FrameCtl*)t;
    unsigned long long* status = (unsigned long long*)(t + kCtlBytes + kKeyBytes + kValBytes);
    // tile 0's words cleared: epoch 0 and no flag, an entry no look-back accepts
    if (cudaMemsetAsync(ctl, 0, sizeof(FrameCtl), s) != cudaSuccess) return KT_ERR_CUDA;
    if (cudaMemsetAsync(status, 0, 256 * 8, s) != cudaSuccess) return KT_ERR_CUDA;
    if (launch_lookback_timeout_probe(status, ctl, spin_limit, s) != cudaSuccess) return KT_ERR_CUDA;
    return KT_OK;
}
