// sort_no_alloc.cu — gs3d_sort_pairs_no_alloc: the stable pair sort of sort_pairs with its
// scratch in this library's own static device memory instead of caller-provided temp storage.
//
// Who needs it: a caller that cannot hand the library a temporary device buffer. A plain C or
// Julia render loop that keeps its device memory fixed across frames, or that must not call
// into its allocator while a frame is in flight (CUDA.jl's pool may run the garbage collector
// to satisfy an allocation, which stalls the frame), has nowhere to get the temp storage that
// sort_pairs wants; the reference itself reallocates that buffer inside render!
// (forward_core.jl:639-642). This entry point takes no buffer and allocates nothing.
//
// Limits and rules:
//  * at most GS3D_SORT_NO_ALLOC_MAX_ITEMS (2^20) pairs per call; larger calls are rejected
//    with GS3D_ERR_INVALID_ARGUMENT before anything is launched;
//  * the scratch is one array per device, shared by every call on that device: two calls
//    whose work overlaps on the device (different streams without an event between them, or
//    different host threads) race on it and produce garbage. Calls on one stream are safe;
//  * the scratch occupies kScratchBytes of device memory on each device where this module is
//    loaded: under CUDA's default lazy module loading (CUDA_MODULE_LOADING=LAZY) that is the
//    first call of this entry point on the device, otherwise the library's load;
//  * no part of the scratch has to start at zero: the one region the sort accumulates into
//    (the per-digit histograms) is cleared by every call on its own stream before use, and the
//    other regions are fully written before they are read;
//  * every call with nb_items > 0 looks the scratch address of the current device up
//    (cudaGetSymbolAddress, which on the first call also loads this module's device code on that
//    device). Nothing is cached across calls, so a device reset or a new primary context between
//    calls is harmless. Make the first call on a device before capturing any stream on it.
#include "common.cuh"
#include "internal.h"

namespace gs3d {
namespace {

// 2^20 pairs need 12,853,504 bytes of sort scratch (8 MiB of alternate keys, 4 MiB of alternate
// values, 256 tiles x 256 digit counters, 8 x 256 global counters, each region 256-aligned);
// 13 MiB leaves room for the alignment of every region. The first call checks the fit.
constexpr size_t kScratchBytes = (size_t)13 << 20;

static __device__ __align__(256) unsigned char g_sort_scratch[kScratchBytes];

// Address of the current device's scratch. Looked up on every call (a cheap host-side query)
// rather than cached, because a cached address goes stale when the device's context is torn
// down and re-created (cudaDeviceReset), after which it would point at memory this module no
// longer owns.
int scratch_for_current_device(void** out) {
    const size_t need = radix_sort_workspace_bytes(GS3D_SORT_NO_ALLOC_MAX_ITEMS);
    if (need > kScratchBytes)
        return set_error("gs3d_sort_pairs_no_alloc: static scratch of %zu bytes is smaller "
                         "than the %zu bytes %d pairs need",
                         kScratchBytes, need, GS3D_SORT_NO_ALLOC_MAX_ITEMS),
               GS3D_ERR_UNSUPPORTED;
    void* p = nullptr;
    GS3D_CUDA(cudaGetSymbolAddress(&p, g_sort_scratch), "cudaGetSymbolAddress(sort scratch)");
    if (!p || (reinterpret_cast<uintptr_t>(p) & 255u) != 0)
        return set_error("gs3d_sort_pairs_no_alloc: scratch address %p is not 256-aligned", p),
               GS3D_ERR_CUDA;
    *out = p;
    return GS3D_OK;
}

}  // namespace
}  // namespace gs3d

extern "C" GS3D_API int gs3d_sort_pairs_no_alloc(const int64_t* keys_in, int64_t* keys_out,
                                                 const int32_t* values_in, int32_t* values_out,
                                                 int nb_items, int highest_key_bit,
                                                 gs3d_stream_t stream) {
    using namespace gs3d;
    if (nb_items < 0) return invalid("gs3d_sort_pairs_no_alloc: nb_items = %d", nb_items);
    if (nb_items > GS3D_SORT_NO_ALLOC_MAX_ITEMS)
        return invalid("gs3d_sort_pairs_no_alloc: nb_items = %d exceeds the fixed scratch limit "
                       "of %d pairs; use sort_pairs with caller-provided temp storage",
                       nb_items, GS3D_SORT_NO_ALLOC_MAX_ITEMS);
    if (nb_items == 0) return GS3D_OK;
    if (!keys_in || !keys_out || !values_in || !values_out)
        return invalid("gs3d_sort_pairs_no_alloc: NULL pointer");
    void* scratch = nullptr;
    GS3D_RETURN_IF(scratch_for_current_device(&scratch));
    return radix_sort_pairs(scratch, kScratchBytes, keys_in, keys_out, values_in, values_out,
                            nb_items, nullptr, nb_items, highest_key_bit,
                            reinterpret_cast<cudaStream_t>(stream));
}
