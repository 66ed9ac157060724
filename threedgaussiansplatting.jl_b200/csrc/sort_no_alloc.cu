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
//  * the scratch occupies kScratchBytes of device memory on each device where this library's
//    device code is loaded, whether or not this entry point is ever called;
//  * no part of the scratch has to start at zero: the one region the sort accumulates into
//    (the per-digit histograms) is cleared by every call on its own stream before use, and the
//    other regions are fully written before they are read;
//  * the first call with nb_items > 0 on a device does per-device setup on the host: it looks
//    the scratch address up (cudaGetSymbolAddress, which also loads this library's device code
//    on that device if it is not yet loaded) and sets the sort kernel's shared-memory limit.
//    Make that first call before capturing any stream on the device.
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace gs3d {
namespace {

// 2^20 pairs need 12,853,504 bytes of sort scratch (8 MiB of alternate keys, 4 MiB of alternate
// values, 256 tiles x 256 digit counters, 8 x 256 global counters, each region 256-aligned);
// 13 MiB leaves room for the alignment of every region. The first call checks the fit.
constexpr size_t kScratchBytes = (size_t)13 << 20;

static __device__ __align__(256) unsigned char g_sort_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Address of this device's scratch, looked up once per device (the device must be current).
int scratch_for_current_device(void** out) {
    int dev = -1;
    GS3D_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices)
        return set_error("gs3d_sort_pairs_no_alloc: device ordinal %d outside [0, %d)", dev,
                         kMaxDevices),
               GS3D_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_scratch_ptr[dev]) {
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
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
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
