// abi.cu — error plumbing, version, and the drop-in replacement of the reference's only
// native component, deps/cub_sort_pairs/cub_sort_pairs_wrapper.cu (sort_pairs and
// determine_sort_pairs_temp_storage, same signatures, bound by forward_core.jl:629-659).
#include <cstdarg>
#include <cstdlib>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace gs3d {

namespace {
thread_local char g_error[512] = "no error";
}

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
}

int cuda_fail(cudaError_t e, const char* what) {
    set_error("CUDA error in %s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
    return GS3D_ERR_CUDA;
}

int invalid(const char* fmt, ...) {
    char buf[400];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    set_error("invalid argument: %s", buf);
    return GS3D_ERR_INVALID_ARGUMENT;
}

namespace {
struct ProfRecord {
    const char* stage;
    cudaEvent_t start, stop;
    bool closed;
};
bool g_prof_enabled = false;
std::vector<ProfRecord> g_prof;
std::vector<cudaEvent_t> g_event_pool;

cudaEvent_t pool_event() {
    if (!g_event_pool.empty()) {
        cudaEvent_t e = g_event_pool.back();
        g_event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}
}  // namespace

void prof_begin(const char* stage, cudaStream_t stream) {
    if (!g_prof_enabled) return;
    ProfRecord r{stage, pool_event(), pool_event(), false};
    cudaEventRecord(r.start, stream);
    g_prof.push_back(r);
}

void prof_end(const char* stage, cudaStream_t stream) {
    if (!g_prof_enabled) return;
    for (auto it = g_prof.rbegin(); it != g_prof.rend(); ++it)
        if (!it->closed && std::strcmp(it->stage, stage) == 0) {
            cudaEventRecord(it->stop, stream);
            it->closed = true;
            return;
        }
}

int device_sm_count() {
    int dev = 0, sms = kSMs;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

}  // namespace gs3d

using namespace gs3d;

extern "C" {

GS3D_API const char* gs3d_last_error_string(void) { return g_error; }

GS3D_API int gs3d_version(void) { return 1; }

GS3D_API int gs3d_profile_enable(int enable) {
    for (auto& r : g_prof) {
        g_event_pool.push_back(r.start);
        g_event_pool.push_back(r.stop);
    }
    g_prof.clear();
    g_prof_enabled = enable != 0;
    return GS3D_OK;
}

GS3D_API int gs3d_profile_report(char* buf, size_t len) {
    if (!buf || len == 0) return invalid("NULL report buffer");
    struct Acc { const char* stage; int n; double ms; };
    std::vector<Acc> acc;
    for (auto& r : g_prof) {
        if (!r.closed) continue;
        GS3D_CUDA(cudaEventSynchronize(r.stop), "profile event");
        float ms = 0.0f;
        GS3D_CUDA(cudaEventElapsedTime(&ms, r.start, r.stop), "profile elapsed");
        auto it = std::find_if(acc.begin(), acc.end(),
                               [&](const Acc& a) { return std::strcmp(a.stage, r.stage) == 0; });
        if (it == acc.end()) acc.push_back({r.stage, 1, ms});
        else { it->n += 1; it->ms += ms; }
    }
    size_t off = 0;
    buf[0] = 0;
    for (auto& a : acc) {
        const int w = snprintf(buf + off, len - off, "%s %d %.6f\n", a.stage, a.n, a.ms);
        if (w < 0 || (size_t)w >= len - off) break;
        off += (size_t)w;
    }
    return GS3D_OK;
}

GS3D_API size_t determine_sort_pairs_temp_storage(const int64_t* keys_in, int64_t* keys_out,
                                                  const int32_t* values_in, int32_t* values_out,
                                                  int nb_items, int highest_key_bit) {
    (void)keys_in; (void)keys_out; (void)values_in; (void)values_out;
    const int64_t n = nb_items > 0 ? nb_items : 1;
    size_t bytes = radix_sort_workspace_bytes(n);
    if (bucket_sort_applies(n, highest_key_bit))
        bytes = std::max(bytes, bucket_sort_workspace_bytes(n, highest_key_bit));
    return bytes;
}

GS3D_API int gs3d_sort_pairs_async(void* temp_storage, size_t temp_storage_bytes,
                                   const int64_t* keys_in, int64_t* keys_out,
                                   const int32_t* values_in, int32_t* values_out, int nb_items,
                                   int highest_key_bit, gs3d_stream_t stream) {
    if (nb_items < 0) return invalid("nb_items = %d", nb_items);
    if (nb_items == 0) return GS3D_OK;
    if (!temp_storage || !keys_in || !keys_out || !values_in || !values_out)
        return invalid("NULL pointer");
    // 33 .. 46 key bits (the reference's keys: 33 + floor(log2 #tiles)): bucket by the bits
    // above 32, sort each bucket in shared memory; other widths: LSD radix sort
    if (bucket_sort_applies(nb_items, highest_key_bit) &&
        temp_storage_bytes >= bucket_sort_workspace_bytes(nb_items, highest_key_bit))
        return bucket_sort_pairs(temp_storage, temp_storage_bytes, keys_in, keys_out, values_in,
                                 values_out, nb_items, highest_key_bit,
                                 reinterpret_cast<cudaStream_t>(stream));
    return radix_sort_pairs(temp_storage, temp_storage_bytes, keys_in, keys_out, values_in,
                            values_out, nb_items, nullptr, nb_items, highest_key_bit,
                            reinterpret_cast<cudaStream_t>(stream));
}

// The reference's wrapper drops CUB's status and passes no stream (legacy default stream);
// this one keeps that signature. Errors are available through gs3d_last_error_string().
GS3D_API void sort_pairs(void* temp_storage, size_t temp_storage_bytes, const int64_t* keys_in,
                         int64_t* keys_out, const int32_t* values_in, int32_t* values_out,
                         int nb_items, int highest_key_bit) {
    (void)gs3d_sort_pairs_async(temp_storage, temp_storage_bytes, keys_in, keys_out, values_in,
                                values_out, nb_items, highest_key_bit, nullptr);
}

}  // extern "C"
