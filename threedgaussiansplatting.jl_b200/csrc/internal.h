// internal.h — host-side interfaces shared between libgs3d translation units.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace gs3d {

// Round a byte count up to 256 (every workspace region starts 256-byte aligned).
inline size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

// LSD radix sort of (int64 key, int32 value) pairs on bits [0, highest_key_bit), stable.
// The item count is read from count_dev[0] on the device (clamped to capacity) when
// count_dev is not NULL, else count_host is used. keys_in / values_in are not modified.
size_t radix_sort_workspace_bytes(int64_t capacity);
int radix_sort_pairs(void* ws, size_t ws_bytes, const int64_t* keys_in, int64_t* keys_out,
                     const int32_t* values_in, int32_t* values_out, int64_t capacity,
                     const int32_t* count_dev, int64_t count_host, int highest_key_bit,
                     cudaStream_t stream);

// Tile-bucket sort of the duplicated keys (tile_sort.cu). tile_sort_count writes the per-tile
// inclusive ends into tiles_end and D into counts[1] (status bit on overflow);
// tile_sort_order then fills the sorted keys and values. The counts F / D are read on the device.
size_t tile_sort_workspace_bytes(int64_t capacity_dup, int nb_tiles);
int tile_sort_max_tiles();  // more tiles than this take the reference-order pipeline
int tile_sort_count(void* ws, size_t ws_bytes, int32_t* counts, const int4* ranges,
                    int64_t capacity_n, int tiles_x, int nb_tiles, int64_t capacity_dup,
                    int32_t* tiles_end, cudaStream_t stream);
int tile_sort_order(void* ws, const int32_t* counts, const int4* ranges, const float* depths,
                    int64_t capacity_n, int tiles_x, int nb_tiles, int64_t capacity_dup,
                    const int32_t* tiles_end, int64_t* keys_scratch, int64_t* sorted_codes,
                    int32_t* sorted_vals, cudaStream_t stream);

// Stable pair sort of n (int64 key, int32 value) pairs on bits [0, highest_key_bit) for
// 32 < highest_key_bit <= 46 (bucket_sort_applies): the tile pipeline's histogram, scatter
// and per-segment sort with bits [32, highest_key_bit) as the bucket (tile_sort.cu).
bool bucket_sort_applies(int64_t n, int highest_key_bit);
size_t bucket_sort_workspace_bytes(int64_t n, int highest_key_bit);
int bucket_sort_pairs(void* ws, size_t ws_bytes, const int64_t* keys_in, int64_t* keys_out,
                      const int32_t* vals_in, int32_t* vals_out, int64_t n, int highest_key_bit,
                      cudaStream_t stream);

// Device-wide scans over int32 with the length on the device (len_dev[0]) or on the host.
size_t scan_workspace_bytes(int64_t capacity);
// inclusive scan of in[0, len) into out; the total is written to total_dev[0].
int inclusive_scan_i32(const int32_t* in, int32_t* out, int64_t capacity, const int32_t* len_dev,
                       int64_t len_host, int32_t* total_dev, void* ws, cudaStream_t stream);

// Exclusive scan in place of the per-chunk sums of a chunked scan (chunk = 4096 items):
// nchunks = ceil(len / 4096); the grand total goes to total_dev[0] (may be NULL).
int scan_spine(int32_t* sums, int64_t capacity, const int32_t* len_dev, int64_t len_host,
               int32_t* total_dev, cudaStream_t stream);

int device_sm_count();

// Opt-in stage timers (gs3d_profile_enable): CUDA events recorded on the launching stream
// around each stage; no effect when disabled.
void prof_begin(const char* stage, cudaStream_t stream);
void prof_end(const char* stage, cudaStream_t stream);

struct ProfScope {
    const char* stage;
    cudaStream_t stream;
    ProfScope(const char* s, cudaStream_t st) : stage(s), stream(st) { prof_begin(s, st); }
    ~ProfScope() { prof_end(stage, stream); }
};

}  // namespace gs3d
