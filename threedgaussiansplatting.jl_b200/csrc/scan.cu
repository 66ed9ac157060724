// scan.cu — device-wide int32 scans whose length lives in device memory, so a render needs
// no host round trip to size them (the reference reads each scan's total back to the host:
// forward_core.jl:231-233, :259-264). Reduce-then-scan in three launches: per-chunk sums,
// one block scanning the chunk sums, per-chunk rescan with the chunk's offset. No block ever
// waits on another, so there is no spin loop anywhere.
#include "common.cuh"
#include "internal.h"

namespace gs3d {

namespace {

__device__ __forceinline__ int64_t read_len(const int32_t* len_dev, int64_t len_host,
                                            int64_t capacity) {
    int64_t len = len_dev ? (int64_t)len_dev[0] : len_host;
    if (len > capacity) len = capacity;
    if (len < 0) len = 0;
    return len;
}

__global__ void __launch_bounds__(kChunkThreads) k_chunk_sums(const int32_t* __restrict__ in,
                                                              int64_t capacity,
                                                              const int32_t* len_dev,
                                                              int64_t len_host,
                                                              int32_t* __restrict__ sums) {
    __shared__ int sm[33];
    const int64_t len = read_len(len_dev, len_host, capacity);
    const int64_t base = (int64_t)blockIdx.x * kChunk;
    if (base >= len) return;
    int s = 0;
#pragma unroll
    for (int k = 0; k < kChunkItems; ++k) {
        const int64_t i = base + k * kChunkThreads + threadIdx.x;
        if (i < len) s += in[i];
    }
    int total;
    block_exclusive_scan(s, sm, &total);
    if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// One block of 1024 threads: exclusive scan of sums[0, nchunks) in place, total -> total_dev.
__global__ void __launch_bounds__(1024) k_chunk_spine(int32_t* __restrict__ sums, int64_t capacity,
                                                      const int32_t* len_dev, int64_t len_host,
                                                      int32_t* total_dev) {
    __shared__ int sm[33];
    const int64_t len = read_len(len_dev, len_host, capacity);
    const int64_t nchunks = (len + kChunk - 1) / kChunk;
    int carry = 0;
    for (int64_t b = 0; b < nchunks; b += 1024) {
        const int64_t i = b + threadIdx.x;
        const int v = i < nchunks ? sums[i] : 0;
        int tot;
        const int ex = block_exclusive_scan(v, sm, &tot);
        if (i < nchunks) sums[i] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0 && total_dev) total_dev[0] = carry;
}

__global__ void __launch_bounds__(kChunkThreads) k_chunk_rescan(const int32_t* __restrict__ in,
                                                                int32_t* __restrict__ out,
                                                                int64_t capacity,
                                                                const int32_t* len_dev,
                                                                int64_t len_host,
                                                                const int32_t* __restrict__ sums) {
    __shared__ int sm[33];
    const int64_t len = read_len(len_dev, len_host, capacity);
    const int64_t base = (int64_t)blockIdx.x * kChunk;
    if (base >= len) return;
    const int64_t mine = base + (int64_t)threadIdx.x * kChunkItems;  // blocked arrangement
    int v[kChunkItems];
    int s = 0;
#pragma unroll
    for (int k = 0; k < kChunkItems; ++k) {
        const int64_t i = mine + k;
        v[k] = i < len ? in[i] : 0;
        s += v[k];
    }
    int total;
    int run = block_exclusive_scan(s, sm, &total) + sums[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kChunkItems; ++k) {
        const int64_t i = mine + k;
        run += v[k];
        if (i < len) out[i] = run;
    }
}

}  // namespace

int scan_spine(int32_t* sums, int64_t capacity, const int32_t* len_dev, int64_t len_host,
               int32_t* total_dev, cudaStream_t stream) {
    k_chunk_spine<<<1, 1024, 0, stream>>>(sums, capacity, len_dev, len_host, total_dev);
    GS3D_LAUNCHED("k_chunk_spine");
    return GS3D_OK;
}

size_t scan_workspace_bytes(int64_t capacity) {
    return align256((size_t)(ceil_div(capacity, kChunk) + 1) * sizeof(int32_t));
}

int inclusive_scan_i32(const int32_t* in, int32_t* out, int64_t capacity, const int32_t* len_dev,
                       int64_t len_host, int32_t* total_dev, void* ws, cudaStream_t stream) {
    const int64_t nchunks = ceil_div(capacity, kChunk);
    int32_t* sums = static_cast<int32_t*>(ws);
    if (nchunks > 0) {
        k_chunk_sums<<<(unsigned)nchunks, kChunkThreads, 0, stream>>>(in, capacity, len_dev,
                                                                      len_host, sums);
        GS3D_LAUNCHED("k_chunk_sums");
    }
    k_chunk_spine<<<1, 1024, 0, stream>>>(sums, capacity, len_dev, len_host, total_dev);
    GS3D_LAUNCHED("k_chunk_spine");
    if (nchunks > 0) {
        k_chunk_rescan<<<(unsigned)nchunks, kChunkThreads, 0, stream>>>(in, out, capacity, len_dev,
                                                                        len_host, sums);
        GS3D_LAUNCHED("k_chunk_rescan");
    }
    return GS3D_OK;
}

}  // namespace gs3d
