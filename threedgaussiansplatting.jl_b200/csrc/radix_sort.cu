// radix_sort.cu — stable LSD radix sort of (int64 key, int32 value) pairs on bits
// [0, highest_key_bit), the operation deps/cub_sort_pairs/cub_sort_pairs_wrapper.cu:31-43
// delegates to CUB and forward_core.jl:618-660 calls once per render.
//
// Per 8-bit digit pass (reduce-then-scan; no inter-block waits):
//   upsweep   : per 4096-item tile, digit histogram -> hist[digit][tile]
//   spine     : one block per digit scans its row and adds the digit's global base
//               (from a single global histogram of all passes, taken once up front)
//   downsweep : per tile, stable rank (warp match_any + per-warp digit counters), stage the
//               tile in shared memory in digit order, then write runs out contiguously.
// The item count may live on the device (the render's duplicate count), so no host sync.
#include "common.cuh"
#include "internal.h"

namespace gs3d {

namespace {

constexpr int RS_THREADS = 256;
constexpr int RS_WARPS = RS_THREADS / 32;
constexpr int RS_TILE = 4096;
constexpr int RS_ROUNDS = RS_TILE / RS_THREADS;  // 16 rounds of 32 items per warp
constexpr int RS_MAX_PASSES = 8;

__device__ __forceinline__ int64_t rs_count(const int32_t* count_dev, int64_t count_host,
                                            int64_t capacity) {
    int64_t c = count_dev ? (int64_t)count_dev[0] : count_host;
    if (c > capacity) c = capacity;
    if (c < 0) c = 0;
    return c;
}

__device__ __forceinline__ uint32_t digit_of(int64_t key, int shift, uint32_t mask) {
    return (uint32_t)(((uint64_t)key >> shift) & mask);
}

// Global digit histograms of every pass, grid-stride over tiles.
__global__ void __launch_bounds__(RS_THREADS) k_rs_global_hist(const int64_t* __restrict__ keys,
                                                               int64_t capacity,
                                                               const int32_t* count_dev,
                                                               int64_t count_host, int passes,
                                                               int highest_bit,
                                                               int32_t* __restrict__ ghist) {
    __shared__ int sh[RS_MAX_PASSES][256];
    for (int i = threadIdx.x; i < RS_MAX_PASSES * 256; i += RS_THREADS) (&sh[0][0])[i] = 0;
    __syncthreads();
    const int64_t count = rs_count(count_dev, count_host, capacity);
    for (int64_t i = (int64_t)blockIdx.x * RS_THREADS + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * RS_THREADS) {
        const int64_t k = keys[i];
        for (int p = 0; p < passes; ++p) {
            const int shift = 8 * p;
            const int nb = min(8, highest_bit - shift);
            atomicAdd(&sh[p][digit_of(k, shift, (1u << nb) - 1u)], 1);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < passes * 256; i += RS_THREADS) {
        const int v = (&sh[0][0])[i];
        if (v) atomicAdd(&ghist[i], v);
    }
}

__global__ void __launch_bounds__(RS_THREADS) k_rs_upsweep(const int64_t* __restrict__ keys,
                                                           int64_t capacity,
                                                           const int32_t* count_dev,
                                                           int64_t count_host, int shift,
                                                           uint32_t mask,
                                                           int32_t* __restrict__ hist) {
    __shared__ int wh[RS_WARPS][256];
    const int64_t count = rs_count(count_dev, count_host, capacity);
    const int64_t ntiles = (count + RS_TILE - 1) / RS_TILE;
    const int64_t t = blockIdx.x;
    if (t >= ntiles) return;
    for (int i = threadIdx.x; i < RS_WARPS * 256; i += RS_THREADS) (&wh[0][0])[i] = 0;
    __syncthreads();
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t base = t * RS_TILE;
#pragma unroll 4
    for (int r = 0; r < RS_ROUNDS; ++r) {
        const int64_t i = base + w * (RS_ROUNDS * 32) + r * 32 + lane;
        if (i < count) atomicAdd(&wh[w][digit_of(keys[i], shift, mask)], 1);
    }
    __syncthreads();
    const int d = threadIdx.x;  // 256 threads <-> 256 digits
    int s = 0;
#pragma unroll
    for (int ww = 0; ww < RS_WARPS; ++ww) s += wh[ww][d];
    hist[(int64_t)d * ntiles + t] = s;
}

// Block d: exclusive scan of row d of hist (over tiles), offset by the global base of d.
__global__ void __launch_bounds__(RS_THREADS) k_rs_spine(int32_t* __restrict__ hist,
                                                         int64_t capacity,
                                                         const int32_t* count_dev,
                                                         int64_t count_host,
                                                         const int32_t* __restrict__ ghist_pass) {
    __shared__ int sm[33];
    __shared__ int base_sh;
    const int64_t count = rs_count(count_dev, count_host, capacity);
    const int64_t ntiles = (count + RS_TILE - 1) / RS_TILE;
    const int d = blockIdx.x;
    int tot;
    const int ex = block_exclusive_scan(ghist_pass[threadIdx.x], sm, &tot);
    if (threadIdx.x == d) base_sh = ex;
    __syncthreads();
    int carry = base_sh;
    int32_t* row = hist + (int64_t)d * ntiles;
    for (int64_t b = 0; b < ntiles; b += RS_THREADS) {
        const int64_t i = b + threadIdx.x;
        const int v = i < ntiles ? row[i] : 0;
        const int e = block_exclusive_scan(v, sm, &tot);
        if (i < ntiles) row[i] = carry + e;
        carry += tot;
    }
}

struct DownSmem {
    int64_t keys[RS_TILE];
    int32_t vals[RS_TILE];
    int wcount[RS_WARPS][256];
    int tile_start[256];
    int goff[256];
    int scan[33];
};

__global__ void __launch_bounds__(RS_THREADS) k_rs_downsweep(
    const int64_t* __restrict__ keys_in, const int32_t* __restrict__ vals_in,
    int64_t* __restrict__ keys_out, int32_t* __restrict__ vals_out, int64_t capacity,
    const int32_t* count_dev, int64_t count_host, int shift, uint32_t mask,
    const int32_t* __restrict__ hist) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    DownSmem& S = *reinterpret_cast<DownSmem*>(smem_raw);
    const int64_t count = rs_count(count_dev, count_host, capacity);
    const int64_t ntiles = (count + RS_TILE - 1) / RS_TILE;
    const int64_t t = blockIdx.x;
    if (t >= ntiles) return;
    const int64_t base = t * RS_TILE;
    const int n_here = (int)min((int64_t)RS_TILE, count - base);
    for (int i = threadIdx.x; i < RS_WARPS * 256; i += RS_THREADS) (&S.wcount[0][0])[i] = 0;
    __syncthreads();

    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned lt_mask = (1u << lane) - 1u;
    int64_t key[RS_ROUNDS];
    int32_t val[RS_ROUNDS];
    int rank[RS_ROUNDS];
#pragma unroll
    for (int r = 0; r < RS_ROUNDS; ++r) {
        const int li = w * (RS_ROUNDS * 32) + r * 32 + lane;
        const bool valid = li < n_here;
        key[r] = valid ? keys_in[base + li] : 0;
        val[r] = valid ? vals_in[base + li] : 0;
        const uint32_t d = valid ? digit_of(key[r], shift, mask) : 256u;
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        const int before = valid ? S.wcount[w][d] : 0;
        rank[r] = before + __popc(peers & lt_mask);
        __syncwarp();
        if (valid && (peers & lt_mask) == 0) S.wcount[w][d] = before + __popc(peers);
        __syncwarp();
    }
    __syncthreads();
    {
        const int d = threadIdx.x;
        int run = 0;
#pragma unroll
        for (int ww = 0; ww < RS_WARPS; ++ww) {
            const int c = S.wcount[ww][d];
            S.wcount[ww][d] = run;
            run += c;
        }
        int tot;
        const int st = block_exclusive_scan(run, S.scan, &tot);
        S.tile_start[d] = st;
        S.goff[d] = hist[(int64_t)d * ntiles + t];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < RS_ROUNDS; ++r) {
        const int li = w * (RS_ROUNDS * 32) + r * 32 + lane;
        if (li < n_here) {
            const uint32_t d = digit_of(key[r], shift, mask);
            const int lp = S.tile_start[d] + S.wcount[w][d] + rank[r];
            S.keys[lp] = key[r];
            S.vals[lp] = val[r];
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n_here; i += RS_THREADS) {
        const int64_t k = S.keys[i];
        const uint32_t d = digit_of(k, shift, mask);
        const int64_t o = (int64_t)S.goff[d] + (i - S.tile_start[d]);
        keys_out[o] = k;
        vals_out[o] = S.vals[i];
    }
}

__global__ void k_rs_copy(const int64_t* __restrict__ ki, const int32_t* __restrict__ vi,
                          int64_t* __restrict__ ko, int32_t* __restrict__ vo, int64_t capacity,
                          const int32_t* count_dev, int64_t count_host) {
    const int64_t count = rs_count(count_dev, count_host, capacity);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x) {
        ko[i] = ki[i];
        vo[i] = vi[i];
    }
}

struct RsLayout {
    size_t alt_keys, alt_vals, hist, ghist, total;
};

RsLayout rs_layout(int64_t capacity) {
    RsLayout L;
    const int64_t ntiles = ceil_div(capacity, RS_TILE);
    size_t off = 0;
    L.alt_keys = off; off += align256((size_t)capacity * 8);
    L.alt_vals = off; off += align256((size_t)capacity * 4);
    L.hist = off;     off += align256((size_t)(ntiles * 256 + 1) * 4);
    L.ghist = off;    off += align256((size_t)RS_MAX_PASSES * 256 * 4);
    L.total = off;
    return L;
}

}  // namespace

size_t radix_sort_workspace_bytes(int64_t capacity) {
    if (capacity < 1) capacity = 1;
    return rs_layout(capacity).total;
}

int radix_sort_pairs(void* ws, size_t ws_bytes, const int64_t* keys_in, int64_t* keys_out,
                     const int32_t* values_in, int32_t* values_out, int64_t capacity,
                     const int32_t* count_dev, int64_t count_host, int highest_key_bit,
                     cudaStream_t stream) {
    if (capacity <= 0) return GS3D_OK;
    if (highest_key_bit > 64) highest_key_bit = 64;
    const RsLayout L = rs_layout(capacity);
    if (ws_bytes < L.total)
        return set_error("radix sort workspace too small: %zu < %zu", ws_bytes, L.total),
               GS3D_ERR_WORKSPACE;
    unsigned char* w = static_cast<unsigned char*>(ws);
    int64_t* alt_keys = reinterpret_cast<int64_t*>(w + L.alt_keys);
    int32_t* alt_vals = reinterpret_cast<int32_t*>(w + L.alt_vals);
    int32_t* hist = reinterpret_cast<int32_t*>(w + L.hist);
    int32_t* ghist = reinterpret_cast<int32_t*>(w + L.ghist);
    const int64_t ntiles_cap = ceil_div(capacity, RS_TILE);
    const int passes = highest_key_bit <= 0 ? 0 : (highest_key_bit + 7) / 8;
    if (passes == 0) {
        k_rs_copy<<<kSMs * 4, 256, 0, stream>>>(keys_in, values_in, keys_out, values_out, capacity,
                                               count_dev, count_host);
        GS3D_LAUNCHED("k_rs_copy");
        return GS3D_OK;
    }
    GS3D_CUDA(cudaMemsetAsync(ghist, 0, (size_t)RS_MAX_PASSES * 256 * 4, stream), "memset ghist");
    const unsigned gh_blocks = (unsigned)std::min<int64_t>(ntiles_cap * (RS_TILE / RS_THREADS), kSMs * 8);
    k_rs_global_hist<<<gh_blocks, RS_THREADS, 0, stream>>>(keys_in, capacity, count_dev, count_host,
                                                           passes, highest_key_bit, ghist);
    GS3D_LAUNCHED("k_rs_global_hist");
    // set on every call: the attribute belongs to the current context (lost on a device reset),
    // the call is a cheap host-side update, and it needs no per-device state shared between
    // host threads
    GS3D_CUDA(cudaFuncSetAttribute(k_rs_downsweep, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)sizeof(DownSmem)),
              "downsweep smem attribute");
    const int64_t* src_k = keys_in;
    const int32_t* src_v = values_in;
    for (int p = 0; p < passes; ++p) {
        const bool to_out = ((passes - 1 - p) % 2) == 0;
        int64_t* dk = to_out ? keys_out : alt_keys;
        int32_t* dv = to_out ? values_out : alt_vals;
        const int shift = 8 * p;
        const int nb = std::min(8, highest_key_bit - shift);
        const uint32_t mask = (nb >= 32) ? 0xffffffffu : ((1u << nb) - 1u);
        k_rs_upsweep<<<(unsigned)ntiles_cap, RS_THREADS, 0, stream>>>(src_k, capacity, count_dev,
                                                                      count_host, shift, mask, hist);
        GS3D_LAUNCHED("k_rs_upsweep");
        k_rs_spine<<<256, RS_THREADS, 0, stream>>>(hist, capacity, count_dev, count_host,
                                                   ghist + 256 * p);
        GS3D_LAUNCHED("k_rs_spine");
        k_rs_downsweep<<<(unsigned)ntiles_cap, RS_THREADS, sizeof(DownSmem), stream>>>(
            src_k, src_v, dk, dv, capacity, count_dev, count_host, shift, mask, hist);
        GS3D_LAUNCHED("k_rs_downsweep");
        src_k = dk;
        src_v = dv;
    }
    return GS3D_OK;
}

}  // namespace gs3d
