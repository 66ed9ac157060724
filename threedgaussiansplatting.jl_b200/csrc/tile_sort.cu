// tile_sort.cu — the duplicated-key stage of render! (forward_core.jl:259-264 counts,
// :531-603 keys, :618-660 sort_pairs, :676-734 tile ranges) as a tile-bucket sort.
//
// The reference writes one key  tile << 32 | depth bits  per (filtered Gaussian, overlapped
// tile) in filtered-index order and sorts them stably on bits [0, 33 + floor(log2 #tiles)):
// within a tile, entries end up by depth, equal depths by filtered index. The same order is
// produced here without a device-wide multi-pass sort:
//   k_tile_hist     entries per (block, tile): each of kHistBlocks blocks takes a contiguous
//                   range of filtered Gaussians and counts in a shared-memory histogram;
//   k_tile_colscan  per tile, exclusive prefix over the blocks and the tile total;
//   k_tile_scan     inclusive scan over tiles = tiles_end (F7's output), the segment starts,
//                   and D;
//   k_tile_scatter  one 64-bit key  depth bits << 32 | filtered index  per entry into its
//                   tile's segment, each block within its own sub-range (claimed with
//                   shared-memory cursors; the order inside a segment does not matter,
//                   because these keys are unique);
//   k_tile_segsort  one CTA per tile sorts its segment ascending (up to kRadixCap entries: a
//                   shared-memory radix sort on the depth bits, then runs of equal depth by
//                   filtered index; up to kSegCap: a bitonic network in shared memory; larger
//                   segments in a scratch region with the network's long-stride stages in
//                   global memory and the short ones chunk-wise in shared memory) and writes
//                   the sorted keys tile << 32 | depth bits and values filtered index + 1.
// Sorting (depth bits, filtered index) inside each tile is exactly the stable sort of the
// reference's keys, so sdf2dgs_codes, sdfgidx_to_fgidx and tiles_end are bit-identical.
#include "common.cuh"
#include "internal.h"

namespace gs3d {
namespace {

constexpr int kSegCap = 4096;   // segment entries sorted in shared memory (32 KB)
constexpr int kSegThreads = 256;

// Block b of kHistBlocks takes the filtered Gaussians [b chunk, (b + 1) chunk) (chunk =
// ceil(F / kHistBlocks)) and counts their tile entries in a shared-memory histogram over all
// tiles, written to bcount[b][t].
constexpr int kHistBlocks = 148;
constexpr int kHistThreads = 1024;

__device__ __forceinline__ void block_chunk(const int32_t* counts, int& f0, int& f1) {
    const int F = counts[0];
    const int chunk = (F + kHistBlocks - 1) / kHistBlocks;
    f0 = min(F, (int)blockIdx.x * chunk);
    f1 = min(F, f0 + chunk);
}

__global__ void __launch_bounds__(kHistThreads) k_tile_hist(const int32_t* __restrict__ counts,
                                                           const int4* __restrict__ ranges,
                                                           int tiles_x, int nb_tiles,
                                                           int32_t* __restrict__ bcount) {
    extern __shared__ int32_t hist[];
    for (int i = threadIdx.x; i < nb_tiles; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    int f0, f1;
    block_chunk(counts, f0, f1);
    for (int f = f0 + threadIdx.x; f < f1; f += blockDim.x) {
        const int4 r = ranges[f];
        for (int ty = r.y; ty <= r.w; ++ty)
            for (int tx = r.x; tx <= r.z; ++tx) atomicAdd(&hist[(ty - 1) * tiles_x + (tx - 1)], 1);
    }
    __syncthreads();
    int32_t* out = bcount + (size_t)blockIdx.x * nb_tiles;
    for (int i = threadIdx.x; i < nb_tiles; i += blockDim.x) out[i] = hist[i];
}

// Per tile: exclusive prefix of the block counts (in place) and the tile total. A CTA takes 32
// tiles (one per lane, coalesced) and splits the kHistBlocks blocks over its 8 warps.
__global__ void __launch_bounds__(256) k_tile_colscan(int32_t* __restrict__ bcount, int nb_tiles,
                                                      int32_t* __restrict__ tcount) {
    constexpr int G = 8, PER = (kHistBlocks + G - 1) / G;
    __shared__ int part[G][32];
    const int tl = threadIdx.x & 31, g = threadIdx.x >> 5;
    const int t = blockIdx.x * 32 + tl;
    const int b0 = g * PER, b1 = min(kHistBlocks, b0 + PER);
    int v[PER];
    int sum = 0;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const int b = b0 + k;
        v[k] = (t < nb_tiles && b < b1) ? bcount[(size_t)b * nb_tiles + t] : 0;
        sum += v[k];
    }
    part[g][tl] = sum;
    __syncthreads();
    if (g == 0) {
        int run = 0;
#pragma unroll
        for (int q = 0; q < G; ++q) {
            const int c = part[q][tl];
            part[q][tl] = run;
            run += c;
        }
        if (t < nb_tiles) tcount[t] = run;
    }
    __syncthreads();
    int run = part[g][tl];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const int b = b0 + k;
        if (t < nb_tiles && b < b1) bcount[(size_t)b * nb_tiles + t] = run;
        run += v[k];
    }
}

// One CTA of 1024 threads: thread i scans tiles [i per, (i + 1) per).
__global__ void __launch_bounds__(1024) k_tile_scan(const int32_t* __restrict__ tcount, int nb_tiles,
                                                    int64_t capacity, int32_t* __restrict__ tiles_end,
                                                    int32_t* __restrict__ cursor,
                                                    int32_t* __restrict__ counts) {
    __shared__ int sm[33];
    const int per = (nb_tiles + 1023) / 1024;
    const int t0 = threadIdx.x * per;
    int s = 0;
    for (int k = 0; k < per; ++k)
        if (t0 + k < nb_tiles) s += tcount[t0 + k];
    int total;
    int run = block_exclusive_scan(s, sm, &total);
    for (int k = 0; k < per; ++k) {
        const int t = t0 + k;
        if (t >= nb_tiles) break;
        cursor[t] = run;
        run += tcount[t];
        tiles_end[t] = run;
    }
    if (threadIdx.x == 0) {
        counts[1] = total;
        if ((int64_t)total > capacity) atomicOr(&counts[2], (int)GS3D_STATUS_DUP_OVERFLOW);
    }
}

// Same block partition as k_tile_hist: block b's entries of tile t go to positions
// tile start + bcount[b][t] + ..., claimed with shared-memory cursors.
__global__ void __launch_bounds__(kHistThreads) k_tile_scatter(
    const int32_t* __restrict__ counts, const int4* __restrict__ ranges,
    const float* __restrict__ depths, int tiles_x, int nb_tiles, int64_t capacity,
    const int32_t* __restrict__ tile_start, const int32_t* __restrict__ bcount,
    uint64_t* __restrict__ keys) {
    extern __shared__ int32_t cur[];
    if ((int64_t)counts[1] > capacity) return;  // overflow: flagged by k_tile_scan
    const int32_t* base = bcount + (size_t)blockIdx.x * nb_tiles;
    for (int i = threadIdx.x; i < nb_tiles; i += blockDim.x) cur[i] = tile_start[i] + base[i];
    __syncthreads();
    int f0, f1;
    block_chunk(counts, f0, f1);
    for (int f = f0 + threadIdx.x; f < f1; f += blockDim.x) {
        const int4 r = ranges[f];
        if (r.x > r.z || r.y > r.w) continue;
        const uint64_t key = ((uint64_t)f2u(depths[f]) << 32) | (uint32_t)f;
        for (int ty = r.y; ty <= r.w; ++ty)
            for (int tx = r.x; tx <= r.z; ++tx) {
                const int pos = atomicAdd(&cur[(ty - 1) * tiles_x + (tx - 1)], 1);
                keys[pos] = key;
            }
    }
}

// ---- the generic stable pair sort (sort_pairs) on the same machinery -----------------------
// Keys of highest_key_bit = 32 + B bits (1 <= B <= kMaxBucketBits): bits [32, 32 + B) pick one
// of 2^B buckets, which play the tiles' part; inside a bucket the entries are sorted by
// (bits [0, 32) of the key, input index), i.e. stably. Block b of kHistBlocks takes the items
// [b chunk, (b + 1) chunk), chunk = ceil(n / kHistBlocks).
constexpr int kMaxBucketBits = 14;

__device__ __forceinline__ void item_chunk(int64_t n, int64_t& i0, int64_t& i1) {
    const int64_t chunk = (n + kHistBlocks - 1) / kHistBlocks;
    i0 = min(n, (int64_t)blockIdx.x * chunk);
    i1 = min(n, i0 + chunk);
}

__global__ void __launch_bounds__(kHistThreads) k_key_hist(const int64_t* __restrict__ keys, int64_t n,
                                                          int nb_buckets, int32_t* __restrict__ bcount,
                                                          int32_t* __restrict__ counts) {
    extern __shared__ int32_t hist[];
    for (int i = threadIdx.x; i < nb_buckets; i += blockDim.x) hist[i] = 0;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        counts[0] = 1;  // non-zero: the segment sort's "something to sort" test
        counts[2] = 0;
    }
    __syncthreads();
    int64_t i0, i1;
    item_chunk(n, i0, i1);
    const uint32_t bmask = (uint32_t)nb_buckets - 1u;
    for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x)
        atomicAdd(&hist[(uint32_t)((uint64_t)keys[i] >> 32) & bmask], 1);
    __syncthreads();
    int32_t* out = bcount + (size_t)blockIdx.x * nb_buckets;
    for (int i = threadIdx.x; i < nb_buckets; i += blockDim.x) out[i] = hist[i];
}

// Item i goes to its bucket's sub-range of block b as (low 32 key bits) << 32 | i; the order
// inside a sub-range does not matter (the entries are unique and sorted afterwards).
__global__ void __launch_bounds__(kHistThreads) k_key_scatter(
    const int64_t* __restrict__ keys, int64_t n, int nb_buckets,
    const int32_t* __restrict__ bucket_start, const int32_t* __restrict__ bcount,
    uint64_t* __restrict__ out) {
    extern __shared__ int32_t cur[];
    const int32_t* base = bcount + (size_t)blockIdx.x * nb_buckets;
    for (int i = threadIdx.x; i < nb_buckets; i += blockDim.x) cur[i] = bucket_start[i] + base[i];
    __syncthreads();
    int64_t i0, i1;
    item_chunk(n, i0, i1);
    const uint32_t bmask = (uint32_t)nb_buckets - 1u;
    for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const uint64_t k = (uint64_t)keys[i];
        const int pos = atomicAdd(&cur[(uint32_t)(k >> 32) & bmask], 1);
        out[pos] = (k << 32) | (uint64_t)(uint32_t)i;
    }
}

// Compare-exchange of the bitonic network: pair p of stage (k, j) is (i, i + j), ascending
// when bit k of the (global) index i is clear.
__device__ __forceinline__ void bitonic_pair(int p, int j, int& i, int& l) {
    i = ((p & ~(j - 1)) << 1) | (p & (j - 1));
    l = i + j;
}

// All stages j = jtop .. 1 of every k in [k_lo, k_hi] on s[0, P) (s = chunk of a sequence whose
// first element has global index base; P a power of two <= kSegCap).
__device__ void bitonic_local(uint64_t* s, int P, int base, int k_lo, int k_hi, int jtop) {
    for (int k = k_lo; k <= k_hi; k <<= 1) {
        for (int j = min(k >> 1, jtop); j > 0; j >>= 1) {
            for (int p = threadIdx.x; p < P / 2; p += blockDim.x) {
                int i, l;
                bitonic_pair(p, j, i, l);
                const bool asc = ((base + i) & k) == 0;
                const uint64_t a = s[i], b = s[l];
                if ((a > b) == asc) {
                    s[i] = b;
                    s[l] = a;
                }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ void emit(int64_t pos, uint64_t key, uint64_t tile_hi,
                                     int64_t* __restrict__ codes, int32_t* __restrict__ vals) {
    // the reference's key: tile << 32 | depth bits (depth bits widened as a signed word)
    const uint64_t dcode = (uint64_t)(int64_t)(int32_t)(uint32_t)(key >> 32);
    codes[pos] = (int64_t)(tile_hi | dcode);
    vals[pos] = (int32_t)(uint32_t)key + 1;
}

// Segments up to kRadixCap entries: LSD radix sort on the depth bits (4 passes of 8 bits) in
// shared memory, stable: warp w ranks its contiguous block of entries 32 at a time in order
// (peers by __match_any_sync, running per-warp digit counters), and the (digit, warp) offsets
// come from one block scan. Entries of equal depth then sit in scatter order; each such run is
// put in filtered-index order afterwards (insertion sort by one thread per run; runs longer
// than kMaxRun make the whole segment take the bitonic network instead).
constexpr int kRadixCap = 2048;
constexpr int kRadixRounds = kRadixCap / (kSegThreads / 32) / 32;  // 8 rounds of 32 per warp
constexpr int kMaxRun = 64;
constexpr int kSegSmemBytes = 2 * kRadixCap * 8 + (kSegThreads / 32) * 256 * 4;  // 40 KB
static_assert(kSegCap * 8 <= kSegSmemBytes, "bitonic buffer must fit the shared buffer");

// Four passes: the sorted entries end in kA again.
__device__ void radix_depth_sort(uint64_t* kA, uint64_t* kB, int* wc, int* scan_sm, int m) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const unsigned lt = (1u << lane) - 1u;
    const int per_warp = (m + 7) / 8;
    const int R = (per_warp + 31) / 32;
    const int B = R * 32;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 32 + 8 * pass;
        for (int i = threadIdx.x; i < 8 * 256; i += blockDim.x) wc[i] = 0;
        __syncthreads();
        uint64_t kreg[kRadixRounds];
        int rank[kRadixRounds];
#pragma unroll
        for (int r = 0; r < kRadixRounds; ++r) {
            kreg[r] = 0;
            rank[r] = 0;
            if (r >= R) continue;
            const int i = w * B + r * 32 + lane;
            const bool valid = i < m;
            const uint64_t k = valid ? kA[i] : 0ull;
            const unsigned d = valid ? (unsigned)((k >> shift) & 255u) : 256u;
            const unsigned peers = __match_any_sync(0xffffffffu, d);
            const int before = valid ? wc[w * 256 + d] : 0;
            rank[r] = before + __popc(peers & lt);
            kreg[r] = k;
            __syncwarp();
            if (valid && (peers & lt) == 0) wc[w * 256 + d] = before + __popc(peers);
            __syncwarp();
        }
        __syncthreads();
        {  // thread d: digit total over the warps, block scan over digits, per-warp offsets
            const int d = threadIdx.x;
            int tot = 0;
#pragma unroll
            for (int ww = 0; ww < 8; ++ww) tot += wc[ww * 256 + d];
            int all;
            int base = block_exclusive_scan(tot, scan_sm, &all);
#pragma unroll
            for (int ww = 0; ww < 8; ++ww) {
                const int c = wc[ww * 256 + d];
                wc[ww * 256 + d] = base;
                base += c;
            }
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < kRadixRounds; ++r) {
            if (r >= R) continue;
            const int i = w * B + r * 32 + lane;
            if (i >= m) continue;
            const unsigned d = (unsigned)((kreg[r] >> shift) & 255u);
            kB[wc[w * 256 + d] + rank[r]] = kreg[r];
        }
        __syncthreads();
        uint64_t* t = kA;
        kA = kB;
        kB = t;
    }
}

#ifndef GS3D_SEGSORT_MINB
#define GS3D_SEGSORT_LB __launch_bounds__(kSegThreads)
#else
#define GS3D_SEGSORT_LB __launch_bounds__(kSegThreads, GS3D_SEGSORT_MINB)
#endif

// Output of one sorted entry. The render's tile pipeline: the reference's code and value
// (emit). The generic pair sort (Pairs non-NULL): the entry's low 32 bits are its input index,
// whose key and value are copied.
struct Pairs {
    const int64_t* keys_in;
    const int32_t* vals_in;
};

__device__ __forceinline__ void emit_any(const Pairs& pr, int64_t pos, uint64_t key, uint64_t tile_hi,
                                         int64_t* __restrict__ codes, int32_t* __restrict__ vals) {
    if (pr.keys_in) {
        const uint32_t idx = (uint32_t)key;
        codes[pos] = pr.keys_in[idx];
        vals[pos] = pr.vals_in[idx];
    } else {
        emit(pos, key, tile_hi, codes, vals);
    }
}

__global__ void GS3D_SEGSORT_LB k_tile_segsort(
    const int32_t* __restrict__ counts, int64_t capacity, const int32_t* __restrict__ tiles_end,
    const uint64_t* __restrict__ keys, uint64_t* __restrict__ scratch, int64_t* __restrict__ codes,
    int32_t* __restrict__ vals, const Pairs pr) {
    __shared__ __align__(16) unsigned char raw[kSegSmemBytes];
    __shared__ int scan_sm[33];
    const int64_t D = counts[1];
    if (counts[0] == 0 || D == 0 || D > capacity) return;
    const int t = blockIdx.x;
    const int start = t == 0 ? 0 : tiles_end[t - 1];
    const int m = tiles_end[t] - start;
    if (m <= 0) return;
    const uint64_t tile_hi = (uint64_t)(uint32_t)(t + 1) << 32;
    int P = 1;
    while (P < m) P <<= 1;
    uint64_t* s = reinterpret_cast<uint64_t*>(raw);
    if (m <= kRadixCap) {
        uint64_t* kA = s;
        uint64_t* kB = s + kRadixCap;
        int* wc = reinterpret_cast<int*>(s + 2 * kRadixCap);
        for (int i = threadIdx.x; i < m; i += blockDim.x) kA[i] = keys[start + i];
        __syncthreads();
        radix_depth_sort(kA, kB, wc, scan_sm, m);
        // runs of equal depth: find them (reads only), then order each by filtered index
        int rs[kRadixCap / kSegThreads], rl[kRadixCap / kSegThreads];
        bool long_run = false;
#pragma unroll
        for (int q = 0; q < kRadixCap / kSegThreads; ++q) {
            rs[q] = -1;
            rl[q] = 0;
            const int i = threadIdx.x + q * kSegThreads;
            if (i + 1 >= m) continue;
            const uint32_t di = (uint32_t)(kA[i] >> 32);
            if ((uint32_t)(kA[i + 1] >> 32) != di) continue;
            if (i > 0 && (uint32_t)(kA[i - 1] >> 32) == di) continue;
            int e = i + 1;
            while (e < m && (uint32_t)(kA[e] >> 32) == di && e - i <= kMaxRun) ++e;
            if (e - i > kMaxRun) long_run = true;
            rs[q] = i;
            rl[q] = e - i;
        }
        if (__syncthreads_or(long_run)) {
            for (int i = m + threadIdx.x; i < P; i += blockDim.x) kA[i] = ~0ull;
            __syncthreads();
            bitonic_local(kA, P, 0, 2, P, P);
        } else {
#pragma unroll
            for (int q = 0; q < kRadixCap / kSegThreads; ++q) {
                if (rs[q] < 0) continue;
                uint64_t* run = kA + rs[q];
                for (int a = 1; a < rl[q]; ++a) {  // whole-key compare: the depths are equal
                    const uint64_t v = run[a];
                    int b = a - 1;
                    while (b >= 0 && run[b] > v) {
                        run[b + 1] = run[b];
                        --b;
                    }
                    run[b + 1] = v;
                }
            }
            __syncthreads();
        }
        for (int i = threadIdx.x; i < m; i += blockDim.x) emit_any(pr, start + i, kA[i], tile_hi, codes, vals);
        return;
    }
    if (P <= kSegCap) {
        for (int i = threadIdx.x; i < P; i += blockDim.x) s[i] = i < m ? keys[start + i] : ~0ull;
        __syncthreads();
        bitonic_local(s, P, 0, 2, P, P);
        for (int i = threadIdx.x; i < m; i += blockDim.x) emit_any(pr, start + i, s[i], tile_hi, codes, vals);
        return;
    }
    // large segment: padded copy in scratch[2 start, 2 start + P) (P < 2 m, so the regions of
    // different tiles do not overlap); stages with j >= kSegCap in global memory, the others
    // chunk-wise in shared memory
    uint64_t* g = scratch + 2 * (int64_t)start;
    for (int i = threadIdx.x; i < P; i += blockDim.x) g[i] = i < m ? keys[start + i] : ~0ull;
    __syncthreads();
    for (int k = 2; k <= P; k <<= 1) {
        if (k > kSegCap) {
            for (int j = k >> 1; j >= kSegCap; j >>= 1) {
                for (int p = threadIdx.x; p < P / 2; p += blockDim.x) {
                    int i, l;
                    bitonic_pair(p, j, i, l);
                    const bool asc = (i & k) == 0;
                    const uint64_t a = g[i], b = g[l];
                    if ((a > b) == asc) {
                        g[i] = b;
                        g[l] = a;
                    }
                }
                __syncthreads();
            }
        }
        // stages j < kSegCap of this k (for k <= kSegCap: every k up to kSegCap at once)
        const int k_hi = k <= kSegCap ? kSegCap : k;
        for (int c = 0; c < P; c += kSegCap) {
            for (int i = threadIdx.x; i < kSegCap; i += blockDim.x) s[i] = g[c + i];
            __syncthreads();
            bitonic_local(s, kSegCap, c, k, k_hi, kSegCap >> 1);
            for (int i = threadIdx.x; i < kSegCap; i += blockDim.x) g[c + i] = s[i];
            __syncthreads();
        }
        if (k <= kSegCap) k = kSegCap;  // every k <= kSegCap was just done
    }
    for (int i = threadIdx.x; i < m; i += blockDim.x) emit_any(pr, start + i, g[i], tile_hi, codes, vals);
}

}  // namespace

// workspace: tile counts, tile starts (2 nb_tiles int32), block counts (kHistBlocks x
// nb_tiles int32), large-segment scratch (2 capacity_dup uint64)
size_t tile_sort_workspace_bytes(int64_t capacity_dup, int nb_tiles) {
    if (capacity_dup < 1) capacity_dup = 1;
    return align256((size_t)2 * nb_tiles * sizeof(int32_t)) +
           align256((size_t)kHistBlocks * nb_tiles * sizeof(int32_t)) +
           align256((size_t)2 * capacity_dup * sizeof(uint64_t));
}

int tile_sort_max_tiles() {
    // the per-block tile histograms live in shared memory
    return (int)((200u * 1024u) / sizeof(int32_t));
}

namespace {
struct TsLayout {
    int32_t *tcount, *cursor, *bcount;
    uint64_t* big;
};
TsLayout ts_layout(void* ws, int nb_tiles) {
    unsigned char* w = static_cast<unsigned char*>(ws);
    TsLayout L;
    L.tcount = reinterpret_cast<int32_t*>(w);
    L.cursor = L.tcount + nb_tiles;
    w += align256((size_t)2 * nb_tiles * sizeof(int32_t));
    L.bcount = reinterpret_cast<int32_t*>(w);
    w += align256((size_t)kHistBlocks * nb_tiles * sizeof(int32_t));
    L.big = reinterpret_cast<uint64_t*>(w);
    return L;
}

// Set on every call: the attribute belongs to the current context (lost on a device reset), the
// call is a cheap host-side update, and it needs no per-device state shared between host threads.
int set_hist_smem() {
    const int want = tile_sort_max_tiles() * (int)sizeof(int32_t);
    GS3D_CUDA(cudaFuncSetAttribute(k_tile_hist, cudaFuncAttributeMaxDynamicSharedMemorySize, want),
              "tile histogram shared memory");
    GS3D_CUDA(cudaFuncSetAttribute(k_tile_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize, want),
              "tile scatter shared memory");
    return GS3D_OK;
}
}  // namespace

int tile_sort_count(void* ws, size_t ws_bytes, int32_t* counts, const int4* ranges,
                    int64_t capacity_n, int tiles_x, int nb_tiles, int64_t capacity_dup,
                    int32_t* tiles_end, cudaStream_t stream) {
    (void)capacity_n;
    if (ws_bytes < tile_sort_workspace_bytes(capacity_dup, nb_tiles))
        return set_error("tile sort workspace too small"), GS3D_ERR_WORKSPACE;
    if (nb_tiles > tile_sort_max_tiles())
        return set_error("%d tiles exceed the tile sort's %d", nb_tiles, tile_sort_max_tiles()),
               GS3D_ERR_UNSUPPORTED;
    GS3D_RETURN_IF(set_hist_smem());
    const TsLayout L = ts_layout(ws, nb_tiles);
    const size_t smem = (size_t)nb_tiles * sizeof(int32_t);
    k_tile_hist<<<kHistBlocks, kHistThreads, smem, stream>>>(counts, ranges, tiles_x, nb_tiles, L.bcount);
    GS3D_LAUNCHED("k_tile_hist");
    k_tile_colscan<<<(unsigned)ceil_div(nb_tiles, 32), 256, 0, stream>>>(L.bcount, nb_tiles, L.tcount);
    GS3D_LAUNCHED("k_tile_colscan");
    k_tile_scan<<<1, 1024, 0, stream>>>(L.tcount, nb_tiles, capacity_dup, tiles_end, L.cursor, counts);
    GS3D_LAUNCHED("k_tile_scan");
    return GS3D_OK;
}

int tile_sort_order(void* ws, const int32_t* counts, const int4* ranges, const float* depths,
                    int64_t capacity_n, int tiles_x, int nb_tiles, int64_t capacity_dup,
                    const int32_t* tiles_end, int64_t* keys_scratch, int64_t* sorted_codes,
                    int32_t* sorted_vals, cudaStream_t stream) {
    (void)capacity_n;
    const TsLayout L = ts_layout(ws, nb_tiles);
    uint64_t* keys = reinterpret_cast<uint64_t*>(keys_scratch);
    const size_t smem = (size_t)nb_tiles * sizeof(int32_t);
    k_tile_scatter<<<kHistBlocks, kHistThreads, smem, stream>>>(counts, ranges, depths, tiles_x, nb_tiles,
                                                                capacity_dup, L.cursor, L.bcount, keys);
    GS3D_LAUNCHED("k_tile_scatter");
    k_tile_segsort<<<(unsigned)nb_tiles, kSegThreads, 0, stream>>>(counts, capacity_dup, tiles_end, keys,
                                                                   L.big, sorted_codes, sorted_vals,
                                                                   Pairs{nullptr, nullptr});
    GS3D_LAUNCHED("k_tile_segsort");
    return GS3D_OK;
}

// ---- generic pair sort --------------------------------------------------------------------
// workspace: counts (4 int32), bucket counts + starts (2 T int32), bucket ends (T int32), block
// counts (kHistBlocks x T int32), large-segment scratch (2 n uint64), entries (n uint64)
bool bucket_sort_applies(int64_t n, int highest_key_bit) {
    return highest_key_bit > 32 && highest_key_bit <= 32 + kMaxBucketBits && n < ((int64_t)1 << 31);
}

size_t bucket_sort_workspace_bytes(int64_t n, int highest_key_bit) {
    if (n < 1) n = 1;
    const int T = 1 << std::max(1, std::min(kMaxBucketBits, highest_key_bit - 32));
    return align256(4 * sizeof(int32_t)) + align256((size_t)T * sizeof(int32_t)) +
           tile_sort_workspace_bytes(n, T) + align256((size_t)n * sizeof(uint64_t));
}

int bucket_sort_pairs(void* ws, size_t ws_bytes, const int64_t* keys_in, int64_t* keys_out,
                      const int32_t* vals_in, int32_t* vals_out, int64_t n, int highest_key_bit,
                      cudaStream_t stream) {
    if (!bucket_sort_applies(n, highest_key_bit))
        return set_error("bucket sort: %d key bits / %lld items not supported", highest_key_bit,
                         (long long)n),
               GS3D_ERR_UNSUPPORTED;
    if (ws_bytes < bucket_sort_workspace_bytes(n, highest_key_bit))
        return set_error("sort temp storage too small: %zu < %zu", ws_bytes,
                         bucket_sort_workspace_bytes(n, highest_key_bit)),
               GS3D_ERR_WORKSPACE;
    if (n == 0) return GS3D_OK;
    const int T = 1 << (highest_key_bit - 32);
    unsigned char* w = static_cast<unsigned char*>(ws);
    int32_t* counts = reinterpret_cast<int32_t*>(w);
    w += align256(4 * sizeof(int32_t));
    int32_t* ends = reinterpret_cast<int32_t*>(w);
    w += align256((size_t)T * sizeof(int32_t));
    const TsLayout L = ts_layout(w, T);
    w += tile_sort_workspace_bytes(n, T);
    uint64_t* entries = reinterpret_cast<uint64_t*>(w);
    const int smem = T * (int)sizeof(int32_t);
    GS3D_CUDA(cudaFuncSetAttribute(k_key_hist, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
              "key histogram shared memory");
    GS3D_CUDA(cudaFuncSetAttribute(k_key_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
              "key scatter shared memory");
    k_key_hist<<<kHistBlocks, kHistThreads, smem, stream>>>(keys_in, n, T, L.bcount, counts);
    GS3D_LAUNCHED("k_key_hist");
    k_tile_colscan<<<(unsigned)ceil_div(T, 32), 256, 0, stream>>>(L.bcount, T, L.tcount);
    GS3D_LAUNCHED("k_tile_colscan");
    k_tile_scan<<<1, 1024, 0, stream>>>(L.tcount, T, n, ends, L.cursor, counts);
    GS3D_LAUNCHED("k_tile_scan");
    k_key_scatter<<<kHistBlocks, kHistThreads, smem, stream>>>(keys_in, n, T, L.cursor, L.bcount, entries);
    GS3D_LAUNCHED("k_key_scatter");
    k_tile_segsort<<<(unsigned)T, kSegThreads, 0, stream>>>(counts, n, ends, entries, L.big, keys_out,
                                                           vals_out, Pairs{keys_in, vals_in});
    GS3D_LAUNCHED("k_tile_segsort");
    return GS3D_OK;
}

}  // namespace gs3d
