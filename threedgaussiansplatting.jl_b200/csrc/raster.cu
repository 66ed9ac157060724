// raster.cu — front-to-back tile alpha blend, render_tiles_kernel! (forward_core.jl:756-993).
//
// One CTA per tile (tile_width x tile_height threads, one pixel each). The duplicated Gaussians
// of the tile are staged BATCH = blockDim at a time in shared memory in the reference's
// precomputed form (forward_core.jl:877-897): six quadratic-form coefficients with log(opacity)
// absorbed, the colour and the depth. Per pixel the arithmetic and its order are the
// reference's: alpha = min(max_alpha, exp(q)), skip alpha < min_alpha, stop when
// T (1 - alpha) < min_transmittance.
//
// Work saved without changing any pixel's result:
//   * warps cover compact 4 x 8 pixel blocks (when the tile allows; otherwise pixel columns)
//     made of two 16-lane groups of 4 x 4 pixels (PixelGroups); 32 staged entries at a time
//     are tested against each group's block with the entry's alpha >= min_alpha ellipse box
//     (inflated by a safety margin), and each group then evaluates, in order, only the
//     entries that can reach one of its pixels;
//   * q below log(min_alpha) - 0.01 skips the exponential (exp(q) < min_alpha there);
//   * the CTA leaves once every pixel has stopped (__syncthreads_count).
// A CTA reads F and D from device memory and draws the void image itself when there is
// nothing to draw (render_void!, forward_structs.jl:743-757), so no host sync is needed.
#include "common.cuh"
#include "internal.h"

namespace gs3d {

namespace {

struct RasterArgs {
    const int32_t* sfgidx;      // sorted dup -> fgidx (1-based)
    const int32_t* tiles_end;   // per tile, inclusive 1-based end
    const float* f2d;           // 9 x F
    const float* depths;        // F
    const int32_t* counts;      // [0] F, [1] D
    int64_t capacity_dup;
    float* rgb;
    float* trans;
    float* depth_img;
    int32_t* last;
    int32_t width, height;
    int32_t tile_w, tile_h, tiles_x;
    int32_t compact;            // 4 x 8 warp blocks
    float bg0, bg1, bg2;
    float min_alpha, max_alpha, min_T, q_skip, log_min_alpha;
    // contribution masks for the backward blend (NULL: none); see k_raster
    uint32_t* cmask;
    int64_t cmask_words;
    float min_alpha_mark;
    int32_t* mask_flag;         // device_counts[3]
    const int32_t* order;       // tiles longest first (NULL: row-major)
    int32_t nb_tiles;
};

#ifndef GS3D_RASTER_MINB
#define GS3D_RASTER_MINB 3
#endif

// MASKS: write the contribution masks (when a.cmask is set and they fit); without, the blend
// carries no marking work at all.
template <int GS, bool MASKS>
__global__ void __launch_bounds__(512, GS3D_RASTER_MINB) k_raster(const RasterArgs a) {
    extern __shared__ __align__(16) float4 sm4[];
    const int nthr = blockDim.x;
    float4* sA = sm4;                 // p1 p2 p3 p4
    float4* sB = sm4 + nthr;          // p5 p6 r g
    float4* sC = sm4 + 2 * nthr;      // b depth cx cy
    float2* sR = reinterpret_cast<float2*>(sm4 + 3 * nthr);  // box half-widths rx ry

    const int t = threadIdx.x;
    const int lane = t & 31;
    int lu, lv;  // 0-based pixel in tile
    const PixelGroups<GS> pg(a.compact, a.tile_w, a.tile_h, t, lu, lv);
    int txi, tyi;
    if (!block_tile(a.order, a.tiles_x, a.nb_tiles, txi, tyi)) return;
    const int u0 = txi * a.tile_w, v0 = tyi * a.tile_h;
    const int U = u0 + lu + 1, V = v0 + lv + 1;
    const bool inside = U <= a.width && V <= a.height;
    const size_t px = (size_t)(V - 1) + (size_t)a.height * (size_t)(U - 1);

    const int F = a.counts[0];
    const int64_t Draw = a.counts[1];
    // render_void! when there is nothing to draw, and also when the duplicated keys overflowed
    // the buffers (flagged in counts[2]; the sorted arrays and tile ends are then not valid)
    if (F == 0 || Draw == 0 || Draw > a.capacity_dup) {
        if (inside) {
            if (a.rgb) { a.rgb[3 * px] = a.bg0; a.rgb[3 * px + 1] = a.bg1; a.rgb[3 * px + 2] = a.bg2; }
            if (a.trans) a.trans[px] = 1.0f;
            if (a.depth_img) a.depth_img[px] = u2f(0x7f800000u);
            if (a.last) a.last[px] = 0;
        }
        return;
    }
    const int tile = txi + tyi * a.tiles_x + 1;  // 1-based linear, x-contiguous
    const int start = tile == 1 ? 0 : a.tiles_end[tile - 2];
    const int end = a.tiles_end[tile - 1];
    // contribution masks: row (start / 32 + tile - 1 + c) holds, for chunk c of 32 consecutive
    // entries of this tile, one 32-bit word per warp; bit j of warp w's word is set when one of
    // the warp's pixels blended entry 32 c + j, or evaluated it with alpha within 0.1% below
    // min_alpha, before it stopped (the entry that stops a pixel comes after its last
    // contributor, where the backward never looks). Rows of distinct tiles never overlap, and
    // D / 32 + #tiles + 1 rows of nthr / 32 words cover every tile.
    const int nwarps = nthr >> 5;
    const bool wmask = MASKS && a.cmask != nullptr && (nthr & 31) == 0 &&
                       (Draw / 32 + (int64_t)a.nb_tiles + 1) * nwarps <= a.cmask_words;
    if (wmask && t == 0 && blockIdx.x == 0 && blockIdx.y == 0) *a.mask_flag = 1;
    uint32_t* const mrow =
        wmask ? a.cmask + ((int64_t)(start >> 5) + (tile - 1)) * nwarps + (t >> 5) : nullptr;

    const float cu = (float)(lu + 1) - 0.5f, cv = (float)(lv + 1) - 0.5f;
    const float uu = cu * cu, uv = cu * cv, vv = cv * cv;
    float T = 1.0f, c0 = 0.0f, c1 = 0.0f, c2 = 0.0f, dep = 0.0f;
    int32_t lastc = 0;
    bool done = !inside;

    for (int base = start; base < end; base += nthr) {
        if (__syncthreads_count(!done) == 0) break;  // also guards shared-memory reuse
        const int idx = base + t;
        if (idx < end) {
            const int fg = a.sfgidx[idx] - 1;
            const float* r = a.f2d + 9 * (size_t)fg;
            const float x = r[0], y = r[1], op = r[2];
            const float ic11 = r[3], ic21 = r[4], ic22 = r[5];
            const float du = x - (float)u0;
            const float dv = y - (float)v0;
            const float ic11_du = ic11 * du, ic21_du = ic21 * du, ic22_dv = ic22 * dv;
            const float p1 = -0.5f * ic11, p2 = -0.5f * ic22, p3 = -ic21;
            const float p4 = ic11_du + ic21 * dv;
            const float p5 = ic21_du + ic22_dv;
            const float lop = gs_logf(op);
            const float p6 = -0.5f * (ic11_du * du + ic22_dv * dv) - ic21_du * dv + lop;
            sA[t] = make_float4(p1, p2, p3, p4);
            sB[t] = make_float4(p5, p6, r[6], r[7]);
            sC[t] = make_float4(r[8], a.depths[fg], du, dv);
            sR[t] = cull_box(ic11, ic21, ic22, lop, a.log_min_alpha);
        }
        __syncthreads();
        if (__any_sync(0xffffffffu, !done)) {
            const int nb = min(nthr, end - base);
            for (int ch = 0; ch < nb; ch += 32) {
                const int j = ch + lane;
                const bool valid = j < nb;
                float eu0 = 0.0f, eu1 = 0.0f, ev0 = 0.0f, ev1 = 0.0f;
                if (valid) {
                    const float4 C = sC[j];
                    const float2 R = sR[j];
                    eu0 = C.z - R.x; eu1 = C.z + R.x;
                    ev0 = C.w - R.y; ev1 = C.w + R.y;
                }
                unsigned mask = pg.relevant(valid, eu0, eu1, ev0, ev1);
                const int iters = PixelGroups<GS>::iterations(mask);
                uint32_t mw = 0;
                for (int it = 0; it < iters; ++it) {
                    if (!mask) continue;
                    const int jj = ch + __ffs(mask) - 1;
                    mask &= mask - 1;
                    if (done) continue;
                    const float4 A = sA[jj];
                    const float4 B = sB[jj];
                    const float q = A.x * uu + A.y * vv + A.z * uv + A.w * cu + B.x * cv + B.y;
                    if (q < a.q_skip) continue;
                    const float alpha = min_hi(a.max_alpha, gs_expf_blend(q));
                    if (alpha < a.min_alpha) {
                        if (MASKS && alpha >= a.min_alpha_mark) mw |= 1u << (jj - ch);
                        continue;
                    }
                    const float nT = T * (1.0f - alpha);
                    if (nT < a.min_T) { done = true; continue; }
                    if (MASKS) mw |= 1u << (jj - ch);
                    const float w = T * alpha;
                    const float4 C = sC[jj];
                    c0 += w * B.z;
                    c1 += w * B.w;
                    c2 += w * C.x;
                    T = nT;
                    dep += w * C.y;
                    lastc = base + jj + 1;
                }
                if (MASKS && mrow) {
                    const uint32_t ww = __reduce_or_sync(0xffffffffu, mw);
                    if (lane == 0) mrow[(int64_t)((base - start + ch) >> 5) * nwarps] = ww;
                }
                if (__all_sync(0xffffffffu, done)) break;
            }
        }
    }
    if (inside) {
        if (a.rgb) {
            a.rgb[3 * px] = c0 + T * a.bg0;
            a.rgb[3 * px + 1] = c1 + T * a.bg1;
            a.rgb[3 * px + 2] = c2 + T * a.bg2;
        }
        if (a.trans) a.trans[px] = T;
        if (a.depth_img) a.depth_img[px] = dep;
        if (a.last) a.last[px] = lastc;
    }
}

// Work counts of the blend as the reference performs it (render_tiles_kernel!,
// forward_core.jl:928-968): every pixel examines its tile's entries in sorted order until it
// stops. blends = (pixel, entry) evaluations, the terminating one included; contributions =
// evaluations blended into the pixel (alpha >= min_alpha and T (1 - alpha) >= min_T). Same
// staging and arithmetic as k_raster, without its culling, so the counts are the ones the
// reference's loop would reach. For rooflines and tests only; not on the render path.
__global__ void __launch_bounds__(512) k_raster_counts(const RasterArgs a,
                                                       unsigned long long* __restrict__ out) {
    extern __shared__ __align__(16) float4 sm4[];
    __shared__ unsigned long long blk[2];
    const int nthr = blockDim.x;
    float4* sA = sm4;
    float4* sB = sm4 + nthr;
    const int t = threadIdx.x;
    if (t < 2) blk[t] = 0ull;
    int lu, lv;
    tile_pixel(a.compact, a.tile_w, a.tile_h, t, lu, lv);
    const int txi = blockIdx.x, tyi = blockIdx.y;
    const int u0 = txi * a.tile_w, v0 = tyi * a.tile_h;
    const bool inside = u0 + lu + 1 <= a.width && v0 + lv + 1 <= a.height;
    const int F = a.counts[0];
    const int64_t Draw = a.counts[1];
    __syncthreads();
    if (F == 0 || Draw == 0 || Draw > a.capacity_dup) return;
    const int tile = txi + tyi * a.tiles_x + 1;
    const int start = tile == 1 ? 0 : a.tiles_end[tile - 2];
    const int end = a.tiles_end[tile - 1];
    const float cu = (float)(lu + 1) - 0.5f, cv = (float)(lv + 1) - 0.5f;
    const float uu = cu * cu, uv = cu * cv, vv = cv * cv;
    float T = 1.0f;
    bool done = !inside;
    unsigned long long nb = 0, nc = 0;
    for (int base = start; base < end; base += nthr) {
        if (__syncthreads_count(!done) == 0) break;
        const int idx = base + t;
        if (idx < end) {
            const int fg = a.sfgidx[idx] - 1;
            const float* r = a.f2d + 9 * (size_t)fg;
            const float du = r[0] - (float)u0, dv = r[1] - (float)v0;
            const float ic11 = r[3], ic21 = r[4], ic22 = r[5];
            const float ic11_du = ic11 * du, ic21_du = ic21 * du, ic22_dv = ic22 * dv;
            const float p6 = -0.5f * (ic11_du * du + ic22_dv * dv) - ic21_du * dv + gs_logf(r[2]);
            sA[t] = make_float4(-0.5f * ic11, -0.5f * ic22, -ic21, ic11_du + ic21 * dv);
            sB[t] = make_float4(ic21_du + ic22_dv, p6, 0.0f, 0.0f);
        }
        __syncthreads();
        const int n = min(nthr, end - base);
        for (int j = 0; j < n && !done; ++j) {
            const float4 A = sA[j], B = sB[j];
            const float q = A.x * uu + A.y * vv + A.z * uv + A.w * cu + B.x * cv + B.y;
            ++nb;
            if (q < a.q_skip) continue;
            const float alpha = min_hi(a.max_alpha, gs_expf_blend(q));
            if (alpha < a.min_alpha) continue;
            const float nT = T * (1.0f - alpha);
            if (nT < a.min_T) { done = true; break; }
            T = nT;
            ++nc;
        }
    }
    atomicAdd(&blk[0], nb);
    atomicAdd(&blk[1], nc);
    __syncthreads();
    if (t == 0) {
        atomicAdd(out, blk[0]);
        atomicAdd(out + 1, blk[1]);
    }
}

}  // namespace

namespace {
RasterArgs raster_args(const gs3d_render_outputs& out, const gs3d_camera& cam,
                       const gs3d_tiling& til, const gs3d_render_options& opt,
                       const gs3d_render_buffers& buf) {
    RasterArgs a;
    a.sfgidx = buf.sdfgidx_to_fgidx;
    a.tiles_end = buf.tiles_end_sdfgidx;
    a.f2d = buf.means2d_opacities_inverse_covariances_colors;
    a.depths = buf.depths;
    a.counts = buf.device_counts;
    a.capacity_dup = buf.capacity_dup;
    a.rgb = out.rgb;
    a.trans = out.transmittance;
    a.depth_img = out.depth;
    a.last = out.last_contributing_sdfgids;
    a.width = cam.width;
    a.height = cam.height;
    a.tile_w = til.tile_width;
    a.tile_h = til.tile_height;
    a.tiles_x = til.nb_tiles_x;
    a.compact = compact_tiles(til.tile_width, til.tile_height);
    a.bg0 = opt.background[0];
    a.bg1 = opt.background[1];
    a.bg2 = opt.background[2];
    a.min_alpha = opt.min_alpha;
    a.max_alpha = opt.max_alpha;
    a.min_T = opt.min_transmittance;
    // exp(q) < min_alpha for every q < log(min_alpha) - 0.01 (margin >> 2 ulp)
    a.log_min_alpha = opt.min_alpha > 0.0f ? gs_logf(opt.min_alpha) : -INFINITY;
    a.q_skip = opt.min_alpha > 0.0f ? a.log_min_alpha - 0.01f : -INFINITY;
    a.cmask = buf.contrib_masks;
    a.cmask_words = buf.contrib_mask_words;
    a.min_alpha_mark = opt.min_alpha * 0.999f;
    a.mask_flag = buf.device_counts + 3;
    a.order = nullptr;
    a.nb_tiles = til.nb_tiles_x * til.nb_tiles_y;
    return a;
}

// Bucket of a tile with n duplicated entries: 0 for none, else 1 + 8 floor(log2 n) + the next
// three bits of n (at most 248).
__device__ __forceinline__ int order_bucket(int n) {
    if (n <= 0) return 0;
    const int e = 31 - __clz(n);
    const int m = e >= 3 ? (n >> (e - 3)) & 7 : (n << (3 - e)) & 7;
    return 1 + 8 * e + m;
}

// One block: the tiles by descending bucket of their duplicate counts (a counting sort over 256
// buckets; the order within a bucket is that of the shared-memory atomics). Any tile ends give
// a permutation (a void render's are not read).
__global__ void __launch_bounds__(1024) k_tile_order(const int32_t* __restrict__ tiles_end,
                                                     const int32_t* __restrict__ counts,
                                                     int64_t capacity_dup, int nb_tiles,
                                                     int32_t* __restrict__ order) {
    __shared__ int hist[256];
    __shared__ int offs[256];
    const int t = threadIdx.x;
    const int64_t D = counts[1];
    const bool valid = counts[0] > 0 && D > 0 && D <= capacity_dup;
    for (int k = t; k < 256; k += blockDim.x) hist[k] = 0;
    __syncthreads();
    for (int i = t; i < nb_tiles; i += blockDim.x) {
        const int n = valid ? tiles_end[i] - (i ? tiles_end[i - 1] : 0) : 0;
        atomicAdd(&hist[order_bucket(n)], 1);
    }
    __syncthreads();
    if (t < 32) {
        // lane L: buckets 255 - 8 L down to 248 - 8 L; exclusive prefix over lanes, descending
        int local = 0;
        for (int k = 0; k < 8; ++k) local += hist[255 - 8 * t - k];
        int incl = local;
        for (int d = 1; d < 32; d <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, incl, d);
            if (t >= d) incl += o;
        }
        int run = incl - local;
        for (int k = 0; k < 8; ++k) {
            offs[255 - 8 * t - k] = run;
            run += hist[255 - 8 * t - k];
        }
    }
    __syncthreads();
    for (int i = t; i < nb_tiles; i += blockDim.x) {
        const int n = valid ? tiles_end[i] - (i ? tiles_end[i - 1] : 0) : 0;
        order[atomicAdd(&offs[order_bucket(n)], 1)] = i;
    }
}
}  // namespace

int launch_raster_counts(const gs3d_camera& cam, const gs3d_tiling& til,
                         const gs3d_render_options& opt, const gs3d_render_buffers& buf,
                         unsigned long long* counts_out, cudaStream_t stream) {
    const gs3d_render_outputs none = {};
    RasterArgs a = raster_args(none, cam, til, opt, buf);
    a.cmask = nullptr;
    const int nthr = til.tile_width * til.tile_height;
    GS3D_CUDA(cudaMemsetAsync(counts_out, 0, 2 * sizeof(unsigned long long), stream),
              "zero work counts");
    k_raster_counts<<<dim3(til.nb_tiles_x, til.nb_tiles_y), nthr, (size_t)nthr * 2 * sizeof(float4),
                      stream>>>(a, counts_out);
    GS3D_LAUNCHED("k_raster_counts");
    return GS3D_OK;
}

int launch_raster(const gs3d_render_outputs& out, const gs3d_camera& cam, const gs3d_tiling& til,
                  const gs3d_render_options& opt, const gs3d_render_buffers& buf, bool masks,
                  cudaStream_t stream) {
    RasterArgs a = raster_args(out, cam, til, opt, buf);
    if (!masks) a.cmask = nullptr;
    if (buf.tile_order && a.nb_tiles > 0) {
        k_tile_order<<<1, 1024, 0, stream>>>(buf.tiles_end_sdfgidx, buf.device_counts,
                                            buf.capacity_dup, a.nb_tiles, buf.tile_order);
        GS3D_LAUNCHED("k_tile_order");
        a.order = buf.tile_order;
    }
    const int nthr = til.tile_width * til.tile_height;
    const size_t smem = (size_t)nthr * (3 * sizeof(float4) + sizeof(float2));
    dim3 grid(til.nb_tiles_x, til.nb_tiles_y);
    // Compact tiles: 16-lane groups (4 x 4 pixels), measured fastest on the 1080p training
    // workload (8 lanes: equal, 32: 6% slower); other tiles: whole warps over pixel columns.
    if (a.cmask) {
        if (a.compact) k_raster<16, true><<<grid, nthr, smem, stream>>>(a);
        else k_raster<32, true><<<grid, nthr, smem, stream>>>(a);
    } else {
        if (a.compact) k_raster<16, false><<<grid, nthr, smem, stream>>>(a);
        else k_raster<32, false><<<grid, nthr, smem, stream>>>(a);
    }
    GS3D_LAUNCHED("k_raster");
    return GS3D_OK;
}

}  // namespace gs3d
