// bwd_raster.cu — B2 of backward! (backward_core.jl:37-72): the reverse blend,
// backward_render_tiles_kernel! (backward_core.jl:96-293). Per pixel, back to front from its
// last contributor, T recovered by division by (1 - alpha), the reference's per-pair gradient
// formulas. The gradients are float-atomic sums compared within a tolerance (in the reference
// too), so this file is compiled with floating-point contraction allowed and uses the fast
// exponential and reciprocal intrinsics; the set of (pixel, Gaussian) pairs taken is decided
// exactly: where alpha falls within 4e-6 (relative) of min_alpha the exact exponential
// (gs_expf_blend) decides. The 9 gradients of a (warp, Gaussian) pair are summed across the
// warp with register shuffles before atomics (the reference issues 9 atomics per pixel-pair;
// its TODO at backward_core.jl:282).
//   k_bwd_raster_masks  the forward's contribution masks name each warp's candidate entries
//   k_bwd_raster        without masks: each warp tests every staged entry's cull box
#include "common.cuh"
#include "internal.h"

namespace gs3d {
namespace {

struct BwdArgs {
    const int32_t* sfgidx;
    const int32_t* tiles_end;
    const float* f2d;
    const int32_t* counts;
    int64_t capacity_dup;
    const float* trans;
    const int32_t* last;
    const float* rgb_grad;
    float* mean2d_g;
    float* opacity_g;
    float* licov_g;
    float* color_g;
    int32_t width, height, tile_w, tile_h, tiles_x, compact;
    float bg0, bg1, bg2, min_alpha, max_alpha, log_min_alpha;
    int32_t use_masks;  // the masks kernel is launched too (it takes renders with masks)
    const int32_t* order;  // tiles longest first (NULL: row-major)
    int32_t nb_tiles;
};

// Sum 9 per-lane values over the warp by recursive halving: at each of the five xor levels a
// lane pair exchanges half of its remaining values, 12 shuffles in all. Afterwards the even
// lanes hold complete sums, lane L the sum of value reduce9_index(L) (or padding).
__device__ __forceinline__ float reduce9(const float (&v)[9], int lane) {
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
    float a[5];
#pragma unroll
    for (int k = 0; k < 5; ++k) {
        const float hi = k + 5 < 9 ? v[k + 5] : 0.0f;
        a[k] = (b4 ? hi : v[k]) + __shfl_xor_sync(0xffffffffu, b4 ? v[k] : hi, 16);
    }
    float b[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float hi = k + 3 < 5 ? a[k + 3] : 0.0f;
        b[k] = (b3 ? hi : a[k]) + __shfl_xor_sync(0xffffffffu, b3 ? a[k] : hi, 8);
    }
    float c[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const float hi = k + 2 < 3 ? b[k + 2] : 0.0f;
        c[k] = (b2 ? hi : b[k]) + __shfl_xor_sync(0xffffffffu, b2 ? b[k] : hi, 4);
    }
    const float d = (b1 ? c[1] : c[0]) + __shfl_xor_sync(0xffffffffu, b1 ? c[0] : c[1], 2);
    return d + __shfl_xor_sync(0xffffffffu, d, 1);
}

// Value index whose total reduce9 leaves in lane L (even lanes), or -1 for padding.
__device__ __forceinline__ int reduce9_index(int lane) {
    const int b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1, b1 = (lane >> 1) & 1;
    const int s3 = 2 * b2 + b1;
    if (s3 >= 3) return -1;
    const int s2 = 3 * b3 + s3;
    if (s2 >= 5) return -1;
    const int idx = 5 * b4 + s2;
    return idx < 9 && (lane & 1) == 0 ? idx : -1;
}

#ifndef GS3D_BWD_PX
#define GS3D_BWD_PX 2
#endif
constexpr int kBwdPixelsPerThread = GS3D_BWD_PX;

#ifndef GS3D_BWD_DIRECT_MAX
#define GS3D_BWD_DIRECT_MAX 8
#endif

#ifndef GS3D_BWDRASTER_MINB
#define GS3D_BWDRASTER_MINB 2
#endif

__global__ void __launch_bounds__(512, GS3D_BWDRASTER_MINB) k_bwd_raster(const BwdArgs a) {
    extern __shared__ __align__(16) float4 sm4[];
    const int nthr = blockDim.x;
    float4* sA = sm4;                                          // x y opacity ic11
    float4* sB = sm4 + nthr;                                   // ic21 ic22 r g
    float4* sC = sm4 + 2 * nthr;                               // b q_threshold cx cy
    float2* sR = reinterpret_cast<float2*>(sm4 + 3 * nthr);    // box half-widths
    int* sF = reinterpret_cast<int*>(sR + nthr);               // fgidx (0-based)
    __shared__ int red[32];

    const int F = a.counts[0];
    const int64_t Draw = a.counts[1];
    if (F == 0 || Draw == 0 || Draw > a.capacity_dup) return;  // nothing drawn (or overflow)
    if (a.use_masks && a.counts[3] == 1) return;  // k_bwd_raster_masks does this render

    const int t = threadIdx.x;
    const int lane = t & 31, warp = t >> 5;
    int lu, lv;
    tile_pixel(a.compact, a.tile_w, a.tile_h, t, lu, lv);
    int txi, tyi;
    if (!block_tile(a.order, a.tiles_x, a.nb_tiles, txi, tyi)) return;
    const int u0 = txi * a.tile_w, v0 = tyi * a.tile_h;
    const int U = u0 + lu + 1, V = v0 + lv + 1;
    const bool inside = U <= a.width && V <= a.height;
    const size_t px = (size_t)(V - 1) + (size_t)a.height * (size_t)(U - 1);
    const int tile = txi + tyi * a.tiles_x + 1;
    const int start = tile == 1 ? 0 : a.tiles_end[tile - 2];
    const int end = a.tiles_end[tile - 1];

    float T = 0.0f, g0 = 0.0f, g1 = 0.0f, g2 = 0.0f;
    int lastc = 0;
    if (inside) {
        lastc = a.last[px];
        T = a.trans[px];
        g0 = a.rgb_grad[3 * px];
        g1 = a.rgb_grad[3 * px + 1];
        g2 = a.rgb_grad[3 * px + 2];
    }
    float p0 = T * a.bg0, p1 = T * a.bg1, p2 = T * a.bg2;
    const float cpu = (float)U - 0.5f, cpv = (float)V - 0.5f;
    const float wu0 = (float)__reduce_min_sync(0xffffffffu, (unsigned)lu) + 0.5f;
    const float wu1 = (float)__reduce_max_sync(0xffffffffu, (unsigned)lu) + 0.5f;
    const float wv0 = (float)__reduce_min_sync(0xffffffffu, (unsigned)lv) + 0.5f;
    const float wv1 = (float)__reduce_max_sync(0xffffffffu, (unsigned)lv) + 0.5f;

    // this lane's share of the warp-reduced atomics: pointer and stride of value reduce9_index
    const int vi = reduce9_index(lane);
    float* vptr = nullptr;
    int vstride = 0;
    if (vi >= 0) {
        if (vi < 2) { vptr = a.mean2d_g + vi; vstride = 2; }
        else if (vi == 2) { vptr = a.opacity_g; vstride = 1; }
        else if (vi < 6) { vptr = a.licov_g + (vi - 3); vstride = 3; }
        else { vptr = a.color_g + (vi - 6); vstride = 3; }
    }

    // warp / block maxima of the last contributor (1-based sorted index)
    const int wlast = (int)__reduce_max_sync(0xffffffffu, (unsigned)lastc);
    if (lane == 0) red[warp] = wlast;
    __syncthreads();
    int blast = 0;
    for (int w = 0; w < (nthr >> 5); ++w) blast = max(blast, red[w]);
    const int eff_end = min(end, blast);  // exclusive 0-based == inclusive 1-based

    for (int bend = eff_end; bend > start; bend -= nthr) {
        const int bstart = max(start, bend - nthr);
        const int nb = bend - bstart;
        __syncthreads();
        if (t < nb) {
            const int fg = a.sfgidx[bstart + t] - 1;
            const float* r = a.f2d + 9 * (size_t)fg;
            const float op = r[2];
            const float lop = gs_logf(op);
            sA[t] = make_float4(r[0], r[1], op, r[3]);
            sB[t] = make_float4(r[4], r[5], r[6], r[7]);
            // op * exp(q) < min_alpha whenever q < log(min_alpha) - log(op) - 0.01
            const float thr = op > 0.0f ? a.log_min_alpha - lop - 0.01f : -INFINITY;
            sC[t] = make_float4(r[8], thr, r[0] - (float)u0, r[1] - (float)v0);
            sR[t] = cull_box(r[3], r[4], r[5], lop, a.log_min_alpha);
            sF[t] = fg;
        }
        __syncthreads();
        const int jend = min(nb, wlast - bstart);  // warp-uniform, exclusive
        for (int c1 = jend; c1 > 0; c1 -= 32) {
            const int c0 = max(0, c1 - 32);
            const int j = c0 + lane;
            bool rel = false;
            if (j < c1) {
                const float4 C = sC[j];
                const float2 R = sR[j];
                rel = C.z + R.x >= wu0 && C.z - R.x <= wu1 && C.w + R.y >= wv0 && C.w - R.y <= wv1;
            }
            unsigned mask = __ballot_sync(0xffffffffu, rel);
            while (mask) {
                const int hb = 31 - __clz(mask);
                mask &= ~(1u << hb);
                const int jj = c0 + hb;
                bool contrib = false;
                float v[9] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                if (inside && bstart + jj + 1 <= lastc) {
                    const float4 A = sA[jj];
                    const float4 B = sB[jj];
                    const float4 Cc = sC[jj];
                    const float du = cpu - A.x, dv = cpv - A.y;
                    const float ic11 = A.w, ic21 = B.x, ic22 = B.y;
                    const float du2 = du * du, dv2 = dv * dv, duv = du * dv;
                    const float q = fmaf(-0.5f, fmaf(ic11, du2, ic22 * dv2), -ic21 * duv);
                    if (q >= Cc.y) {
                        // __expf (within 8 ulp for |q| < 6); where alpha falls within 4e-6
                        // (relative) of min_alpha the exact exponential decides, so the
                        // pairs taken are those the forward blended
                        float ge = __expf(q);
                        float alpha = min_hi(a.max_alpha, A.z * ge);
                        if (fabsf(alpha - a.min_alpha) <= 4e-6f * a.min_alpha) {
                            ge = gs_expf_blend(q);
                            alpha = min_hi(a.max_alpha, A.z * ge);
                        }
                        if (alpha >= a.min_alpha) {
                            contrib = true;
                            const float inv1m = __fdividef(1.0f, 1.0f - alpha);
                            T *= inv1m;
                            const float tc0 = T * B.z, tc1 = T * B.w, tc2 = T * Cc.x;
                            p0 = fmaf(alpha, tc0, p0);
                            p1 = fmaf(alpha, tc1, p1);
                            p2 = fmaf(alpha, tc2, p2);
                            const float ag =
                                inv1m * fmaf(g0, tc0 - p0, fmaf(g1, tc1 - p1, g2 * (tc2 - p2)));
                            const float aga = alpha * ag;
                            const float sc = -0.5f * aga;
                            const float g21 = sc * duv;
                            v[0] = aga * fmaf(du, ic11, dv * ic21);
                            v[1] = aga * fmaf(du, ic21, dv * ic22);
                            v[2] = ge * ag;
                            v[3] = sc * du2;
                            v[4] = g21 + g21;
                            v[5] = sc * dv2;
                            const float ta = T * alpha;
                            v[6] = ta * g0;
                            v[7] = ta * g1;
                            v[8] = ta * g2;
                        }
                    }
                }
                const unsigned cmask = __ballot_sync(0xffffffffu, contrib);
                if (cmask == 0) continue;
                const int fg = sF[jj];
                if (__popc(cmask) <= GS3D_BWD_DIRECT_MAX) {
                    if (contrib) {
                        atomicAdd(a.mean2d_g + 2 * fg, v[0]);
                        atomicAdd(a.mean2d_g + 2 * fg + 1, v[1]);
                        atomicAdd(a.opacity_g + fg, v[2]);
                        atomicAdd(a.licov_g + 3 * fg, v[3]);
                        atomicAdd(a.licov_g + 3 * fg + 1, v[4]);
                        atomicAdd(a.licov_g + 3 * fg + 2, v[5]);
                        atomicAdd(a.color_g + 3 * fg, v[6]);
                        atomicAdd(a.color_g + 3 * fg + 1, v[7]);
                        atomicAdd(a.color_g + 3 * fg + 2, v[8]);
                    }
                } else {
                    const float s = reduce9(v, lane);
                    if (vi >= 0) atomicAdd(vptr + (size_t)vstride * fg, s);
                }
            }
        }
    }
}

// ---- over the forward's contribution masks ---------------------------------------------------
// The pairs the reference's backward differentiates are a subset of the pairs the forward marked
// in render_buffers.contrib_masks (every pair it blended, plus those within 0.1% below
// min_alpha: the backward recomputes alpha as opacity x exp(conic form) while the forward folds
// log(opacity) into the exponent, and the two roundings differ by a few ulps). Mask rows are
// those k_raster writes: row (start / 32 + tile - 1 + c) holds chunk c (32 consecutive entries
// of the tile), one word per thread, for the forward's thread -> pixel map (fwd_pixel). A warp
// walks, back to front, only the entries one of its pixels marked (the OR of its lanes' words):
// no cull box, no exponent threshold per staged entry, no iteration without a candidate pixel.
// Every lane runs the same instructions for each entry: a lane that does not take the pair
// (its bit unset, or alpha below min_alpha) carries alpha = 0, exp = 0 and 1 / (1 - alpha) = 1
// through the update, which leaves its T and colour sums exactly unchanged (T x 1, colour +
// 0 x c) and makes its 9 gradients exactly zero, so there are no divergent branches on the
// common path. The same
// pairs in the same order per pixel as k_bwd_raster.
__device__ __forceinline__ void fwd_pixel(int compact, int tw, int th, int t, int& lu, int& lv) {
    if (compact) {
        const PixelGroups<16> pg(compact, tw, th, t, lu, lv);
        (void)pg;
    } else {
        tile_pixel(compact, tw, th, t, lu, lv);
    }
}

// One pixel's state in the reverse walk.
struct PixelState {
    float T, p0, p1, p2, g0, g1, g2, cpu, cpv;
    int rl;  // entries [0, rl) of the tile may be taken (relative to its start)
};

// The reference's per-pair update for one pixel (backward_core.jl:226-286), branch-free: a pair
// not taken (take == false) leaves the state exactly unchanged and gives exact zeros. ADD: add
// the 9 gradients to v, else write them.
template <bool ADD>
__device__ __forceinline__ bool pair_update(PixelState& s, bool mine, const float4 A, const float4 B,
                                            float cb, float min_alpha, float max_alpha, float (&v)[9]) {
    const float du = s.cpu - A.x, dv = s.cpv - A.y;
    const float ic11 = A.z, ic21 = A.w, ic22 = B.x;
    const float du2 = du * du, dv2 = dv * dv, duv = du * dv;
    const float q = fmaf(-0.5f, fmaf(ic11, du2, ic22 * dv2), -ic21 * duv);
    float ge = __expf(q);
    float alpha = min_hi(max_alpha, B.y * ge);
    if (mine && fabsf(alpha - min_alpha) <= 4e-6f * min_alpha) {
        ge = gs_expf_blend(q);
        alpha = min_hi(max_alpha, B.y * ge);
    }
    const bool take = mine && alpha >= min_alpha;
    const float al = take ? alpha : 0.0f;
    ge = take ? ge : 0.0f;
    const float inv1m = take ? __fdividef(1.0f, 1.0f - alpha) : 1.0f;
    s.T *= inv1m;
    const float tc0 = s.T * B.z, tc1 = s.T * B.w, tc2 = s.T * cb;
    s.p0 = fmaf(al, tc0, s.p0);
    s.p1 = fmaf(al, tc1, s.p1);
    s.p2 = fmaf(al, tc2, s.p2);
    const float ag = inv1m * fmaf(s.g0, tc0 - s.p0, fmaf(s.g1, tc1 - s.p1, s.g2 * (tc2 - s.p2)));
    const float aga = al * ag;
    const float sc = -0.5f * aga;
    const float g21 = sc * duv;
    const float ta = s.T * al;
    const float w[9] = {aga * fmaf(du, ic11, dv * ic21), aga * fmaf(du, ic21, dv * ic22), ge * ag,
                        sc * du2, g21 + g21, sc * dv2, ta * s.g0, ta * s.g1, ta * s.g2};
#pragma unroll
    for (int k = 0; k < 9; ++k) v[k] = ADD ? v[k] + w[k] : w[k];
    return take;
}

// PX pixels per thread: thread t of warp w takes the forward's threads (PX w + p) 32 + lane,
// p < PX, i.e. PX of the forward's 4 x 8 warp blocks side by side, so one walk over the entries
// the PX blocks marked serves PX pixels per lane, and one warp reduction per entry covers them.
// An entry a block marked is a candidate for every pixel of that block: a lane takes it when it
// lies before its pixel's last contributor and alpha >= min_alpha, the reference's test (where
// its own pixel did not mark the entry, alpha is below 0.999 min_alpha there and the test fails,
// as it does in k_bwd_raster). A pixel whose block did not mark the entry skips it as a whole.
// Two-pixel blocks: 4 resident per SM (64 registers, a 16-byte spill) measured 1.123 ms at 3M
// Gaussians, 1080p, against 1.169 ms for 3 (75 registers, no spill).
#ifndef GS3D_BWDMASK_MINB
#define GS3D_BWDMASK_MINB 4
#endif

template <int PX>  // 1 or 2
__global__ void __launch_bounds__(512 / PX, PX == 1 ? 2 : GS3D_BWDMASK_MINB) k_bwd_raster_masks(const BwdArgs a,
                                                                               const uint32_t* cmask) {
    extern __shared__ __align__(16) float4 sm4[];
    const int nthr = blockDim.x;
    const int npx = nthr * PX;                               // tile pixels (forward threads)
    float4* E0 = sm4;                                        // x y ic11 ic21
    float4* E1 = sm4 + npx;                                  // ic22 opacity r g
    float* E2 = reinterpret_cast<float*>(sm4 + 2 * npx);     // b
    int* EF = reinterpret_cast<int*>(E2 + npx);              // fgidx (0-based)
    __shared__ int red[32];

    const int F = a.counts[0];
    const int64_t Draw = a.counts[1];
    if (F == 0 || Draw == 0 || Draw > a.capacity_dup || a.counts[3] != 1) return;

    const int t = threadIdx.x;
    const int lane = t & 31, warp = t >> 5;
    int txi, tyi;
    if (!block_tile(a.order, a.tiles_x, a.nb_tiles, txi, tyi)) return;
    const int tile = txi + tyi * a.tiles_x + 1;
    const int start = tile == 1 ? 0 : a.tiles_end[tile - 2];
    const int end = a.tiles_end[tile - 1];
    const int fwarps = npx >> 5;  // the forward's warps per tile: mask words per row
    const uint32_t* mrow = cmask + ((int64_t)(start >> 5) + (tile - 1)) * fwarps + warp * PX;
    PixelState st[PX];
    int lrl = 0;
#pragma unroll
    for (int p = 0; p < PX; ++p) {
        const int ft = (warp * PX + p) * 32 + lane;
        int lu, lv;
        fwd_pixel(a.compact, a.tile_w, a.tile_h, ft, lu, lv);
        const int U = txi * a.tile_w + lu + 1, V = tyi * a.tile_h + lv + 1;
        const bool inside = U <= a.width && V <= a.height;
        const size_t px = (size_t)(V - 1) + (size_t)a.height * (size_t)(U - 1);
        PixelState& s = st[p];
        s.T = s.g0 = s.g1 = s.g2 = 0.0f;
        int lastc = 0;
        if (inside) {
            lastc = a.last[px];
            s.T = a.trans[px];
            s.g0 = a.rgb_grad[3 * px];
            s.g1 = a.rgb_grad[3 * px + 1];
            s.g2 = a.rgb_grad[3 * px + 2];
        }
        s.p0 = s.T * a.bg0;
        s.p1 = s.T * a.bg1;
        s.p2 = s.T * a.bg2;
        s.cpu = (float)U - 0.5f;
        s.cpv = (float)V - 0.5f;
        s.rl = lastc > start ? lastc - start : 0;
        lrl = max(lrl, s.rl);
    }

    // this lane's share of the warp-reduced atomics: pointer and stride of value reduce9_index
    const int vi = reduce9_index(lane);
    float* vptr = nullptr;
    int vstride = 0;
    if (vi >= 0) {
        if (vi < 2) { vptr = a.mean2d_g + vi; vstride = 2; }
        else if (vi == 2) { vptr = a.opacity_g; vstride = 1; }
        else if (vi < 6) { vptr = a.licov_g + (vi - 3); vstride = 3; }
        else { vptr = a.color_g + (vi - 6); vstride = 3; }
    }

    const int wrl = (int)__reduce_max_sync(0xffffffffu, (unsigned)lrl);
    if (lane == 0) red[warp] = wrl;
    __syncthreads();
    int brl = 0;
    for (int w = 0; w < (nthr >> 5); ++w) brl = max(brl, red[w]);
    const float min_alpha = a.min_alpha, max_alpha = a.max_alpha;

    for (int b0 = brl > 0 ? ((brl - 1) / npx) * npx : -1; b0 >= 0; b0 -= npx) {
        __syncthreads();  // every warp is done with the previous batch's entries
#pragma unroll
        for (int p = 0; p < PX; ++p) {
            const int k = t + p * nthr;
            const int e = start + b0 + k;
            if (e < end) {
                const int fg = a.sfgidx[e] - 1;
                const float* r = a.f2d + 9 * (size_t)fg;
                E0[k] = make_float4(r[0], r[1], r[3], r[4]);
                E1[k] = make_float4(r[5], r[2], r[6], r[7]);
                E2[k] = r[8];
                EF[k] = fg;
            }
        }
        __syncthreads();
        const int whi = min(wrl - b0, npx);  // the warp's exclusive bound inside the batch
        if (whi <= 0) continue;
        int w = (whi - 1) >> 5;
        // the PX forward warps' words of row w of the batch: pixel p takes part in an entry
        // only when its own 4 x 8 block marked it (a warp-uniform test)
        uint32_t nxt[PX];
#pragma unroll
        for (int p = 0; p < PX; ++p) nxt[p] = mrow[(int64_t)((b0 >> 5) + w) * fwarps + p];
        for (; w >= 0; --w) {
            uint32_t wp[PX];
            uint32_t wm = 0;
            const int nb = whi - (w << 5);  // drop bits at or beyond the warp's bound
            const uint32_t keep = nb < 32 ? (1u << nb) - 1u : 0xffffffffu;
#pragma unroll
            for (int p = 0; p < PX; ++p) {
                wp[p] = nxt[p] & keep;
                if (w > 0) nxt[p] = mrow[(int64_t)((b0 >> 5) + w - 1) * fwarps + p];
                wm |= wp[p];
            }
            while (wm) {
                const int j = 31 - __clz(wm);
                wm &= ~(1u << j);
                const int en = (w << 5) + j;
                const int rel = b0 + en;
                const float4 A = E0[en];
                const float4 B = E1[en];
                const float cb = E2[en];
                float v[9];
                bool take;
                const bool u0 = (wp[0] >> j) & 1u;
                if (PX == 1 || !((wp[PX - 1] >> j) & 1u)) {
                    take = pair_update<false>(st[0], rel < st[0].rl, A, B, cb, min_alpha, max_alpha, v);
                } else if (!u0) {
                    take = pair_update<false>(st[PX - 1], rel < st[PX - 1].rl, A, B, cb, min_alpha,
                                              max_alpha, v);
                } else {
                    take = pair_update<false>(st[0], rel < st[0].rl, A, B, cb, min_alpha, max_alpha, v);
                    take |= pair_update<true>(st[PX - 1], rel < st[PX - 1].rl, A, B, cb, min_alpha,
                                              max_alpha, v);
                }
                const unsigned cm = __ballot_sync(0xffffffffu, take);
                if (cm == 0) continue;
                const int fg = EF[en];
                if (__popc(cm) <= GS3D_BWD_DIRECT_MAX) {
                    if (take) {
                        atomicAdd(a.mean2d_g + 2 * fg, v[0]);
                        atomicAdd(a.mean2d_g + 2 * fg + 1, v[1]);
                        atomicAdd(a.opacity_g + fg, v[2]);
                        atomicAdd(a.licov_g + 3 * fg, v[3]);
                        atomicAdd(a.licov_g + 3 * fg + 1, v[4]);
                        atomicAdd(a.licov_g + 3 * fg + 2, v[5]);
                        atomicAdd(a.color_g + 3 * fg, v[6]);
                        atomicAdd(a.color_g + 3 * fg + 1, v[7]);
                        atomicAdd(a.color_g + 3 * fg + 2, v[8]);
                    }
                } else {
                    const float sum = reduce9(v, lane);
                    if (vi >= 0) atomicAdd(vptr + (size_t)vstride * fg, sum);
                }
            }
        }
    }
}

}  // namespace

int launch_bwd_raster(const gs3d_fgradients* fg, const float* rgb_grad,
                      const gs3d_render_outputs* out, const gs3d_camera* cam,
                      const gs3d_tiling* til, const gs3d_render_options* opt,
                      const gs3d_render_buffers* buf, cudaStream_t stream) {
    BwdArgs a;
    a.sfgidx = buf->sdfgidx_to_fgidx;
    a.tiles_end = buf->tiles_end_sdfgidx;
    a.f2d = buf->means2d_opacities_inverse_covariances_colors;
    a.counts = buf->device_counts;
    a.capacity_dup = buf->capacity_dup;
    a.trans = out->transmittance;
    a.last = out->last_contributing_sdfgids;
    a.rgb_grad = rgb_grad;
    a.mean2d_g = fg->mean2d_grads;
    a.opacity_g = fg->opacity_grads;
    a.licov_g = fg->licov2d_grads;
    a.color_g = fg->color_grads;
    a.width = cam->width;
    a.height = cam->height;
    a.tile_w = til->tile_width;
    a.tile_h = til->tile_height;
    a.tiles_x = til->nb_tiles_x;
    a.compact = compact_tiles(til->tile_width, til->tile_height);
    a.bg0 = opt->background[0];
    a.bg1 = opt->background[1];
    a.bg2 = opt->background[2];
    a.min_alpha = opt->min_alpha;
    a.max_alpha = opt->max_alpha;
    a.log_min_alpha = opt->min_alpha > 0.0f ? gs_logf(opt->min_alpha) : -INFINITY;
    a.order = buf->tile_order;  // the forward blend's order
    a.nb_tiles = til->nb_tiles_x * til->nb_tiles_y;
    const int nthr = til->tile_width * til->tile_height;
    const size_t smem = (size_t)nthr * (3 * sizeof(float4) + sizeof(float2) + sizeof(int));
    // with contribution masks: k_bwd_raster_masks takes renders that wrote them
    // (device_counts[3]), k_bwd_raster the others; each returns at once on the other's
    a.use_masks = (buf->contrib_masks != nullptr && (nthr & 31) == 0) ? 1 : 0;
    const size_t smem_m = (size_t)nthr * (2 * sizeof(float4) + sizeof(float) + sizeof(int));
    ProfScope prof("bwd_raster", stream);
    const dim3 grid(til->nb_tiles_x, til->nb_tiles_y);
    if (a.use_masks) {
        // two pixels per thread when the tile's warps pair up
        if ((nthr & 63) == 0 && kBwdPixelsPerThread == 2)
            k_bwd_raster_masks<2><<<grid, nthr / 2, smem_m, stream>>>(a, buf->contrib_masks);
        else
            k_bwd_raster_masks<1><<<grid, nthr, smem_m, stream>>>(a, buf->contrib_masks);
        GS3D_LAUNCHED("k_bwd_raster_masks");
    }
    k_bwd_raster<<<grid, nthr, smem, stream>>>(a);
    GS3D_LAUNCHED("k_bwd_raster");
    return GS3D_OK;
}

}  // namespace gs3d
