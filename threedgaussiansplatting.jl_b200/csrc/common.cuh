// common.cuh — shared device/host helpers of libgs3d.so (sm_100a).
//
// Numerics contract: every translation unit is compiled with -fmad=false, so a*b+c is two
// IEEE roundings unless written fmaf(); division and sqrt are IEEE round-to-nearest
// (nvcc's default -prec-div/-prec-sqrt). exp and log are this file's gs_expf / gs_logf,
// implemented from published methods so that results are reproducible off the GPU:
//   * gs_expf: Cody & Waite reduction x = k ln2 + r (|r| <= ln2/2) and the degree-7 Taylor
//     polynomial of e^r (Horner, fused multiply-adds), scaled by 2^k in two exact steps.
//   * gs_logf: x = 2^e m, m in [sqrt(1/2), sqrt(2)); log m = 2 atanh((m-1)/(m+1)) by the
//     odd Taylor series of atanh through the 9th power.
// Both are within about 2 ulp of the true value.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <climits>
#include <cstring>
#include <algorithm>

#include "../../include/gs3d.h"

#define GS_HD __host__ __device__ __forceinline__

namespace gs3d {

// ---- error plumbing (defined in abi.cu) ------------------------------------------------
void set_error(const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
int invalid(const char* fmt, ...);

#define GS3D_CUDA(expr, what)                                           \
    do {                                                                \
        cudaError_t e_ = (expr);                                        \
        if (e_ != cudaSuccess) return ::gs3d::cuda_fail(e_, what);      \
    } while (0)
#define GS3D_LAUNCHED(what)                                             \
    do {                                                                \
        cudaError_t e_ = cudaGetLastError();                            \
        if (e_ != cudaSuccess) return ::gs3d::cuda_fail(e_, what);      \
    } while (0)
#define GS3D_RETURN_IF(status)                                          \
    do {                                                                \
        int s_ = (status);                                              \
        if (s_ != GS3D_OK) return s_;                                   \
    } while (0)

// ---- bit casts ----------------------------------------------------------------------------
GS_HD float u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f; memcpy(&f, &u, 4); return f;
#endif
}
GS_HD uint32_t f2u(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    uint32_t u; memcpy(&u, &f, 4); return u;
#endif
}

// ---- exp / log (see header comment) --------------------------------------------------------
GS_HD float gs_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return u2f(0x7f800000u);
    if (x < -104.0f) return 0.0f;
    const float k = rintf(x * 1.44269502162933349609375f);
    float r = fmaf(-k, 0.693147182464599609375f, x);
    r = fmaf(-k, -1.904654323148236e-09f, r);
    float p = 1.98412698e-04f;
    p = fmaf(p, r, 1.38888892e-03f);
    p = fmaf(p, r, 8.33333377e-03f);
    p = fmaf(p, r, 4.16666679e-02f);
    p = fmaf(p, r, 1.66666672e-01f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ki = (int)k;
    const int k1 = ki / 2;
    const int k2 = ki - k1;
    return (p * u2f((uint32_t)(k1 + 127) << 23)) * u2f((uint32_t)(k2 + 127) << 23);
}

// gs_expf for the alpha-blend exponents, bit for bit: for -80 <= x <= 0.5 the result p 2^k is a
// normal number, so gs_expf's two exact scalings by 2^(k/2) and 2^(k - k/2) equal one exact
// scaling by 2^k; outside that range (and for NaN) it is gs_expf itself.
GS_HD float gs_expf_blend(float x) {
    if (!(x >= -80.0f && x <= 0.5f)) return gs_expf(x);
    const float k = rintf(x * 1.44269502162933349609375f);
    float r = fmaf(-k, 0.693147182464599609375f, x);
    r = fmaf(-k, -1.904654323148236e-09f, r);
    float p = 1.98412698e-04f;
    p = fmaf(p, r, 1.38888892e-03f);
    p = fmaf(p, r, 8.33333377e-03f);
    p = fmaf(p, r, 4.16666679e-02f);
    p = fmaf(p, r, 1.66666672e-01f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return p * u2f((uint32_t)((int)k + 127) << 23);
}

GS_HD float gs_logf(float x) {
    if (x != x) return x;
    if (x < 0.0f) return u2f(0x7fc00000u);
    if (x == 0.0f) return u2f(0xff800000u);
    if (x == u2f(0x7f800000u)) return x;
    int e_adj = 0;
    if (x < 1.17549435e-38f) { x = x * 8388608.0f; e_adj = -23; }
    const uint32_t u = f2u(x);
    int e = (int)((u >> 23) & 0xffu) - 127 + e_adj;
    float m = u2f((u & 0x007fffffu) | 0x3f800000u);
    if (m > 1.41421353816986083984375f) { m = m * 0.5f; e += 1; }
    const float f = m - 1.0f;
    const float s = f / (2.0f + f);
    const float s2 = s * s;
    float p = fmaf(s2, 0.111111112f, 0.142857149f);
    p = fmaf(p, s2, 0.2f);
    p = fmaf(p, s2, 0.333333343f);
    const float t = (s * s2) * p;
    const float logm = 2.0f * s + 2.0f * t;
    const float ef = (float)e;
    return fmaf(ef, 0.693147182464599609375f, fmaf(ef, -1.904654323148236e-09f, logm));
}

// x / b, correctly rounded, for a divisor b > 0 fixed for a whole launch with rb = RN(1/b)
// from the host: q0 = RN(x rb), r = x - b q0 (exact with one FMA), q = RN(q0 + r rb) equals
// RN(x/b) while x, the remainder and the quotient stay clear of underflow and overflow
// (P. Markstein, "Computation of elementary functions on the IBM RISC System/6000 processor",
// IBM J. Res. Dev. 34(1), 1990), i.e. for 2^-100 <= |x| <= 2^80 and b in [2^-40, 1] (the
// bias corrections 1 - beta^t). The other x take exact detours instead of the division's slow
// path: +-0 / b = +-0; a tiny x is divided as x 2^64 and the quotient scaled back by 2^-64,
// exact while that quotient is normal; what is left (subnormal quotients, huge or non-finite
// x, b outside that range) is the ordinary division.
GS_HD float markstein_quotient(float x, float b, float rb) {
    const float q0 = x * rb;
    const float r = fmaf(-b, q0, x);
    return fmaf(r, rb, q0);
}

GS_HD float div_by_const(float x, float b, float rb) {
    const float ax = fabsf(x);
    const bool b_ok = b >= 0x1p-40f && b <= 1.0f;
    if (b_ok && ax >= 0x1p-100f && ax <= 0x1p80f) return markstein_quotient(x, b, rb);
    if (ax == 0.0f && b > 0.0f) return x;
    if (b_ok && ax < 0x1p-100f) {
        const float qs = markstein_quotient(x * 0x1p64f, b, rb);
        if (fabsf(qs) >= 0x1p-62f) return qs * 0x1p-64f;
    }
    return x / b;
}

// num / d (IEEE, correctly rounded) with zero and small numerators kept off the division's
// slow path: +-0 / d = +-0 for d > 0; for |num| < 2^-60 the quotient of num 2^64 is scaled back
// by 2^-64, exact while it is normal and finite; NaN, infinite and the remaining cases divide
// directly.
GS_HD float div_small_num(float num, float d) {
    const float an = fabsf(num);
    if (!(an < 0x1p-60f)) return num / d;
    if (an == 0.0f && d > 0.0f) return num;
    const float qs = (num * 0x1p64f) / d;
    const float aq = fabsf(qs);
    return (aq >= 0x1p-62f && aq <= 0x1p127f) ? qs * 0x1p-64f : num / d;
}

GS_HD float gs_sigmoid(float x) { return 1.0f / (1.0f + gs_expf(-x)); }
GS_HD float gs_logit(float x) { return -gs_logf(1.0f / x - 1.0f); }
GS_HD float jl_clamp(float x, float lo, float hi) { return x > hi ? hi : (x < lo ? lo : x); }
// Julia min(a, b) for floats: NaN if either argument is NaN
GS_HD float fmin_jl(float a, float b) { return (a != a || b != b) ? a + b : (b < a ? b : a); }
// fmin_jl(hi, x) for a hi that is not NaN (callers check): a NaN x fails the comparison and
// stays NaN, every other x gives the same value.
GS_HD float min_hi(float hi, float x) { return x > hi ? hi : x; }

// float -> int32, saturating, NaN -> 0 (NaN / overflowing boxes become empty)
GS_HD int32_t sat_i32(float v) {
    if (v != v) return 0;
    if (v >= 2147483520.0f) return INT32_MAX;
    if (v <= -2147483648.0f) return INT32_MIN;
    return (int32_t)v;
}

// SH constants SH_CONSTS_F64[i] (sh.jl:1-18) rounded to float, i 1-based; folds to a
// literal when i is a compile-time constant.
GS_HD float sh_c(int i) {
    switch (i) {
        case 1: return (float)0.28209479177387814;
        case 2: return (float)0.4886025119029199;
        case 3: return (float)0.4886025119029199;
        case 4: return (float)0.4886025119029199;
        case 5: return (float)1.0925484305920792;
        case 6: return (float)-1.0925484305920792;
        case 7: return (float)0.31539156525252005;
        case 8: return (float)-1.0925484305920792;
        case 9: return (float)0.5462742152960396;
        case 10: return (float)-0.5900435899266435;
        case 11: return (float)2.890611442640554;
        case 12: return (float)-0.4570457994644658;
        case 13: return (float)0.3731763325901154;
        case 14: return (float)-0.4570457994644658;
        case 15: return (float)1.445305721320277;
        case 16: return (float)-0.5900435899266435;
        default: return 0.0f;
    }
}

// evaluate_sh_basis_function (sh.jl:123-149), i 1-based (constant after unrolling)
GS_HD float sh_basis(int i, float x, float y, float z) {
    switch (i) {
        case 1: return sh_c(1);
        case 2: return -y * sh_c(2);
        case 3: return z * sh_c(3);
        case 4: return -x * sh_c(4);
        case 5: return x * y * sh_c(5);
        case 6: return y * z * sh_c(6);
        case 7: return (2.0f * (z * z) - x * x - y * y) * sh_c(7);
        case 8: return x * z * sh_c(8);
        case 9: return (x * x - y * y) * sh_c(9);
        case 10: return y * (3.0f * (x * x) - y * y) * sh_c(10);
        case 11: return x * y * z * sh_c(11);
        case 12: return y * (4.0f * (z * z) - x * x - y * y) * sh_c(12);
        case 13: return z * (2.0f * (z * z) - 3.0f * (x * x + y * y)) * sh_c(13);
        case 14: return x * (4.0f * (z * z) - x * x - y * y) * sh_c(14);
        case 15: return z * (x * x - y * y) * sh_c(15);
        case 16: return x * (x * x - 3.0f * (y * y)) * sh_c(16);
        default: return 0.0f;
    }
}

// ---- tile rasterisation helpers ---------------------------------------------------------
// Pixels of a tile CTA: compact 4 (u) x 8 (v) blocks per warp when the tile allows (v fastest
// inside a block, so a warp stores 4 runs of 8 consecutive pixels of the column-major
// images), else pixel columns (v fastest).
GS_HD int compact_tiles(int tw, int th) { return (tw % 4 == 0 && th % 8 == 0) ? 1 : 0; }

// The tile (0-based column txi, row tyi) a block of a (tiles_x, tiles_y) grid takes: tile
// blockIdx.y * tiles_x + blockIdx.x, or with an order (a permutation of the 0-based tiles) that
// entry of it; false (skip the block) for an entry out of range.
__device__ __forceinline__ bool block_tile(const int32_t* order, int tiles_x, int nb_tiles, int& txi,
                                           int& tyi) {
    int b = blockIdx.x + blockIdx.y * gridDim.x;
    if (order) {
        b = order[b];
        if (b < 0 || b >= nb_tiles) return false;
    }
    txi = b % tiles_x;
    tyi = b / tiles_x;
    return true;
}

__device__ __forceinline__ void tile_pixel(int compact, int tw, int th, int t, int& lu, int& lv) {
    if (compact) {
        const int w = t >> 5, lane = t & 31;
        const int bpr = tw >> 2;
        lu = (w % bpr) * 4 + (lane >> 3);
        lv = (w / bpr) * 8 + (lane & 7);
    } else {
        lv = t % th;
        lu = t / th;
    }
}

// Lane groups of a warp for the rasterisers: GS consecutive lanes (GS = 8, 16 or 32) share one
// rectangle of pixels and walk, in order, only the staged Gaussians whose cull box reaches that
// rectangle, independently of the warp's other groups. Small Gaussians then cost a smaller
// share of the warp. With compact tiles a warp covers a 4 (u) x 8 (v) pixel block split into
// groups of GW x GH pixels (32: 4 x 8, 16: 4 x 4, 8: 2 x 4); otherwise GS is 32 and the warp
// covers pixel columns (tile_pixel).
template <int GS>
struct PixelGroups {
    static constexpr int GW = GS == 8 ? 2 : 4;
    static constexpr int GH = GS == 32 ? 8 : 4;
    static constexpr int NGU = 4 / GW, NGV = 8 / GH, NG = NGU * NGV;
    static_assert(GS == 8 || GS == 16 || GS == 32, "group size");
    int group;
    float r_u0, r_u1, r_v0, r_v1;  // GS == 32: the warp's pixel-centre rectangle
    float b_u, b_v;                // GS < 32: centre of the warp block's first pixel

    // Pixel (lu, lv), 0-based in the tile, of thread t; GS < 32 needs compact tiles.
    __device__ __forceinline__ PixelGroups(int compact, int tw, int th, int t, int& lu, int& lv) {
        const int lane = t & 31;
        if (GS == 32) {
            tile_pixel(compact, tw, th, t, lu, lv);
            group = 0;
            r_u0 = (float)__reduce_min_sync(0xffffffffu, (unsigned)lu) + 0.5f;
            r_u1 = (float)__reduce_max_sync(0xffffffffu, (unsigned)lu) + 0.5f;
            r_v0 = (float)__reduce_min_sync(0xffffffffu, (unsigned)lv) + 0.5f;
            r_v1 = (float)__reduce_max_sync(0xffffffffu, (unsigned)lv) + 0.5f;
            b_u = b_v = 0.0f;
        } else {
            const int w = t >> 5, bpr = tw >> 2;
            const int bu = (w % bpr) * 4, bv = (w / bpr) * 8;
            group = lane / GS;
            const int i = lane % GS;
            lu = bu + (group % NGU) * GW + i / GH;
            lv = bv + (group / NGU) * GH + i % GH;
            b_u = (float)bu + 0.5f;
            b_v = (float)bv + 0.5f;
            r_u0 = r_u1 = r_v0 = r_v1 = 0.0f;
        }
    }

    // Ballot of this lane's group: which of the warp's 32 candidate entries (one per lane,
    // `valid` with box [eu0, eu1] x [ev0, ev1] in tile-local continuous coordinates) overlap
    // the group's pixel-centre rectangle.
    __device__ __forceinline__ unsigned relevant(bool valid, float eu0, float eu1, float ev0,
                                                 float ev1) const {
        if (GS == 32)
            return __ballot_sync(0xffffffffu,
                                 valid && eu1 >= r_u0 && eu0 <= r_u1 && ev1 >= r_v0 && ev0 <= r_v1);
        bool ou[NGU], ov[NGV];
#pragma unroll
        for (int k = 0; k < NGU; ++k) {
            const float u0 = b_u + (float)(k * GW);
            ou[k] = eu1 >= u0 && eu0 <= u0 + (float)(GW - 1);
        }
#pragma unroll
        for (int k = 0; k < NGV; ++k) {
            const float v0 = b_v + (float)(k * GH);
            ov[k] = ev1 >= v0 && ev0 <= v0 + (float)(GH - 1);
        }
        unsigned mine = 0;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
            const unsigned b = __ballot_sync(0xffffffffu, valid && ou[g % NGU] && ov[g / NGU]);
            if (g == group) mine = b;
        }
        return mine;
    }

    // Iterations a warp needs to walk every group's mask.
    __device__ __forceinline__ static int iterations(unsigned mask) {
        if (GS == 32) return __popc(mask);
        return (int)__reduce_max_sync(0xffffffffu, (unsigned)__popc(mask));
    }
};

// Half-widths (rx, ry) of the box, around the mean, outside which a Gaussian with conic
// (ic11, ic21, ic22) and log-opacity lop has alpha < min_alpha at every point: the
// alpha = min_alpha ellipse d'M d = 2 (lop - log(min_alpha)) widened by 0.1 in that form and by
// 0.1% + 0.01 px, far beyond the rounding of either raster kernel's exponent. (+inf, +inf)
// when the conic is degenerate or non-finite (never culled); (-inf, -inf) when no point can
// reach min_alpha.
__device__ __forceinline__ float2 cull_box(float ic11, float ic21, float ic22, float lop,
                                           float log_min_alpha) {
    const float det = ic11 * ic22 - ic21 * ic21;
    const float gamma = 2.0f * (lop - log_min_alpha) + 0.1f;
    const float inf = u2f(0x7f800000u);
    if (!(det > 0.0f) || !(ic11 > 0.0f) || !(ic22 > 0.0f) || !(gamma == gamma) || gamma == inf ||
        det == inf)
        return make_float2(inf, inf);
    if (gamma <= 0.0f) return make_float2(-inf, -inf);
    return make_float2(sqrtf(gamma * ic22 / det) * 1.001f + 0.01f,
                       sqrtf(gamma * ic11 / det) * 1.001f + 0.01f);
}

// ---- launch geometry ---------------------------------------------------------------------
constexpr int kSMs = 148;
constexpr int kChunk = 4096;          // items per scan / sort tile
constexpr int kChunkThreads = 256;
constexpr int kChunkItems = kChunk / kChunkThreads;

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---- warp / block scans ---------------------------------------------------------------
__device__ __forceinline__ int warp_inclusive_scan(int v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// Exclusive block scan of one int per thread (blockDim.x a multiple of 32, <= 1024).
// smem: >= 33 ints. Returns the exclusive prefix; *total receives the block sum.
__device__ __forceinline__ int block_exclusive_scan(int v, int* smem, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    const int inc = warp_inclusive_scan(v);
    if (lane == 31) smem[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const int w = lane < nwarps ? smem[lane] : 0;
        const int wi = warp_inclusive_scan(w);
        if (lane < nwarps) smem[lane] = wi - w;
        if (lane == nwarps - 1) smem[32] = wi;
    }
    __syncthreads();
    const int res = smem[warp] + inc - v;
    *total = smem[32];
    __syncthreads();
    return res;
}

}  // namespace gs3d
