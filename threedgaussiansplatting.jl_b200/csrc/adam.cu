// adam.cu — update!(opt, fgradients, Val(sh)) (optimizer.jl:964-1009).
//
// The reference launches five kernels (four component groups, then the SH coefficients:
// optimizer.jl:1084-1127, :1165-1248), each walking the F filtered Gaussians. Here two launches
// cover all 59 parameters when every SH array has storage degree 3 (the training configuration):
// k_adam_sh16 (48 words per Gaussian, moved as 16-byte units) and k_adam_geom (the 11 geometry
// scalars). Other storage degrees use one launch, k_adam_warp4, which gives each warp four
// filtered Gaussians at a time; lane s updates scalar slot s of each (SH coefficients first,
// then mean, opacity feature, scales, rotation), so all lanes run the same update with no
// divergence, the SH rows move as consecutive words, and every load of the four Gaussians is in
// flight before the first update.
// Per scalar the reference's update (scalar_adam_update, optimizer.jl:941-953):
//   m1 <- b1 m1 + (1 - b1) g ; m2 <- b2 m2 + (1 - b2) g^2
//   p  <- p - lr (m1 / (1 - b1^t)) / (sqrt(m2 / (1 - b2^t)) + eps),  t = update_count + 1
// Gaussians whose fgidx_to_gidx entry is <= 0 are skipped (optimizer.jl:1099-1103). SH
// coefficient 1 of each channel uses the DC learning rate, the others the rest rate.
#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace gs3d {
namespace {

struct AdamArgs {
    float* mo;      // 4 x n
    float* sf;      // 3 x n
    float* rf;      // 4 x n
    float* sh;      // S x 3 x n
    int S;
    float* mm;      // 2 x 3 x n
    float* om;      // 2 x n
    float* sm;      // 2 x 3 x n
    float* rm;      // 2 x 4 x n
    float* shm;     // 2 x Sm x 3 x n
    int Sm;
    const float* g_mean;   // 3 x F
    const float* g_op;     // F
    const float* g_scale;  // 3 x F
    const float* g_rot;    // 4 x F
    const float* g_sh;     // Sg x 3 x F
    int Sg;
    const int32_t* f2g;
    const int32_t* counts;
    int maxo;              // (render degree + 1)^2
    float lr_means, lr_op, lr_scale, lr_rot, lr_dc, lr_rest;
    float b1, b2, eps, bc1, bc2;
    float rbc1, rbc2;      // RN(1 / bc): the bias-correction divisions as div_by_const
    int64_t ncap;          // capacity of fgidx_to_gidx (the Gaussians' n): F is clamped to it
};

// One scalar update: p - (lr (m1 / bc1)) / (sqrt(m2 / bc2) + eps) with every operation
// correctly rounded. Zero gradients and moments are common (clamped colour channels, unused SH
// bands) and the second moments tiny (squared gradients of 1e-10 and below), so the divisions
// go through div_by_const / div_small_num, which give the same bits without the division's
// slow path.
__device__ __forceinline__ float adam_param(float p, float nm1, float nm2, float lr,
                                            const AdamArgs& a) {
    const float h1 = div_by_const(nm1, a.bc1, a.rbc1);
    const float h2 = div_by_const(nm2, a.bc2, a.rbc2);
    return p - div_small_num(lr * h1, sqrtf(h2) + a.eps);
}

__device__ __forceinline__ void adam_scalar(float* p, float g, float* m, float lr, const AdamArgs& a) {
    const float nm1 = a.b1 * m[0] + (1.0f - a.b1) * g;
    const float nm2 = a.b2 * m[1] + (1.0f - a.b2) * (g * g);
    m[0] = nm1;
    m[1] = nm2;
    *p = adam_param(*p, nm1, nm2, lr, a);
}

__device__ __forceinline__ void adam_reg(float& p, float g, float& m1, float& m2, float lr,
                                         const AdamArgs& a) {
    const float nm1 = a.b1 * m1 + (1.0f - a.b1) * g;
    const float nm2 = a.b2 * m2 + (1.0f - a.b2) * (g * g);
    m1 = nm1;
    m2 = nm2;
    p = adam_param(p, nm1, nm2, lr, a);
}

// Scalar slot s of filtered Gaussian f / Gaussian gi: parameter, first moment (m2 follows),
// gradient and learning rate (slot order as in k_adam_warp).
template <int MAXO>
__device__ __forceinline__ void adam_slot(const AdamArgs& a, int s, int64_t f, size_t gi, float*& p,
                                          float*& m, const float*& g, float& lr) {
    constexpr int NSH = 3 * MAXO;
    if (s < NSH) {
        const int ch = s / MAXO, i = s - ch * MAXO;
        p = a.sh + gi * 3 * a.S + (size_t)(ch * a.S + i);
        g = a.g_sh + (size_t)f * 3 * a.Sg + (size_t)(ch * a.Sg + i);
        m = a.shm + 2 * (gi * 3 * a.Sm + (size_t)(ch * a.Sm + i));
        lr = i == 0 ? a.lr_dc : a.lr_rest;
    } else {
        const int k = s - NSH;
        if (k < 3) {
            p = a.mo + 4 * gi + k; g = a.g_mean + 3 * (size_t)f + k; m = a.mm + 6 * gi + 2 * k; lr = a.lr_means;
        } else if (k == 3) {
            p = a.mo + 4 * gi + 3; g = a.g_op + f; m = a.om + 2 * gi; lr = a.lr_op;
        } else if (k < 7) {
            const int q = k - 4;
            p = a.sf + 3 * gi + q; g = a.g_scale + 3 * (size_t)f + q; m = a.sm + 6 * gi + 2 * q; lr = a.lr_scale;
        } else {
            const int q = k - 7;
            p = a.rf + 4 * gi + q; g = a.g_rot + 4 * (size_t)f + q; m = a.rm + 8 * gi + 2 * q; lr = a.lr_rot;
        }
    }
}

// Four filtered Gaussians per warp iteration, every load issued before any update so that a
// warp keeps up to 8 independent parameter / moment / gradient loads per lane in flight.
template <int MAXO>
__global__ void __launch_bounds__(256) k_adam_warp4(const AdamArgs a) {
    constexpr int G = 4;
    constexpr int NSLOT = 3 * MAXO + 11;
    constexpr int R = (NSLOT + 31) / 32;
    const int F = a.counts[0];
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t base = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * G; base < F;
         base += nwarps * G) {
        const int64_t mine = base + (lane & (G - 1));
        const int gl = (lane < G && mine < F) ? a.f2g[mine] : 0;
        float* pp[G * R];
        float* mp[G * R];
        float pv[G * R], gv[G * R], lr[G * R];
        float2 mv[G * R];
        bool on[G * R];
#pragma unroll
        for (int k = 0; k < G; ++k) {
            const int gidx = __shfl_sync(0xffffffffu, gl, k);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int e = k * R + r;
                const int s = r * 32 + lane;
                on[e] = gidx > 0 && s < NSLOT;
                if (on[e]) {
                    const float* gp;
                    adam_slot<MAXO>(a, s, base + k, (size_t)gidx - 1, pp[e], mp[e], gp, lr[e]);
                    pv[e] = *pp[e];
                    mv[e] = *reinterpret_cast<const float2*>(mp[e]);
                    gv[e] = *gp;
                }
            }
        }
#pragma unroll
        for (int e = 0; e < G * R; ++e) {
            if (!on[e]) continue;
            adam_reg(pv[e], gv[e], mv[e].x, mv[e].y, lr[e], a);
            *pp[e] = pv[e];
            *reinterpret_cast<float2*>(mp[e]) = mv[e];
        }
    }
}

// Storage degree 3 everywhere (Gaussians, moments, gradients): 48 SH words per Gaussian, so
// every Gaussian's SH rows, moment rows and gradient rows are whole 16-byte units.
//   k_adam_sh16: thread 12 f + c updates SH unit c of filtered Gaussian f, words 4c..4c+3 of
//                the parameter row with their 8 interleaved moments and 4 gradients, as four
//                16-byte loads; 12 consecutive threads cover one Gaussian's 192-byte row.
//   k_adam_geom: one thread per filtered Gaussian for the 11 geometry scalars (mean, opacity
//                feature, scales, rotation).
// Grids are sized for the host-known n >= F, one item per thread, so the SMs keep as many
// independent loads in flight as they hold threads (the SH kernel needs few registers and runs
// at full occupancy). Same per-scalar update as above.
__device__ __forceinline__ void adam4(float4& p, const float4& g, float4& m01, float4& m23,
                                      float lr0, float lr, int nup, const AdamArgs& a) {
    adam_reg(p.x, g.x, m01.x, m01.y, lr0, a);
    if (nup > 1) adam_reg(p.y, g.y, m01.z, m01.w, lr, a);
    if (nup > 2) adam_reg(p.z, g.z, m23.x, m23.y, lr, a);
    if (nup > 3) adam_reg(p.w, g.w, m23.z, m23.w, lr, a);
}

#ifndef GS3D_ADAM_GEOM_MINB
#define GS3D_ADAM_GEOM_MINB 5
#endif
#ifndef GS3D_ADAM_DGEOM_MINB
#define GS3D_ADAM_DGEOM_MINB 4
#endif
#ifndef GS3D_ADAM_SH_MINB
#define GS3D_ADAM_SH_MINB 8
#endif

template <int Q>
__device__ __forceinline__ float4 sh_basis4(float x, float y, float z) {
    return make_float4(sh_basis(4 * Q + 1, x, y, z), sh_basis(4 * Q + 2, x, y, z),
                       sh_basis(4 * Q + 3, x, y, z), sh_basis(4 * Q + 4, x, y, z));
}

// SH gradients of coefficients 4q + 1 .. 4q + 4 (1-based) of one colour channel for one view,
// as the projection backward computes them (compute_sh_coeffs_grad!, backward_core.jl:936-964):
// live ? cg * basis_k(d) : 0, d = normalize(mean - camera position), same operations.
__device__ __forceinline__ float4 sh_grad_unit(int q, float cg, bool live, const float4& mo,
                                               float px, float py, float pz) {
    const float vx = mo.x - px, vy = mo.y - py, vz = mo.z - pz;
    const float inv_vn = 1.0f / sqrtf(vx * vx + vy * vy + vz * vz);
    const float nd0 = vx * inv_vn, nd1 = vy * inv_vn, nd2 = vz * inv_vn;
    float4 b;
    switch (q) {
        case 0: b = sh_basis4<0>(nd0, nd1, nd2); break;
        case 1: b = sh_basis4<1>(nd0, nd1, nd2); break;
        case 2: b = sh_basis4<2>(nd0, nd1, nd2); break;
        default: b = sh_basis4<3>(nd0, nd1, nd2); break;
    }
    return live ? make_float4(cg * b.x, cg * b.y, cg * b.z, cg * b.w)
                : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
}

// k_adam_sh16 with the unit's SH gradients recomputed from the filtered Gaussian's colour
// gradient (fgradients' color_grads), its projected colour (row f of the render buffers'
// projected array, floats 6..8: live where >= 0) and the camera position; runs before
// k_adam_geom, which updates the means it reads.
__global__ void __launch_bounds__(256, GS3D_ADAM_SH_MINB) k_adam_sh16_rebuild(const AdamArgs a,
                                                           const float* __restrict__ color_g,
                                                           const float* __restrict__ projected,
                                                           float px, float py, float pz) {
    const uint32_t F = (uint32_t)max(0, min(a.counts[0], (int32_t)a.ncap));
    const uint32_t it = blockIdx.x * blockDim.x + threadIdx.x;
    if (it >= 12u * F) return;
    const uint32_t f = it / 12u;
    const int c = (int)(it - f * 12u);
    const int ch = c >> 2, q = c & 3, i0 = 4 * q;
    if (i0 >= a.maxo) return;
    const int gidx = a.f2g[f];
    if (gidx <= 0) return;
    const size_t gi = (size_t)gidx - 1;
    const float4 mo = reinterpret_cast<const float4*>(a.mo)[gi];
    const float cg = __ldg(color_g + 3 * (size_t)f + ch);
    const bool live = __ldg(projected + 9 * (size_t)f + 6 + ch) >= 0.0f;
    const float4 g = sh_grad_unit(q, cg, live, mo, px, py, pz);
    float4* pp = reinterpret_cast<float4*>(a.sh + gi * 48) + c;
    float4* mp = reinterpret_cast<float4*>(a.shm + gi * 96) + 2 * c;
    float4 p = *pp, m01 = mp[0], m23 = mp[1];
    adam4(p, g, m01, m23, i0 == 0 ? a.lr_dc : a.lr_rest, a.lr_rest, min(4, a.maxo - i0), a);
    *pp = p;
    mp[0] = m01;
    mp[1] = m23;
}

__global__ void __launch_bounds__(256, GS3D_ADAM_SH_MINB) k_adam_sh16(const AdamArgs a) {
    // 32-bit indices: the host only takes this path when 12 n < 2^31
    const uint32_t F = (uint32_t)max(0, min(a.counts[0], (int32_t)a.ncap));
    const uint32_t it = blockIdx.x * blockDim.x + threadIdx.x;
    if (it >= 12u * F) return;
    const uint32_t f = it / 12u;
    const int c = (int)(it - f * 12u);
    const int i0 = 4 * (c & 3);  // coefficient index of the unit's first word
    if (i0 >= a.maxo) return;
    const int gidx = a.f2g[f];
    if (gidx <= 0) return;
    const size_t gi = (size_t)gidx - 1;
    float4* pp = reinterpret_cast<float4*>(a.sh + gi * 48) + c;
    float4* mp = reinterpret_cast<float4*>(a.shm + gi * 96) + 2 * c;
    const float4 g = __ldg(reinterpret_cast<const float4*>(a.g_sh + (size_t)f * 48) + c);
    float4 p = *pp, m01 = mp[0], m23 = mp[1];
    const int nup = min(4, a.maxo - i0);
    adam4(p, g, m01, m23, i0 == 0 ? a.lr_dc : a.lr_rest, a.lr_rest, nup, a);
    *pp = p;
    mp[0] = m01;
    mp[1] = m23;
}


__global__ void __launch_bounds__(256, GS3D_ADAM_GEOM_MINB) k_adam_geom(const AdamArgs a) {
    const int64_t F = max((int64_t)0, min((int64_t)a.counts[0], a.ncap));
    const int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (f >= F) return;
    const int gidx = a.f2g[f];
    if (gidx <= 0) return;
    const size_t gi = (size_t)gidx - 1;
    float4* mop = reinterpret_cast<float4*>(a.mo) + gi;
    float4* rfp = reinterpret_cast<float4*>(a.rf) + gi;
    float2* mmp = reinterpret_cast<float2*>(a.mm) + 3 * gi;
    float2* omp = reinterpret_cast<float2*>(a.om) + gi;
    float2* smp = reinterpret_cast<float2*>(a.sm) + 3 * gi;
    float4* rmp = reinterpret_cast<float4*>(a.rm) + 2 * gi;
    float* sfp = a.sf + 3 * gi;
    float4 mo = *mop, rf = *rfp, rm0 = rmp[0], rm1 = rmp[1];
    float2 mm0 = mmp[0], mm1 = mmp[1], mm2 = mmp[2], om = *omp;
    float2 sm0 = smp[0], sm1 = smp[1], sm2 = smp[2];
    float s0 = sfp[0], s1 = sfp[1], s2 = sfp[2];
    const float gm0 = __ldg(a.g_mean + 3 * f), gm1 = __ldg(a.g_mean + 3 * f + 1),
                gm2 = __ldg(a.g_mean + 3 * f + 2), go = __ldg(a.g_op + f);
    const float gs0 = __ldg(a.g_scale + 3 * f), gs1 = __ldg(a.g_scale + 3 * f + 1),
                gs2 = __ldg(a.g_scale + 3 * f + 2);
    const float4 gr = __ldg(reinterpret_cast<const float4*>(a.g_rot) + f);
    adam_reg(mo.x, gm0, mm0.x, mm0.y, a.lr_means, a);
    adam_reg(mo.y, gm1, mm1.x, mm1.y, a.lr_means, a);
    adam_reg(mo.z, gm2, mm2.x, mm2.y, a.lr_means, a);
    adam_reg(mo.w, go, om.x, om.y, a.lr_op, a);
    adam_reg(s0, gs0, sm0.x, sm0.y, a.lr_scale, a);
    adam_reg(s1, gs1, sm1.x, sm1.y, a.lr_scale, a);
    adam_reg(s2, gs2, sm2.x, sm2.y, a.lr_scale, a);
    adam_reg(rf.x, gr.x, rm0.x, rm0.y, a.lr_rot, a);
    adam_reg(rf.y, gr.y, rm0.z, rm0.w, a.lr_rot, a);
    adam_reg(rf.z, gr.z, rm1.x, rm1.y, a.lr_rot, a);
    adam_reg(rf.w, gr.w, rm1.z, rm1.w, a.lr_rot, a);
    *mop = mo;
    *rfp = rf;
    rmp[0] = rm0;
    rmp[1] = rm1;
    mmp[0] = mm0; mmp[1] = mm1; mmp[2] = mm2;
    *omp = om;
    smp[0] = sm0; smp[1] = sm1; smp[2] = sm2;
    sfp[0] = s0; sfp[1] = s1; sfp[2] = s2;
}

bool aligned(const void* p, uintptr_t b) { return (reinterpret_cast<uintptr_t>(p) & (b - 1)) == 0; }

// The k_adam_sh16 / k_adam_geom layout, apart from the SH gradients.
bool flat16_params_ok(const AdamArgs& a, int64_t n) {
    return n > 0 && 12 * n < ((int64_t)1 << 31) && a.S == 16 && a.Sm == 16 && aligned(a.sh, 16) &&
           aligned(a.shm, 16) && aligned(a.mo, 16) && aligned(a.rf, 16) && aligned(a.rm, 16) &&
           aligned(a.g_rot, 16) && aligned(a.mm, 8) && aligned(a.om, 8) && aligned(a.sm, 8);
}

bool flat16_ok(const AdamArgs& a, int64_t n) {
    return flat16_params_ok(a, n) && a.Sg == 16 && aligned(a.g_sh, 16);
}

int launch_adam_warp(const AdamArgs& a, cudaStream_t stream) {
    const int blocks = device_sm_count() * 8;
    switch (a.maxo) {
        case 1: k_adam_warp4<1><<<blocks, 256, 0, stream>>>(a); break;
        case 4: k_adam_warp4<4><<<blocks, 256, 0, stream>>>(a); break;
        case 9: k_adam_warp4<9><<<blocks, 256, 0, stream>>>(a); break;
        default: k_adam_warp4<16><<<blocks, 256, 0, stream>>>(a); break;
    }
    GS3D_LAUNCHED("k_adam_warp4");
    return GS3D_OK;
}

// Multi-view data parallelism: the gradients of one view are written into a dense row per
// Gaussian (by gs3d_backward_dense directly, or scattered from the F-compact arrays by
// k_scatter_dense), kDenseRow floats: SH 3 x 16 channel-major at 0 (16-byte aligned),
// mean 48, opacity feature 51, scaling features 52, rotation features 55, touched flag 59.
// Rows are summed across ranks (NCCL), then the dense kernels step every touched Gaussian of
// a range [g_begin, g_end) whose rows start at dense[0], with the summed gradients.
constexpr int kDenseRow = GS3D_DENSE_ROW;
constexpr int kDMean = 48, kDOpacity = 51, kDScale = 52, kDRot = 55, kDTouched = 59;
constexpr int kGeomRow = GS3D_GEOM_ROW;

__global__ void __launch_bounds__(256) k_scatter_dense(const AdamArgs a, float* __restrict__ dense) {
    const int F = a.counts[0];
    const int nc = 11 + 3 * a.maxo;
    const int64_t total = (int64_t)F * (nc + 1);
    for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < total;
         it += (int64_t)gridDim.x * blockDim.x) {
        const int f = (int)(it / (nc + 1));
        const int c = (int)(it - (int64_t)f * (nc + 1));
        const int gidx = a.f2g[f];
        if (gidx <= 0) continue;
        float* row = dense + (size_t)(gidx - 1) * kDenseRow;
        if (c == nc) { row[kDTouched] = 1.0f; continue; }
        float v;
        int col;
        if (c < 3) { v = a.g_mean[3 * (size_t)f + c]; col = kDMean + c; }
        else if (c == 3) { v = a.g_op[f]; col = kDOpacity; }
        else if (c < 7) { v = a.g_scale[3 * (size_t)f + (c - 4)]; col = kDScale + (c - 4); }
        else if (c < 11) { v = a.g_rot[4 * (size_t)f + (c - 7)]; col = kDRot + (c - 7); }
        else {
            const int k = c - 11, ch = k / a.maxo, i = k - ch * a.maxo;
            v = a.g_sh[(size_t)f * 3 * a.Sg + (size_t)(ch * a.Sg + i)];
            col = ch * 16 + i;
        }
        row[col] = v;
    }
}

// Any storage degree: one thread per (Gaussian, scalar slot).
__global__ void __launch_bounds__(256) k_adam_dense(const AdamArgs a, const float* __restrict__ dense,
                                                    int64_t g_begin, int64_t g_end) {
    const int nc = 11 + 3 * a.maxo;
    const int64_t total = (g_end - g_begin) * nc;
    for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < total;
         it += (int64_t)gridDim.x * blockDim.x) {
        const int64_t lr_ = it / nc;
        const int c = (int)(it - lr_ * nc);
        const float* row = dense + (size_t)lr_ * kDenseRow;
        if (!(row[kDTouched] > 0.0f)) continue;
        const size_t gi = (size_t)(g_begin + lr_);
        if (c < 3) {
            adam_scalar(a.mo + 4 * gi + c, row[kDMean + c], a.mm + 6 * gi + 2 * c, a.lr_means, a);
        } else if (c == 3) {
            adam_scalar(a.mo + 4 * gi + 3, row[kDOpacity], a.om + 2 * gi, a.lr_op, a);
        } else if (c < 7) {
            const int k = c - 4;
            adam_scalar(a.sf + 3 * gi + k, row[kDScale + k], a.sm + 6 * gi + 2 * k, a.lr_scale, a);
        } else if (c < 11) {
            const int k = c - 7;
            adam_scalar(a.rf + 4 * gi + k, row[kDRot + k], a.rm + 8 * gi + 2 * k, a.lr_rot, a);
        } else {
            const int k = c - 11;
            const int ch = k / a.maxo, i = k - ch * a.maxo;
            adam_scalar(a.sh + gi * 3 * a.S + (size_t)(ch * a.S + i), row[ch * 16 + i],
                        a.shm + gi * 6 * a.Sm + 2 * (size_t)(ch * a.Sm + i),
                        i == 0 ? a.lr_dc : a.lr_rest, a);
        }
    }
}

// Storage degree 3 (the k_adam_sh16 / k_adam_geom forms over dense rows): thread
// 12 (g - g_begin) + c updates SH unit c of Gaussian g from the row's 16-byte unit c.
__global__ void __launch_bounds__(256, GS3D_ADAM_SH_MINB) k_adam_dense_sh16(const AdamArgs a,
                                                         const float* __restrict__ dense,
                                                         int64_t g_begin, int64_t g_end) {
    const int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (it >= 12 * (g_end - g_begin)) return;
    const int64_t lr_ = it / 12;
    const int c = (int)(it - lr_ * 12);
    const int i0 = 4 * (c & 3);
    if (i0 >= a.maxo) return;
    const float* row = dense + (size_t)lr_ * kDenseRow;
    if (!(__ldg(row + kDTouched) > 0.0f)) return;
    const size_t gi = (size_t)(g_begin + lr_);
    float4* pp = reinterpret_cast<float4*>(a.sh + gi * 48) + c;
    float4* mp = reinterpret_cast<float4*>(a.shm + gi * 96) + 2 * c;
    const float4 g = __ldg(reinterpret_cast<const float4*>(row) + c);
    float4 p = *pp, m01 = mp[0], m23 = mp[1];
    adam4(p, g, m01, m23, i0 == 0 ? a.lr_dc : a.lr_rest, a.lr_rest, min(4, a.maxo - i0), a);
    *pp = p;
    mp[0] = m01;
    mp[1] = m23;
}

// Geometry part of a row: 12 floats at `geom` + (g - g_begin) * stride (the dense row's last 12,
// stride kDenseRow, or a factored geometry row, stride kGeomRow).
__global__ void __launch_bounds__(256, GS3D_ADAM_DGEOM_MINB) k_adam_dense_geom(const AdamArgs a,
                                                         const float* __restrict__ geom, int stride,
                                                         int64_t g_begin, int64_t g_end) {
    const int64_t lr_ = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (lr_ >= g_end - g_begin) return;
    const float4* row4 = reinterpret_cast<const float4*>(geom + (size_t)lr_ * stride);
    const float4 r12 = __ldg(row4), r13 = __ldg(row4 + 1), r14 = __ldg(row4 + 2);
    // r12: mean x y z, opacity; r13: scale 0 1 2, rotation 0; r14: rotation 1 2 3, touched
    if (!(r14.w > 0.0f)) return;
    const size_t gi = (size_t)(g_begin + lr_);
    float4* mop = reinterpret_cast<float4*>(a.mo) + gi;
    float4* rfp = reinterpret_cast<float4*>(a.rf) + gi;
    float2* mmp = reinterpret_cast<float2*>(a.mm) + 3 * gi;
    float2* omp = reinterpret_cast<float2*>(a.om) + gi;
    float2* smp = reinterpret_cast<float2*>(a.sm) + 3 * gi;
    float4* rmp = reinterpret_cast<float4*>(a.rm) + 2 * gi;
    float* sfp = a.sf + 3 * gi;
    float4 mo = *mop, rf = *rfp, rm0 = rmp[0], rm1 = rmp[1];
    float2 mm0 = mmp[0], mm1 = mmp[1], mm2 = mmp[2], om = *omp;
    float2 sm0 = smp[0], sm1 = smp[1], sm2 = smp[2];
    float s0 = sfp[0], s1 = sfp[1], s2 = sfp[2];
    adam_reg(mo.x, r12.x, mm0.x, mm0.y, a.lr_means, a);
    adam_reg(mo.y, r12.y, mm1.x, mm1.y, a.lr_means, a);
    adam_reg(mo.z, r12.z, mm2.x, mm2.y, a.lr_means, a);
    adam_reg(mo.w, r12.w, om.x, om.y, a.lr_op, a);
    adam_reg(s0, r13.x, sm0.x, sm0.y, a.lr_scale, a);
    adam_reg(s1, r13.y, sm1.x, sm1.y, a.lr_scale, a);
    adam_reg(s2, r13.z, sm2.x, sm2.y, a.lr_scale, a);
    adam_reg(rf.x, r13.w, rm0.x, rm0.y, a.lr_rot, a);
    adam_reg(rf.y, r14.x, rm0.z, rm0.w, a.lr_rot, a);
    adam_reg(rf.z, r14.y, rm1.x, rm1.y, a.lr_rot, a);
    adam_reg(rf.w, r14.z, rm1.z, rm1.w, a.lr_rot, a);
    *mop = mo;
    *rfp = rf;
    rmp[0] = rm0;
    rmp[1] = rm1;
    mmp[0] = mm0; mmp[1] = mm1; mmp[2] = mm2;
    *omp = om;
    smp[0] = sm0; smp[1] = sm1; smp[2] = sm2;
    sfp[0] = s0; sfp[1] = s1; sfp[2] = s2;
}

// Factored rows (sharded multi-view step): the SH gradient of Gaussian g is rebuilt from the
// colour rows of the views, sum over v = 0 .. nv - 1 of live_c(v) cg_c(v) basis_k(d_v), d_v the
// unit direction from camera v to the Gaussian's mean, each term the expression the projection
// backward uses for one view (compute_sh_coeffs_grad!, backward_core.jl:936-964), the terms added
// in view order starting from the first view that filtered the Gaussian (one view: the
// single-view gradient bit for bit). Thread 12 (g - g_begin) + c updates SH unit c; it reads the
// mean, so it runs before k_adam_dense_geom updates it.
struct ViewPositions {
    float p[GS3D_MAX_FACTORED_VIEWS][3];
};

__global__ void __launch_bounds__(256, GS3D_ADAM_SH_MINB) k_adam_factored_sh16(const AdamArgs a,
                                                            const float* __restrict__ geom,
                                                            const float4* __restrict__ colour,
                                                            int nv, int64_t view_stride,
                                                            const ViewPositions vp,
                                                            int64_t g_begin, int64_t g_end) {
    const int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (it >= 12 * (g_end - g_begin)) return;
    const int64_t lr_ = it / 12;
    const int c = (int)(it - lr_ * 12);
    const int ch = c >> 2, q = c & 3, i0 = 4 * q;
    if (i0 >= a.maxo) return;
    if (!(__ldg(geom + (size_t)lr_ * kGeomRow + (kGeomRow - 1)) > 0.0f)) return;
    const size_t gi = (size_t)(g_begin + lr_);
    const float4 mo = reinterpret_cast<const float4*>(a.mo)[gi];
    float4 g = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    bool first = true;
    for (int v = 0; v < nv; ++v) {
        const float4 cr = __ldg(colour + (size_t)v * view_stride + lr_);
        if (!(cr.w > 0.0f)) continue;  // not filtered in view v
        const int fl = (int)cr.w;
        const bool live = ((fl >> (1 + ch)) & 1) != 0;
        const float cg = ch == 0 ? cr.x : (ch == 1 ? cr.y : cr.z);
        const float4 t = sh_grad_unit(q, cg, live, mo, vp.p[v][0], vp.p[v][1], vp.p[v][2]);
        if (first) {
            g = t;
            first = false;
        } else {
            g.x = g.x + t.x; g.y = g.y + t.y; g.z = g.z + t.z; g.w = g.w + t.w;
        }
    }
    float4* pp = reinterpret_cast<float4*>(a.sh + gi * 48) + c;
    float4* mp = reinterpret_cast<float4*>(a.shm + gi * 96) + 2 * c;
    float4 p = *pp, m01 = mp[0], m23 = mp[1];
    adam4(p, g, m01, m23, i0 == 0 ? a.lr_dc : a.lr_rest, a.lr_rest, min(4, a.maxo - i0), a);
    *pp = p;
    mp[0] = m01;
    mp[1] = m23;
}

}  // namespace

// 1 - beta^t rounded to float, t = update_count + 1 (the bias corrections of
// scalar_adam_update; beta^t is taken in double and rounded once).
float adam_bias_correction(float beta, int32_t update_count) {
    return 1.0f - (float)std::pow((double)beta, (double)update_count + 1.0);
}

}  // namespace gs3d

using namespace gs3d;

namespace {

// Shared argument set-up; g / m / p may be NULL only where the caller does not need them.
int make_args(const gs3d_gaussians* g, const gs3d_adam_moments* m, const gs3d_fgradients* fg,
              const int32_t* fgidx_to_gidx, const int32_t* device_counts,
              const gs3d_adam_params* p, AdamArgs& a) {
    a = AdamArgs{};
    if (!p) return invalid("NULL Adam parameters");
    if (p->sh_degree < 0 || p->sh_degree > 3) return invalid("Adam SH degree %d", p->sh_degree);
    if (g && (p->sh_degree > g->sh_degree)) return invalid("SH degree exceeds the Gaussians'");
    if (m && (p->sh_degree > m->sh_degree)) return invalid("SH degree exceeds the moments'");
    if (fg && (p->sh_degree > fg->sh_degree)) return invalid("SH degree exceeds the gradients'");
    if (p->update_count < 0) return invalid("update_count %d", p->update_count);
    if (g) {
        a.mo = g->means_opacity_features; a.sf = g->scaling_features; a.rf = g->rotation_features;
        a.sh = g->sh_coeffs; a.S = (g->sh_degree + 1) * (g->sh_degree + 1);
    }
    if (m) {
        a.mm = m->means_moments; a.om = m->opacity_features_moments; a.sm = m->scaling_features_moments;
        a.rm = m->rotation_features_moments; a.shm = m->sh_coeffs_moments;
        a.Sm = (m->sh_degree + 1) * (m->sh_degree + 1);
    }
    if (fg) {
        a.g_mean = fg->mean3d_grads; a.g_op = fg->opacity_feature_grads;
        a.g_scale = fg->scaling_features_grads; a.g_rot = fg->rotation_features_grads;
        a.g_sh = fg->sh_coeffs_grads; a.Sg = (fg->sh_degree + 1) * (fg->sh_degree + 1);
    }
    a.f2g = fgidx_to_gidx;
    a.counts = device_counts;
    a.maxo = (p->sh_degree + 1) * (p->sh_degree + 1);
    a.lr_means = p->lr_means; a.lr_op = p->lr_opacity_features; a.lr_scale = p->lr_scaling_features;
    a.lr_rot = p->lr_rotation_features; a.lr_dc = p->lr_sh_dc; a.lr_rest = p->lr_sh_rest;
    a.b1 = p->beta1; a.b2 = p->beta2; a.eps = p->epsilon;
    a.bc1 = adam_bias_correction(p->beta1, p->update_count);
    a.bc2 = adam_bias_correction(p->beta2, p->update_count);
    a.rbc1 = 1.0f / a.bc1;
    a.rbc2 = 1.0f / a.bc2;
    return GS3D_OK;
}

}  // namespace

extern "C" GS3D_API int gs3d_adam_step(const gs3d_gaussians* g, const gs3d_adam_moments* m,
                                       const gs3d_fgradients* fg, const int32_t* fgidx_to_gidx,
                                       const int32_t* device_counts, const gs3d_adam_params* p,
                                       gs3d_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (!g || !m || !fg || !fgidx_to_gidx || !device_counts || !p) return invalid("NULL argument");
    AdamArgs a;
    GS3D_RETURN_IF(make_args(g, m, fg, fgidx_to_gidx, device_counts, p, a));
    ProfScope prof("adam", stream);
    if (flat16_ok(a, g->n)) {
        a.ncap = g->n;
        k_adam_sh16<<<(unsigned)ceil_div(12 * (int64_t)g->n, 256), 256, 0, stream>>>(a);
        GS3D_LAUNCHED("k_adam_sh16");
        k_adam_geom<<<(unsigned)ceil_div((int64_t)g->n, 256), 256, 0, stream>>>(a);
        GS3D_LAUNCHED("k_adam_geom");
        return GS3D_OK;
    }
    GS3D_RETURN_IF(launch_adam_warp(a, stream));
    return GS3D_OK;
}

extern "C" GS3D_API int gs3d_scatter_dense_grads(const gs3d_fgradients* fg,
                                                 const int32_t* fgidx_to_gidx,
                                                 const int32_t* device_counts, int32_t sh_degree,
                                                 float* dense, int32_t n, gs3d_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (!fg || !fgidx_to_gidx || !device_counts || !dense || n < 0) return invalid("NULL argument");
    gs3d_adam_params p{};
    p.sh_degree = sh_degree;
    p.beta1 = 0.5f;
    p.beta2 = 0.5f;
    AdamArgs a;
    GS3D_RETURN_IF(make_args(nullptr, nullptr, fg, fgidx_to_gidx, device_counts, &p, a));
    ProfScope prof("scatter_dense", stream);
    GS3D_CUDA(cudaMemsetAsync(dense, 0, (size_t)n * kDenseRow * sizeof(float), stream), "zero dense");
    k_scatter_dense<<<device_sm_count() * 8, 256, 0, stream>>>(a, dense);
    GS3D_LAUNCHED("k_scatter_dense");
    return GS3D_OK;
}

extern "C" GS3D_API int gs3d_adam_step_dense_range(const gs3d_gaussians* g,
                                                   const gs3d_adam_moments* m, const float* dense,
                                                   int32_t g_begin, int32_t g_end,
                                                   const gs3d_adam_params* p,
                                                   gs3d_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (!g || !m || !dense || !p) return invalid("NULL argument");
    if (g_begin < 0 || g_end < g_begin || g_end > g->n)
        return invalid("Gaussian range [%d, %d) of n = %d", g_begin, g_end, g->n);
    AdamArgs a;
    GS3D_RETURN_IF(make_args(g, m, nullptr, nullptr, nullptr, p, a));
    if (g_end == g_begin) return GS3D_OK;
    ProfScope prof("adam_dense", stream);
    const int64_t cnt = (int64_t)g_end - g_begin;
    const bool flat = a.S == 16 && a.Sm == 16 && aligned(dense, 16) && aligned(a.sh, 16) &&
                      aligned(a.shm, 16) && aligned(a.mo, 16) && aligned(a.rf, 16) &&
                      aligned(a.rm, 16) && aligned(a.mm, 8) && aligned(a.om, 8) && aligned(a.sm, 8);
    if (flat) {
        k_adam_dense_sh16<<<(unsigned)ceil_div(12 * cnt, 256), 256, 0, stream>>>(a, dense, g_begin, g_end);
        GS3D_LAUNCHED("k_adam_dense_sh16");
        k_adam_dense_geom<<<(unsigned)ceil_div(cnt, 256), 256, 0, stream>>>(a, dense + kDMean, kDenseRow,
                                                                            g_begin, g_end);
        GS3D_LAUNCHED("k_adam_dense_geom");
    } else {
        k_adam_dense<<<device_sm_count() * 8, 256, 0, stream>>>(a, dense, g_begin, g_end);
        GS3D_LAUNCHED("k_adam_dense");
    }
    return GS3D_OK;
}

extern "C" GS3D_API int gs3d_adam_step_dense(const gs3d_gaussians* g, const gs3d_adam_moments* m,
                                             const float* dense, const gs3d_adam_params* p,
                                             gs3d_stream_t stream) {
    if (!g) return invalid("NULL argument");
    return gs3d_adam_step_dense_range(g, m, dense, 0, g->n, p, stream);
}

extern "C" GS3D_API int gs3d_adam_step_factored_range(
    const gs3d_gaussians* g, const gs3d_adam_moments* m, const float* geom_rows,
    const float* colour_rows, int32_t n_views, int64_t view_stride, const float* view_positions,
    int32_t g_begin, int32_t g_end, const gs3d_adam_params* p, gs3d_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (!g || !m || !geom_rows || !colour_rows || !view_positions || !p) return invalid("NULL argument");
    if (g_begin < 0 || g_end < g_begin || g_end > g->n)
        return invalid("Gaussian range [%d, %d) of n = %d", g_begin, g_end, g->n);
    if (n_views < 1 || n_views > GS3D_MAX_FACTORED_VIEWS)
        return invalid("%d views (1 .. %d)", n_views, GS3D_MAX_FACTORED_VIEWS);
    if (view_stride < (int64_t)g_end - g_begin) return invalid("view stride %lld < range", (long long)view_stride);
    AdamArgs a;
    GS3D_RETURN_IF(make_args(g, m, nullptr, nullptr, nullptr, p, a));
    if (!(a.S == 16 && a.Sm == 16 && aligned(geom_rows, 16) && aligned(colour_rows, 16) &&
          aligned(a.sh, 16) && aligned(a.shm, 16) && aligned(a.mo, 16) && aligned(a.rf, 16) &&
          aligned(a.rm, 16) && aligned(a.mm, 8) && aligned(a.om, 8) && aligned(a.sm, 8)))
        return invalid("factored Adam needs storage degree 3 and 16-byte aligned arrays");
    if (g_end == g_begin) return GS3D_OK;
    ViewPositions vp{};
    for (int v = 0; v < n_views; ++v)
        for (int k = 0; k < 3; ++k) vp.p[v][k] = view_positions[3 * v + k];
    ProfScope prof("adam_dense", stream);
    const int64_t cnt = (int64_t)g_end - g_begin;
    k_adam_factored_sh16<<<(unsigned)ceil_div(12 * cnt, 256), 256, 0, stream>>>(
        a, geom_rows, reinterpret_cast<const float4*>(colour_rows), n_views, view_stride, vp, g_begin, g_end);
    GS3D_LAUNCHED("k_adam_factored_sh16");
    k_adam_dense_geom<<<(unsigned)ceil_div(cnt, 256), 256, 0, stream>>>(a, geom_rows, kGeomRow, g_begin, g_end);
    GS3D_LAUNCHED("k_adam_dense_geom");
    return GS3D_OK;
}

extern "C" GS3D_API int gs3d_adam_step_rebuild_sh(const gs3d_gaussians* g, const gs3d_adam_moments* m,
                                                  const gs3d_fgradients* fg,
                                                  const int32_t* fgidx_to_gidx,
                                                  const int32_t* device_counts,
                                                  const float* projected,
                                                  const float* camera_position,
                                                  const gs3d_adam_params* p, gs3d_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (!g || !m || !fg || !fgidx_to_gidx || !device_counts || !projected || !camera_position || !p)
        return invalid("NULL argument");
    if (!fg->color_grads) return invalid("NULL colour gradients");
    AdamArgs a;
    GS3D_RETURN_IF(make_args(g, m, fg, fgidx_to_gidx, device_counts, p, a));
    // the SH gradients are not read: only the other arrays need the flat layout
    if (!flat16_params_ok(a, g->n))
        return invalid("rebuilt SH update needs storage degree 3 and aligned arrays");
    ProfScope prof("adam", stream);
    a.ncap = g->n;
    k_adam_sh16_rebuild<<<(unsigned)ceil_div(12 * (int64_t)g->n, 256), 256, 0, stream>>>(
        a, fg->color_grads, projected, camera_position[0], camera_position[1], camera_position[2]);
    GS3D_LAUNCHED("k_adam_sh16_rebuild");
    k_adam_geom<<<(unsigned)ceil_div((int64_t)g->n, 256), 256, 0, stream>>>(a);
    GS3D_LAUNCHED("k_adam_geom");
    return GS3D_OK;
}
