// backward.cu — backward! (backward_core.jl:37-72).
//   k_zero_2d        zero_2d_grads! over the F filtered Gaussians (backward_structs.jl:250-257)
//   (B2, the reverse blend, is in bwd_raster.cu: launch_bwd_raster)
//   k_bwd_project    backward_project_fgaussians_kernel! (backward_core.jl:309-452) with
//                    compute_cov2d_lower_grad, Transposed_dsigma_dm / dv / dv_ds, DL_dR,
//                    compute_normed_q_grad, compute_sh_coeffs_grad! and the colour/direction
//                    Jacobian of sh.jl:175-267 (coefficient 15 in its last term unless
//                    GS3D_BACKWARD_FIX_SH16).
#include "common.cuh"
#include "internal.h"

namespace gs3d {

int check_render_common(const gs3d_gaussians* g, const gs3d_camera* cam, const gs3d_tiling* til,
                        const gs3d_render_options* opt);
int launch_bwd_raster(const gs3d_fgradients* fg, const float* rgb_grad,
                      const gs3d_render_outputs* out, const gs3d_camera* cam,
                      const gs3d_tiling* til, const gs3d_render_options* opt,
                      const gs3d_render_buffers* buf, cudaStream_t stream);

namespace {

__global__ void __launch_bounds__(256) k_zero_2d(const int32_t* __restrict__ counts,
                                                 float* __restrict__ m2, float* __restrict__ op,
                                                 float* __restrict__ li, float* __restrict__ co) {
    const int F = counts[0];
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 3 * F; i += gridDim.x * blockDim.x) {
        li[i] = 0.0f;
        co[i] = 0.0f;
        if (i < 2 * F) m2[i] = 0.0f;
        if (i < F) op[i] = 0.0f;
    }
}

// ---- projection backward -------------------------------------------------------------------
__device__ __forceinline__ int low3(int i, int j) {
    // column-major lower index of a symmetric 3x3: (0,0)0 (1,0)1 (2,0)2 (1,1)3 (2,1)4 (2,2)5
    const int hi = i > j ? i : j, lo = i > j ? j : i;
    return lo == 0 ? hi : (lo == 1 ? 2 + hi : 5);
}

// The colour -> direction Jacobian of sh.jl:175-267 for the channels whose colour is positive
// (`pos`): Jt[i][c] = d colour_c / d direction_i at the unit direction (x, y, z), from the SH row
// read linearly as the reference does (hc = mys + c MAXO: coefficients 0 .. 3 MAXO - 1 of the
// row, sh.jl:196); coefficient 15 in the last degree-3 term unless fix_sh16.
template <int DEG>
__device__ __forceinline__ void colour_dir_jacobian(const float* mys, float x, float y, float z,
                                                    const bool (&pos)[3], int fix_sh16,
                                                    float (&Jt)[3][3]) {
    constexpr int MAXO = (DEG + 1) * (DEG + 1);
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int c = 0; c < 3; ++c) Jt[i][c] = 0.0f;
    if (DEG > 0) {
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            if (!pos[c]) continue;
            const float* hc = mys + c * MAXO;
            float dy = -sh_c(2) * hc[1];
            float dz = sh_c(3) * hc[2];
            float dx = -sh_c(4) * hc[3];
            if (DEG >= 2) {
                { const float q = sh_c(5) * hc[4]; dx += y * q; dy += x * q; }
                { const float q = sh_c(6) * hc[5]; dy += z * q; dz += y * q; }
                { const float q = sh_c(7) * hc[6]; dx -= 2.0f * x * q; dy -= 2.0f * y * q; dz += 4.0f * z * q; }
                { const float q = sh_c(8) * hc[7]; dx += z * q; dz += x * q; }
                { const float q = sh_c(9) * hc[8]; dx += 2.0f * x * q; dy -= 2.0f * y * q; }
                if (DEG >= 3) {
                    { const float q = sh_c(10) * hc[9]; dx += 6.0f * x * y * q; dy += 3.0f * (x * x - y * y) * q; }
                    { const float q = sh_c(11) * hc[10]; dx += y * z * q; dy += x * z * q; dz += x * y * q; }
                    { const float q = sh_c(12) * hc[11];
                      dx -= 2.0f * x * y * q;
                      dy += (4.0f * (z * z) - x * x - 3.0f * (y * y)) * q;
                      dz += 8.0f * y * z * q; }
                    { const float q = sh_c(13) * hc[12];
                      dx -= 6.0f * x * z * q;
                      dy -= 6.0f * y * z * q;
                      dz += 3.0f * (2.0f * (z * z) - x * x - y * y) * q; }
                    { const float q = sh_c(14) * hc[13];
                      dx += (4.0f * (z * z) - 3.0f * (x * x) - y * y) * q;
                      dy -= 2.0f * x * y * q;
                      dz += 8.0f * x * z * q; }
                    { const float q = sh_c(15) * hc[14]; dx += 2.0f * x * z * q; dy -= 2.0f * y * z * q; dz += (x * x - y * y) * q; }
                    { const float q = sh_c(16) * (fix_sh16 ? hc[15] : hc[14]);
                      dx += 3.0f * (x * x - y * y) * q;
                      dy -= 6.0f * x * y * q; }
                }
            }
            Jt[0][c] = dx; Jt[1][c] = dy; Jt[2][c] = dz;
        }
    }
}

// m3 += the mean3d gradient through the direction's normalisation: inv_vn (I - nd nd^T) Jt cgr.
__device__ __forceinline__ void add_colour_dir_term(const float (&Jt)[3][3], const float (&cgr)[3],
                                                    const float (&nd)[3], float inv_vn, float (&m3)[3]) {
    float ndg[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) ndg[i] = Jt[i][0] * cgr[0] + Jt[i][1] * cgr[1] + Jt[i][2] * cgr[2];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        float w = 0.0f;
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            const float Nij = i == j ? 1.0f - nd[i] * nd[i] : -nd[i < j ? i : j] * nd[i < j ? j : i];
            w = w + Nij * ndg[j];
        }
        m3[i] = m3[i] + inv_vn * w;
    }
}

struct BProjArgs {
    const float4* mo4;
    const float* scal;
    const float4* rot4;
    const float* sh;
    int sh_stride;
    const int32_t* f2g;
    const float* f2d;
    const int32_t* counts;
    const float* mean2d_g;
    const float* opacity_g;
    const float* licov_g;
    const float* color_g;
    float* mean3d_g;
    float* opf_g;
    float* scale_g;
    float* rot_g;
    float* sh_g;
    int sh_grad_stride;
    int fix_sh16;
    int skip_sh;  // GS3D_BACKWARD_SKIP_SH_GRADS: no SH gradients (F-compact output only)
    int no_dir;   // GS3D_BACKWARD_NO_COLOUR_DIRECTION: no colour -> direction term, SH not read
    int accumulate;  // GS3D_BACKWARD_ACCUMULATE_ROWS: add into dense / geometry rows
    // NULL, or dense gradient rows indexed by Gaussian (kDenseRow floats, layout in gs3d.h):
    // the 3D gradients then go to row gidx - g_begin instead of the F-compact arrays above
    float* dense;
    // NULL, or the factored rows (dense == NULL): geometry row gidx - g_begin (kGeomRow floats,
    // the dense row's last 12) and colour row gidx - g_begin (the three colour gradients and
    // the flags 1 + 2 live0 + 4 live1 + 8 live2 + 16 pos0 + 32 pos1 + 64 pos2) instead of the
    // SH gradients
    float* geom;
    float4* colour;
    // only filtered Gaussians whose 0-based Gaussian index is in [g_begin, g_end) are done
    int32_t g_begin, g_end;
};

// Dense gradient row (GS3D_DENSE_ROW): SH 3 x 16 channel-major at 0, mean 48, opacity feature
// 51, scaling features 52, rotation features 55, touched flag 59.
// Offsets below are relative to the geometry part (dense row + 48, or the factored geometry row).
constexpr int kDenseRow = GS3D_DENSE_ROW;
constexpr int kDGeom = 48, kGeomRow = GS3D_GEOM_ROW;
constexpr int kDMean = 0, kDOpacity = 3, kDScale = 4, kDRot = 7, kDTouched = 11;

#ifndef GS3D_BWDPROJ_MINB
#define GS3D_BWDPROJ_MINB 4
#endif

template <int DEG>
__global__ void __launch_bounds__(128, GS3D_BWDPROJ_MINB) k_bwd_project(const BProjArgs a, const gs3d_camera cam,
                                                     const gs3d_render_options opt) {
    const int F = a.counts[0];
    float Ps[3][3];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) Ps[i][j] = cam.P[i + 3 * j];
    const int L2I[3] = {0, 1, 1}, L2J[3] = {0, 0, 1};
    const int L3I[6] = {0, 1, 2, 1, 2, 2}, L3J[6] = {0, 0, 0, 1, 1, 2};
    constexpr int MAXO = (DEG + 1) * (DEG + 1);
    constexpr int NSH = 3 * MAXO;
    // per-warp staging of the SH rows: the coefficients are loaded into it as float4, the
    // Jacobian reads them from it, the SH gradients replace them and the warp then stores its
    // 32 consecutive gradient rows with coalesced writes
    __shared__ float stage[4][32][NSH + 1];
    const int lane = threadIdx.x & 31;
    float* mys = &stage[threadIdx.x >> 5][lane][0];
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t fb = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 32; fb < F;
         fb += nwarps * 32) {
      const int f = (int)fb + lane;
      const int gi0 = f < F ? a.f2g[f] - 1 : -1;
      const int gi = (gi0 >= a.g_begin && gi0 < a.g_end) ? gi0 : -1;
      if (gi >= 0) {
        float* const drow = a.dense ? a.dense + (size_t)(gi - a.g_begin) * kDenseRow + kDGeom
                                    : a.geom ? a.geom + (size_t)(gi - a.g_begin) * kGeomRow : nullptr;
        const float* r = a.f2d + 9 * (size_t)f;
        const float4 mo = a.mo4[gi];
        const float orig_op = gs_sigmoid(mo.w);
        const float depth = Ps[2][0] * mo.x + Ps[2][1] * mo.y + Ps[2][2] * mo.z + cam.P[11];
        const float opac = opt.use_antialiasing ? r[2] : orig_op;
        const float og = a.opacity_g[f];
        const float opf = opt.use_antialiasing ? og * opac * (1.0f - orig_op) : og * opac * (1.0f - opac);
        if (drow) {
            drow[kDOpacity] = a.accumulate ? drow[kDOpacity] + opf : opf;
            drow[kDTouched] = 1.0f;
        } else {
            a.opf_g[f] = opf;
        }

        // compute_cov2d_lower_grad (backward_core.jl:465-493)
        const float ia = r[3], ib = r[4], id = r[5];
        const float a_sq = ia * ia, ab = ia * ib, b_sq = ib * ib, bd = ib * id, d_sq = id * id, ad = ia * id;
        const float ab2 = ab + ab, bd2 = bd + bd;
        const float M[3][3] = {{a_sq, ab, b_sq}, {ab2, b_sq + ad, bd2}, {ib * ib, bd, d_sq}};
        const float lg0 = a.licov_g[3 * (size_t)f], lg1 = a.licov_g[3 * (size_t)f + 1],
                    lg2 = a.licov_g[3 * (size_t)f + 2];
        float cg[3];
#pragma unroll
        for (int i = 0; i < 3; ++i) cg[i] = -(M[i][0] * lg0 + M[i][1] * lg1 + M[i][2] * lg2);
        if (opt.use_antialiasing) {
            const float Dx = opt.dilation_x, Dy = opt.dilation_y;
            const float det = (ad - b_sq) * Dx * Dy;
            const float b2 = ib + ib;
            const float k = orig_op * og;
            const float e0 = a_sq * Dx + b_sq * Dx - ia * det;
            const float e1 = b2 * (ia * Dx + id * Dy - det);
            const float e2 = b_sq * Dx + (id * id) * Dy - id * det;
            cg[0] = cg[0] + k * e0;
            cg[1] = cg[1] + k * e1;
            cg[2] = cg[2] + k * e2;
        }

        // mean3d gradient from mean2d
        const float mx = r[0], my = r[1];
        float cmx = mx, cmy = my;
        const bool clampmode = opt.clipping_mode == 0;
        if (clampmode) {
            cmx = jl_clamp(mx, opt.clip_x_min, opt.clip_x_max);
            cmy = jl_clamp(my, opt.clip_y_min, opt.clip_y_max);
        }
        const float idepth = 1.0f / depth;
        float J[2][3];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            J[0][j] = idepth * (Ps[0][j] + (-cmx) * Ps[2][j]);
            J[1][j] = idepth * (Ps[1][j] + (-cmy) * Ps[2][j]);
        }
        const float gx = a.mean2d_g[2 * (size_t)f], gy = a.mean2d_g[2 * (size_t)f + 1];
        float m3[3];
        if (!clampmode) {
#pragma unroll
            for (int j = 0; j < 3; ++j) m3[j] = J[0][j] * gx + J[1][j] * gy;
        } else {
            const float t0 = gx, t1 = gy, t2 = -(mx * gx + my * gy);
#pragma unroll
            for (int j = 0; j < 3; ++j) m3[j] = idepth * (Ps[0][j] * t0 + Ps[1][j] * t1 + Ps[2][j] * t2);
        }

        // 3D covariance lower (V), scales, rotation
        const float s[3] = {gs_expf(a.scal[3 * (size_t)gi]), gs_expf(a.scal[3 * (size_t)gi + 1]),
                            gs_expf(a.scal[3 * (size_t)gi + 2])};
        const float4 qf = a.rot4[gi];
        float R[3][3];
        {
            const float qss = qf.x * qf.x + qf.y * qf.y + qf.z * qf.z + qf.w * qf.w;
            const float qs = sqrtf(2.0f * (1.0f / qss));
            const float rr = qf.x * qs, x = qf.y * qs, y = qf.z * qs, z = qf.w * qs;
            R[0][0] = 1.0f - (y * y + z * z); R[0][1] = x * y - rr * z; R[0][2] = x * z + rr * y;
            R[1][0] = x * y + rr * z; R[1][1] = 1.0f - (x * x + z * z); R[1][2] = y * z - rr * x;
            R[2][0] = x * z - rr * y; R[2][1] = y * z + rr * x; R[2][2] = 1.0f - (x * x + y * y);
        }
        float V[6];
        {
            float RS[3][3];
#pragma unroll
            for (int i = 0; i < 3; ++i)
#pragma unroll
                for (int j = 0; j < 3; ++j) RS[i][j] = R[i][j] * s[j];
#pragma unroll
            for (int k = 0; k < 6; ++k) {
                const int i = L3I[k], j = L3J[k];
                V[k] = RS[i][0] * RS[j][0] + RS[i][1] * RS[j][1] + RS[i][2] * RS[j][2];
            }
        }
        // mean3d gradient from cov2d (Transposed_dsigma_dm, backward_core.jl:789-922). The
        // reference contracts dSigma/dm_k = dJ_k V J^T + J V dJ_k^T (dJ_k: 2x3, 18 entries per k)
        // with the lower-triangle cov2d gradient G. V is symmetric, so with W_i = V J_i^T the
        // contraction is sum_al dJ[0][al][k] U0[al] + dJ[1][al][k] U1[al], U0 = 2 G00 W0 + G10 W1,
        // U1 = 2 G11 W1 + G10 W0; each dJ[i][al][k] is e_i[al] Ps[i][k] + r_i[al] Ps[2][k], so the
        // sum is Ps[0][k] a0 + Ps[1][k] a1 + Ps[2][k] (b0 + b1): ~50 operations instead of ~470
        // (same value up to rounding).
        {
            const float c2x = cmx + cmx, c2y = cmy + cmy;
            float dlx = 1.0f, dly = 1.0f;
            if (clampmode) {
                dlx = (opt.clip_x_min < cmx && cmx <= opt.clip_x_max) ? 1.0f : 0.0f;
                dly = (opt.clip_y_min < cmy && cmy <= opt.clip_y_max) ? 1.0f : 0.0f;
            }
            float a0 = 0.0f, b0 = 0.0f, a1 = 0.0f, b1 = 0.0f;
#pragma unroll
            for (int al = 0; al < 3; ++al) {
                const float w0 = V[low3(al, 0)] * J[0][0] + V[low3(al, 1)] * J[0][1] + V[low3(al, 2)] * J[0][2];
                const float w1 = V[low3(al, 0)] * J[1][0] + V[low3(al, 1)] * J[1][1] + V[low3(al, 2)] * J[1][2];
                const float u0 = 2.0f * cg[0] * w0 + cg[1] * w1;
                const float u1 = 2.0f * cg[2] * w1 + cg[1] * w0;
                const float r0 = Ps[0][al] - c2x * Ps[2][al];
                const float r1 = Ps[1][al] - c2y * Ps[2][al];
                a0 = a0 + (dlx * Ps[2][al]) * u0;
                b0 = b0 + r0 * u0;
                a1 = a1 + (dly * Ps[2][al]) * u1;
                b1 = b1 + r1 * u1;
            }
            const float sc = -(1.0f / (depth * depth));
            const float b01 = b0 + b1;
#pragma unroll
            for (int k = 0; k < 3; ++k)
                m3[k] = m3[k] + sc * (Ps[0][k] * a0 + Ps[1][k] * a1 + Ps[2][k] * b01);
        }
        // mean3d gradient from the view-dependent colour
        const float vx = mo.x - cam.position[0], vy = mo.y - cam.position[1], vz = mo.z - cam.position[2];
        const float inv_vn = 1.0f / sqrtf(vx * vx + vy * vy + vz * vz);
        const float nd0 = vx * inv_vn, nd1 = vy * inv_vn, nd2 = vz * inv_vn;
        const float col[3] = {r[6], r[7], r[8]};
        const float cgr[3] = {a.color_g[3 * (size_t)f], a.color_g[3 * (size_t)f + 1],
                              a.color_g[3 * (size_t)f + 2]};
        const float* h = a.sh + (size_t)gi * 3 * a.sh_stride;
        // colour channels that take part in the direction term (positive colour)
        const bool pos[3] = {!(col[0] <= 0.0f), !(col[1] <= 0.0f), !(col[2] <= 0.0f)};
        if (!a.no_dir) {
            // the Jacobian reads coefficients 0 .. 3 MAXO - 1 of the row linearly (sh.jl:196)
            if (DEG > 0) {
                if ((NSH % 4) == 0 && (reinterpret_cast<uintptr_t>(h) & 15) == 0) {
#pragma unroll
                    for (int k = 0; k < NSH / 4; ++k) {
                        const float4 v4 = reinterpret_cast<const float4*>(h)[k];
                        mys[4 * k] = v4.x; mys[4 * k + 1] = v4.y; mys[4 * k + 2] = v4.z; mys[4 * k + 3] = v4.w;
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < NSH; ++k) mys[k] = h[k];
                }
            }
            float Jt[3][3];
            colour_dir_jacobian<DEG>(mys, nd0, nd1, nd2, pos, a.fix_sh16, Jt);
            const float nd[3] = {nd0, nd1, nd2};
            add_colour_dir_term(Jt, cgr, nd, inv_vn, m3);
        }
        float* const m3out = drow ? drow + kDMean : a.mean3d_g + 3 * (size_t)f;
        const bool acc = drow && a.accumulate;
        m3out[0] = acc ? m3out[0] + m3[0] : m3[0];
        m3out[1] = acc ? m3out[1] + m3[1] : m3[1];
        m3out[2] = acc ? m3out[2] + m3[2] : m3[2];

        // scaling features: v gradient = Transposed_dsigma_dv(J) * cg
        float vg[6];
#pragma unroll
        for (int jv = 0; jv < 6; ++jv) {
            const int rr = L3I[jv], ss = L3J[jv];
            float tt = 0.0f;
#pragma unroll
            for (int p = 0; p < 3; ++p) {
                const int pp = L2I[p], qq = L2J[p];
                float e = J[pp][rr] * J[qq][ss];
                if (rr != ss) e = e + J[pp][ss] * J[qq][rr];
                tt = tt + e * cg[p];
            }
            vg[jv] = tt;
        }
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            float tt = 0.0f;
#pragma unroll
            for (int i = 0; i < 6; ++i) tt = tt + (s[j] * R[L3I[i]][j] * R[L3J[i]][j]) * vg[i];
            float* const so = (drow ? drow + kDScale : a.scale_g + 3 * (size_t)f) + j;
            *so = acc ? *so + (2.0f * tt) * s[j] : (2.0f * tt) * s[j];
        }
        // rotation features
        {
            const float ssq[3] = {s[0] * s[0], s[1] * s[1], s[2] * s[2]};
            float Rg[3][3];
#pragma unroll
            for (int k = 0; k < 3; ++k)
#pragma unroll
                for (int l = 0; l < 3; ++l) {
                    float tt = vg[low3(k, k)] * R[k][l];
#pragma unroll
                    for (int i = 0; i < 3; ++i) tt = tt + vg[low3(i, k)] * R[i][l];
                    Rg[k][l] = ssq[l] * tt;
                }
            const float qss = qf.x * qf.x + qf.y * qf.y + qf.z * qf.z + qf.w * qf.w;
            const float inv_qn = 1.0f / sqrtf(qss);
            const float nq[4] = {qf.x * inv_qn, qf.y * inv_qn, qf.z * inv_qn, qf.w * inv_qn};
            const float rq = nq[0], xq = nq[1], yq = nq[2], zq = nq[3];
            const float m2x = -(xq + xq), m2y = -(yq + yq), m2z = -(zq + zq);
            const float A[4][3][3] = {
                {{0.0f, -zq, yq}, {zq, 0.0f, -xq}, {-yq, xq, 0.0f}},
                {{0.0f, yq, zq}, {yq, m2x, -rq}, {zq, rq, m2x}},
                {{m2y, xq, rq}, {xq, 0.0f, zq}, {-rq, zq, m2y}},
                {{m2z, -rq, xq}, {rq, m2z, yq}, {xq, yq, 0.0f}}};
            float nqg[4];
#pragma unroll
            for (int t4 = 0; t4 < 4; ++t4) {
                float dsum = 0.0f;
#pragma unroll
                for (int c3 = 0; c3 < 3; ++c3)
#pragma unroll
                    for (int r3 = 0; r3 < 3; ++r3) dsum = dsum + A[t4][r3][c3] * Rg[r3][c3];
                nqg[t4] = 2.0f * dsum;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float w = 0.0f;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float Nij = i == j ? 1.0f - nq[i] * nq[i] : -nq[i < j ? i : j] * nq[i < j ? j : i];
                    w = w + Nij * nqg[j];
                }
                float* const ro = (drow ? drow + kDRot : a.rot_g + 4 * (size_t)f) + i;
                *ro = acc ? *ro + inv_qn * w : inv_qn * w;
            }
        }
        // SH coefficients (compute_sh_coeffs_grad!, backward_core.jl:936-964), staged; or
        // their factors: the colour gradients and which channels are live
        if (a.colour) {
            const float fl = 1.0f + (col[0] >= 0.0f ? 2.0f : 0.0f) + (col[1] >= 0.0f ? 4.0f : 0.0f) +
                             (col[2] >= 0.0f ? 8.0f : 0.0f) + (pos[0] ? 16.0f : 0.0f) +
                             (pos[1] ? 32.0f : 0.0f) + (pos[2] ? 64.0f : 0.0f);
            a.colour[gi - a.g_begin] = make_float4(cgr[0], cgr[1], cgr[2], fl);
        } else if (!a.skip_sh) {
#pragma unroll
          for (int l = 0; l < 3; ++l) {
            const bool live = col[l] >= 0.0f;
#pragma unroll
            for (int k = 1; k <= MAXO; ++k)
                mys[(k - 1) + l * MAXO] = live ? cgr[l] * sh_basis(k, nd0, nd1, nd2) : 0.0f;
          }
        }
      }
      __syncwarp();
      const int nrows = (int)min((int64_t)32, (int64_t)F - fb);
      float* const warp_stage = &stage[threadIdx.x >> 5][0][0];
      if (a.colour || a.skip_sh) {
          // factored rows: written per Gaussian above; or no SH gradients
      } else if (a.dense) {  // row `row` of the warp goes to dense row gidx - g_begin (if in range)
          const int rel = gi >= 0 ? gi - a.g_begin : -1;
          for (int e = lane; e < 32 * NSH; e += 32) {
              const int row = e / NSH, rem = e - row * NSH;
              const int grow = __shfl_sync(0xffffffffu, rel, row);
              if (row >= nrows || grow < 0) continue;
              const int c = rem / MAXO, k = rem - c * MAXO;
              float* const d = a.dense + (size_t)grow * kDenseRow + (size_t)(c * 16 + k);
              const float val = warp_stage[row * (NSH + 1) + rem];
              *d = a.accumulate ? *d + val : val;
          }
      } else {
          for (int e = lane; e < nrows * NSH; e += 32) {
              const int row = e / NSH, rem = e - row * NSH;
              const int c = rem / MAXO, k = rem - c * MAXO;
              a.sh_g[(size_t)(fb + row) * 3 * a.sh_grad_stride + (size_t)(c * a.sh_grad_stride + k)] =
                  warp_stage[row * (NSH + 1) + rem];
          }
      }
      __syncwarp();
    }
}

// Camera positions of up to GS3D_MAX_FACTORED_VIEWS views, passed by value.
struct DirViews {
    float p[GS3D_MAX_FACTORED_VIEWS][3];
};

// The colour -> direction part of the mean3d gradient, added to factored geometry rows whose
// projection backward left it out (GS3D_BACKWARD_NO_COLOUR_DIRECTION): for Gaussian g_begin + i
// and each view v that filtered it (colour row flag > 0), in order v = 0, 1, ..., the term
// k_bwd_project adds for that view (the same SH row, mean, camera position, colour gradients
// and positive-colour flags, the same operations), added to the row's mean gradient. With one
// view this gives the row k_bwd_project writes without the flag, bit for bit.
template <int DEG>
__global__ void __launch_bounds__(128) k_colour_dir_rows(const float4* __restrict__ mo4,
                                                         const float* __restrict__ sh, int sh_stride,
                                                         float* __restrict__ geom,
                                                         const float4* __restrict__ colour, int nv,
                                                         int64_t view_stride, const DirViews vp,
                                                         int fix_sh16, int64_t g_begin, int64_t g_end) {
    constexpr int MAXO = (DEG + 1) * (DEG + 1);
    constexpr int NSH = 3 * MAXO;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= g_end - g_begin) return;
    float* row = geom + (size_t)i * kGeomRow;
    if (!(row[kDTouched] > 0.0f)) return;
    const size_t gi = (size_t)(g_begin + i);
    const float4 mo = mo4[gi];
    float mys[NSH];
    if (DEG > 0) {
        const float* h = sh + gi * 3 * (size_t)sh_stride;
        if ((NSH % 4) == 0 && (reinterpret_cast<uintptr_t>(h) & 15) == 0) {
#pragma unroll
            for (int k = 0; k < NSH / 4; ++k) {
                const float4 v4 = __ldg(reinterpret_cast<const float4*>(h) + k);
                mys[4 * k] = v4.x; mys[4 * k + 1] = v4.y; mys[4 * k + 2] = v4.z; mys[4 * k + 3] = v4.w;
            }
        } else {
#pragma unroll
            for (int k = 0; k < NSH; ++k) mys[k] = h[k];
        }
    }
    float m3[3] = {row[kDMean], row[kDMean + 1], row[kDMean + 2]};
    for (int v = 0; v < nv; ++v) {
        const float4 cr = colour[(size_t)v * view_stride + i];
        if (!(cr.w > 0.0f)) continue;  // not filtered in view v
        const int fl = (int)cr.w;
        const bool pos[3] = {((fl >> 4) & 1) != 0, ((fl >> 5) & 1) != 0, ((fl >> 6) & 1) != 0};
        const float vx = mo.x - vp.p[v][0], vy = mo.y - vp.p[v][1], vz = mo.z - vp.p[v][2];
        const float inv_vn = 1.0f / sqrtf(vx * vx + vy * vy + vz * vz);
        const float nd0 = vx * inv_vn, nd1 = vy * inv_vn, nd2 = vz * inv_vn;
        const float cgr[3] = {cr.x, cr.y, cr.z};
        float Jt[3][3];
        colour_dir_jacobian<DEG>(mys, nd0, nd1, nd2, pos, fix_sh16, Jt);
        const float nd[3] = {nd0, nd1, nd2};
        add_colour_dir_term(Jt, cgr, nd, inv_vn, m3);
    }
    row[kDMean] = m3[0];
    row[kDMean + 1] = m3[1];
    row[kDMean + 2] = m3[2];
}

int grid_for(int64_t items, int threads, int per_sm) {
    int64_t b = ceil_div(items, threads);
    const int64_t cap = (int64_t)kSMs * per_sm;
    if (b > cap) b = cap;
    if (b < 1) b = 1;
    return (int)b;
}

}  // namespace
}  // namespace gs3d

using namespace gs3d;

namespace {

constexpr unsigned kPhaseRaster = 1u, kPhaseProject = 2u;

// backward! in phases: kPhaseRaster = B1 + B2 (the 2D gradients), kPhaseProject = B3 + B4 for
// the filtered Gaussians with index in [g_begin, g_end), with the 3D gradients into the
// F-compact arrays of fg (dense == NULL, geom == NULL), into dense rows (row gidx - g_begin;
// zeroed here first when zero_rows > 0: rows [0, zero_rows) of dense), or into factored
// geometry and colour rows (row gidx - g_begin of each).
int backward_impl(const gs3d_fgradients* fg, const float* rgb_grad,
                  const gs3d_render_outputs* out, const gs3d_gaussians* g, const gs3d_camera* cam,
                  const gs3d_tiling* til, const gs3d_render_options* opt,
                  const gs3d_render_buffers* buf, uint32_t flags, unsigned phases, float* dense,
                  int32_t zero_rows, int32_t g_begin, int32_t g_end, cudaStream_t stream,
                  float* geom = nullptr, float* colour = nullptr) {
    GS3D_RETURN_IF(check_render_common(g, cam, til, opt));
    if (!fg || !buf) return invalid("NULL argument");
    if ((phases & kPhaseRaster) &&
        (!rgb_grad || !out || !out->transmittance || !out->last_contributing_sdfgids))
        return invalid("backward needs the gradient image, transmittance and last-contributor images");
    if (!fg->mean2d_grads || !fg->opacity_grads || !fg->licov2d_grads || !fg->color_grads)
        return invalid("NULL 2D gradient array");
    const bool compact_out = (phases & kPhaseProject) && !dense && !geom;
    if (compact_out && (!fg->mean3d_grads || !fg->opacity_feature_grads ||
                        !fg->scaling_features_grads || !fg->rotation_features_grads ||
                        (!fg->sh_coeffs_grads && !(flags & GS3D_BACKWARD_SKIP_SH_GRADS))))
        return invalid("NULL gradient array");
    if (g_begin < 0 || g_end < g_begin) return invalid("Gaussian range [%d, %d)", g_begin, g_end);
    if (compact_out && (fg->sh_degree < opt->sh_degree || fg->sh_degree > 3))
        return invalid("gradient SH degree %d < render degree %d", fg->sh_degree, opt->sh_degree);
    const int64_t cap_n = buf->capacity_n > 0 ? buf->capacity_n : 1;
    if (dense && zero_rows > 0) {
        ProfScope prof("zero_dense", stream);
        GS3D_CUDA(cudaMemsetAsync(dense, 0, (size_t)zero_rows * kDenseRow * sizeof(float), stream),
                  "zero dense rows");
    }
    if (phases & kPhaseRaster) {
        {
            ProfScope prof("zero_2d", stream);
            k_zero_2d<<<grid_for(3 * cap_n, 256, 8), 256, 0, stream>>>(
                buf->device_counts, fg->mean2d_grads, fg->opacity_grads, fg->licov2d_grads,
                fg->color_grads);
            GS3D_LAUNCHED("k_zero_2d");
        }
        GS3D_RETURN_IF(launch_bwd_raster(fg, rgb_grad, out, cam, til, opt, buf, stream));
    }
    if (!(phases & kPhaseProject)) return GS3D_OK;

    BProjArgs p;
    p.mo4 = reinterpret_cast<const float4*>(g->means_opacity_features);
    p.scal = g->scaling_features;
    p.rot4 = reinterpret_cast<const float4*>(g->rotation_features);
    p.sh = g->sh_coeffs;
    p.sh_stride = (g->sh_degree + 1) * (g->sh_degree + 1);
    p.f2g = buf->fgidx_to_gidx;
    p.f2d = buf->means2d_opacities_inverse_covariances_colors;
    p.counts = buf->device_counts;
    p.mean2d_g = fg->mean2d_grads;
    p.opacity_g = fg->opacity_grads;
    p.licov_g = fg->licov2d_grads;
    p.color_g = fg->color_grads;
    p.mean3d_g = fg->mean3d_grads;
    p.opf_g = fg->opacity_feature_grads;
    p.scale_g = fg->scaling_features_grads;
    p.rot_g = fg->rotation_features_grads;
    p.sh_g = fg->sh_coeffs_grads;
    p.sh_grad_stride = (fg->sh_degree + 1) * (fg->sh_degree + 1);
    p.fix_sh16 = (flags & GS3D_BACKWARD_FIX_SH16) ? 1 : 0;
    p.skip_sh = (compact_out && (flags & GS3D_BACKWARD_SKIP_SH_GRADS)) ? 1 : 0;
    p.no_dir = (geom && (flags & GS3D_BACKWARD_NO_COLOUR_DIRECTION)) ? 1 : 0;
    p.accumulate = (!compact_out && (flags & GS3D_BACKWARD_ACCUMULATE_ROWS)) ? 1 : 0;
    p.dense = dense;
    p.geom = geom;
    p.colour = reinterpret_cast<float4*>(colour);
    p.g_begin = g_begin;
    p.g_end = g_end;
    const int grid = grid_for(cap_n, 128, 16);
    ProfScope prof("bwd_project", stream);
    switch (opt->sh_degree) {
        case 0: k_bwd_project<0><<<grid, 128, 0, stream>>>(p, *cam, *opt); break;
        case 1: k_bwd_project<1><<<grid, 128, 0, stream>>>(p, *cam, *opt); break;
        case 2: k_bwd_project<2><<<grid, 128, 0, stream>>>(p, *cam, *opt); break;
        default: k_bwd_project<3><<<grid, 128, 0, stream>>>(p, *cam, *opt); break;
    }
    GS3D_LAUNCHED("k_bwd_project");
    return GS3D_OK;
}

}  // namespace

extern "C" GS3D_API int gs3d_backward(const gs3d_fgradients* fg, const float* rgb_grad,
                                      const gs3d_render_outputs* out, const gs3d_gaussians* g,
                                      const gs3d_camera* cam, const gs3d_tiling* til,
                                      const gs3d_render_options* opt,
                                      const gs3d_render_buffers* buf, uint32_t flags,
                                      gs3d_stream_t stream) {
    return backward_impl(fg, rgb_grad, out, g, cam, til, opt, buf, flags,
                         kPhaseRaster | kPhaseProject, nullptr, 0, 0, INT32_MAX,
                         reinterpret_cast<cudaStream_t>(stream));
}

extern "C" GS3D_API int gs3d_backward_dense(const gs3d_fgradients* fg, const float* rgb_grad,
                                            const gs3d_render_outputs* out,
                                            const gs3d_gaussians* g, const gs3d_camera* cam,
                                            const gs3d_tiling* til,
                                            const gs3d_render_options* opt,
                                            const gs3d_render_buffers* buf, uint32_t flags,
                                            float* dense, int32_t n, gs3d_stream_t stream) {
    if (!dense) return invalid("NULL dense rows");
    if (!g || n < g->n) return invalid("dense rows %d < n", n);
    return backward_impl(fg, rgb_grad, out, g, cam, til, opt, buf, flags,
                         kPhaseRaster | kPhaseProject, dense, n, 0, g->n,
                         reinterpret_cast<cudaStream_t>(stream));
}

extern "C" GS3D_API int gs3d_backward_raster(const gs3d_fgradients* fg, const float* rgb_grad,
                                             const gs3d_render_outputs* out,
                                             const gs3d_gaussians* g, const gs3d_camera* cam,
                                             const gs3d_tiling* til,
                                             const gs3d_render_options* opt,
                                             const gs3d_render_buffers* buf, uint32_t flags,
                                             gs3d_stream_t stream) {
    return backward_impl(fg, rgb_grad, out, g, cam, til, opt, buf, flags, kPhaseRaster, nullptr,
                         0, 0, 0, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" GS3D_API int gs3d_backward_project_dense(const gs3d_fgradients* fg,
                                                    const gs3d_gaussians* g, const gs3d_camera* cam,
                                                    const gs3d_tiling* til,
                                                    const gs3d_render_options* opt,
                                                    const gs3d_render_buffers* buf, uint32_t flags,
                                                    float* dense_rows, int32_t g_begin,
                                                    int32_t g_end, gs3d_stream_t stream) {
    if (!dense_rows) return invalid("NULL dense rows");
    if (!g || g_end > g->n) return invalid("Gaussian range end %d > n", g_end);
    return backward_impl(fg, nullptr, nullptr, g, cam, til, opt, buf, flags, kPhaseProject,
                         dense_rows, 0, g_begin, g_end, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" GS3D_API int gs3d_factored_colour_direction_range(
    const gs3d_gaussians* g, float* geom_rows, const float* colour_rows, int32_t n_views,
    int64_t view_stride, const float* view_positions, int32_t g_begin, int32_t g_end,
    int32_t sh_degree, uint32_t flags, gs3d_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (!g || !geom_rows || !colour_rows || !view_positions) return invalid("NULL argument");
    if (sh_degree < 0 || sh_degree > 3 || sh_degree > g->sh_degree)
        return invalid("SH degree %d (storage %d)", sh_degree, g->sh_degree);
    if (g_begin < 0 || g_end < g_begin || g_end > g->n)
        return invalid("Gaussian range [%d, %d) of n = %d", g_begin, g_end, g->n);
    if (n_views < 1 || n_views > GS3D_MAX_FACTORED_VIEWS)
        return invalid("%d views (1 .. %d)", n_views, GS3D_MAX_FACTORED_VIEWS);
    if (view_stride < (int64_t)g_end - g_begin) return invalid("view stride %lld < range", (long long)view_stride);
    if ((reinterpret_cast<uintptr_t>(colour_rows) & 15) != 0 ||
        (reinterpret_cast<uintptr_t>(g->means_opacity_features) & 15) != 0)
        return invalid("colour rows and means must be 16-byte aligned");
    if (g_end == g_begin) return GS3D_OK;
    DirViews vp{};
    for (int v = 0; v < n_views; ++v)
        for (int k = 0; k < 3; ++k) vp.p[v][k] = view_positions[3 * v + k];
    const int64_t cnt = (int64_t)g_end - g_begin;
    const unsigned grid = (unsigned)ceil_div(cnt, 128);
    const float4* mo4 = reinterpret_cast<const float4*>(g->means_opacity_features);
    const float4* col = reinterpret_cast<const float4*>(colour_rows);
    const int stride = (g->sh_degree + 1) * (g->sh_degree + 1);
    const int fix = (flags & GS3D_BACKWARD_FIX_SH16) ? 1 : 0;
    ProfScope prof("bwd_project", stream);
    switch (sh_degree) {
        case 0: k_colour_dir_rows<0><<<grid, 128, 0, stream>>>(mo4, g->sh_coeffs, stride, geom_rows, col, n_views, view_stride, vp, fix, g_begin, g_end); break;
        case 1: k_colour_dir_rows<1><<<grid, 128, 0, stream>>>(mo4, g->sh_coeffs, stride, geom_rows, col, n_views, view_stride, vp, fix, g_begin, g_end); break;
        case 2: k_colour_dir_rows<2><<<grid, 128, 0, stream>>>(mo4, g->sh_coeffs, stride, geom_rows, col, n_views, view_stride, vp, fix, g_begin, g_end); break;
        default: k_colour_dir_rows<3><<<grid, 128, 0, stream>>>(mo4, g->sh_coeffs, stride, geom_rows, col, n_views, view_stride, vp, fix, g_begin, g_end); break;
    }
    GS3D_LAUNCHED("k_colour_dir_rows");
    return GS3D_OK;
}

extern "C" GS3D_API int gs3d_backward_project_factored(const gs3d_fgradients* fg,
                                                       const gs3d_gaussians* g,
                                                       const gs3d_camera* cam,
                                                       const gs3d_tiling* til,
                                                       const gs3d_render_options* opt,
                                                       const gs3d_render_buffers* buf,
                                                       uint32_t flags, float* geom_rows,
                                                       float* colour_rows, int32_t g_begin,
                                                       int32_t g_end, gs3d_stream_t stream) {
    if (!geom_rows || !colour_rows) return invalid("NULL factored rows");
    if ((reinterpret_cast<uintptr_t>(colour_rows) & 15) != 0)
        return invalid("colour rows not 16-byte aligned");
    if (!g || g_end > g->n) return invalid("Gaussian range end %d > n", g_end);
    return backward_impl(fg, nullptr, nullptr, g, cam, til, opt, buf, flags, kPhaseProject,
                         nullptr, 0, g_begin, g_end, reinterpret_cast<cudaStream_t>(stream),
                         geom_rows, colour_rows);
}
