// backward.cpp — TEST INFRASTRUCTURE ONLY: CPU oracle of gs3d's backward pass.
// Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it.
//
// Restates ThreeDGaussianSplatting.jl's `backward!` (src/backward_core.jl:37-72):
//   reverse tile blend ........ backward_core.jl:96-293 (per-pair gradients; the
//                               reference's float atomics are summed here in double)
//   projection backward ....... backward_core.jl:309-452
//   cov2d gradient ............ backward_core.jl:465-493
//   d(sigma)/d(v) ............. backward_core.jl:513-563
//   d(v)/d(s) ................. backward_core.jl:574-637
//   dL/dR ..................... backward_core.jl:646-726
//   normalised-q gradient ..... backward_core.jl:734-774
//   d(sigma)/d(m) ............. backward_core.jl:789-922
//   SH coefficient gradient ... backward_core.jl:936-964
//   colour/direction Jacobian . sh.jl:175-267 (the degree-3 term 16 reads coefficient 15
//                               unless GS3D_BACKWARD_FIX_SH16 is passed, as sh.jl:249 does)
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

#include "../include/gs3d.h"
#include "oracle_math.h"

using namespace oracle;

namespace {

// lower-triangle index of a symmetric 3x3 matrix, column-major: (0,0)0 (1,0)1 (2,0)2
// (1,1)3 (2,1)4 (2,2)5
inline int low3(int i, int j) {
    if (i < j) std::swap(i, j);
    static const int t[3][3] = {{0, -1, -1}, {1, 3, -1}, {2, 4, 5}};
    return t[i][j];
}
// lower index of a symmetric 2x2 matrix: 0 -> (0,0), 1 -> (1,0), 2 -> (1,1)
const int L2I[3] = {0, 1, 1};
const int L2J[3] = {0, 0, 1};
const int L3I[6] = {0, 1, 2, 1, 2, 2};
const int L3J[6] = {0, 0, 0, 1, 1, 2};

struct J23 { float a[2][3]; };

inline J23 lin_proj(const gs3d_camera& c, float u, float v, float depth) {
    const float* P = c.P;
    const float idepth = 1.0f / depth;
    J23 J;
    for (int j = 0; j < 3; ++j) {
        J.a[0][j] = idepth * (P[0 + 3 * j] + (-u) * P[2 + 3 * j]);
        J.a[1][j] = idepth * (P[1 + 3 * j] + (-v) * P[2 + 3 * j]);
    }
    return J;
}

inline void quat_to_rot(const float q[4], float R[3][3]) {
    const float ss = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3];
    const float s = std::sqrt(2.0f * (1.0f / ss));
    const float r = q[0] * s, x = q[1] * s, y = q[2] * s, z = q[3] * s;
    R[0][0] = 1.0f - (y * y + z * z); R[0][1] = x * y - r * z;         R[0][2] = x * z + r * y;
    R[1][0] = x * y + r * z;         R[1][1] = 1.0f - (x * x + z * z); R[1][2] = y * z - r * x;
    R[2][0] = x * z - r * y;         R[2][1] = y * z + r * x;         R[2][2] = 1.0f - (x * x + y * y);
}

// transposed_color_normalized_direction_jacobian (sh.jl:175-267): Jt[a][c] = dc_c/dd_a
void color_dir_jacobian_t(int deg, const float col[3], const float nd[3], const float* h,
                          bool fix_sh16, float Jt[3][3]) {
    for (int a = 0; a < 3; ++a) for (int c = 0; c < 3; ++c) Jt[a][c] = 0.0f;
    if (deg == 0) return;
    const int MAXO = (deg + 1) * (deg + 1);
    const float x = nd[0], y = nd[1], z = nd[2];
    for (int c = 0; c < 3; ++c) {
        if (col[c] <= 0.0f) continue;
        const float* hc = h + c * MAXO;  // linear indexing with the options order (sh.jl:196)
        float dy = -SH_C[1] * hc[1];
        float dz = SH_C[2] * hc[2];
        float dx = -SH_C[3] * hc[3];
        if (deg >= 2) {
            { const float s = SH_C[4] * hc[4]; dx += y * s; dy += x * s; }
            { const float s = SH_C[5] * hc[5]; dy += z * s; dz += y * s; }
            { const float s = SH_C[6] * hc[6]; dx -= 2.0f * x * s; dy -= 2.0f * y * s; dz += 4.0f * z * s; }
            { const float s = SH_C[7] * hc[7]; dx += z * s; dz += x * s; }
            { const float s = SH_C[8] * hc[8]; dx += 2.0f * x * s; dy -= 2.0f * y * s; }
            if (deg >= 3) {
                { const float s = SH_C[9] * hc[9]; dx += 6.0f * x * y * s; dy += 3.0f * (x * x - y * y) * s; }
                { const float s = SH_C[10] * hc[10]; dx += y * z * s; dy += x * z * s; dz += x * y * s; }
                { const float s = SH_C[11] * hc[11];
                  dx -= 2.0f * x * y * s;
                  dy += (4.0f * (z * z) - x * x - 3.0f * (y * y)) * s;
                  dz += 8.0f * y * z * s; }
                { const float s = SH_C[12] * hc[12];
                  dx -= 6.0f * x * z * s;
                  dy -= 6.0f * y * z * s;
                  dz += 3.0f * (2.0f * (z * z) - x * x - y * y) * s; }
                { const float s = SH_C[13] * hc[13];
                  dx += (4.0f * (z * z) - 3.0f * (x * x) - y * y) * s;
                  dy -= 2.0f * x * y * s;
                  dz += 8.0f * x * z * s; }
                { const float s = SH_C[14] * hc[14]; dx += 2.0f * x * z * s; dy -= 2.0f * y * z * s; dz += (x * x - y * y) * s; }
                { const float s = SH_C[15] * hc[fix_sh16 ? 15 : 14];
                  dx += 3.0f * (x * x - y * y) * s;
                  dy -= 6.0f * x * y * s; }
            }
        }
        Jt[0][c] = dx; Jt[1][c] = dy; Jt[2][c] = dz;
    }
}

}  // namespace

extern "C" {

// Reverse blend (B2) + projection backward (B3). Inputs are the forward's outputs in the
// reference layouts; F is the number of filtered Gaussians. All gradient outputs are
// F-indexed (fgradients layout) and fully written (2D ones are zeroed first, B1).
// oracle_backward with two test-only options: `project_only` != 0 skips B1 + B2 and takes
// mean2d_g, opacity_g, licov_g and color_g as inputs (to check the projection backward on given
// 2D gradients); `mag` (NULL or 9 x F floats) receives, per filtered Gaussian and per 2D
// gradient component (mean2d 2, opacity 1, licov 3, colour 3), the sum over its per-pixel terms
// of each term evaluated on absolute values (with its colour differences T c - (colour behind)
// taken as |T c| + |behind|): the scale of the rounding errors of any float evaluation and
// summation order, also where the terms or the sum cancel.
int oracle_backward_ex(const gs3d_gaussians* gp, const gs3d_camera* camp, const gs3d_tiling* tp,
                       const gs3d_render_options* op, int32_t F, const int32_t* fgidx_to_gidx,
                       const float* f2d, const int32_t* sfgidx, const int32_t* tiles_end,
                       const float* trans, const int32_t* last, const float* rgb_grad,
                       uint32_t flags, float* mean2d_g, float* opacity_g, float* licov_g,
                       float* color_g, float* mean3d_g, float* opf_g, float* scale_g,
                       float* rot_g, float* sh_g, int32_t sh_grad_degree, int32_t project_only,
                       float* mag);

int oracle_backward(const gs3d_gaussians* gp, const gs3d_camera* camp, const gs3d_tiling* tp,
                    const gs3d_render_options* op, int32_t F, const int32_t* fgidx_to_gidx,
                    const float* f2d, const int32_t* sfgidx, const int32_t* tiles_end,
                    const float* trans, const int32_t* last, const float* rgb_grad,
                    uint32_t flags, float* mean2d_g, float* opacity_g, float* licov_g,
                    float* color_g, float* mean3d_g, float* opf_g, float* scale_g,
                    float* rot_g, float* sh_g, int32_t sh_grad_degree) {
    return oracle_backward_ex(gp, camp, tp, op, F, fgidx_to_gidx, f2d, sfgidx, tiles_end, trans,
                              last, rgb_grad, flags, mean2d_g, opacity_g, licov_g, color_g,
                              mean3d_g, opf_g, scale_g, rot_g, sh_g, sh_grad_degree, 0, nullptr);
}

int oracle_backward_ex(const gs3d_gaussians* gp, const gs3d_camera* camp, const gs3d_tiling* tp,
                       const gs3d_render_options* op, int32_t F, const int32_t* fgidx_to_gidx,
                       const float* f2d, const int32_t* sfgidx, const int32_t* tiles_end,
                       const float* trans, const int32_t* last, const float* rgb_grad,
                       uint32_t flags, float* mean2d_g, float* opacity_g, float* licov_g,
                       float* color_g, float* mean3d_g, float* opf_g, float* scale_g,
                       float* rot_g, float* sh_g, int32_t sh_grad_degree, int32_t project_only,
                       float* mag) {
    const gs3d_gaussians& g = *gp;
    const gs3d_camera& cam = *camp;
    const gs3d_tiling& til = *tp;
    const gs3d_render_options& opt = *op;
    const int W = cam.width, H = cam.height;
    const bool fix16 = (flags & GS3D_BACKWARD_FIX_SH16) != 0;

    // B1 + B2 with double accumulators
    std::vector<double> acc(project_only ? 0 : (size_t)F * 9, 0.0);  // mean2d(2) opacity(1) licov(3) color(3)
    std::vector<double> macc(mag && !project_only ? (size_t)F * 9 : 0, 0.0);
    const int TW = til.tile_width, TH = til.tile_height;
    parallel_for(0, project_only ? 0 : (int64_t)til.nb_tiles_x * til.nb_tiles_y, [&](int64_t tl) {
            const int txi = (int)(tl % til.nb_tiles_x) + 1, tyi = (int)(tl / til.nb_tiles_x) + 1;
            const int tile = txi + (tyi - 1) * til.nb_tiles_x;
            const int first = tile == 1 ? 1 : tiles_end[tile - 2] + 1;
            const int u0 = (txi - 1) * TW, v0 = (tyi - 1) * TH;
            for (int pv = 1; pv <= TH; ++pv)
                for (int pu = 1; pu <= TW; ++pu) {
                    const int U = pu + u0, V = pv + v0;
                    if (!(U >= 1 && U <= W && V >= 1 && V <= H)) continue;
                    const size_t px = (size_t)(V - 1) + (size_t)H * (U - 1);
                    const float cpu = (float)U - 0.5f, cpv = (float)V - 0.5f;
                    float T = trans[px];
                    const int lastc = last[px];
                    const float gr[3] = {rgb_grad[3 * px], rgb_grad[3 * px + 1], rgb_grad[3 * px + 2]};
                    float part[3] = {T * opt.background[0], T * opt.background[1], T * opt.background[2]};
                    for (int s = lastc; s >= first; --s) {
                        const int fg = sfgidx[s - 1] - 1;
                        const float* r = f2d + 9 * (size_t)fg;
                        const float x = r[0], y = r[1], opac = r[2];
                        const float ic11 = r[3], ic21 = r[4], ic22 = r[5];
                        const float du = cpu - x, dv = cpv - y;
                        const float q = -0.5f * (ic11 * (du * du) + ic22 * (dv * dv)) - ic21 * du * dv;
                        const float geval = o_expf(q);
                        const float alpha = o_min(opt.max_alpha, opac * geval);
                        if (alpha < opt.min_alpha) continue;
                        const float inv1m = 1.0f / (1.0f - alpha);
                        T *= inv1m;
                        float tc[3];
                        for (int c = 0; c < 3; ++c) {
                            tc[c] = T * r[6 + c];
                            part[c] += alpha * tc[c];
                        }
                        const float ag = inv1m * (gr[0] * (tc[0] - part[0]) + gr[1] * (tc[1] - part[1]) +
                                                  gr[2] * (tc[2] - part[2]));
                        const float opg = geval * ag;
                        const float aga = alpha * ag;
                        const float sc = -0.5f * aga;
                        const float g11 = sc * (du * du), g21 = sc * (dv * du), g22 = sc * (dv * dv);
                        const float m0 = aga * (du * ic11 + dv * ic21);
                        const float m1 = aga * (du * ic21 + dv * ic22);
                        const float ta = T * alpha;
                        double* a = &acc[9 * (size_t)fg];
                        atomic_add(&a[0], m0); atomic_add(&a[1], m1); atomic_add(&a[2], opg);
                        atomic_add(&a[3], g11); atomic_add(&a[4], g21 + g21); atomic_add(&a[5], g22);
                        atomic_add(&a[6], ta * gr[0]); atomic_add(&a[7], ta * gr[1]);
                        atomic_add(&a[8], ta * gr[2]);
                        if (!macc.empty()) {
                            // each term evaluated on absolute values, with the colour
                            // differences T c - (colour behind) replaced by |T c| + |behind|:
                            // the size that rounding errors scale with, even where the term
                            // itself cancels
                            double* b = &macc[9 * (size_t)fg];
                            const double agm = (double)inv1m *
                                (std::fabs(gr[0]) * ((double)std::fabs(tc[0]) + std::fabs(part[0])) +
                                 std::fabs(gr[1]) * ((double)std::fabs(tc[1]) + std::fabs(part[1])) +
                                 std::fabs(gr[2]) * ((double)std::fabs(tc[2]) + std::fabs(part[2])));
                            const double agam = alpha * agm, scm = 0.5 * agam;
                            const double adu = std::fabs(du), adv = std::fabs(dv);
                            const double t9[9] = {agam * (adu * std::fabs(ic11) + adv * std::fabs(ic21)),
                                                  agam * (adu * std::fabs(ic21) + adv * std::fabs(ic22)),
                                                  geval * agm, scm * adu * adu, 2.0 * scm * adu * adv,
                                                  scm * adv * adv, std::fabs(ta * gr[0]),
                                                  std::fabs(ta * gr[1]), std::fabs(ta * gr[2])};
                            for (int k = 0; k < 9; ++k) atomic_add(&b[k], t9[k]);
                        }
                    }
                }
        });
    if (!macc.empty())
        for (size_t k = 0; k < (size_t)F * 9; ++k) mag[k] = (float)macc[k];
    for (int f = 0; f < (project_only ? 0 : F); ++f) {
        const double* a = &acc[9 * (size_t)f];
        mean2d_g[2 * f] = (float)a[0]; mean2d_g[2 * f + 1] = (float)a[1];
        opacity_g[f] = (float)a[2];
        licov_g[3 * f] = (float)a[3]; licov_g[3 * f + 1] = (float)a[4]; licov_g[3 * f + 2] = (float)a[5];
        color_g[3 * f] = (float)a[6]; color_g[3 * f + 1] = (float)a[7]; color_g[3 * f + 2] = (float)a[8];
    }

    // B3
    const float* P = cam.P;
    float Ps[3][3];
    for (int i = 0; i < 3; ++i) for (int j = 0; j < 3; ++j) Ps[i][j] = P[i + 3 * j];
    const int deg = opt.sh_degree;
    const int MAXO = (deg + 1) * (deg + 1);
    const int S_store = (g.sh_degree + 1) * (g.sh_degree + 1);
    const int S_grad = (sh_grad_degree + 1) * (sh_grad_degree + 1);
    parallel_for(0, F, [&](int64_t ff) {
        const int f = (int)ff;
        const int gi = fgidx_to_gidx[f] - 1;
        const float* r = f2d + 9 * (size_t)f;
        const float* mo = g.means_opacity_features + 4 * (size_t)gi;
        const float m[3] = {mo[0], mo[1], mo[2]};
        const float orig_op = o_sigmoid(mo[3]);
        const float depth = P[2] * m[0] + P[5] * m[1] + P[8] * m[2] + P[11];
        const float opac = opt.use_antialiasing ? r[2] : orig_op;
        const float og = opacity_g[f];
        opf_g[f] = opt.use_antialiasing ? og * opac * (1.0f - orig_op) : og * opac * (1.0f - opac);

        // compute_cov2d_lower_grad
        const float a = r[3], b = r[4], d = r[5];
        const float a_sq = a * a, ab = a * b, b_sq = b * b, bd = b * d, d_sq = d * d, ad = a * d;
        const float ab2 = ab + ab, bd2 = bd + bd;
        const float M[3][3] = {{a_sq, ab, b_sq}, {ab2, b_sq + ad, bd2}, {b * b, bd, d_sq}};
        const float* lg = licov_g + 3 * (size_t)f;
        float cg[3];
        for (int i = 0; i < 3; ++i) cg[i] = -(M[i][0] * lg[0] + M[i][1] * lg[1] + M[i][2] * lg[2]);
        if (opt.use_antialiasing) {
            const float Dx = opt.dilation_x, Dy = opt.dilation_y;
            const float det = (ad - b_sq) * Dx * Dy;
            const float b2 = b + b;
            const float k = orig_op * og;
            const float e0 = a_sq * Dx + b_sq * Dx - a * det;
            const float e1 = b2 * (a * Dx + d * Dy - det);
            const float e2 = b_sq * Dx + (d * d) * Dy - d * det;
            cg[0] = cg[0] + k * e0; cg[1] = cg[1] + k * e1; cg[2] = cg[2] + k * e2;
        }

        // mean3d gradient from mean2d
        const float mx = r[0], my = r[1];
        float cmx = mx, cmy = my;
        const bool clampmode = opt.clipping_mode == 0;
        if (clampmode) {
            cmx = o_clamp(mx, opt.clip_x_min, opt.clip_x_max);
            cmy = o_clamp(my, opt.clip_y_min, opt.clip_y_max);
        }
        const J23 J = lin_proj(cam, cmx, cmy, depth);
        const float gx = mean2d_g[2 * f], gy = mean2d_g[2 * f + 1];
        float m3[3];
        if (!clampmode) {
            for (int j = 0; j < 3; ++j) m3[j] = J.a[0][j] * gx + J.a[1][j] * gy;
        } else {
            const float t[3] = {gx, gy, -(mx * gx + my * gy)};
            const float idepth = 1.0f / depth;
            for (int j = 0; j < 3; ++j) m3[j] = idepth * (Ps[0][j] * t[0] + Ps[1][j] * t[1] + Ps[2][j] * t[2]);
        }

        // mean3d gradient from cov2d (Transposed_dsigma_dm)
        float V[6];
        float s[3];
        const float* sf = g.scaling_features + 3 * (size_t)gi;
        for (int j = 0; j < 3; ++j) s[j] = o_expf(sf[j]);
        float R[3][3];
        const float* qf = g.rotation_features + 4 * (size_t)gi;
        quat_to_rot(qf, R);
        {
            float RS[3][3];
            for (int i = 0; i < 3; ++i) for (int j = 0; j < 3; ++j) RS[i][j] = R[i][j] * s[j];
            for (int k = 0; k < 6; ++k) {
                const int i = L3I[k], j = L3J[k];
                V[k] = RS[i][0] * RS[j][0] + RS[i][1] * RS[j][1] + RS[i][2] * RS[j][2];
            }
        }
        {
            const float c2x = cmx + cmx, c2y = cmy + cmy;
            float dlx = 1.0f, dly = 1.0f;
            if (clampmode) {
                dlx = (opt.clip_x_min < cmx && cmx <= opt.clip_x_max) ? 1.0f : 0.0f;
                dly = (opt.clip_y_min < cmy && cmy <= opt.clip_y_max) ? 1.0f : 0.0f;
            }
            // dJ[i][al][k] = d Jc[i][al] / d m_k  (times -depth^2)
            float dJ[2][3][3];
            for (int al = 0; al < 3; ++al) {
                const float r0 = Ps[0][al] - c2x * Ps[2][al];
                const float r1 = Ps[1][al] - c2y * Ps[2][al];
                const float e0 = dlx * Ps[2][al];
                const float e1 = dly * Ps[2][al];
                for (int k = 0; k < 3; ++k) {
                    dJ[0][al][k] = e0 * Ps[0][k] + r0 * Ps[2][k];
                    dJ[1][al][k] = e1 * Ps[1][k] + r1 * Ps[2][k];
                }
            }
            const float sc = -(1.0f / (depth * depth));
            for (int k = 0; k < 3; ++k) {
                float acc3 = 0.0f;
                for (int p = 0; p < 3; ++p) {
                    const int i = L2I[p], j = L2J[p];
                    float t = 0.0f;
                    for (int al = 0; al < 3; ++al)
                        for (int be = 0; be < 3; ++be)
                            t = t + V[low3(al, be)] * (dJ[i][al][k] * J.a[j][be] + J.a[i][al] * dJ[j][be][k]);
                    acc3 = acc3 + t * cg[p];
                }
                m3[k] = m3[k] + sc * acc3;
            }
        }
        // mean3d gradient from the colour's view dependence
        const float vx = m[0] - cam.position[0], vy = m[1] - cam.position[1], vz = m[2] - cam.position[2];
        const float inv_vn = 1.0f / std::sqrt(vx * vx + vy * vy + vz * vz);
        const float nd[3] = {vx * inv_vn, vy * inv_vn, vz * inv_vn};
        const float col[3] = {r[6], r[7], r[8]};
        const float* cgr = color_g + 3 * (size_t)f;
        const float* h = g.sh_coeffs + (size_t)gi * 3 * S_store;
        float Jt[3][3];
        color_dir_jacobian_t(deg, col, nd, h, fix16, Jt);
        float ndg[3];
        for (int a3 = 0; a3 < 3; ++a3) ndg[a3] = Jt[a3][0] * cgr[0] + Jt[a3][1] * cgr[1] + Jt[a3][2] * cgr[2];
        for (int a3 = 0; a3 < 3; ++a3) {
            float w = 0.0f;
            for (int b3 = 0; b3 < 3; ++b3) {
                const float Nab = a3 == b3 ? 1.0f - nd[a3] * nd[a3]
                                           : -nd[std::min(a3, b3)] * nd[std::max(a3, b3)];
                w = w + Nab * ndg[b3];
            }
            m3[a3] = m3[a3] + inv_vn * w;
        }
        for (int j = 0; j < 3; ++j) mean3d_g[3 * (size_t)f + j] = m3[j];

        // scaling features: cov3d lower gradient = Transposed_dsigma_dv(Jc) * cg
        float vg[6];
        for (int jv = 0; jv < 6; ++jv) {
            const int rr = L3I[jv], ss = L3J[jv];
            float t = 0.0f;
            for (int p = 0; p < 3; ++p) {
                const int pp = L2I[p], qq = L2J[p];
                float e = J.a[pp][rr] * J.a[qq][ss];
                if (rr != ss) e = e + J.a[pp][ss] * J.a[qq][rr];
                t = t + e * cg[p];
            }
            vg[jv] = t;
        }
        for (int j = 0; j < 3; ++j) {
            float t = 0.0f;
            for (int i = 0; i < 6; ++i) t = t + (s[j] * R[L3I[i]][j] * R[L3J[i]][j]) * vg[i];
            scale_g[3 * (size_t)f + j] = (2.0f * t) * s[j];
        }
        // rotation features
        const float ssq[3] = {s[0] * s[0], s[1] * s[1], s[2] * s[2]};
        float Rg[3][3];
        for (int k = 0; k < 3; ++k)
            for (int l = 0; l < 3; ++l) {
                float t = vg[low3(k, k)] * R[k][l];
                for (int i = 0; i < 3; ++i) t = t + vg[low3(i, k)] * R[i][l];
                Rg[k][l] = ssq[l] * t;
            }
        const float qss = qf[0] * qf[0] + qf[1] * qf[1] + qf[2] * qf[2] + qf[3] * qf[3];
        const float inv_qn = 1.0f / std::sqrt(qss);
        const float nq[4] = {qf[0] * inv_qn, qf[1] * inv_qn, qf[2] * inv_qn, qf[3] * inv_qn};
        {
            const float rq = nq[0], xq = nq[1], yq = nq[2], zq = nq[3];
            const float m2x = -(xq + xq), m2y = -(yq + yq), m2z = -(zq + zq);
            const float A[4][3][3] = {
                {{0.0f, -zq, yq}, {zq, 0.0f, -xq}, {-yq, xq, 0.0f}},
                {{0.0f, yq, zq}, {yq, m2x, -rq}, {zq, rq, m2x}},
                {{m2y, xq, rq}, {xq, 0.0f, zq}, {-rq, zq, m2y}},
                {{m2z, -rq, xq}, {rq, m2z, yq}, {xq, yq, 0.0f}}};
            float nqg[4];
            for (int t4 = 0; t4 < 4; ++t4) {
                float dsum = 0.0f;
                for (int col3 = 0; col3 < 3; ++col3)
                    for (int row3 = 0; row3 < 3; ++row3) dsum = dsum + A[t4][row3][col3] * Rg[row3][col3];
                nqg[t4] = 2.0f * dsum;
            }
            for (int a4 = 0; a4 < 4; ++a4) {
                float w = 0.0f;
                for (int b4 = 0; b4 < 4; ++b4) {
                    const float Nab = a4 == b4 ? 1.0f - nq[a4] * nq[a4]
                                               : -nq[std::min(a4, b4)] * nq[std::max(a4, b4)];
                    w = w + Nab * nqg[b4];
                }
                rot_g[4 * (size_t)f + a4] = inv_qn * w;
            }
        }
        // SH coefficients (compute_sh_coeffs_grad!)
        float* shg = sh_g + (size_t)f * 3 * S_grad;
        for (int l = 0; l < 3; ++l) {
            if (col[l] >= 0.0f) {
                for (int k = 1; k <= MAXO; ++k) shg[(k - 1) + l * S_grad] = cgr[l] * o_sh_basis(k, nd[0], nd[1], nd[2]);
            } else {
                for (int k = 1; k <= MAXO; ++k) shg[(k - 1) + l * S_grad] = 0.0f;
            }
        }
    });
    return 0;
}

}  // extern "C"
