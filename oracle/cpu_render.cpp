// cpu_render.cpp — TEST INFRASTRUCTURE ONLY: restatement of ThreeDGaussianSplatting.jl's
// single-threaded CPU `render!` (src/forward_core.jl:25-177), used as the timed CPU
// baseline and as a second, independent cross-check of the GPU-path oracle (the reference
// compares the two at atol 1e-3: test/forward_core.jl:78-141).
//
// Differences from the GPU path are the reference's own: no tiles, one global depth sort
// (sortperm, stable), per-Gaussian exact pixel extents (:117-150), and a Gaussian whose
// contribution would push T below min_transmittance is skipped, not a stop (:155).
//
// nthreads > 1 splits the image into column strips; every pixel still sees the Gaussians in
// the same depth order, so the result does not depend on the thread count.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <numeric>
#include <thread>
#include <vector>

#include "../include/gs3d.h"
#include "oracle_math.h"

using namespace oracle;

namespace {

struct F2D { float x, y, opacity, depth, p, q, r, col[3]; };

inline void quat_to_rot(const float q[4], float R[3][3]) {
    const float ss = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3];
    const float s = std::sqrt(2.0f * (1.0f / ss));
    const float r = q[0] * s, x = q[1] * s, y = q[2] * s, z = q[3] * s;
    R[0][0] = 1.0f - (y * y + z * z); R[0][1] = x * y - r * z;         R[0][2] = x * z + r * y;
    R[1][0] = x * y + r * z;         R[1][1] = 1.0f - (x * x + z * z); R[1][2] = y * z - r * x;
    R[2][0] = x * z - r * y;         R[2][1] = y * z + r * x;         R[2][2] = 1.0f - (x * x + y * y);
}

}  // namespace

extern "C" {

// Outputs rgb (3 x h x w), trans (h x w), depth (h x w, may be NULL). Returns F.
int32_t oracle_cpu_render(const gs3d_gaussians* gp, const gs3d_camera* camp,
                          const gs3d_render_options* op, float* rgb, float* trans,
                          float* depth_img, int32_t nthreads) {
    const gs3d_gaussians& g = *gp;
    const gs3d_camera& cam = *camp;
    const gs3d_render_options& opt = *op;
    const int W = cam.width, H = cam.height;
    const float* P = cam.P;
    const int S = (g.sh_degree + 1) * (g.sh_degree + 1);
    std::vector<F2D> fv;
    fv.reserve(g.n / 4 + 16);
    for (int i = 0; i < g.n; ++i) {
        const float* mo = g.means_opacity_features + 4 * (size_t)i;
        const float m[3] = {mo[0], mo[1], mo[2]};
        float opacity = o_sigmoid(mo[3]);
        if (!(opacity >= opt.min_alpha)) continue;
        const float h0 = P[0] * m[0] + P[3] * m[1] + P[6] * m[2] + P[9];
        const float h1 = P[1] * m[0] + P[4] * m[1] + P[7] * m[2] + P[10];
        const float depth = P[2] * m[0] + P[5] * m[1] + P[8] * m[2] + P[11];
        const float mx = h0 / depth, my = h1 / depth;
        if (!(cam.near_z < depth && depth <= cam.far_z)) continue;
        if (opt.clipping_mode == 1 &&
            !(opt.clip_x_min < mx && mx <= opt.clip_x_max && opt.clip_y_min < my && my <= opt.clip_y_max))
            continue;
        float cu = mx, cv = my;
        if (opt.clipping_mode == 0) {
            cu = o_clamp(mx, opt.clip_x_min, opt.clip_x_max);
            cv = o_clamp(my, opt.clip_y_min, opt.clip_y_max);
        }
        const float idepth = 1.0f / depth;
        float J[2][3];
        for (int j = 0; j < 3; ++j) {
            J[0][j] = idepth * (P[0 + 3 * j] + (-cu) * P[2 + 3 * j]);
            J[1][j] = idepth * (P[1 + 3 * j] + (-cv) * P[2 + 3 * j]);
        }
        const float* sf = g.scaling_features + 3 * (size_t)i;
        const float s[3] = {o_expf(sf[0]), o_expf(sf[1]), o_expf(sf[2])};
        float R[3][3];
        quat_to_rot(g.rotation_features + 4 * (size_t)i, R);
        float A[2][3];
        for (int a = 0; a < 2; ++a)
            for (int k = 0; k < 3; ++k)
                A[a][k] = J[a][0] * (R[0][k] * s[k]) + J[a][1] * (R[1][k] * s[k]) + J[a][2] * (R[2][k] * s[k]);
        float c11 = A[0][0] * A[0][0] + A[0][1] * A[0][1] + A[0][2] * A[0][2];
        const float c21 = A[1][0] * A[0][0] + A[1][1] * A[0][1] + A[1][2] * A[0][2];
        float c22 = A[1][0] * A[1][0] + A[1][1] * A[1][1] + A[1][2] * A[1][2];
        float und = 0.0f;
        if (opt.use_antialiasing) und = std::max(c11 * c22 - c21 * c21, 0.0f);
        c11 += opt.dilation_x;
        c22 += opt.dilation_y;
        const float idet = 1.0f / (c11 * c22 - c21 * c21);
        if (opt.use_antialiasing) opacity *= std::max(opt.antialiasing_min_factor, std::sqrt(und * idet));
        F2D f;
        f.x = mx; f.y = my; f.opacity = opacity; f.depth = depth;
        f.p = c22 * idet; f.q = -c21 * idet; f.r = c11 * idet;
        const float vx = m[0] - cam.position[0], vy = m[1] - cam.position[1], vz = m[2] - cam.position[2];
        const float inv = 1.0f / std::sqrt(vx * vx + vy * vy + vz * vz);
        const float x = vx * inv, y = vy * inv, z = vz * inv;
        const float* h = g.sh_coeffs + (size_t)i * 3 * S;
        for (int c = 0; c < 3; ++c) {
            const float* hc = h + c * S;
            const int deg = opt.sh_degree;
            float cc = o_sh_basis(1, x, y, z) * hc[0];
            if (deg >= 1) {
                cc += (o_sh_basis(2, x, y, z) * hc[1] + o_sh_basis(3, x, y, z) * hc[2] + o_sh_basis(4, x, y, z) * hc[3]);
                if (deg >= 2) {
                    cc += (o_sh_basis(5, x, y, z) * hc[4] + o_sh_basis(6, x, y, z) * hc[5] +
                           o_sh_basis(7, x, y, z) * hc[6] + o_sh_basis(8, x, y, z) * hc[7] +
                           o_sh_basis(9, x, y, z) * hc[8]);
                    if (deg >= 3)
                        cc += (o_sh_basis(10, x, y, z) * hc[9] + o_sh_basis(11, x, y, z) * hc[10] +
                               o_sh_basis(12, x, y, z) * hc[11] + o_sh_basis(13, x, y, z) * hc[12] +
                               o_sh_basis(14, x, y, z) * hc[13] + o_sh_basis(15, x, y, z) * hc[14] +
                               o_sh_basis(16, x, y, z) * hc[15]);
                }
            }
            cc += 0.5f;
            if (cc < 0.0f) cc = 0.0f;
            f.col[c] = cc;
        }
        fv.push_back(f);
    }
    const int F = (int)fv.size();
    std::vector<int> sp(F);
    std::iota(sp.begin(), sp.end(), 0);
    std::stable_sort(sp.begin(), sp.end(), [&](int a, int b) { return fv[a].depth < fv[b].depth; });

    for (size_t k = 0; k < (size_t)W * H; ++k) {
        trans[k] = 1.0f;
        rgb[3 * k] = rgb[3 * k + 1] = rgb[3 * k + 2] = 0.0f;
        if (depth_img) depth_img[k] = 0.0f;
    }
    auto strip = [&](int ua, int ub) {  // columns [ua, ub], 1-based
        for (int fi : sp) {
            const F2D& f = fv[fi];
            const float idet = f.p * f.r - f.q * f.q;
            const float gamma = 2.0f * o_logf(f.opacity / opt.min_alpha) / idet;
            const float xr = std::sqrt(f.r * gamma);
            int u_start = std::max(1, o_ceil_i32(f.x - xr + 0.5f));
            int u_end = std::min(W, o_round_i32(f.x + xr));
            u_start = std::max(u_start, ua);
            u_end = std::min(u_end, ub);
            for (int u = u_start; u <= u_end; ++u) {
                const float ucts = (float)u - 0.5f;
                const float du = ucts - f.x;
                const float disc = f.r * gamma - du * du;
                const float sq = disc <= 0.0f ? 0.0f : std::sqrt(idet * disc);
                const float qdu = f.q * du;
                const float ir = 1.0f / f.r;
                const float top = f.y + (-qdu - sq) * ir;
                const float bot = f.y + (-qdu + sq) * ir;
                const int v_start = std::max(1, o_ceil_i32(top + 0.5f));
                const int v_stop = std::min(H, o_round_i32(bot));
                for (int v = v_start; v <= v_stop; ++v) {
                    const float ddu = ((float)u - 0.5f) - f.x;
                    const float ddv = ((float)v - 0.5f) - f.y;
                    const float val = f.opacity * o_expf(-0.5f * (f.p * (ddu * ddu) + f.r * (ddv * ddv)) - f.q * ddu * ddv);
                    const float alpha = o_min(opt.max_alpha, val);
                    const size_t px = (size_t)(v - 1) + (size_t)H * (u - 1);
                    const float cT = trans[px];
                    const float nT = cT * (1.0f - alpha);
                    if (nT < opt.min_transmittance) continue;
                    const float w = alpha * cT;
                    rgb[3 * px] += w * f.col[0];
                    rgb[3 * px + 1] += w * f.col[1];
                    rgb[3 * px + 2] += w * f.col[2];
                    trans[px] = nT;
                    if (depth_img) depth_img[px] += w * f.depth;
                }
            }
        }
    };
    if (nthreads <= 1) {
        strip(1, W);
    } else {
        std::vector<std::thread> th;
        const int per = (W + nthreads - 1) / nthreads;
        for (int t = 0; t < nthreads; ++t) {
            const int ua = 1 + t * per, ub = std::min(W, (t + 1) * per);
            if (ua > ub) break;
            th.emplace_back(strip, ua, ub);
        }
        for (auto& t : th) t.join();
    }
    for (size_t k = 0; k < (size_t)W * H; ++k)
        for (int c = 0; c < 3; ++c) rgb[3 * k + c] += trans[k] * opt.background[c];
    return F;
}

}  // extern "C"
