// forward.cpp — TEST INFRASTRUCTURE ONLY: CPU oracle of gs3d's render forward.
// Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it, and
// only as the checker or the timed CPU baseline, never as a product path.
//
// Restates the GPU path of ThreeDGaussianSplatting.jl's `render!`
// (src/forward_core.jl:196-314) step by step, single-threaded, in Float32 with the
// reference's operation order and no contraction (-ffp-contract=off):
//   keep mask ............ forward_core.jl:326-355 (cameras.jl:679-692)
//   scan + compaction .... forward_core.jl:231-244, :371-386
//   projection ........... forward_core.jl:411-517 (cameras.jl:714-774,
//                          gaussians.jl:1320-1331, misc.jl:133-141, sh.jl:38-112,
//                          forward_structs.jl:727-739, :1303-1316, :1372-1411, :517-528)
//   duplication keys ..... forward_core.jl:531-603 (forward_structs.jl:436-459)
//   stable key sort ...... forward_core.jl:618-660 (cub_sort_pairs_wrapper.cu:31-43)
//   tile ends ............ forward_core.jl:676-734
//   tile alpha blend ..... forward_core.jl:756-993
//   void render .......... forward_structs.jl:743-757
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <numeric>
#include <vector>

#include "../include/gs3d.h"
#include "oracle_math.h"

using namespace oracle;

namespace oracle {

struct Mat23 { float a[2][3]; };

// project_with_depth (cameras.jl:714-722): P[1:3,1:3] * m .+ P[1:3,4], mean2d = p[1:2]/p[3]
static inline void project_point(const gs3d_camera& c, const float m[3], float& px, float& py,
                                 float& depth) {
    const float* P = c.P;  // column-major 3x4
    const float h0 = P[0] * m[0] + P[3] * m[1] + P[6] * m[2] + P[9];
    const float h1 = P[1] * m[0] + P[4] * m[1] + P[7] * m[2] + P[10];
    const float h2 = P[2] * m[0] + P[5] * m[1] + P[8] * m[2] + P[11];
    depth = h2;
    px = h0 / h2;
    py = h1 / h2;
}

// get_depth (cameras.jl:679-682)
static inline float point_depth(const gs3d_camera& c, const float m[3]) {
    const float* P = c.P;
    return P[2] * m[0] + P[5] * m[1] + P[8] * m[2] + P[11];
}

// get_linearized_projection_2d (cameras.jl:755-774):
// J = (1/depth) * [1 0 -u; 0 1 -v] * P[1:3,1:3]
static inline Mat23 linearized_projection(const gs3d_camera& c, float u, float v, float depth) {
    const float* P = c.P;
    const float idepth = 1.0f / depth;
    Mat23 J;
    for (int j = 0; j < 3; ++j) {
        J.a[0][j] = idepth * (P[0 + 3 * j] + (-u) * P[2 + 3 * j]);
        J.a[1][j] = idepth * (P[1 + 3 * j] + (-v) * P[2 + 3 * j]);
    }
    return J;
}

// quaternion_to_rotation_matrix (misc.jl:133-141)
static inline void quat_to_rot(const float q[4], float R[3][3]) {
    const float ss = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3];
    const float s = std::sqrt(2.0f * (1.0f / ss));
    const float r = q[0] * s, x = q[1] * s, y = q[2] * s, z = q[3] * s;
    R[0][0] = 1.0f - (y * y + z * z); R[0][1] = x * y - r * z;         R[0][2] = x * z + r * y;
    R[1][0] = x * y + r * z;         R[1][1] = 1.0f - (x * x + z * z); R[1][2] = y * z - r * x;
    R[2][0] = x * z - r * y;         R[2][1] = y * z + r * x;         R[2][2] = 1.0f - (x * x + y * y);
}

// sh_coeffs_to_color (sh.jl:38-112); h points at coefficient 1 of channel 1 of this
// Gaussian, `stride` is the storage order (d_storage+1)^2.
static inline void sh_to_color(int deg, const float* h, int stride, float x, float y, float z,
                               float out[3]) {
    for (int c = 0; c < 3; ++c) {
        const float* hc = h + c * stride;
        float cc = o_sh_basis(1, x, y, z) * hc[0];
        if (deg >= 1) {
            cc += (o_sh_basis(2, x, y, z) * hc[1] + o_sh_basis(3, x, y, z) * hc[2] +
                   o_sh_basis(4, x, y, z) * hc[3]);
            if (deg >= 2) {
                cc += (o_sh_basis(5, x, y, z) * hc[4] + o_sh_basis(6, x, y, z) * hc[5] +
                       o_sh_basis(7, x, y, z) * hc[6] + o_sh_basis(8, x, y, z) * hc[7] +
                       o_sh_basis(9, x, y, z) * hc[8]);
                if (deg >= 3) {
                    cc += (o_sh_basis(10, x, y, z) * hc[9] + o_sh_basis(11, x, y, z) * hc[10] +
                           o_sh_basis(12, x, y, z) * hc[11] + o_sh_basis(13, x, y, z) * hc[12] +
                           o_sh_basis(14, x, y, z) * hc[13] + o_sh_basis(15, x, y, z) * hc[14] +
                           o_sh_basis(16, x, y, z) * hc[15]);
                }
            }
        }
        cc += 0.5f;
        if (cc < 0.0f) cc = 0.0f;
        out[c] = cc;
    }
}

// Normalised viewing direction: (m - o) .* inv(sqrt(sum(abs2)))  (backward_core.jl:383-385;
// the forward's normalize() is taken to be the same operation).
static inline void view_direction(const gs3d_camera& c, const float m[3], float d[3]) {
    const float vx = m[0] - c.position[0], vy = m[1] - c.position[1], vz = m[2] - c.position[2];
    const float inv = 1.0f / std::sqrt(vx * vx + vy * vy + vz * vz);
    d[0] = vx * inv; d[1] = vy * inv; d[2] = vz * inv;
}

// Covariance of the projected Gaussian, lower triangle (gaussians.jl:1328-1331):
// JRS = J * (R .* s'), Sigma = JRS * JRS'
static inline void project_covariance(const Mat23& J, const float R[3][3], const float s[3],
                                      float& c11, float& c21, float& c22) {
    float RS[3][3];
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) RS[i][j] = R[i][j] * s[j];
    float A[2][3];
    for (int i = 0; i < 2; ++i)
        for (int k = 0; k < 3; ++k)
            A[i][k] = J.a[i][0] * RS[0][k] + J.a[i][1] * RS[1][k] + J.a[i][2] * RS[2][k];
    c11 = A[0][0] * A[0][0] + A[0][1] * A[0][1] + A[0][2] * A[0][2];
    c21 = A[1][0] * A[0][0] + A[1][1] * A[0][1] + A[1][2] * A[0][2];
    c22 = A[1][0] * A[1][0] + A[1][1] * A[1][1] + A[1][2] * A[1][2];
}

// Render-only input (RenderOnlyGaussiansVector, gaussians.jl:342-392): the 2D covariance is the
// congruence transform J V J^T of the stored 3D covariance (gaussians.jl:1324-1327,
// special_sarrays.jl:1801-1810): T = J V, then the lower entries of T J^T, each sum in index
// order (the order the kernel uses; StaticArrays' unrolling is not recoverable).
static void project_covariance_given(const Mat23& J, const float* cv, float& c11, float& c21,
                                     float& c22) {
    const float V[3][3] = {{cv[0], cv[1], cv[2]}, {cv[1], cv[3], cv[4]}, {cv[2], cv[4], cv[5]}};
    float T[2][3];
    for (int i = 0; i < 2; ++i)
        for (int k = 0; k < 3; ++k)
            T[i][k] = J.a[i][0] * V[0][k] + J.a[i][1] * V[1][k] + J.a[i][2] * V[2][k];
    c11 = T[0][0] * J.a[0][0] + T[0][1] * J.a[0][1] + T[0][2] * J.a[0][2];
    c21 = T[1][0] * J.a[0][0] + T[1][1] * J.a[0][1] + T[1][2] * J.a[0][2];
    c22 = T[1][0] * J.a[1][0] + T[1][1] * J.a[1][1] + T[1][2] * J.a[1][2];
}

struct Projected {
    float mx, my, depth, opacity, ic11, ic21, ic22, col[3];
    int32_t rect[4];  // tile xmin, ymin, xmax, ymax
    int32_t count;
};

// project_fgaussians_kernel! body (forward_core.jl:425-515) for one filtered Gaussian.
// cov != NULL: render-only input (opacity stored as is, covariances 6 x n lower).
static Projected project_one(const gs3d_gaussians& g, const float* cov, int gidx0,
                             const gs3d_camera& cam, const gs3d_tiling& til,
                             const gs3d_render_options& opt) {
    Projected p;
    const float* mo = g.means_opacity_features + 4 * (size_t)gidx0;
    const float m[3] = {mo[0], mo[1], mo[2]};
    float opacity = cov ? mo[3] : o_sigmoid(mo[3]);
    float mx, my, depth;
    project_point(cam, m, mx, my, depth);
    float cu = mx, cv = my;
    if (opt.clipping_mode == 0) {
        cu = o_clamp(mx, opt.clip_x_min, opt.clip_x_max);
        cv = o_clamp(my, opt.clip_y_min, opt.clip_y_max);
    }
    const Mat23 J = linearized_projection(cam, cu, cv, depth);
    float c11, c21, c22;
    if (cov) {
        project_covariance_given(J, cov + 6 * (size_t)gidx0, c11, c21, c22);
    } else {
        const float* sf = g.scaling_features + 3 * (size_t)gidx0;
        const float s[3] = {o_expf(sf[0]), o_expf(sf[1]), o_expf(sf[2])};
        float R[3][3];
        quat_to_rot(g.rotation_features + 4 * (size_t)gidx0, R);
        project_covariance(J, R, s, c11, c21, c22);
    }
    float undilated_det = 0.0f;
    if (opt.use_antialiasing) undilated_det = std::max(c11 * c22 - c21 * c21, 0.0f);
    c11 += opt.dilation_x;
    c22 += opt.dilation_y;
    const float icov_det = 1.0f / (c11 * c22 - c21 * c21);
    if (opt.use_antialiasing)
        opacity *= std::max(opt.antialiasing_min_factor, std::sqrt(undilated_det * icov_det));

    // _get_bbox_cts_px_cov + _get_bbox_discrete_px
    bool empty = true;
    int32_t left = 0, top = 0, right = -1, bottom = -1;
    if (opacity >= opt.min_alpha) {
        const float gamma = 2.0f * o_logf(opacity / opt.min_alpha);
        const float xr = std::sqrt(gamma * c11);
        const float yr = std::sqrt(gamma * c22);
        left = std::max(1, o_ceil_i32((mx - xr) + 0.5f));
        top = std::max(1, o_ceil_i32((my - yr) + 0.5f));
        right = std::min(cam.width, o_round_i32(mx + xr));
        bottom = std::min(cam.height, o_round_i32(my + yr));
        empty = left > right || top > bottom;
    }
    p.mx = mx; p.my = my; p.depth = depth; p.opacity = opacity;
    p.ic11 = c22 * icov_det;
    p.ic21 = -c21 * icov_det;
    p.ic22 = c11 * icov_det;
    float d[3];
    view_direction(cam, m, d);
    sh_to_color(opt.sh_degree, g.sh_coeffs + (size_t)gidx0 * 3 * (g.sh_degree + 1) * (g.sh_degree + 1),
                (g.sh_degree + 1) * (g.sh_degree + 1), d[0], d[1], d[2], p.col);
    if (empty) {
        p.count = 0;
        p.rect[0] = 1; p.rect[1] = 1; p.rect[2] = 0; p.rect[3] = 0;
    } else {
        // rectangle_to_tile_ids without clamping: ceil(px / tile size) on positive ints
        p.rect[0] = (left + til.tile_width - 1) / til.tile_width;
        p.rect[1] = (top + til.tile_height - 1) / til.tile_height;
        p.rect[2] = (right + til.tile_width - 1) / til.tile_width;
        p.rect[3] = (bottom + til.tile_height - 1) / til.tile_height;
        p.count = (p.rect[2] - p.rect[0] + 1) * (p.rect[3] - p.rect[1] + 1);
    }
    return p;
}

// fill_keep_gaussians_kernel! body (forward_core.jl:337-352)
static bool keep_one(const gs3d_gaussians& g, const float* cov, int gidx0, const gs3d_camera& cam,
                     const gs3d_render_options& opt) {
    const float* mo = g.means_opacity_features + 4 * (size_t)gidx0;
    const float m[3] = {mo[0], mo[1], mo[2]};
    const float opacity = cov ? mo[3] : o_sigmoid(mo[3]);
    bool keep = opacity >= opt.min_alpha;
    if (keep) {
        if (opt.clipping_mode == 1) {
            float mx, my, depth;
            project_point(cam, m, mx, my, depth);
            const bool on = opt.clip_x_min < mx && mx <= opt.clip_x_max &&
                            opt.clip_y_min < my && my <= opt.clip_y_max;
            keep = on && (cam.near_z < depth && depth <= cam.far_z) && opacity > opt.min_alpha;
        } else {
            const float depth = point_depth(cam, m);
            keep = cam.near_z < depth && depth <= cam.far_z;
        }
    }
    return keep;
}

}  // namespace oracle

extern "C" {

int64_t oracle_dup_keys(int32_t F, const int32_t* ntiles, const int32_t* ranges,
                        const float* depths, int32_t tiles_x, int64_t* codes, int32_t* dfgidx);
void oracle_tiles_end(const int64_t* scodes, int64_t D, int32_t nb_tiles, int32_t* tiles_end);

// Stable sort of (key, value) pairs on bits [0, highest_key_bit) — the semantics of
// cub::DeviceRadixSort::SortPairs(begin_bit = 0, end_bit = highest_key_bit).
int oracle_sort_pairs(const int64_t* keys_in, int64_t* keys_out, const int32_t* vals_in,
                      int32_t* vals_out, int64_t n, int highest_key_bit) {
    const uint64_t mask = highest_key_bit >= 64 ? ~0ull : ((1ull << highest_key_bit) - 1ull);
    std::vector<int64_t> idx(n);
    std::iota(idx.begin(), idx.end(), 0);
    std::stable_sort(idx.begin(), idx.end(), [&](int64_t a, int64_t b) {
        return ((uint64_t)keys_in[a] & mask) < ((uint64_t)keys_in[b] & mask);
    });
    for (int64_t i = 0; i < n; ++i) {
        keys_out[i] = keys_in[idx[i]];
        vals_out[i] = vals_in[idx[i]];
    }
    return 0;
}

// accumulate!(+) of the keep mask and fill_fgidx_to_gidx_kernel! (forward_core.jl:231-244,
// :371-386). Returns F.
int32_t oracle_compact(const uint8_t* keep, int64_t n, int32_t* keep_cs, int32_t* fgidx_to_gidx) {
    int32_t cs = 0;
    for (int64_t i = 0; i < n; ++i) {
        cs += keep[i] ? 1 : 0;
        keep_cs[i] = cs;
        if (keep[i]) fgidx_to_gidx[cs - 1] = (int32_t)(i + 1);
    }
    return cs;
}

// fill_df2dgs_codes_and_dfgidx_to_fgidx_kernel! (forward_core.jl:531-603) given the counts,
// tile ranges (xmin, ymin, xmax, ymax per filtered Gaussian) and depths. Returns D.
int64_t oracle_dup_keys(int32_t F, const int32_t* ntiles, const int32_t* ranges,
                        const float* depths, int32_t tiles_x, int64_t* codes, int32_t* dfgidx) {
    int64_t d = 0;
    for (int f = 0; f < F; ++f) {
        if (ntiles[f] == 0) continue;
        uint32_t dbits;
        std::memcpy(&dbits, &depths[f], 4);
        const int32_t* rr = ranges + 4 * (size_t)f;
        for (int ty = rr[1]; ty <= rr[3]; ++ty)
            for (int tx = rr[0]; tx <= rr[2]; ++tx) {
                const int32_t tile = tx + (ty - 1) * tiles_x;
                codes[d] = (int64_t)(((uint64_t)(uint32_t)tile << 32) |
                                     (uint64_t)(int64_t)(int32_t)dbits);
                dfgidx[d] = f + 1;
                ++d;
            }
    }
    return d;
}

// fill_tiles_end_sdfgidx_kernel! (forward_core.jl:676-734), restated as: tiles_end[t] =
// number of sorted entries whose tile index is <= t.
void oracle_tiles_end(const int64_t* scodes, int64_t D, int32_t nb_tiles, int32_t* tiles_end) {
    int64_t d = 0;
    for (int t = 1; t <= nb_tiles; ++t) {
        while (d < D && (int32_t)((uint64_t)scodes[d] >> 32) <= t) ++d;
        tiles_end[t - 1] = (int32_t)d;
    }
}

// Full GPU-path render. Arrays use the reference layouts (see gs3d.h). Returns 0, or
// GS3D_ERR_CAPACITY when D > dup_capacity (counts still written: counts[0] = F,
// counts[1] = D). Any output image pointer may be NULL.
// Render-only input: gp's means_opacity_features hold x y z opacity, cov the 6 x n lower
// covariances (scaling / rotation features unused). Otherwise as oracle_render.
int oracle_render_ro(const gs3d_gaussians* gp, const float* cov, const gs3d_camera* camp,
                     const gs3d_tiling* tp, const gs3d_render_options* op, uint8_t* keep,
                     int32_t* keep_cs, int32_t* fgidx_to_gidx, float* depths, float* f2d,
                     int32_t* ranges, int32_t* ntiles, int32_t* ntiles_cs, int64_t dup_capacity,
                     int64_t* codes, int32_t* dfgidx, int64_t* scodes, int32_t* sfgidx,
                     int32_t* tiles_end, float* rgb, float* trans, float* depth_img, int32_t* last,
                     int64_t* counts);

int oracle_render(const gs3d_gaussians* gp, const gs3d_camera* camp, const gs3d_tiling* tp,
                  const gs3d_render_options* op, uint8_t* keep, int32_t* keep_cs,
                  int32_t* fgidx_to_gidx, float* depths, float* f2d, int32_t* ranges,
                  int32_t* ntiles, int32_t* ntiles_cs, int64_t dup_capacity, int64_t* codes,
                  int32_t* dfgidx, int64_t* scodes, int32_t* sfgidx, int32_t* tiles_end,
                  float* rgb, float* trans, float* depth_img, int32_t* last, int64_t* counts) {
    return oracle_render_ro(gp, nullptr, camp, tp, op, keep, keep_cs, fgidx_to_gidx, depths, f2d,
                            ranges, ntiles, ntiles_cs, dup_capacity, codes, dfgidx, scodes, sfgidx,
                            tiles_end, rgb, trans, depth_img, last, counts);
}

int oracle_render_ro(const gs3d_gaussians* gp, const float* cov, const gs3d_camera* camp,
                     const gs3d_tiling* tp, const gs3d_render_options* op, uint8_t* keep,
                     int32_t* keep_cs, int32_t* fgidx_to_gidx, float* depths, float* f2d,
                     int32_t* ranges, int32_t* ntiles, int32_t* ntiles_cs, int64_t dup_capacity,
                     int64_t* codes, int32_t* dfgidx, int64_t* scodes, int32_t* sfgidx,
                     int32_t* tiles_end, float* rgb, float* trans, float* depth_img, int32_t* last,
                     int64_t* counts) {
    const gs3d_gaussians& g = *gp;
    const gs3d_camera& cam = *camp;
    const gs3d_tiling& til = *tp;
    const gs3d_render_options& opt = *op;
    const int n = g.n;
    const int W = cam.width, H = cam.height;
    const int nb_tiles = til.nb_tiles_x * til.nb_tiles_y;

    // F1 + F2
    parallel_for(0, n, [&](int64_t i) { keep[i] = keep_one(g, cov, (int)i, cam, opt) ? 1 : 0; });
    int32_t cs = 0;
    for (int i = 0; i < n; ++i) {
        cs += keep[i];
        if (keep_cs) keep_cs[i] = cs;
        if (keep[i]) fgidx_to_gidx[cs - 1] = i + 1;
    }
    const int F = cs;

    auto render_void = [&]() {
        for (int u = 0; u < W; ++u)
            for (int v = 0; v < H; ++v) {
                const size_t px = (size_t)v + (size_t)H * u;
                if (rgb) for (int c = 0; c < 3; ++c) rgb[3 * px + c] = opt.background[c];
                if (trans) trans[px] = 1.0f;
                if (depth_img) depth_img[px] = INFINITY;
                if (last) last[px] = 0;
            }
    };
    counts[0] = F;
    counts[1] = 0;
    if (F == 0) { render_void(); return 0; }

    // F3 + F4
    parallel_for(0, F, [&](int64_t f) {
        const Projected p = project_one(g, cov, fgidx_to_gidx[f] - 1, cam, til, opt);
        depths[f] = p.depth;
        float* r = f2d + 9 * (size_t)f;
        r[0] = p.mx; r[1] = p.my; r[2] = p.opacity; r[3] = p.ic11; r[4] = p.ic21; r[5] = p.ic22;
        r[6] = p.col[0]; r[7] = p.col[1]; r[8] = p.col[2];
        for (int k = 0; k < 4; ++k) ranges[4 * (size_t)f + k] = p.rect[k];
        ntiles[f] = p.count;
    });
    int64_t D = 0;
    for (int f = 0; f < F; ++f) {
        D += ntiles[f];
        ntiles_cs[f] = (int32_t)D;
    }
    counts[1] = D;
    if (D == 0) { render_void(); return 0; }
    if (D > dup_capacity) return GS3D_ERR_CAPACITY;

    // F5: keys, tiles enumerated y-outer / x-inner, linear tile = x + (y-1) * tiles_x
    oracle_dup_keys(F, ntiles, ranges, depths, til.nb_tiles_x, codes, dfgidx);
    // F6
    int highest = 33;
    { int t = nb_tiles; while (t > 1) { t >>= 1; ++highest; } }  // 33 + floor(log2(T))
    oracle_sort_pairs(codes, scodes, dfgidx, sfgidx, D, highest);
    // F7
    oracle_tiles_end(scodes, D, nb_tiles, tiles_end);
    // F8: tile alpha blend (render_tiles_kernel!)
    const int TW = til.tile_width, TH = til.tile_height;
    parallel_for(0, (int64_t)til.nb_tiles_x * til.nb_tiles_y, [&](int64_t tl) {
            const int txi = (int)(tl % til.nb_tiles_x) + 1, tyi = (int)(tl / til.nb_tiles_x) + 1;
            const int tile = txi + (tyi - 1) * til.nb_tiles_x;
            const int start = tile == 1 ? 0 : tiles_end[tile - 2];
            const int end = tiles_end[tile - 1];
            const int u0 = (txi - 1) * TW, v0 = (tyi - 1) * TH;
            for (int pv = 1; pv <= TH; ++pv)
                for (int pu = 1; pu <= TW; ++pu) {
                    const int U = pu + u0, V = pv + v0;
                    if (!(U >= 1 && U <= W && V >= 1 && V <= H)) continue;
                    const float cu = (float)pu - 0.5f, cv = (float)pv - 0.5f;
                    const float uu = cu * cu, uv = cu * cv, vv = cv * cv;
                    float T = 1.0f, col[3] = {0.0f, 0.0f, 0.0f}, dep = 0.0f;
                    int32_t lastc = 0;
                    for (int s = start + 1; s <= end; ++s) {
                        const int fg = sfgidx[s - 1] - 1;
                        const float* r = f2d + 9 * (size_t)fg;
                        const float du = r[0] - (float)u0;
                        const float dv = r[1] - (float)v0;
                        const float ic11 = r[3], ic21 = r[4], ic22 = r[5];
                        const float ic11_du = ic11 * du, ic21_du = ic21 * du, ic22_dv = ic22 * dv;
                        const float p1 = -0.5f * ic11, p2 = -0.5f * ic22, p3 = -ic21;
                        const float p4 = ic11_du + ic21 * dv;
                        const float p5 = ic21_du + ic22_dv;
                        const float p6 = -0.5f * (ic11_du * du + ic22_dv * dv) - ic21_du * dv +
                                         o_logf(r[2]);
                        const float q = p1 * uu + p2 * vv + p3 * uv + p4 * cu + p5 * cv + p6;
                        const float alpha = o_min(opt.max_alpha, o_expf(q));
                        if (alpha < opt.min_alpha) continue;
                        const float nextT = T * (1.0f - alpha);
                        if (nextT < opt.min_transmittance) break;
                        const float w = T * alpha;
                        col[0] += w * r[6]; col[1] += w * r[7]; col[2] += w * r[8];
                        T = nextT;
                        dep += w * depths[fg];
                        lastc = s;
                    }
                    const size_t px = (size_t)(V - 1) + (size_t)H * (U - 1);
                    if (rgb)
                        for (int c = 0; c < 3; ++c) rgb[3 * px + c] = col[c] + T * opt.background[c];
                    if (trans) trans[px] = T;
                    if (depth_img) depth_img[px] = dep;
                    if (last) last[px] = lastc;
                }
        });
    return 0;
}

// Work counts of the blend loop (render_tiles_kernel!, forward_core.jl:928-968) over the
// arrays a render left: out[0] = (pixel, Gaussian) evaluations until each pixel stops (the
// terminating evaluation included), out[1] = evaluations blended into the pixel.
void oracle_work_counts(const float* f2d, const int32_t* sfgidx, const int32_t* tiles_end,
                        const gs3d_camera* camp, const gs3d_tiling* tp,
                        const gs3d_render_options* op, int64_t* out) {
    const gs3d_camera& cam = *camp;
    const gs3d_tiling& til = *tp;
    const gs3d_render_options& opt = *op;
    const int W = cam.width, H = cam.height;
    const int TW = til.tile_width, TH = til.tile_height;
    const int64_t T = (int64_t)til.nb_tiles_x * til.nb_tiles_y;
    std::vector<int64_t> nb(T, 0), nc(T, 0);
    parallel_for(0, T, [&](int64_t tl) {
        const int txi = (int)(tl % til.nb_tiles_x) + 1, tyi = (int)(tl / til.nb_tiles_x) + 1;
        const int tile = txi + (tyi - 1) * til.nb_tiles_x;
        const int start = tile == 1 ? 0 : tiles_end[tile - 2];
        const int end = tiles_end[tile - 1];
        const int u0 = (txi - 1) * TW, v0 = (tyi - 1) * TH;
        for (int pv = 1; pv <= TH; ++pv)
            for (int pu = 1; pu <= TW; ++pu) {
                if (!(pu + u0 <= W && pv + v0 <= H)) continue;
                const float cu = (float)pu - 0.5f, cv = (float)pv - 0.5f;
                const float uu = cu * cu, uv = cu * cv, vv = cv * cv;
                float Tr = 1.0f;
                for (int s = start + 1; s <= end; ++s) {
                    const float* r = f2d + 9 * (size_t)(sfgidx[s - 1] - 1);
                    const float du = r[0] - (float)u0, dv = r[1] - (float)v0;
                    const float ic11 = r[3], ic21 = r[4], ic22 = r[5];
                    const float ic11_du = ic11 * du, ic21_du = ic21 * du, ic22_dv = ic22 * dv;
                    const float p1 = -0.5f * ic11, p2 = -0.5f * ic22, p3 = -ic21;
                    const float p4 = ic11_du + ic21 * dv;
                    const float p5 = ic21_du + ic22_dv;
                    const float p6 = -0.5f * (ic11_du * du + ic22_dv * dv) - ic21_du * dv +
                                     o_logf(r[2]);
                    const float q = p1 * uu + p2 * vv + p3 * uv + p4 * cu + p5 * cv + p6;
                    ++nb[tl];
                    const float alpha = o_min(opt.max_alpha, o_expf(q));
                    if (alpha < opt.min_alpha) continue;
                    const float nextT = Tr * (1.0f - alpha);
                    if (nextT < opt.min_transmittance) break;
                    Tr = nextT;
                    ++nc[tl];
                }
            }
    });
    out[0] = out[1] = 0;
    for (int64_t t = 0; t < T; ++t) {
        out[0] += nb[t];
        out[1] += nc[t];
    }
}

void oracle_set_threads(int32_t n) { thread_count() = n < 1 ? 1 : n; }

// Exposed for the oracle self-tests.
float oracle_expf(float x) { return o_expf(x); }
float oracle_logf(float x) { return o_logf(x); }

}  // extern "C"
