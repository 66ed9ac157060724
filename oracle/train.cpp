// train.cpp — TEST INFRASTRUCTURE ONLY: CPU oracle of gs3d's optimizer, loss and
// densification. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
// load it.
//
// Restates ThreeDGaussianSplatting.jl:
//   sparse Adam .............. optimizer.jl:941-953 (scalar), :964-1009, :1084-1127,
//                              :1165-1248 (SH: DC lr for coefficient 1, rest lr otherwise)
//   loss ..................... training.jl:196-217: L = (1-w) L1 + w DSSIM,
//                              dL/dK = +-(1-w)/N (">" so ties get -) + w dDSSIM/dK.
//                              DSSIM = 1 - SSIM (docs/src/math.md:125). SSIM itself lives in
//                              FastCUDASSIM v0.2.1, which is not vendored: this build uses
//                              Wang et al. 2004 (11-tap Gaussian window, sigma 1.5, zero
//                              padding, C1 = 0.01^2, C2 = 0.03^2, mean over 3 x h x w).
//                              PARITY UNPINNED for the SSIM term.
//   ADC statistics ........... training.jl:472-497
//   ADC masks / counts / scan  training.jl:325-397, :557-580
//   ADC apply ................ gaussians.jl:1526-1694, optimizer.jl:1304-1378,
//                              training.jl:514-541 (split means use this build's
//                              counter-based normal sampler, not CUDA.jl randn)
//   opacity reset ............ gaussians.jl:1093-1101, optimizer.jl:754-756
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

#include "../include/gs3d.h"
#include "oracle_math.h"

using namespace oracle;

namespace {

inline float adam_scalar(float param, float grad, float& m1, float& m2, float lr, float b1,
                         float b2, float eps, float bc1, float bc2) {
    const float nm1 = b1 * m1 + (1.0f - b1) * grad;
    const float nm2 = b2 * m2 + (1.0f - b2) * (grad * grad);
    const float h1 = nm1 / bc1;
    const float h2 = nm2 / bc2;
    m1 = nm1;
    m2 = nm2;
    return param - lr * h1 / (std::sqrt(h2) + eps);
}

// 11-tap Gaussian window, sigma 1.5, normalised in double then rounded to float.
void gauss_window(float w[11]) {
    double g[11], s = 0.0;
    for (int i = 0; i < 11; ++i) { g[i] = std::exp(-((i - 5) * (i - 5)) / (2.0 * 1.5 * 1.5)); s += g[i]; }
    for (int i = 0; i < 11; ++i) w[i] = (float)(g[i] / s);
}

// zero-padded separable 'same' blur of an h x w plane (v fastest: index v + h*u)
void blur(const std::vector<double>& in, std::vector<double>& out, int h, int W, const float w[11]) {
    std::vector<double> tmp((size_t)h * W, 0.0);
    for (int u = 0; u < W; ++u)
        for (int v = 0; v < h; ++v) {
            double s = 0.0;
            for (int k = -5; k <= 5; ++k) {
                const int vv = v + k;
                if (vv < 0 || vv >= h) continue;
                s += (double)w[k + 5] * in[(size_t)vv + (size_t)h * u];
            }
            tmp[(size_t)v + (size_t)h * u] = s;
        }
    for (int u = 0; u < W; ++u)
        for (int v = 0; v < h; ++v) {
            double s = 0.0;
            for (int k = -5; k <= 5; ++k) {
                const int uu = u + k;
                if (uu < 0 || uu >= W) continue;
                s += (double)w[k + 5] * tmp[(size_t)v + (size_t)h * uu];
            }
            out[(size_t)v + (size_t)h * u] = s;
        }
}

// counter-based uniform in (0,1) and normal (Marsaglia polar) keyed by (seed, key, i)
inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
inline float uniform_pm1(uint64_t seed, uint64_t key, uint32_t ctr) {
    const uint64_t r = splitmix64(seed ^ splitmix64(key * 0x100000001B3ull + ctr));
    // 24 random bits -> (-1, 1) exactly representable
    const int32_t b = (int32_t)(r >> 40);                // [0, 2^24)
    return ((float)b - 8388607.5f) * (1.0f / 8388608.0f);
}
// six standard normals for one split Gaussian
void split_normals(uint64_t seed, uint64_t key, float out[6]) {
    uint32_t ctr = 0;
    for (int k = 0; k < 6; k += 2) {
        float z0 = 0.0f, z1 = 0.0f;
        for (int it = 0; it < 64; ++it) {
            const float u = uniform_pm1(seed, key, ctr++);
            const float v = uniform_pm1(seed, key, ctr++);
            const float s = u * u + v * v;
            if (s >= 1.0f || s == 0.0f) continue;
            const float f = std::sqrt(-2.0f * o_logf(s) / s);
            z0 = u * f; z1 = v * f;
            break;
        }
        out[k] = z0; out[k + 1] = z1;
    }
}

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

// update!(opt, fgradients, Val(sh)) — all F filtered Gaussians; gidx <= 0 skipped.
// bc1 = 1 - beta1^t and bc2 = 1 - beta2^t with t = update_count + 1 (host-computed).
int oracle_adam(const gs3d_gaussians* gp, const gs3d_adam_moments* mp, const gs3d_fgradients* fp,
                const int32_t* fgidx_to_gidx, int32_t F, const gs3d_adam_params* ap, float bc1,
                float bc2) {
    const gs3d_gaussians& g = *gp;
    const gs3d_adam_moments& mo = *mp;
    const gs3d_fgradients& fg = *fp;
    const gs3d_adam_params& a = *ap;
    const int S_store = (g.sh_degree + 1) * (g.sh_degree + 1);
    const int S_grad = (fg.sh_degree + 1) * (fg.sh_degree + 1);
    const int S_mom = (mo.sh_degree + 1) * (mo.sh_degree + 1);
    const int MAXO = (a.sh_degree + 1) * (a.sh_degree + 1);
    for (int f = 0; f < F; ++f) {
        const int gidx = fgidx_to_gidx[f];
        if (gidx <= 0) continue;
        const size_t gi = (size_t)gidx - 1;
        float* mof = g.means_opacity_features + 4 * gi;
        for (int i = 0; i < 3; ++i) {
            float* m = mo.means_moments + 6 * gi + 2 * i;
            mof[i] = adam_scalar(mof[i], fg.mean3d_grads[3 * (size_t)f + i], m[0], m[1], a.lr_means,
                                 a.beta1, a.beta2, a.epsilon, bc1, bc2);
        }
        {
            float* m = mo.opacity_features_moments + 2 * gi;
            mof[3] = adam_scalar(mof[3], fg.opacity_feature_grads[f], m[0], m[1], a.lr_opacity_features,
                                 a.beta1, a.beta2, a.epsilon, bc1, bc2);
        }
        for (int i = 0; i < 3; ++i) {
            float* m = mo.scaling_features_moments + 6 * gi + 2 * i;
            float* p = g.scaling_features + 3 * gi + i;
            *p = adam_scalar(*p, fg.scaling_features_grads[3 * (size_t)f + i], m[0], m[1],
                             a.lr_scaling_features, a.beta1, a.beta2, a.epsilon, bc1, bc2);
        }
        for (int i = 0; i < 4; ++i) {
            float* m = mo.rotation_features_moments + 8 * gi + 2 * i;
            float* p = g.rotation_features + 4 * gi + i;
            *p = adam_scalar(*p, fg.rotation_features_grads[4 * (size_t)f + i], m[0], m[1],
                             a.lr_rotation_features, a.beta1, a.beta2, a.epsilon, bc1, bc2);
        }
        // SH: linear index into the (MAXO x 3) view of each array, as adam_sh_coeffs_update_kernel!
        // does when the options degree differs from the storage degree (views are contiguous
        // per Gaussian only when the degrees agree; we index [i, c] explicitly).
        for (int c = 0; c < 3; ++c)
            for (int i = 0; i < MAXO; ++i) {
                float* p = g.sh_coeffs + gi * 3 * S_store + (size_t)(i + c * S_store);
                const float gr = fg.sh_coeffs_grads[(size_t)f * 3 * S_grad + (size_t)(i + c * S_grad)];
                float* m = mo.sh_coeffs_moments + gi * 6 * S_mom + 2 * (size_t)(i + c * S_mom);
                *p = adam_scalar(*p, gr, m[0], m[1], i == 0 ? a.lr_sh_dc : a.lr_sh_rest, a.beta1,
                                 a.beta2, a.epsilon, bc1, bc2);
            }
    }
    return 0;
}

// L1 + weight * DSSIM and its gradient; images are 3 x h x w (c fastest, then v, then u).
// out_loss[0] = loss, [1] = L1, [2] = DSSIM (double precision accumulation).
int oracle_loss(const float* K, const float* I, int32_t W, int32_t h, float weight,
                double* out_loss, float* grad) {
    const size_t np = (size_t)W * h;
    const double N = 3.0 * (double)np;
    float win[11];
    gauss_window(win);
    const double C1 = 0.01 * 0.01, C2 = 0.03 * 0.03;
    double l1 = 0.0;
    for (size_t i = 0; i < 3 * np; ++i) l1 += std::fabs((double)K[i] - (double)I[i]);
    l1 /= N;
    const float l1w = (1.0f - weight) / (float)(3 * np);
    double ssim_sum = 0.0;
    std::vector<double> x(np), y(np), xx(np), yy(np), xy(np);
    std::vector<double> mx(np), my(np), exx(np), eyy(np), exy(np), d1(np), d2(np), d3(np), b1(np),
        b2(np), b3(np);
    for (int c = 0; c < 3; ++c) {
        for (size_t p = 0; p < np; ++p) {
            x[p] = K[3 * p + c]; y[p] = I[3 * p + c];
            xx[p] = x[p] * x[p]; yy[p] = y[p] * y[p]; xy[p] = x[p] * y[p];
        }
        blur(x, mx, h, W, win); blur(y, my, h, W, win);
        blur(xx, exx, h, W, win); blur(yy, eyy, h, W, win); blur(xy, exy, h, W, win);
        for (size_t p = 0; p < np; ++p) {
            const double ux = mx[p], uy = my[p];
            const double sx = exx[p] - ux * ux, sy = eyy[p] - uy * uy, sxy = exy[p] - ux * uy;
            const double A1 = 2.0 * ux * uy + C1, A2 = 2.0 * sxy + C2;
            const double B1 = ux * ux + uy * uy + C1, B2 = sx + sy + C2;
            const double S = (A1 * A2) / (B1 * B2);
            ssim_sum += S;
            d1[p] = (2.0 * uy * A2 + A1 * (-2.0 * uy)) / (B1 * B2) - S * (2.0 * ux / B1 - 2.0 * ux / B2);
            d2[p] = -S / B2;
            d3[p] = 2.0 * A1 / (B1 * B2);
        }
        blur(d1, b1, h, W, win); blur(d2, b2, h, W, win); blur(d3, b3, h, W, win);
        for (size_t p = 0; p < np; ++p) {
            const double dS = b1[p] + 2.0 * x[p] * b2[p] + y[p] * b3[p];
            const double g_dssim = -dS / N;
            const float gl1 = K[3 * p + c] > I[3 * p + c] ? l1w : -l1w;
            grad[3 * p + c] = (float)((double)gl1 + (double)weight * g_dssim);
        }
    }
    const double dssim = 1.0 - ssim_sum / N;
    out_loss[1] = l1;
    out_loss[2] = dssim;
    out_loss[0] = (1.0 - weight) * l1 + weight * dssim;
    return 0;
}

// update_adc_stats_kernel! (training.jl:472-497)
int oracle_adc_stats(float* acc, int32_t* cnt, const float* mean2d_g, const int32_t* fgidx_to_gidx,
                     int32_t F, int32_t W, int32_t h) {
    const double sqw4 = (double)W * W / 4.0, sqh4 = (double)h * h / 4.0;
    for (int f = 0; f < F; ++f) {
        const int gidx = fgidx_to_gidx[f];
        const float gx = mean2d_g[2 * f], gy = mean2d_g[2 * f + 1];
        if (gx != 0.0f || gy != 0.0f) {
            const double nn = std::sqrt((double)(gx * gx) * sqw4 + (double)(gy * gy) * sqh4);
            acc[gidx - 1] = (float)((double)acc[gidx - 1] + nn);
            cnt[gidx - 1] += 1;
        }
    }
    return 0;
}

// Masks, counts, inclusive scan and ngidx_to_gidx (training.jl:325-397, :557-580).
// Returns n'.
int32_t oracle_adc_plan(const gs3d_gaussians* gp, const float* acc, const int32_t* cnt,
                        const gs3d_adc_params* pp, float* max_sf, uint8_t* prune, uint8_t* densify,
                        uint8_t* clone, uint8_t* counts, int32_t* counts_cs, int32_t* ngidx_to_gidx) {
    const gs3d_gaussians& g = *gp;
    const gs3d_adc_params& p = *pp;
    const float prune_thr = o_logit(p.pruning_min_opacity);
    const float scale_thr = o_logf(p.pruning_3d_max_scale);
    const float size_thr = o_logf(p.densification_size_threshold);
    int32_t cs = 0;
    for (int i = 0; i < g.n; ++i) {
        const float avg = cnt[i] >= 1 ? acc[i] / (float)cnt[i] : 0.0f;
        const float* sf = g.scaling_features + 3 * (size_t)i;
        const float ms = std::max(std::max(sf[0], sf[1]), sf[2]);
        max_sf[i] = ms;
        const float opf = g.means_opacity_features[4 * (size_t)i + 3];
        bool pr = opf < prune_thr;
        if (p.use_max_scale_pruning) pr = pr || ms > scale_thr;
        const bool de = !pr && avg >= p.densification_mean2d_grad_norm_threshold_ndc;
        const bool cl = de && ms <= size_thr;
        prune[i] = pr; densify[i] = de; clone[i] = cl;
        counts[i] = (uint8_t)((pr ? 0 : 1) + (de ? 1 : 0));
        cs += counts[i];
        counts_cs[i] = cs;
        if (!pr) {
            if (de) { ngidx_to_gidx[cs - 2] = i + 1; ngidx_to_gidx[cs - 1] = i + 1; }
            else ngidx_to_gidx[cs - 1] = i + 1;
        }
    }
    return cs;
}

// Apply the plan: new Gaussians, new moments (zero-initialised by the caller is NOT
// assumed: every new entry is written) and retargeted fgidx_to_gidx.
int oracle_adc_apply(const gs3d_gaussians* og, const gs3d_adam_moments* om, const gs3d_gaussians* ng,
                     const gs3d_adam_moments* nm, const uint8_t* prune, const uint8_t* densify,
                     const uint8_t* clone, const int32_t* counts_cs, int32_t* fgidx_to_gidx, int32_t F,
                     float log_split, uint64_t seed) {
    const int S = (og->sh_degree + 1) * (og->sh_degree + 1);
    const int Sm = (om->sh_degree + 1) * (om->sh_degree + 1);
    auto copy_moments = [&](size_t from, size_t to, bool zero) {
        for (int k = 0; k < 6; ++k) nm->means_moments[6 * to + k] = zero ? 0.0f : om->means_moments[6 * from + k];
        for (int k = 0; k < 2; ++k) nm->opacity_features_moments[2 * to + k] = zero ? 0.0f : om->opacity_features_moments[2 * from + k];
        for (int k = 0; k < 6; ++k) nm->scaling_features_moments[6 * to + k] = zero ? 0.0f : om->scaling_features_moments[6 * from + k];
        for (int k = 0; k < 8; ++k) nm->rotation_features_moments[8 * to + k] = zero ? 0.0f : om->rotation_features_moments[8 * from + k];
        for (int k = 0; k < 6 * Sm; ++k) nm->sh_coeffs_moments[6 * Sm * to + k] = zero ? 0.0f : om->sh_coeffs_moments[6 * Sm * from + k];
    };
    auto copy_rest = [&](size_t from, size_t to) {
        for (int k = 0; k < 4; ++k) ng->rotation_features[4 * to + k] = og->rotation_features[4 * from + k];
        for (int k = 0; k < 3 * S; ++k) ng->sh_coeffs[3 * S * to + k] = og->sh_coeffs[3 * S * from + k];
    };
    for (int i = 0; i < og->n; ++i) {
        if (prune[i]) continue;
        const size_t last = (size_t)counts_cs[i] - 1;
        const float* mo = og->means_opacity_features + 4 * (size_t)i;
        const float* sf = og->scaling_features + 3 * (size_t)i;
        if (densify[i]) {
            const size_t first = last - 1;
            if (clone[i]) {
                for (int k = 0; k < 4; ++k) { ng->means_opacity_features[4 * first + k] = mo[k]; ng->means_opacity_features[4 * last + k] = mo[k]; }
                for (int k = 0; k < 3; ++k) { ng->scaling_features[3 * first + k] = sf[k]; ng->scaling_features[3 * last + k] = sf[k]; }
                copy_moments(i, first, false);
                copy_moments(i, last, true);
            } else {
                float R[3][3];
                quat_to_rot(og->rotation_features + 4 * (size_t)i, R);
                const float s[3] = {o_expf(sf[0]), o_expf(sf[1]), o_expf(sf[2])};
                float nrm[6];
                split_normals(seed, (uint64_t)i + 1, nrm);  // nrm[j + 3k] = N[j][k]
                for (int k = 0; k < 2; ++k) {
                    const size_t to = k == 0 ? first : last;
                    for (int r = 0; r < 3; ++r) {
                        const float sh = R[r][0] * (nrm[0 + 3 * k] * s[0]) + R[r][1] * (nrm[1 + 3 * k] * s[1]) +
                                         R[r][2] * (nrm[2 + 3 * k] * s[2]);
                        ng->means_opacity_features[4 * to + r] = mo[r] + sh;
                    }
                    ng->means_opacity_features[4 * to + 3] = mo[3];
                    for (int r = 0; r < 3; ++r) ng->scaling_features[3 * to + r] = sf[r] + log_split;
                }
                copy_moments(i, first, true);
                copy_moments(i, last, true);
            }
            copy_rest(i, first);
            copy_rest(i, last);
        } else {
            for (int k = 0; k < 4; ++k) ng->means_opacity_features[4 * last + k] = mo[k];
            for (int k = 0; k < 3; ++k) ng->scaling_features[3 * last + k] = sf[k];
            copy_moments(i, last, false);
            copy_rest(i, last);
        }
    }
    for (int f = 0; f < F; ++f) {
        const int gidx = fgidx_to_gidx[f];
        int32_t ngidx = 0;
        const int i = gidx - 1;
        if (!prune[i]) {
            if (densify[i]) { if (clone[i]) ngidx = counts_cs[i] - 1; }
            else ngidx = counts_cs[i];
        }
        fgidx_to_gidx[f] = ngidx;
    }
    return 0;
}

int oracle_opacity_reset(const gs3d_gaussians* g, const gs3d_adam_moments* m, float max_opacity) {
    const float thr = o_logit(max_opacity);
    for (int i = 0; i < g->n; ++i) {
        float* p = g->means_opacity_features + 4 * (size_t)i + 3;
        *p = std::min(*p, thr);
        m->opacity_features_moments[2 * (size_t)i] = 0.0f;
        m->opacity_features_moments[2 * (size_t)i + 1] = 0.0f;
    }
    return 0;
}

// exposed for tests: the split sampler's normals
void oracle_split_normals(uint64_t seed, uint64_t key, float* out6) { split_normals(seed, key, out6); }

}  // extern "C"
