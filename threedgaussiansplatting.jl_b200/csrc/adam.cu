// adam.cu — update!(opt, fgradients, Val(sh)) (optimizer.jl:964-1009) as ONE kernel.
//
// The reference launches five kernels (four component groups, then the SH coefficients:
// optimizer.jl:1084-1127, :1165-1248), each walking the F filtered Gaussians. Here one
// grid-stride kernel walks (filtered Gaussian, component) pairs, component-fastest, so a warp
// touches consecutive scalars of one or two Gaussians: the F-compact gradients stream
// contiguously and the scattered parameter / moment rows are read and written once.
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
};

__device__ __forceinline__ void adam_scalar(float* p, float g, float* m, float lr, const AdamArgs& a) {
    const float nm1 = a.b1 * m[0] + (1.0f - a.b1) * g;
    const float nm2 = a.b2 * m[1] + (1.0f - a.b2) * (g * g);
    const float h1 = nm1 / a.bc1;
    const float h2 = nm2 / a.bc2;
    m[0] = nm1;
    m[1] = nm2;
    *p = *p - lr * h1 / (sqrtf(h2) + a.eps);
}

__global__ void __launch_bounds__(256) k_adam(const AdamArgs a) {
    const int F = a.counts[0];
    const int nc = 11 + 3 * a.maxo;
    const int64_t total = (int64_t)F * nc;
    for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < total;
         it += (int64_t)gridDim.x * blockDim.x) {
        const int f = (int)(it / nc);
        const int c = (int)(it - (int64_t)f * nc);
        const int gidx = a.f2g[f];
        if (gidx <= 0) continue;
        const size_t gi = (size_t)gidx - 1;
        if (c < 3) {
            adam_scalar(a.mo + 4 * gi + c, a.g_mean[3 * (size_t)f + c], a.mm + 6 * gi + 2 * c, a.lr_means, a);
        } else if (c == 3) {
            adam_scalar(a.mo + 4 * gi + 3, a.g_op[f], a.om + 2 * gi, a.lr_op, a);
        } else if (c < 7) {
            const int k = c - 4;
            adam_scalar(a.sf + 3 * gi + k, a.g_scale[3 * (size_t)f + k], a.sm + 6 * gi + 2 * k, a.lr_scale, a);
        } else if (c < 11) {
            const int k = c - 7;
            adam_scalar(a.rf + 4 * gi + k, a.g_rot[4 * (size_t)f + k], a.rm + 8 * gi + 2 * k, a.lr_rot, a);
        } else {
            const int k = c - 11;
            const int ch = k / a.maxo, i = k - ch * a.maxo;
            adam_scalar(a.sh + gi * 3 * a.S + (size_t)(ch * a.S + i),
                        a.g_sh[(size_t)f * 3 * a.Sg + (size_t)(ch * a.Sg + i)],
                        a.shm + gi * 6 * a.Sm + 2 * (size_t)(ch * a.Sm + i),
                        i == 0 ? a.lr_dc : a.lr_rest, a);
        }
    }
}

// Multi-view data parallelism: the F-compact gradients of one view are scattered into a
// dense row per Gaussian, kDenseRow floats: mean(3) opacity(1) scale(3) rotation(4)
// SH(3 x 16, channel-major) touched(1). Rows are summed across ranks (NCCL all-reduce),
// then k_adam_dense steps every touched Gaussian with the summed gradient.
constexpr int kDenseRow = 60;
constexpr int kDenseTouched = 59;

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
        if (c == nc) { row[kDenseTouched] = 1.0f; continue; }
        float v;
        int col;
        if (c < 3) { v = a.g_mean[3 * (size_t)f + c]; col = c; }
        else if (c == 3) { v = a.g_op[f]; col = 3; }
        else if (c < 7) { v = a.g_scale[3 * (size_t)f + (c - 4)]; col = c; }
        else if (c < 11) { v = a.g_rot[4 * (size_t)f + (c - 7)]; col = c; }
        else {
            const int k = c - 11, ch = k / a.maxo, i = k - ch * a.maxo;
            v = a.g_sh[(size_t)f * 3 * a.Sg + (size_t)(ch * a.Sg + i)];
            col = 11 + ch * 16 + i;
        }
        row[col] = v;
    }
}

__global__ void __launch_bounds__(256) k_adam_dense(const AdamArgs a, const float* __restrict__ dense,
                                                    int n) {
    const int nc = 11 + 3 * a.maxo;
    const int64_t total = (int64_t)n * nc;
    for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < total;
         it += (int64_t)gridDim.x * blockDim.x) {
        const int g = (int)(it / nc);
        const int c = (int)(it - (int64_t)g * nc);
        const float* row = dense + (size_t)g * kDenseRow;
        if (!(row[kDenseTouched] > 0.0f)) continue;
        const size_t gi = (size_t)g;
        if (c < 3) {
            adam_scalar(a.mo + 4 * gi + c, row[c], a.mm + 6 * gi + 2 * c, a.lr_means, a);
        } else if (c == 3) {
            adam_scalar(a.mo + 4 * gi + 3, row[3], a.om + 2 * gi, a.lr_op, a);
        } else if (c < 7) {
            const int k = c - 4;
            adam_scalar(a.sf + 3 * gi + k, row[c], a.sm + 6 * gi + 2 * k, a.lr_scale, a);
        } else if (c < 11) {
            const int k = c - 7;
            adam_scalar(a.rf + 4 * gi + k, row[c], a.rm + 8 * gi + 2 * k, a.lr_rot, a);
        } else {
            const int k = c - 11;
            const int ch = k / a.maxo, i = k - ch * a.maxo;
            adam_scalar(a.sh + gi * 3 * a.S + (size_t)(ch * a.S + i), row[11 + ch * 16 + i],
                        a.shm + gi * 6 * a.Sm + 2 * (size_t)(ch * a.Sm + i),
                        i == 0 ? a.lr_dc : a.lr_rest, a);
        }
    }
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
    const int blocks = device_sm_count() * 8;
    ProfScope prof("adam", stream);
    k_adam<<<blocks, 256, 0, stream>>>(a);
    GS3D_LAUNCHED("k_adam");
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

extern "C" GS3D_API int gs3d_adam_step_dense(const gs3d_gaussians* g, const gs3d_adam_moments* m,
                                             const float* dense, const gs3d_adam_params* p,
                                             gs3d_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (!g || !m || !dense || !p) return invalid("NULL argument");
    AdamArgs a;
    GS3D_RETURN_IF(make_args(g, m, nullptr, nullptr, nullptr, p, a));
    ProfScope prof("adam_dense", stream);
    k_adam_dense<<<device_sm_count() * 8, 256, 0, stream>>>(a, dense, g->n);
    GS3D_LAUNCHED("k_adam_dense");
    return GS3D_OK;
}
