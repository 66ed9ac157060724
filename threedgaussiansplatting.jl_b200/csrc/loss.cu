// loss.cu — the training loss of training_step! (training.jl:196-217):
//   L = (1 - w) mean|K - I| + w DSSIM(K, I),  dL/dK = +-(1 - w)/N (">" : ties get -)
//       + w dDSSIM/dK,  DSSIM = 1 - SSIM (docs/src/math.md:125), N = 3 h w.
// The reference takes DSSIM and its gradient from FastCUDASSIM v0.2.1, which is not vendored;
// this build uses SSIM as published by Wang et al. (2004): per channel, an 11-tap Gaussian
// window (sigma 1.5) applied separably with zero padding, C1 = 0.01^2, C2 = 0.03^2, averaged
// over all 3 h w values. Its gradient is analytic:
//   dS(q)/dK(p) = w(q-p) [dS/dmu_x(q) + 2 K(p) dS/dE[x^2](q) + I(p) dS/dE[xy](q)],
// i.e. three more zero-padded blurs of per-pixel partials (the window is symmetric).
// Two tiled kernels (forward maps + partials; backward blurs + gradient) and a fixed-order
// final reduction, so the loss value is deterministic.
#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace gs3d {
namespace {

constexpr int TV = 32;            // tile rows (v, contiguous in memory)
constexpr int TU = 16;            // tile columns (u)
constexpr int HALO = 5;
constexpr int RV = TV + 2 * HALO; // 42
constexpr int RU = TU + 2 * HALO; // 26
constexpr int LT = 256;           // threads

struct LossArgs {
    const float* K;   // 3 x h x w  (index 3 (v + h u) + c)
    const float* I;
    float* dmaps;     // 3 maps x 3 channels x (w h): dS/dmu, dS/dE[x^2], dS/dE[xy]
    float* grad;
    float* partial;   // per block: [ssim sum, l1 sum]
    float* loss;
    int W, H;
    float weight, l1w;
    float win[11];
    double invN;
};

__global__ void __launch_bounds__(LT) k_ssim_forward(const LossArgs a) {
    __shared__ float sx[RU][RV];
    __shared__ float sy[RU][RV];
    __shared__ float tmp[5][RU][TV];
    __shared__ float red[LT / 32];
    const int u0 = blockIdx.x * TU, v0 = blockIdx.y * TV;
    const int t = threadIdx.x;
    float ssim_acc = 0.0f;
    const size_t plane = (size_t)a.W * a.H;
    for (int c = 0; c < 3; ++c) {
        __syncthreads();
        for (int i = t; i < RU * RV; i += LT) {
            const int uu = i / RV, vv = i % RV;
            const int u = u0 + uu - HALO, v = v0 + vv - HALO;
            float x = 0.0f, y = 0.0f;
            if (u >= 0 && u < a.W && v >= 0 && v < a.H) {
                const size_t p = 3 * ((size_t)v + (size_t)a.H * u) + c;
                x = a.K[p];
                y = a.I[p];
            }
            sx[uu][vv] = x;
            sy[uu][vv] = y;
        }
        __syncthreads();
        for (int i = t; i < RU * TV; i += LT) {  // blur along v
            const int uu = i / TV, v = i % TV;
            float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f, m4 = 0.f;
#pragma unroll
            for (int k = 0; k < 11; ++k) {
                const float x = sx[uu][v + k], y = sy[uu][v + k], wk = a.win[k];
                m0 += wk * x;
                m1 += wk * y;
                m2 += wk * (x * x);
                m3 += wk * (y * y);
                m4 += wk * (x * y);
            }
            tmp[0][uu][v] = m0; tmp[1][uu][v] = m1; tmp[2][uu][v] = m2;
            tmp[3][uu][v] = m3; tmp[4][uu][v] = m4;
        }
        __syncthreads();
        for (int i = t; i < TU * TV; i += LT) {  // blur along u, SSIM and partials
            const int uu = i / TV, v = i % TV;
            const int u = u0 + uu, vg = v0 + v;
            if (u >= a.W || vg >= a.H) continue;
            float ux = 0.f, uy = 0.f, exx = 0.f, eyy = 0.f, exy = 0.f;
#pragma unroll
            for (int k = 0; k < 11; ++k) {
                const float wk = a.win[k];
                ux += wk * tmp[0][uu + k][v];
                uy += wk * tmp[1][uu + k][v];
                exx += wk * tmp[2][uu + k][v];
                eyy += wk * tmp[3][uu + k][v];
                exy += wk * tmp[4][uu + k][v];
            }
            const float C1 = 0.0001f, C2 = 0.0009f;
            const float vx = exx - ux * ux, vy = eyy - uy * uy, vxy = exy - ux * uy;
            const float A1 = 2.0f * ux * uy + C1, A2 = 2.0f * vxy + C2;
            const float B1 = ux * ux + uy * uy + C1, B2 = vx + vy + C2;
            const float iB = 1.0f / (B1 * B2);
            const float S = A1 * A2 * iB;
            ssim_acc += S;
            const size_t pp = (size_t)vg + (size_t)a.H * u;
            a.dmaps[(0 * 3 + c) * plane + pp] = 2.0f * uy * (A2 - A1) * iB - 2.0f * ux * S * (1.0f / B1 - 1.0f / B2);
            a.dmaps[(1 * 3 + c) * plane + pp] = -S / B2;
            a.dmaps[(2 * 3 + c) * plane + pp] = 2.0f * A1 * iB;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ssim_acc += __shfl_xor_sync(0xffffffffu, ssim_acc, o);
    if ((t & 31) == 0) red[t >> 5] = ssim_acc;
    __syncthreads();
    if (t == 0) {
        float s = 0.0f;
        for (int w = 0; w < LT / 32; ++w) s += red[w];
        a.partial[2 * (blockIdx.y * gridDim.x + blockIdx.x)] = s;
    }
}

__global__ void __launch_bounds__(LT) k_ssim_backward(const LossArgs a) {
    __shared__ float sd[3][RU][RV];
    __shared__ float tmp[3][RU][TV];
    __shared__ float red[LT / 32];
    const int u0 = blockIdx.x * TU, v0 = blockIdx.y * TV;
    const int t = threadIdx.x;
    const size_t plane = (size_t)a.W * a.H;
    float l1_acc = 0.0f;
    for (int c = 0; c < 3; ++c) {
        __syncthreads();
        for (int i = t; i < RU * RV; i += LT) {
            const int uu = i / RV, vv = i % RV;
            const int u = u0 + uu - HALO, v = v0 + vv - HALO;
            const bool in = u >= 0 && u < a.W && v >= 0 && v < a.H;
            const size_t pp = (size_t)v + (size_t)a.H * u;
#pragma unroll
            for (int m = 0; m < 3; ++m) sd[m][uu][vv] = in ? a.dmaps[(m * 3 + c) * plane + pp] : 0.0f;
        }
        __syncthreads();
        for (int i = t; i < RU * TV; i += LT) {
            const int uu = i / TV, v = i % TV;
            float m0 = 0.f, m1 = 0.f, m2 = 0.f;
#pragma unroll
            for (int k = 0; k < 11; ++k) {
                const float wk = a.win[k];
                m0 += wk * sd[0][uu][v + k];
                m1 += wk * sd[1][uu][v + k];
                m2 += wk * sd[2][uu][v + k];
            }
            tmp[0][uu][v] = m0; tmp[1][uu][v] = m1; tmp[2][uu][v] = m2;
        }
        __syncthreads();
        for (int i = t; i < TU * TV; i += LT) {
            const int uu = i / TV, v = i % TV;
            const int u = u0 + uu, vg = v0 + v;
            if (u >= a.W || vg >= a.H) continue;
            float b0 = 0.f, b1 = 0.f, b2 = 0.f;
#pragma unroll
            for (int k = 0; k < 11; ++k) {
                const float wk = a.win[k];
                b0 += wk * tmp[0][uu + k][v];
                b1 += wk * tmp[1][uu + k][v];
                b2 += wk * tmp[2][uu + k][v];
            }
            const size_t p = 3 * ((size_t)vg + (size_t)a.H * u) + c;
            const float x = a.K[p], y = a.I[p];
            const float dS = b0 + 2.0f * x * b1 + y * b2;
            const float gd = -dS * (float)a.invN;
            const float gl = x > y ? a.l1w : -a.l1w;
            a.grad[p] = gl + a.weight * gd;
            l1_acc += fabsf(x - y);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l1_acc += __shfl_xor_sync(0xffffffffu, l1_acc, o);
    if ((t & 31) == 0) red[t >> 5] = l1_acc;
    __syncthreads();
    if (t == 0) {
        float s = 0.0f;
        for (int w = 0; w < LT / 32; ++w) s += red[w];
        a.partial[2 * (blockIdx.y * gridDim.x + blockIdx.x) + 1] = s;
    }
}

__global__ void __launch_bounds__(256) k_loss_final(const LossArgs a, int nblocks) {
    __shared__ double rs[256], rl[256];
    double s = 0.0, l = 0.0;
    for (int i = threadIdx.x; i < nblocks; i += 256) {
        s += (double)a.partial[2 * i];
        l += (double)a.partial[2 * i + 1];
    }
    rs[threadIdx.x] = s;
    rl[threadIdx.x] = l;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
        if (threadIdx.x < o) {
            rs[threadIdx.x] += rs[threadIdx.x + o];
            rl[threadIdx.x] += rl[threadIdx.x + o];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const double l1 = rl[0] * a.invN;
        const double dssim = 1.0 - rs[0] * a.invN;
        a.loss[0] = (float)((1.0 - (double)a.weight) * l1 + (double)a.weight * dssim);
        a.loss[1] = (float)l1;
        a.loss[2] = (float)dssim;
    }
}

size_t loss_ws(int W, int H, int* nblocks) {
    const int bx = (W + TU - 1) / TU, by = (H + TV - 1) / TV;
    if (nblocks) *nblocks = bx * by;
    return align256((size_t)9 * W * H * sizeof(float)) + align256((size_t)2 * bx * by * sizeof(float));
}

}  // namespace
}  // namespace gs3d

using namespace gs3d;

extern "C" {

GS3D_API int gs3d_loss_workspace_size(int32_t width, int32_t height, size_t* bytes) {
    if (!bytes || width <= 0 || height <= 0) return invalid("bad loss workspace query");
    *bytes = loss_ws(width, height, nullptr);
    return GS3D_OK;
}

GS3D_API int gs3d_loss_l1_dssim(const float* rendered, const float* target, int32_t width,
                                int32_t height, float dssim_weight, float* loss_device,
                                float* rgb_image_grad, void* workspace, size_t workspace_bytes,
                                gs3d_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (!rendered || !target || !loss_device || !rgb_image_grad || width <= 0 || height <= 0)
        return invalid("bad loss arguments");
    int nblocks = 0;
    const size_t need = loss_ws(width, height, &nblocks);
    if (!workspace || workspace_bytes < need)
        return set_error("loss workspace %zu < %zu", workspace_bytes, need), GS3D_ERR_WORKSPACE;
    LossArgs a;
    a.K = rendered;
    a.I = target;
    a.dmaps = static_cast<float*>(workspace);
    a.partial = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) +
                                         align256((size_t)9 * width * height * sizeof(float)));
    a.grad = rgb_image_grad;
    a.loss = loss_device;
    a.W = width;
    a.H = height;
    a.weight = dssim_weight;
    const double N = 3.0 * (double)width * (double)height;
    a.invN = 1.0 / N;
    a.l1w = (1.0f - dssim_weight) / (float)(3 * (int64_t)width * height);
    {  // Gaussian window, sigma 1.5, normalised in double
        double g[11], s = 0.0;
        for (int i = 0; i < 11; ++i) { g[i] = std::exp(-((i - 5) * (i - 5)) / (2.0 * 1.5 * 1.5)); s += g[i]; }
        for (int i = 0; i < 11; ++i) a.win[i] = (float)(g[i] / s);
    }
    const dim3 grid((width + TU - 1) / TU, (height + TV - 1) / TV);
    ProfScope prof("loss", stream);
    k_ssim_forward<<<grid, LT, 0, stream>>>(a);
    GS3D_LAUNCHED("k_ssim_forward");
    k_ssim_backward<<<grid, LT, 0, stream>>>(a);
    GS3D_LAUNCHED("k_ssim_backward");
    k_loss_final<<<1, 256, 0, stream>>>(a, nblocks);
    GS3D_LAUNCHED("k_loss_final");
    return GS3D_OK;
}

}  // extern "C"
