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
//
// Both kernels stage a 16 (u) x 32 (v) tile with its 5-pixel halo in shared memory (all three
// channels at once, read as the contiguous runs of the interleaved images) and blur with
// sliding windows held in registers: a thread makes 4 consecutive outputs of the vertical pass
// from 14 staged inputs, and 2 consecutive outputs of the horizontal pass from 12, every tap a
// fused multiply-add.
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
constexpr int RVP = RV + 1;       // padded staged row: the warp's 4 columns x 8 runs hit distinct banks
constexpr int TVP = TV + 1;       // padded row of the vertical pass's output
constexpr int VR = 4;             // vertical-pass outputs per thread
constexpr int UR = 2;             // horizontal-pass outputs per thread
static_assert(RU * (TV / VR) <= LT && TV * (TU / UR) == LT, "pass work must fit one round");

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

// Stage the (RU x RV) halo region of the interleaved images K and I, all three channels, into
// sx / sy [c][uu][vv], zero outside the image. Every load of a thread is issued before its
// first shared-memory store, so each thread keeps 2 NST loads in flight.
constexpr int NST = (RU * 3 * RV + LT - 1) / LT;

__device__ __forceinline__ void stage_rgb2(const float* __restrict__ K, const float* __restrict__ I,
                                           float (*sx)[RU][RVP], float (*sy)[RU][RVP], int u0,
                                           int v0, int W, int H) {
    float xk[NST], yk[NST];
#pragma unroll
    for (int k = 0; k < NST; ++k) {
        const int i = threadIdx.x + k * LT;
        const int uu = i / (3 * RV);
        const int r = i - uu * (3 * RV);
        const int vv = r / 3, c = r - 3 * vv;
        const int u = u0 + uu - HALO, v = v0 + vv - HALO;
        const bool in = i < RU * 3 * RV && u >= 0 && u < W && v >= 0 && v < H;
        const size_t p = in ? 3 * ((size_t)v + (size_t)H * u) + c : 0;
        xk[k] = in ? __ldg(K + p) : 0.0f;
        yk[k] = in ? __ldg(I + p) : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < NST; ++k) {
        const int i = threadIdx.x + k * LT;
        if (i >= RU * 3 * RV) continue;
        const int uu = i / (3 * RV);
        const int r = i - uu * (3 * RV);
        const int vv = r / 3, c = r - 3 * vv;
        sx[c][uu][vv] = xk[k];
        sy[c][uu][vv] = yk[k];
    }
}

#ifndef GS3D_SSIM_MINB
#define GS3D_SSIM_MINB 4
#endif

__global__ void __launch_bounds__(LT, GS3D_SSIM_MINB) k_ssim_forward(const LossArgs a) {
    __shared__ float sx[3][RU][RVP];
    __shared__ float sy[3][RU][RVP];
    __shared__ float tmp[5][RU][TVP];
    __shared__ float red[LT / 32];
    const int u0 = blockIdx.x * TU, v0 = blockIdx.y * TV;
    const int t = threadIdx.x;
    const size_t plane = (size_t)a.W * a.H;
    stage_rgb2(a.K, a.I, sx, sy, u0, v0, a.W, a.H);
    float ssim_acc = 0.0f;
    for (int c = 0; c < 3; ++c) {
        __syncthreads();  // staging done / previous channel's tmp consumed
        if (t < RU * (TV / VR)) {  // vertical pass: column uu, rows vo .. vo + VR - 1
            const int uu = t / (TV / VR), vo = (t % (TV / VR)) * VR;
            float acc[5][VR];
#pragma unroll
            for (int m = 0; m < 5; ++m)
#pragma unroll
                for (int o = 0; o < VR; ++o) acc[m][o] = 0.0f;
#pragma unroll
            for (int j = 0; j < VR + 10; ++j) {
                const float x = sx[c][uu][vo + j], y = sy[c][uu][vo + j];
                const float xx = x * x, yy = y * y, xy = x * y;
#pragma unroll
                for (int o = 0; o < VR; ++o) {
                    const int k = j - o;
                    if (k < 0 || k > 10) continue;
                    const float wk = a.win[k];
                    acc[0][o] = fmaf(wk, x, acc[0][o]);
                    acc[1][o] = fmaf(wk, y, acc[1][o]);
                    acc[2][o] = fmaf(wk, xx, acc[2][o]);
                    acc[3][o] = fmaf(wk, yy, acc[3][o]);
                    acc[4][o] = fmaf(wk, xy, acc[4][o]);
                }
            }
#pragma unroll
            for (int m = 0; m < 5; ++m)
#pragma unroll
                for (int o = 0; o < VR; ++o) tmp[m][uu][vo + o] = acc[m][o];
        }
        __syncthreads();
        {  // horizontal pass: row v, columns uo .. uo + UR - 1; SSIM and its partials
            const int v = t % TV, uo = (t / TV) * UR;
            float acc[5][UR];
#pragma unroll
            for (int m = 0; m < 5; ++m)
#pragma unroll
                for (int o = 0; o < UR; ++o) acc[m][o] = 0.0f;
#pragma unroll
            for (int j = 0; j < UR + 10; ++j) {
                float q[5];
#pragma unroll
                for (int m = 0; m < 5; ++m) q[m] = tmp[m][uo + j][v];
#pragma unroll
                for (int o = 0; o < UR; ++o) {
                    const int k = j - o;
                    if (k < 0 || k > 10) continue;
                    const float wk = a.win[k];
#pragma unroll
                    for (int m = 0; m < 5; ++m) acc[m][o] = fmaf(wk, q[m], acc[m][o]);
                }
            }
            const int vg = v0 + v;
#pragma unroll
            for (int o = 0; o < UR; ++o) {
                const int u = u0 + uo + o;
                if (u >= a.W || vg >= a.H) continue;
                const float ux = acc[0][o], uy = acc[1][o];
                const float C1 = 0.0001f, C2 = 0.0009f;
                const float vx = fmaf(-ux, ux, acc[2][o]), vy = fmaf(-uy, uy, acc[3][o]);
                const float vxy = fmaf(-ux, uy, acc[4][o]);
                const float A1 = fmaf(2.0f * ux, uy, C1), A2 = fmaf(2.0f, vxy, C2);
                const float B1 = fmaf(ux, ux, fmaf(uy, uy, C1)), B2 = vx + vy + C2;
                const float iB = 1.0f / (B1 * B2);
                const float S = A1 * A2 * iB;
                ssim_acc += S;
                // dS/dmu_x = 2 uy (A2 - A1) / (B1 B2) - 2 ux S (1/B1 - 1/B2),
                // dS/dE[x^2] = -S / B2, dS/dE[xy] = 2 A1 / (B1 B2)
                const size_t pp = (size_t)vg + (size_t)a.H * u;
                a.dmaps[(0 * 3 + c) * plane + pp] =
                    2.0f * iB * fmaf(uy, A2 - A1, -ux * S * (B2 - B1));
                a.dmaps[(1 * 3 + c) * plane + pp] = -S * B1 * iB;
                a.dmaps[(2 * 3 + c) * plane + pp] = 2.0f * A1 * iB;
            }
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

__global__ void __launch_bounds__(LT, GS3D_SSIM_MINB) k_ssim_backward(const LossArgs a) {
    __shared__ float sd[3][RU][RVP];
    __shared__ float tmp[3][RU][TVP];
    __shared__ float red[LT / 32];
    const int u0 = blockIdx.x * TU, v0 = blockIdx.y * TV;
    const int t = threadIdx.x;
    const size_t plane = (size_t)a.W * a.H;
    const int v = t % TV, uo = (t / TV) * UR;  // this thread's horizontal-pass outputs
    const int vg = v0 + v;
    float l1_acc = 0.0f;
    const float ginv = (float)a.invN;
    for (int c = 0; c < 3; ++c) {
        // K and I of this channel at the thread's output pixels, loaded ahead of the blurs
        float xs[UR], ys[UR];
#pragma unroll
        for (int o = 0; o < UR; ++o) {
            const int u = u0 + uo + o;
            const bool in = u < a.W && vg < a.H;
            const size_t p = in ? 3 * ((size_t)vg + (size_t)a.H * u) + c : 0;
            xs[o] = in ? __ldg(a.K + p) : 0.0f;
            ys[o] = in ? __ldg(a.I + p) : 0.0f;
        }
        __syncthreads();  // previous channel's sd / tmp consumed
        {  // the three partial maps of channel c, all loads of a thread in flight together
            float d[NST];
#pragma unroll
            for (int k = 0; k < NST; ++k) {
                const int i = t + k * LT;
                const int m = i / (RU * RV);
                const int r = i - m * (RU * RV);
                const int uu = r / RV, vv = r - RV * uu;
                const int u = u0 + uu - HALO, vs = v0 + vv - HALO;
                const bool in = i < 3 * RU * RV && u >= 0 && u < a.W && vs >= 0 && vs < a.H;
                d[k] = in ? __ldg(a.dmaps + (m * 3 + c) * plane + (size_t)vs + (size_t)a.H * u)
                          : 0.0f;
            }
#pragma unroll
            for (int k = 0; k < NST; ++k) {
                const int i = t + k * LT;
                if (i >= 3 * RU * RV) continue;
                const int m = i / (RU * RV);
                const int r = i - m * (RU * RV);
                const int uu = r / RV, vv = r - RV * uu;
                sd[m][uu][vv] = d[k];
            }
        }
        __syncthreads();
        if (t < RU * (TV / VR)) {  // vertical pass
            const int uu = t / (TV / VR), vo = (t % (TV / VR)) * VR;
            float acc[3][VR];
#pragma unroll
            for (int m = 0; m < 3; ++m)
#pragma unroll
                for (int o = 0; o < VR; ++o) acc[m][o] = 0.0f;
#pragma unroll
            for (int j = 0; j < VR + 10; ++j) {
                float q[3];
#pragma unroll
                for (int m = 0; m < 3; ++m) q[m] = sd[m][uu][vo + j];
#pragma unroll
                for (int o = 0; o < VR; ++o) {
                    const int k = j - o;
                    if (k < 0 || k > 10) continue;
                    const float wk = a.win[k];
#pragma unroll
                    for (int m = 0; m < 3; ++m) acc[m][o] = fmaf(wk, q[m], acc[m][o]);
                }
            }
#pragma unroll
            for (int m = 0; m < 3; ++m)
#pragma unroll
                for (int o = 0; o < VR; ++o) tmp[m][uu][vo + o] = acc[m][o];
        }
        __syncthreads();
        float acc[3][UR];
#pragma unroll
        for (int m = 0; m < 3; ++m)
#pragma unroll
            for (int o = 0; o < UR; ++o) acc[m][o] = 0.0f;
#pragma unroll
        for (int j = 0; j < UR + 10; ++j) {  // horizontal pass
            float q[3];
#pragma unroll
            for (int m = 0; m < 3; ++m) q[m] = tmp[m][uo + j][v];
#pragma unroll
            for (int o = 0; o < UR; ++o) {
                const int k = j - o;
                if (k < 0 || k > 10) continue;
                const float wk = a.win[k];
#pragma unroll
                for (int m = 0; m < 3; ++m) acc[m][o] = fmaf(wk, q[m], acc[m][o]);
            }
        }
        // dL/dK(p) of this channel: L1 part + weight * (-(b0 + 2 K(p) b1 + I(p) b2) / N)
#pragma unroll
        for (int o = 0; o < UR; ++o) {
            const int u = u0 + uo + o;
            if (u >= a.W || vg >= a.H) continue;
            const float x = xs[o], y = ys[o];
            const float dS = fmaf(2.0f * x, acc[1][o], fmaf(y, acc[2][o], acc[0][o]));
            const float gl = x > y ? a.l1w : -a.l1w;
            a.grad[3 * ((size_t)vg + (size_t)a.H * u) + c] = fmaf(a.weight, -dS * ginv, gl);
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
