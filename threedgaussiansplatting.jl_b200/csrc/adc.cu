// adc.cu — adaptive density control of training.jl:313-580 / gaussians.jl:1526-1694 /
// optimizer.jl:1304-1378.
//   gs3d_adc_stats          update_adc_stats_kernel! (training.jl:472-497)
//   gs3d_densify_prune_plan masks (training.jl:325-364), counts in {0,1,2}, inclusive scan,
//                           fill_ngidx_to_gidx_kernel! (training.jl:557-580); one host read
//                           of n' (the reference's @allowscalar read, training.jl:388)
//   gs3d_densify_apply      compaction/expansion of all Gaussian arrays and Adam moments
//                           (carry: 1 copy; clone: 2 copies, moments to the first only;
//                           split: 2 resampled means, scale features + log(split factor),
//                           zero moments; prune: nothing) and the retarget of this step's
//                           fgidx_to_gidx (training.jl:514-541)
//   gs3d_opacity_reset      reset_opacities! + zero_opacity_features_adam_moments!
// Split means are mean + R (s .* n) with n standard normal from a counter-based generator
// keyed by (seed, old index): splitmix64 hashing to 24-bit uniforms in (-1, 1) and the
// Marsaglia polar method. Replicas on different GPUs therefore split identically; CUDA.jl's
// device randn (gaussians.jl:1617) is not reproducible anyway.
#include "common.cuh"
#include "internal.h"

namespace gs3d {
namespace {

__global__ void __launch_bounds__(256) k_adc_stats(float* __restrict__ acc, int32_t* __restrict__ cnt,
                                                   const float* __restrict__ m2g,
                                                   const int32_t* __restrict__ f2g,
                                                   const int32_t* __restrict__ counts, double sqw4,
                                                   double sqh4) {
    const int F = counts[0];
    for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < F; f += gridDim.x * blockDim.x) {
        const int gidx = f2g[f];
        const float gx = m2g[2 * (size_t)f], gy = m2g[2 * (size_t)f + 1];
        if (gidx > 0 && (gx != 0.0f || gy != 0.0f)) {
            const double nn = sqrt((double)(gx * gx) * sqw4 + (double)(gy * gy) * sqh4);
            acc[gidx - 1] = (float)((double)acc[gidx - 1] + nn);
            cnt[gidx - 1] += 1;
        }
    }
}

struct PlanArgs {
    const float* acc;
    const int32_t* cnt;
    const float* sf;   // 3 x n
    const float* mo;   // 4 x n
    float* max_sf;
    uint8_t* prune;
    uint8_t* densify;
    uint8_t* clone;
    uint8_t* counts;
    int32_t* counts_cs;
    int32_t* ngidx_to_gidx;
    int32_t* sums;
    int n;
    float grad_thr, prune_thr, scale_thr, size_thr;
    int use_scale;
};

__device__ __forceinline__ int plan_one(const PlanArgs& a, int i) {
    const float c = (float)a.cnt[i];
    const float avg = a.cnt[i] >= 1 ? a.acc[i] / c : 0.0f;
    const float s0 = a.sf[3 * (size_t)i], s1 = a.sf[3 * (size_t)i + 1], s2 = a.sf[3 * (size_t)i + 2];
    const float ms = fmaxf(fmaxf(s0, s1), s2);
    const float opf = a.mo[4 * (size_t)i + 3];
    bool pr = opf < a.prune_thr;
    if (a.use_scale) pr = pr || ms > a.scale_thr;
    const bool de = !pr && avg >= a.grad_thr;
    const bool cl = de && ms <= a.size_thr;
    a.max_sf[i] = ms;
    a.prune[i] = pr;
    a.densify[i] = de;
    a.clone[i] = cl;
    const int k = (pr ? 0 : 1) + (de ? 1 : 0);
    a.counts[i] = (uint8_t)k;
    return k;
}

__global__ void __launch_bounds__(kChunkThreads) k_plan_up(const PlanArgs a) {
    __shared__ int sm[33];
    const int64_t base = (int64_t)blockIdx.x * kChunk;
    int s = 0;
    for (int k = 0; k < kChunkItems; ++k) {
        const int64_t i = base + k * kChunkThreads + threadIdx.x;
        if (i < a.n) s += plan_one(a, (int)i);
    }
    int tot;
    block_exclusive_scan(s, sm, &tot);
    if (threadIdx.x == 0) a.sums[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(kChunkThreads) k_plan_down(const PlanArgs a) {
    __shared__ int sm[33];
    const int64_t base = (int64_t)blockIdx.x * kChunk;
    const int64_t mine = base + (int64_t)threadIdx.x * kChunkItems;
    int v[kChunkItems];
    int s = 0;
#pragma unroll
    for (int k = 0; k < kChunkItems; ++k) {
        const int64_t i = mine + k;
        v[k] = i < a.n ? (int)a.counts[i] : 0;
        s += v[k];
    }
    int tot;
    int run = block_exclusive_scan(s, sm, &tot) + a.sums[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kChunkItems; ++k) {
        const int64_t i = mine + k;
        if (i >= a.n) break;
        run += v[k];
        a.counts_cs[i] = run;
        if (v[k] == 2) {
            a.ngidx_to_gidx[run - 2] = (int32_t)(i + 1);
            a.ngidx_to_gidx[run - 1] = (int32_t)(i + 1);
        } else if (v[k] == 1) {
            a.ngidx_to_gidx[run - 1] = (int32_t)(i + 1);
        }
    }
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

__device__ __forceinline__ float uniform_pm1(uint64_t seed, uint64_t key, uint32_t ctr) {
    const uint64_t r = splitmix64(seed ^ splitmix64(key * 0x100000001B3ull + ctr));
    const int32_t b = (int32_t)(r >> 40);
    return ((float)b - 8388607.5f) * (1.0f / 8388608.0f);
}

__device__ void split_normals(uint64_t seed, uint64_t key, float out[6]) {
    uint32_t ctr = 0;
    for (int k = 0; k < 6; k += 2) {
        float z0 = 0.0f, z1 = 0.0f;
        for (int it = 0; it < 64; ++it) {
            const float u = uniform_pm1(seed, key, ctr++);
            const float v = uniform_pm1(seed, key, ctr++);
            const float s = u * u + v * v;
            if (s >= 1.0f || s == 0.0f) continue;
            const float f = sqrtf(-2.0f * gs_logf(s) / s);
            z0 = u * f;
            z1 = v * f;
            break;
        }
        out[k] = z0;
        out[k + 1] = z1;
    }
}

struct ApplyArgs {
    const uint8_t* prune;
    const uint8_t* densify;
    const uint8_t* clone;
    const int32_t* counts_cs;
    int n;
    // old
    const float* mo; const float* sf; const float* rf; const float* sh; int S;
    const float* mm; const float* om; const float* sm; const float* rm; const float* shm; int Sm;
    // new
    float* nmo; float* nsf; float* nrf; float* nsh;
    float* nmm; float* nom; float* nsm; float* nrm; float* nshm;
    float log_split;
    uint64_t seed;
    int32_t* f2g;
    const int32_t* counts;  // device F
};

// The small per-Gaussian fields are written by the Gaussian's own thread; the SH rows (3 S
// coefficients and 6 S moments per Gaussian: 192 and 384 bytes at degree 3) are copied by the
// whole warp over its 32 Gaussians' contiguous source rows, so reads and writes are coalesced.
__device__ __forceinline__ void copy_small_moments(const ApplyArgs& a, size_t from, size_t to, bool zero) {
    for (int k = 0; k < 6; ++k) a.nmm[6 * to + k] = zero ? 0.0f : a.mm[6 * from + k];
    for (int k = 0; k < 2; ++k) a.nom[2 * to + k] = zero ? 0.0f : a.om[2 * from + k];
    for (int k = 0; k < 6; ++k) a.nsm[6 * to + k] = zero ? 0.0f : a.sm[6 * from + k];
    for (int k = 0; k < 8; ++k) a.nrm[8 * to + k] = zero ? 0.0f : a.rm[8 * from + k];
}

__device__ __forceinline__ void copy_rotation(const ApplyArgs& a, size_t from, size_t to) {
    for (int k = 0; k < 4; ++k) a.nrf[4 * to + k] = a.rf[4 * from + k];
}

// kinds of an old Gaussian
constexpr int kPruned = 0, kCarry = 1, kClone = 2, kSplit = 3;

__global__ void __launch_bounds__(128) k_adc_apply(const ApplyArgs a) {
    __shared__ int wkind[4][32];
    __shared__ int2 wdst[4][32];  // (first, last) new rows
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t i0 = ((int64_t)blockIdx.x * (blockDim.x >> 5) + wib) * 32; i0 < a.n; i0 += nw * 32) {
        const int64_t i = i0 + lane;
        int kind = kPruned;
        int2 d = make_int2(-1, -1);
        if (i < a.n && !a.prune[i]) {
            const size_t last = (size_t)a.counts_cs[i] - 1;
            const float* mo = a.mo + 4 * (size_t)i;
            const float* sf = a.sf + 3 * (size_t)i;
            if (a.densify[i]) {
                const size_t first = last - 1;
                d = make_int2((int)first, (int)last);
                if (a.clone[i]) {
                    kind = kClone;
                    for (int k = 0; k < 4; ++k) { a.nmo[4 * first + k] = mo[k]; a.nmo[4 * last + k] = mo[k]; }
                    for (int k = 0; k < 3; ++k) { a.nsf[3 * first + k] = sf[k]; a.nsf[3 * last + k] = sf[k]; }
                    copy_small_moments(a, i, first, false);
                    copy_small_moments(a, i, last, true);
                } else {
                    kind = kSplit;
                    const float* q = a.rf + 4 * (size_t)i;
                    const float qss = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3];
                    const float qs = sqrtf(2.0f * (1.0f / qss));
                    const float r = q[0] * qs, x = q[1] * qs, y = q[2] * qs, z = q[3] * qs;
                    const float R[3][3] = {{1.0f - (y * y + z * z), x * y - r * z, x * z + r * y},
                                           {x * y + r * z, 1.0f - (x * x + z * z), y * z - r * x},
                                           {x * z - r * y, y * z + r * x, 1.0f - (x * x + y * y)}};
                    const float s[3] = {gs_expf(sf[0]), gs_expf(sf[1]), gs_expf(sf[2])};
                    float nrm[6];
                    split_normals(a.seed, (uint64_t)i + 1, nrm);
                    for (int k = 0; k < 2; ++k) {
                        const size_t to = k == 0 ? first : last;
                        for (int rr = 0; rr < 3; ++rr) {
                            const float sh = R[rr][0] * (nrm[0 + 3 * k] * s[0]) + R[rr][1] * (nrm[1 + 3 * k] * s[1]) +
                                             R[rr][2] * (nrm[2 + 3 * k] * s[2]);
                            a.nmo[4 * to + rr] = mo[rr] + sh;
                        }
                        a.nmo[4 * to + 3] = mo[3];
                        for (int rr = 0; rr < 3; ++rr) a.nsf[3 * to + rr] = sf[rr] + a.log_split;
                    }
                    copy_small_moments(a, i, first, true);
                    copy_small_moments(a, i, last, true);
                }
                copy_rotation(a, i, first);
                copy_rotation(a, i, last);
            } else {
                kind = kCarry;
                d = make_int2(-1, (int)last);
                for (int k = 0; k < 4; ++k) a.nmo[4 * last + k] = mo[k];
                for (int k = 0; k < 3; ++k) a.nsf[3 * last + k] = sf[k];
                copy_small_moments(a, i, last, false);
                copy_rotation(a, i, last);
            }
        }
        wkind[wib][lane] = kind;
        wdst[wib][lane] = d;
        __syncwarp();
        const int cnt = (int)min((int64_t)32, (int64_t)a.n - i0);
        // SH coefficients: every new copy gets the old row
        const int L = 3 * a.S;
        const float* src = a.sh + (size_t)i0 * L;
        for (int e = lane; e < cnt * L; e += 32) {
            const int jg = e / L, col = e - jg * L;
            const int k = wkind[wib][jg];
            if (k == kPruned) continue;
            const float v = src[e];
            const int2 dd = wdst[wib][jg];
            a.nsh[(size_t)dd.y * L + col] = v;
            if (k != kCarry) a.nsh[(size_t)dd.x * L + col] = v;
        }
        // SH moments: carried and first clone keep them, second clone and both splits start at 0
        const int Lm = 6 * a.Sm;
        const float* srcm = a.shm + (size_t)i0 * Lm;
        for (int e = lane; e < cnt * Lm; e += 32) {
            const int jg = e / Lm, col = e - jg * Lm;
            const int k = wkind[wib][jg];
            if (k == kPruned) continue;
            const int2 dd = wdst[wib][jg];
            if (k == kCarry) {
                a.nshm[(size_t)dd.y * Lm + col] = srcm[e];
            } else if (k == kClone) {
                a.nshm[(size_t)dd.x * Lm + col] = srcm[e];
                a.nshm[(size_t)dd.y * Lm + col] = 0.0f;
            } else {
                a.nshm[(size_t)dd.x * Lm + col] = 0.0f;
                a.nshm[(size_t)dd.y * Lm + col] = 0.0f;
            }
        }
        __syncwarp();
    }
    // adjust_fgidx_to_gidx_adc_kernel!
    if (a.f2g) {
        const int F = a.counts[0];
        for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < F; f += gridDim.x * blockDim.x) {
            const int gidx = a.f2g[f];
            int32_t ngidx = 0;
            if (gidx > 0) {
                const int i = gidx - 1;
                if (!a.prune[i]) {
                    if (a.densify[i]) { if (a.clone[i]) ngidx = a.counts_cs[i] - 1; }
                    else ngidx = a.counts_cs[i];
                }
            }
            a.f2g[f] = ngidx;
        }
    }
}

// Dense gradient rows after a densify step: the carried Gaussian and the first clone keep the
// row of their original, every other new row is zero (untouched) — the dense counterpart of
// adjust_fgidx_to_gidx_adc_kernel! (training.jl:514-541).
__global__ void __launch_bounds__(256) k_remap_dense(const uint8_t* __restrict__ prune,
                                                     const uint8_t* __restrict__ densify,
                                                     const uint8_t* __restrict__ clone,
                                                     const int32_t* __restrict__ counts_cs, int n,
                                                     const float* __restrict__ dense_old,
                                                     float* __restrict__ dense_new, int row) {
    const int64_t total = (int64_t)n * row;
    for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < total;
         it += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(it / row);
        const int c = (int)(it - (int64_t)i * row);
        if (prune[i]) continue;
        const int64_t last = (int64_t)counts_cs[i] - 1;
        const float v = dense_old[it];
        if (densify[i]) {
            const int64_t first = last - 1;
            dense_new[last * row + c] = 0.0f;
            dense_new[first * row + c] = clone[i] ? v : 0.0f;
        } else {
            dense_new[last * row + c] = v;
        }
    }
}

__global__ void __launch_bounds__(256) k_opacity_reset(float* __restrict__ mo, float* __restrict__ om,
                                                       int n, float thr) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        float* p = mo + 4 * (size_t)i + 3;
        *p = fmin_jl(*p, thr);
        om[2 * (size_t)i] = 0.0f;
        om[2 * (size_t)i + 1] = 0.0f;
    }
}

int blocks_for(int64_t n, int threads, int per_sm) {
    int64_t b = ceil_div(n, threads);
    const int64_t cap = (int64_t)kSMs * per_sm;
    return (int)std::max<int64_t>(1, std::min<int64_t>(b, cap));
}

}  // namespace
}  // namespace gs3d

using namespace gs3d;

extern "C" {

GS3D_API int gs3d_adc_stats(const gs3d_adc_buffers* adc, const gs3d_fgradients* fg,
                            const int32_t* fgidx_to_gidx, const int32_t* device_counts,
                            int32_t width, int32_t height, gs3d_stream_t stream_) {
    if (!adc || !fg || !fgidx_to_gidx || !device_counts) return invalid("NULL argument");
    if (!adc->accumulated_mean2d_grad_norms_ndc || !adc->rendering_contribution_counts)
        return invalid("NULL ADC statistics arrays");
    const double sqw4 = (double)width * width / 4.0, sqh4 = (double)height * height / 4.0;
    ProfScope prof("adc_stats", reinterpret_cast<cudaStream_t>(stream_));
    k_adc_stats<<<kSMs * 8, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
        adc->accumulated_mean2d_grad_norms_ndc, adc->rendering_contribution_counts,
        fg->mean2d_grads, fgidx_to_gidx, device_counts, sqw4, sqh4);
    GS3D_LAUNCHED("k_adc_stats");
    return GS3D_OK;
}

GS3D_API int gs3d_adc_workspace_size(int32_t n, size_t* bytes) {
    if (!bytes || n < 0) return invalid("bad ADC workspace query");
    *bytes = scan_workspace_bytes(n > 0 ? n : 1);
    return GS3D_OK;
}

GS3D_API int gs3d_densify_prune_plan(const gs3d_adc_buffers* adc, const gs3d_gaussians* g,
                                     const gs3d_adc_params* p, int32_t* new_n,
                                     gs3d_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (!adc || !g || !p || !new_n) return invalid("NULL argument");
    const int n = g->n;
    if (n == 0) { *new_n = 0; return GS3D_OK; }
    if (!adc->workspace || adc->workspace_bytes < scan_workspace_bytes(n))
        return set_error("ADC workspace too small"), GS3D_ERR_WORKSPACE;
    PlanArgs a;
    a.acc = adc->accumulated_mean2d_grad_norms_ndc;
    a.cnt = adc->rendering_contribution_counts;
    a.sf = g->scaling_features;
    a.mo = g->means_opacity_features;
    a.max_sf = adc->max_scale_features;
    a.prune = adc->should_prune;
    a.densify = adc->should_densify;
    a.clone = adc->should_clone;
    a.counts = adc->new_gaussian_counts;
    a.counts_cs = adc->new_gaussian_counts_cs;
    a.ngidx_to_gidx = adc->ngidx_to_gidx;
    a.sums = static_cast<int32_t*>(adc->workspace);
    a.n = n;
    a.grad_thr = p->densification_mean2d_grad_norm_threshold_ndc;
    a.prune_thr = gs_logit(p->pruning_min_opacity);
    a.scale_thr = gs_logf(p->pruning_3d_max_scale);
    a.size_thr = gs_logf(p->densification_size_threshold);
    a.use_scale = p->use_max_scale_pruning;
    const unsigned nch = (unsigned)ceil_div(n, kChunk);
    k_plan_up<<<nch, kChunkThreads, 0, stream>>>(a);
    GS3D_LAUNCHED("k_plan_up");
    int32_t* total = a.sums + nch;  // one spare slot after the chunk sums
    GS3D_RETURN_IF(scan_spine(a.sums, n, nullptr, n, total, stream));
    k_plan_down<<<nch, kChunkThreads, 0, stream>>>(a);
    GS3D_LAUNCHED("k_plan_down");
    GS3D_CUDA(cudaMemcpyAsync(new_n, total, sizeof(int32_t), cudaMemcpyDeviceToHost, stream), "copy n'");
    GS3D_CUDA(cudaStreamSynchronize(stream), "sync n'");
    return GS3D_OK;
}

GS3D_API int gs3d_densify_apply(const gs3d_adc_buffers* adc, const gs3d_gaussians* og,
                                const gs3d_adam_moments* om, const gs3d_gaussians* ng,
                                const gs3d_adam_moments* nm, int32_t* fgidx_to_gidx,
                                const int32_t* device_counts, float log_splitting_scale_factor,
                                uint64_t seed, gs3d_stream_t stream_) {
    if (!adc || !og || !om || !ng || !nm) return invalid("NULL argument");
    if (og->sh_degree != ng->sh_degree || om->sh_degree != nm->sh_degree)
        return invalid("SH degree changes across densification");
    if (fgidx_to_gidx && !device_counts) return invalid("fgidx_to_gidx needs device_counts");
    ApplyArgs a;
    a.prune = adc->should_prune; a.densify = adc->should_densify; a.clone = adc->should_clone;
    a.counts_cs = adc->new_gaussian_counts_cs;
    a.n = og->n;
    a.mo = og->means_opacity_features; a.sf = og->scaling_features; a.rf = og->rotation_features;
    a.sh = og->sh_coeffs; a.S = (og->sh_degree + 1) * (og->sh_degree + 1);
    a.mm = om->means_moments; a.om = om->opacity_features_moments; a.sm = om->scaling_features_moments;
    a.rm = om->rotation_features_moments; a.shm = om->sh_coeffs_moments;
    a.Sm = (om->sh_degree + 1) * (om->sh_degree + 1);
    a.nmo = ng->means_opacity_features; a.nsf = ng->scaling_features; a.nrf = ng->rotation_features;
    a.nsh = ng->sh_coeffs;
    a.nmm = nm->means_moments; a.nom = nm->opacity_features_moments; a.nsm = nm->scaling_features_moments;
    a.nrm = nm->rotation_features_moments; a.nshm = nm->sh_coeffs_moments;
    a.log_split = log_splitting_scale_factor;
    a.seed = seed;
    a.f2g = fgidx_to_gidx;
    a.counts = device_counts;
    k_adc_apply<<<blocks_for(std::max(og->n, 1), 128, 16), 128, 0,
                  reinterpret_cast<cudaStream_t>(stream_)>>>(a);
    GS3D_LAUNCHED("k_adc_apply");
    return GS3D_OK;
}

GS3D_API int gs3d_densify_remap_dense(const gs3d_adc_buffers* adc, int32_t n_old,
                                      const float* dense_old, float* dense_new,
                                      gs3d_stream_t stream_) {
    if (!adc || !dense_old || !dense_new || n_old < 0) return invalid("NULL argument");
    if (n_old == 0) return GS3D_OK;
    k_remap_dense<<<kSMs * 8, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
        adc->should_prune, adc->should_densify, adc->should_clone, adc->new_gaussian_counts_cs,
        n_old, dense_old, dense_new, GS3D_DENSE_ROW);
    GS3D_LAUNCHED("k_remap_dense");
    return GS3D_OK;
}

GS3D_API int gs3d_opacity_reset(const gs3d_gaussians* g, const gs3d_adam_moments* m,
                                float max_opacity, gs3d_stream_t stream_) {
    if (!g || !m) return invalid("NULL argument");
    if (g->n == 0) return GS3D_OK;
    k_opacity_reset<<<blocks_for(g->n, 256, 8), 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
        g->means_opacity_features, m->opacity_features_moments, g->n, gs_logit(max_opacity));
    GS3D_LAUNCHED("k_opacity_reset");
    return GS3D_OK;
}

}  // extern "C"
