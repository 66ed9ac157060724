// forward.cu — render forward, render! GPU (forward_core.jl:196-314):
//   k_keep_*       visibility mask + scan + compaction (F1, F2: forward_core.jl:326-386)
//   k_project      per filtered Gaussian: mean, EWA conic, SH colour, tile rectangle (F3:
//                  forward_core.jl:411-517)
//   scan           duplicate counts -> offsets, D on the device (F4)
//   k_dup_keys     tile << 32 | depth bits keys (F5: forward_core.jl:531-603)
//   radix sort     (F6: radix_sort.cu)
//   k_tiles_end    per-tile end of the sorted range (F7: forward_core.jl:676-734)
//   k_raster       (F8 / F9: raster.cu)
// F and D never leave the device unless the caller asks for them.
#include "common.cuh"
#include "internal.h"

namespace gs3d {

int launch_raster(const gs3d_render_outputs& out, const gs3d_camera& cam, const gs3d_tiling& til,
                  const gs3d_render_options& opt, const gs3d_render_buffers& buf, bool masks,
                  cudaStream_t stream);
int launch_raster_counts(const gs3d_camera& cam, const gs3d_tiling& til,
                         const gs3d_render_options& opt, const gs3d_render_buffers& buf,
                         unsigned long long* counts_out, cudaStream_t stream);

namespace {

// project_with_depth (cameras.jl:714-722)
__device__ __forceinline__ void project_point(const gs3d_camera& c, float m0, float m1, float m2,
                                              float& px, float& py, float& depth) {
    const float* P = c.P;
    const float h0 = P[0] * m0 + P[3] * m1 + P[6] * m2 + P[9];
    const float h1 = P[1] * m0 + P[4] * m1 + P[7] * m2 + P[10];
    const float h2 = P[2] * m0 + P[5] * m1 + P[8] * m2 + P[11];
    depth = h2;
    px = h0 / h2;
    py = h1 / h2;
}

// ro: render-only input, mo.w is the opacity itself
__device__ __forceinline__ bool keep_gaussian(const float4 mo, const gs3d_camera& cam,
                                              const gs3d_render_options& opt, bool ro = false) {
    const float opacity = ro ? mo.w : gs_sigmoid(mo.w);
    bool keep = opacity >= opt.min_alpha;
    if (keep) {
        if (opt.clipping_mode == 1) {  // BoundaryFilter
            float mx, my, depth;
            project_point(cam, mo.x, mo.y, mo.z, mx, my, depth);
            const bool on = opt.clip_x_min < mx && mx <= opt.clip_x_max && opt.clip_y_min < my &&
                            my <= opt.clip_y_max;
            keep = on && (cam.near_z < depth && depth <= cam.far_z) && opacity > opt.min_alpha;
        } else {  // CovarianceBoundaryClamp: check_depth(get_mean_sv(g), camera)
            const float* P = cam.P;
            const float depth = P[2] * mo.x + P[5] * mo.y + P[8] * mo.z + P[11];
            keep = cam.near_z < depth && depth <= cam.far_z;
        }
    }
    return keep;
}

__global__ void __launch_bounds__(kChunkThreads) k_keep_upsweep(const float4* __restrict__ mo4,
                                                                int n, gs3d_camera cam,
                                                                gs3d_render_options opt,
                                                                uint8_t* __restrict__ keep,
                                                                int32_t* __restrict__ sums,
                                                                int ro) {
    __shared__ int sm[33];
    const int64_t base = (int64_t)blockIdx.x * kChunk;
    int cnt = 0;
#pragma unroll 4
    for (int k = 0; k < kChunkItems; ++k) {
        const int64_t i = base + k * kChunkThreads + threadIdx.x;
        if (i < n) {
            const bool kp = keep_gaussian(mo4[i], cam, opt, ro != 0);
            keep[i] = kp ? 1 : 0;
            cnt += kp ? 1 : 0;
        }
    }
    int total;
    block_exclusive_scan(cnt, sm, &total);
    if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// Second pass: each warp owns 16 rows of 32 consecutive Gaussians of the block's chunk; a
// ballot per row gives the row's keep mask, the lanes' prefixes are popcounts of the mask below
// them, and keep_cs / fgidx_to_gidx are written a row (32 consecutive entries) at a time.
__global__ void __launch_bounds__(kChunkThreads) k_keep_downsweep(const uint8_t* __restrict__ keep,
                                                                  int n,
                                                                  const int32_t* __restrict__ sums,
                                                                  int32_t* __restrict__ keep_cs,
                                                                  int32_t* __restrict__ f2g) {
    __shared__ int sm[33];
    constexpr int kRows = kChunk / kChunkThreads;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t wbase = (int64_t)blockIdx.x * kChunk + (int64_t)warp * (32 * kRows);
    uint32_t masks[kRows];
    int cnt = 0;
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
        const int64_t i = wbase + r * 32 + lane;
        masks[r] = __ballot_sync(0xffffffffu, i < n && keep[i] != 0);
        cnt += __popc(masks[r]);
    }
    int total;
    const int wex = block_exclusive_scan(lane == 0 ? cnt : 0, sm, &total);  // lane 0: the warp's offset
    int run = __shfl_sync(0xffffffffu, wex, 0) + sums[blockIdx.x];
    const uint32_t below = (1u << lane) - 1u;
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
        const int64_t i = wbase + r * 32 + lane;
        const uint32_t m = masks[r];
        const uint32_t mine = (m >> lane) & 1u;
        const int incl = run + __popc(m & below) + (int)mine;
        if (i < n) {
            if (keep_cs) keep_cs[i] = incl;
            if (mine) f2g[incl - 1] = (int32_t)(i + 1);
        }
        run += __popc(m);
    }
}

// sh_coeffs_to_color (sh.jl:38-112) for one channel; hc = coefficient 1 of that channel
template <int DEG>
__device__ __forceinline__ float sh_channel(const float* hc, float x, float y, float z) {
    float cc = sh_basis(1, x, y, z) * hc[0];
    if (DEG >= 1) {
        cc += (sh_basis(2, x, y, z) * hc[1] + sh_basis(3, x, y, z) * hc[2] +
               sh_basis(4, x, y, z) * hc[3]);
        if (DEG >= 2) {
            cc += (sh_basis(5, x, y, z) * hc[4] + sh_basis(6, x, y, z) * hc[5] +
                   sh_basis(7, x, y, z) * hc[6] + sh_basis(8, x, y, z) * hc[7] +
                   sh_basis(9, x, y, z) * hc[8]);
            if (DEG >= 3) {
                cc += (sh_basis(10, x, y, z) * hc[9] + sh_basis(11, x, y, z) * hc[10] +
                       sh_basis(12, x, y, z) * hc[11] + sh_basis(13, x, y, z) * hc[12] +
                       sh_basis(14, x, y, z) * hc[13] + sh_basis(15, x, y, z) * hc[14] +
                       sh_basis(16, x, y, z) * hc[15]);
            }
        }
    }
    cc += 0.5f;
    if (cc < 0.0f) cc = 0.0f;
    return cc;
}

struct ProjectArgs {
    const float4* mo4;
    const float* scal;
    const float4* rot4;
    const float* sh;
    int sh_stride;  // (storage degree + 1)^2
    const int32_t* f2g;
    const int32_t* counts;
    float* depths;
    float* f2d;
    int32_t* ranges;
    int32_t* ntiles;
    const float* cov;  // render-only input: 6 x n lower 3D covariances (else NULL)
};

#ifndef GS3D_PROJECT_MINB
#define GS3D_PROJECT_MINB 4
#endif

// Colour of Gaussian gi (mean m) seen from the camera: sh_coeffs_to_color over the normalised
// view direction (sh.jl:38-112).
// The SH rows of Gaussian gi (3 channels x (DEG + 1)^2 coefficients) into registers.
template <int DEG>
__device__ __forceinline__ void load_sh_rows(const ProjectArgs& a, int gi,
                                             float (&hc)[3][(DEG + 1) * (DEG + 1)]) {
    const float* h = a.sh + (size_t)gi * 3 * a.sh_stride;
    constexpr int NC = (DEG + 1) * (DEG + 1);
    if (NC == a.sh_stride && ((3 * NC) % 4) == 0 && (reinterpret_cast<uintptr_t>(a.sh) & 15) == 0) {
        const float4* h4 = reinterpret_cast<const float4*>(h);
#pragma unroll
        for (int k = 0; k < (3 * NC) / 4; ++k) {
            const float4 v = h4[k];
            (&hc[0][0])[4 * k] = v.x; (&hc[0][0])[4 * k + 1] = v.y;
            (&hc[0][0])[4 * k + 2] = v.z; (&hc[0][0])[4 * k + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int i = 0; i < NC; ++i) hc[c][i] = h[c * a.sh_stride + i];
    }
}

// sh_coeffs_to_color (sh.jl:38-112) seen from camera position p: the clamped colour.
template <int DEG>
__device__ __forceinline__ float3 colour_from_sh(const float (&hc)[3][(DEG + 1) * (DEG + 1)],
                                                 const float* p, float mx0, float my0, float mz0) {
    const float vx = mx0 - p[0], vy = my0 - p[1], vz = mz0 - p[2];
    const float inv = 1.0f / sqrtf(vx * vx + vy * vy + vz * vz);
    const float dx = vx * inv, dy = vy * inv, dz = vz * inv;
    return make_float3(sh_channel<DEG>(hc[0], dx, dy, dz), sh_channel<DEG>(hc[1], dx, dy, dz),
                       sh_channel<DEG>(hc[2], dx, dy, dz));
}

template <int DEG>
__device__ __forceinline__ float3 gaussian_colour(const ProjectArgs& a, const gs3d_camera& cam, int gi,
                                                  float mx0, float my0, float mz0) {
    float hc[3][(DEG + 1) * (DEG + 1)];
    load_sh_rows<DEG>(a, gi, hc);
    return colour_from_sh<DEG>(hc, cam.position, mx0, my0, mz0);
}

// RO: render-only input (stored opacity and 3D covariance). COL: also the colour (else left
// for k_project_colour).
template <int DEG, bool RO, bool COL = true>
__global__ void __launch_bounds__(256, GS3D_PROJECT_MINB) k_project(const ProjectArgs a, const gs3d_camera cam,
                                                 const gs3d_tiling til,
                                                 const gs3d_render_options opt) {
    const int F = a.counts[0];
    for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < F; f += gridDim.x * blockDim.x) {
        const int gi = a.f2g[f] - 1;
        const float4 mo = a.mo4[gi];
        float opacity = RO ? mo.w : gs_sigmoid(mo.w);
        float mx, my, depth;
        project_point(cam, mo.x, mo.y, mo.z, mx, my, depth);
        float cu = mx, cv = my;
        if (opt.clipping_mode == 0) {
            cu = jl_clamp(mx, opt.clip_x_min, opt.clip_x_max);
            cv = jl_clamp(my, opt.clip_y_min, opt.clip_y_max);
        }
        // get_linearized_projection_2d (cameras.jl:755-774)
        const float* P = cam.P;
        const float idepth = 1.0f / depth;
        float J[2][3];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            J[0][j] = idepth * (P[0 + 3 * j] + (-cu) * P[2 + 3 * j]);
            J[1][j] = idepth * (P[1 + 3 * j] + (-cv) * P[2 + 3 * j]);
        }
        float c11, c21, c22;
        if (RO) {
            // congruence transform J V J^T of the stored covariance (gaussians.jl:1324-1327):
            // T = J V, then the lower entries of T J^T, each sum in index order
            const float* cv = a.cov + 6 * (size_t)gi;
            const float V[3][3] = {{cv[0], cv[1], cv[2]}, {cv[1], cv[3], cv[4]}, {cv[2], cv[4], cv[5]}};
            float T[2][3];
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int k = 0; k < 3; ++k)
                    T[i][k] = J[i][0] * V[0][k] + J[i][1] * V[1][k] + J[i][2] * V[2][k];
            c11 = T[0][0] * J[0][0] + T[0][1] * J[0][1] + T[0][2] * J[0][2];
            c21 = T[1][0] * J[0][0] + T[1][1] * J[0][1] + T[1][2] * J[0][2];
            c22 = T[1][0] * J[1][0] + T[1][1] * J[1][1] + T[1][2] * J[1][2];
        } else {
            // scale and rotation (gaussians.jl:1280-1331, misc.jl:133-141)
            const float s0 = gs_expf(a.scal[3 * (size_t)gi]);
            const float s1 = gs_expf(a.scal[3 * (size_t)gi + 1]);
            const float s2 = gs_expf(a.scal[3 * (size_t)gi + 2]);
            const float4 q = a.rot4[gi];
            const float qss = q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w;
            const float qs = sqrtf(2.0f * (1.0f / qss));
            const float r = q.x * qs, x = q.y * qs, y = q.z * qs, z = q.w * qs;
            const float R[3][3] = {{1.0f - (y * y + z * z), x * y - r * z, x * z + r * y},
                                   {x * y + r * z, 1.0f - (x * x + z * z), y * z - r * x},
                                   {x * z - r * y, y * z + r * x, 1.0f - (x * x + y * y)}};
            const float s[3] = {s0, s1, s2};
            float RS[3][3];
#pragma unroll
            for (int i = 0; i < 3; ++i)
#pragma unroll
                for (int j = 0; j < 3; ++j) RS[i][j] = R[i][j] * s[j];
            float A[2][3];
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int k = 0; k < 3; ++k)
                    A[i][k] = J[i][0] * RS[0][k] + J[i][1] * RS[1][k] + J[i][2] * RS[2][k];
            c11 = A[0][0] * A[0][0] + A[0][1] * A[0][1] + A[0][2] * A[0][2];
            c21 = A[1][0] * A[0][0] + A[1][1] * A[0][1] + A[1][2] * A[0][2];
            c22 = A[1][0] * A[1][0] + A[1][1] * A[1][1] + A[1][2] * A[1][2];
        }
        float undilated_det = 0.0f;
        if (opt.use_antialiasing) undilated_det = fmaxf(c11 * c22 - c21 * c21, 0.0f);
        c11 += opt.dilation_x;
        c22 += opt.dilation_y;
        const float icov_det = 1.0f / (c11 * c22 - c21 * c21);
        if (opt.use_antialiasing)
            opacity *= fmaxf(opt.antialiasing_min_factor, sqrtf(undilated_det * icov_det));

        // _get_bbox_cts_px_cov + _get_bbox_discrete_px (forward_structs.jl:1303-1411)
        bool empty = true;
        int left = 0, top = 0, right = -1, bottom = -1;
        if (opacity >= opt.min_alpha) {
            const float gamma = 2.0f * gs_logf(opacity / opt.min_alpha);
            const float xr = sqrtf(gamma * c11);
            const float yr = sqrtf(gamma * c22);
            left = max(1, sat_i32(ceilf((mx - xr) + 0.5f)));
            top = max(1, sat_i32(ceilf((my - yr) + 0.5f)));
            right = min(cam.width, sat_i32(rintf(mx + xr)));
            bottom = min(cam.height, sat_i32(rintf(my + yr)));
            empty = left > right || top > bottom;
        }
        float3 col = make_float3(0.0f, 0.0f, 0.0f);
        if (COL) col = gaussian_colour<DEG>(a, cam, gi, mo.x, mo.y, mo.z);

        a.depths[f] = depth;
        float* rr = a.f2d + 9 * (size_t)f;
        rr[0] = mx; rr[1] = my; rr[2] = opacity;
        rr[3] = c22 * icov_det; rr[4] = -c21 * icov_det; rr[5] = c11 * icov_det;
        if (COL) { rr[6] = col.x; rr[7] = col.y; rr[8] = col.z; }
        int4 rect;
        int count;
        if (empty) {
            rect = make_int4(1, 1, 0, 0);
            count = 0;
        } else {  // rectangle_to_tile_ids without clamping (forward_structs.jl:517-528)
            rect.x = (left + til.tile_width - 1) / til.tile_width;
            rect.y = (top + til.tile_height - 1) / til.tile_height;
            rect.z = (right + til.tile_width - 1) / til.tile_width;
            rect.w = (bottom + til.tile_height - 1) / til.tile_height;
            count = (rect.z - rect.x + 1) * (rect.w - rect.y + 1);
        }
        reinterpret_cast<int4*>(a.ranges)[f] = rect;
        a.ntiles[f] = count;
    }
}

// The colours of the filtered Gaussians (floats 6..8 of their 2D records), for a render whose
// projection ran without them (GS3D_RENDER_DEFER_COLOUR).
template <int DEG>
__global__ void __launch_bounds__(256, GS3D_PROJECT_MINB) k_project_colour(const ProjectArgs a,
                                                                           const gs3d_camera cam) {
    const int F = a.counts[0];
    for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < F; f += gridDim.x * blockDim.x) {
        const int gi = a.f2g[f] - 1;
        const float4 mo = a.mo4[gi];
        const float3 col = gaussian_colour<DEG>(a, cam, gi, mo.x, mo.y, mo.z);
        float* rr = a.f2d + 9 * (size_t)f;
        rr[6] = col.x; rr[7] = col.y; rr[8] = col.z;
    }
}

// Camera positions of up to GS3D_MAX_FACTORED_VIEWS views, passed by value.
struct ColourViews {
    float p[GS3D_MAX_FACTORED_VIEWS][3];
};

// The colours of Gaussians [g_begin, g_end) seen from nv cameras: row v * view_stride + (gi -
// g_begin) of out gets view v's colour (the value k_project would store for that Gaussian and
// camera: same loads, same operations), w = 0.
template <int DEG>
__global__ void __launch_bounds__(128) k_shard_colours(const ProjectArgs a, const ColourViews cv,
                                                       int nv, int64_t g_begin, int64_t g_end,
                                                       float4* __restrict__ out, int64_t view_stride) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= g_end - g_begin) return;
    const int gi = (int)(g_begin + i);
    const float4 mo = a.mo4[gi];
    float hc[3][(DEG + 1) * (DEG + 1)];
    load_sh_rows<DEG>(a, gi, hc);
    for (int v = 0; v < nv; ++v) {
        const float3 c = colour_from_sh<DEG>(hc, cv.p[v], mo.x, mo.y, mo.z);
        out[(size_t)v * view_stride + i] = make_float4(c.x, c.y, c.z, 0.0f);
    }
}

// Floats 6..8 of the filtered Gaussians' 2D records from colours computed elsewhere: Gaussian gi
// = c N S + q S + i (0 <= q < N, 0 <= i < S) takes row ((c N + q) V + view) S + i.
__global__ void __launch_bounds__(256) k_fill_colours(const ProjectArgs a,
                                                      const float4* __restrict__ colours,
                                                      int64_t S, int N, int V, int view) {
    const int F = a.counts[0];
    const int64_t C = (int64_t)N * S;
    for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < F; f += gridDim.x * blockDim.x) {
        const int64_t gi = a.f2g[f] - 1;
        const int64_t c = gi / C, rem = gi - c * C, q = rem / S, i = rem - q * S;
        const float4 col = colours[((c * N + q) * V + view) * S + i];
        float* rr = a.f2d + 9 * (size_t)f;
        rr[6] = col.x; rr[7] = col.y; rr[8] = col.z;
    }
}

// fill_df2dgs_codes_and_dfgidx_to_fgidx_kernel! (forward_core.jl:531-603)
__global__ void __launch_bounds__(256) k_dup_keys(const int32_t* __restrict__ counts,
                                                  const int32_t* __restrict__ ntiles,
                                                  const int32_t* __restrict__ ntiles_cs,
                                                  const int4* __restrict__ ranges,
                                                  const float* __restrict__ depths,
                                                  int tiles_x, int64_t capacity,
                                                  int64_t* __restrict__ codes,
                                                  int32_t* __restrict__ dfg,
                                                  int32_t* status) {
    const int F = counts[0];
    for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < F; f += gridDim.x * blockDim.x) {
        const int cnt = ntiles[f];
        if (cnt == 0) continue;
        int64_t d = (int64_t)ntiles_cs[f] - cnt;
        if ((int64_t)ntiles_cs[f] > capacity) atomicOr(status, (int)GS3D_STATUS_DUP_OVERFLOW);
        const int4 r = ranges[f];
        const uint64_t dcode = (uint64_t)(int64_t)(int32_t)f2u(depths[f]);
        for (int ty = r.y; ty <= r.w; ++ty) {
            const int ycontrib = (ty - 1) * tiles_x;
            for (int tx = r.x; tx <= r.z; ++tx, ++d) {
                if (d >= capacity) continue;
                const uint32_t tile = (uint32_t)(tx + ycontrib);
                codes[d] = (int64_t)(((uint64_t)tile << 32) | dcode);
                dfg[d] = f + 1;
            }
        }
    }
}

// fill_tiles_end_sdfgidx_kernel! (forward_core.jl:676-734)
__global__ void __launch_bounds__(256) k_tiles_end(const int32_t* __restrict__ counts,
                                                   int64_t capacity,
                                                   const int64_t* __restrict__ scodes,
                                                   int nb_tiles, int32_t* __restrict__ tiles_end) {
    const int64_t Draw = counts[1];
    const int D = (int)(Draw < capacity ? Draw : capacity);
    if (counts[0] == 0 || D == 0) return;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < D; i += gridDim.x * blockDim.x) {
        const int cur = (int)((uint64_t)scodes[i] >> 32);
        if (i == 0)
            for (int t = 1; t < cur; ++t) tiles_end[t - 1] = 0;
        if (i + 1 < D) {
            const int nxt = (int)((uint64_t)scodes[i + 1] >> 32);
            for (int t = cur; t < nxt; ++t) tiles_end[t - 1] = i + 1;
        } else {
            for (int t = cur; t <= nb_tiles; ++t) tiles_end[t - 1] = D;
        }
    }
}

int grid_for(int64_t items, int threads, int per_sm = 16) {
    int64_t b = ceil_div(items, threads);
    const int64_t cap = (int64_t)kSMs * per_sm;
    if (b > cap) b = cap;
    if (b < 1) b = 1;
    return (int)b;
}

struct FwdLayout {
    size_t sums, sort, total;
};

// scan sums, then one region used either by the radix sort (reference-order pipeline) or by
// the tile-bucket sort
FwdLayout fwd_layout(int64_t capacity_n, int64_t capacity_dup, int nb_tiles) {
    FwdLayout L;
    size_t off = 0;
    L.sums = off; off += scan_workspace_bytes(capacity_n > 0 ? capacity_n : 1);
    L.sort = off;
    off += std::max(radix_sort_workspace_bytes(capacity_dup),
                    tile_sort_workspace_bytes(capacity_dup, nb_tiles > 0 ? nb_tiles : 1));
    L.total = off;
    return L;
}

int check_common(const gs3d_gaussians* g, const gs3d_camera* cam, const gs3d_tiling* til,
                 const gs3d_render_options* opt) {
    if (!g || !cam || !til || !opt) return invalid("NULL argument");
    if (g->n < 0) return invalid("negative Gaussian count %d", g->n);
    if (g->n > 0 && (!g->means_opacity_features || !g->scaling_features || !g->rotation_features ||
                     !g->sh_coeffs))
        return invalid("NULL Gaussian array");
    if (g->sh_degree < 0 || g->sh_degree > 3) return invalid("storage SH degree %d", g->sh_degree);
    if (opt->sh_degree < 0 || opt->sh_degree > g->sh_degree)
        return invalid("render SH degree %d with storage degree %d", opt->sh_degree, g->sh_degree);
    if (cam->width <= 0 || cam->height <= 0) return invalid("camera size %dx%d", cam->width, cam->height);
    // depths of kept Gaussians exceed near_z; a negative near plane would let negative depths
    // into the keys, whose sign bit the reference's key layout does not order
    if (!(cam->near_z >= 0.0f) || !(cam->far_z > cam->near_z))
        return invalid("clip planes near %g, far %g (need 0 <= near < far)", cam->near_z, cam->far_z);
    if (opt->max_alpha != opt->max_alpha || opt->min_alpha != opt->min_alpha ||
        opt->min_transmittance != opt->min_transmittance)
        return invalid("NaN alpha / transmittance threshold in the render options");
    if (til->tile_width <= 0 || til->tile_height <= 0 ||
        til->tile_width * til->tile_height > 512 || (til->tile_width * til->tile_height) % 32 != 0)
        return invalid("tile %dx%d (need a multiple of 32 and <= 512 pixels)", til->tile_width,
                       til->tile_height);
    if ((int64_t)til->nb_tiles_x * til->tile_width < cam->width ||
        (int64_t)til->nb_tiles_y * til->tile_height < cam->height || til->nb_tiles_x <= 0 ||
        til->nb_tiles_y <= 0)
        return invalid("tiling %dx%d of %dx%d does not cover %dx%d", til->nb_tiles_x,
                       til->nb_tiles_y, til->tile_width, til->tile_height, cam->width, cam->height);
    return GS3D_OK;
}

}  // namespace

int check_render_common(const gs3d_gaussians* g, const gs3d_camera* cam, const gs3d_tiling* til,
                        const gs3d_render_options* opt) {
    return check_common(g, cam, til, opt);
}

}  // namespace gs3d

using namespace gs3d;

extern "C" {

GS3D_API int gs3d_render_forward_workspace_size(int64_t capacity_n, int64_t capacity_dup,
                                                int32_t nb_tiles, size_t* bytes) {
    if (!bytes) return invalid("bytes is NULL");
    if (capacity_n < 0 || capacity_dup < 0 || nb_tiles < 0) return invalid("negative capacity");
    *bytes = fwd_layout(capacity_n, capacity_dup, nb_tiles).total;
    return GS3D_OK;
}

// cov != NULL: render-only input (g's means_opacity_features hold the opacities themselves).
static int render_forward_impl(const gs3d_render_outputs* outputs, const gs3d_gaussians* g,
                               const float* cov, const gs3d_camera* cam, const gs3d_tiling* til,
                               const gs3d_render_options* opt, gs3d_render_buffers* buf,
                               int32_t* host_counts, uint32_t flags, gs3d_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    GS3D_RETURN_IF(check_common(g, cam, til, opt));
    if (cov && (flags & GS3D_RENDER_DEFER_COLOUR))
        return invalid("GS3D_RENDER_DEFER_COLOUR is for trainable Gaussians");
    if (!outputs || !buf) return invalid("NULL outputs or buffers");
    if (g->n > buf->capacity_n) return invalid("n = %d exceeds capacity_n = %lld", g->n, (long long)buf->capacity_n);
    if (!buf->keep_gaussians || !buf->fgidx_to_gidx || !buf->depths ||
        !buf->means2d_opacities_inverse_covariances_colors || !buf->intersected_tile_ranges ||
        !buf->nb_overlapped_tiles || !buf->nb_overlapped_tiles_cs || !buf->df2dgs_codes ||
        !buf->dfgidx_to_fgidx || !buf->sdf2dgs_codes || !buf->sdfgidx_to_fgidx ||
        !buf->tiles_end_sdfgidx || !buf->device_counts)
        return invalid("NULL render buffer array");
    if (((uintptr_t)buf->intersected_tile_ranges & 15) || ((uintptr_t)g->means_opacity_features & 15) ||
        (!cov && ((uintptr_t)g->rotation_features & 15)))
        return invalid("tile ranges, means/opacity and rotation arrays must be 16-byte aligned");
    const FwdLayout L = fwd_layout(buf->capacity_n, buf->capacity_dup,
                                   til->nb_tiles_x * til->nb_tiles_y);
    if (!buf->workspace || buf->workspace_bytes < L.total)
        return set_error("render workspace %zu bytes < %zu", buf->workspace_bytes, L.total),
               GS3D_ERR_WORKSPACE;
    unsigned char* ws = static_cast<unsigned char*>(buf->workspace);
    int32_t* sums = reinterpret_cast<int32_t*>(ws + L.sums);
    int32_t* counts = buf->device_counts;
    const int n = g->n;
    const int64_t cap_n = buf->capacity_n > 0 ? buf->capacity_n : 1;
    const int nb_tiles = til->nb_tiles_x * til->nb_tiles_y;

    GS3D_CUDA(cudaMemsetAsync(counts, 0, 4 * sizeof(int32_t), stream), "memset counts");
    // F1 + F2
    if (n > 0) {
        ProfScope prof("keep_compact", stream);
        const unsigned nch = (unsigned)ceil_div(n, kChunk);
        k_keep_upsweep<<<nch, kChunkThreads, 0, stream>>>(
            reinterpret_cast<const float4*>(g->means_opacity_features), n, *cam, *opt,
            buf->keep_gaussians, sums, cov ? 1 : 0);
        GS3D_LAUNCHED("k_keep_upsweep");
        GS3D_RETURN_IF(scan_spine(sums, cap_n, nullptr, n, counts + 0, stream));
        k_keep_downsweep<<<nch, kChunkThreads, 0, stream>>>(buf->keep_gaussians, n, sums,
                                                            buf->keep_gaussians_cs,
                                                            buf->fgidx_to_gidx);
        GS3D_LAUNCHED("k_keep_downsweep");
    }
    // F3
    ProjectArgs pa;
    pa.mo4 = reinterpret_cast<const float4*>(g->means_opacity_features);
    pa.scal = g->scaling_features;
    pa.rot4 = reinterpret_cast<const float4*>(g->rotation_features);
    pa.sh = g->sh_coeffs;
    pa.sh_stride = (g->sh_degree + 1) * (g->sh_degree + 1);
    pa.f2g = buf->fgidx_to_gidx;
    pa.counts = counts;
    pa.depths = buf->depths;
    pa.f2d = buf->means2d_opacities_inverse_covariances_colors;
    pa.ranges = buf->intersected_tile_ranges;
    pa.ntiles = buf->nb_overlapped_tiles;
    pa.cov = cov;
    const int pgrid = grid_for(n, 256, 8);
    {
        ProfScope prof("project", stream);
        if (cov) {
            switch (opt->sh_degree) {
                case 0: k_project<0, true><<<pgrid, 256, 0, stream>>>(pa, *cam, *til, *opt); break;
                case 1: k_project<1, true><<<pgrid, 256, 0, stream>>>(pa, *cam, *til, *opt); break;
                case 2: k_project<2, true><<<pgrid, 256, 0, stream>>>(pa, *cam, *til, *opt); break;
                default: k_project<3, true><<<pgrid, 256, 0, stream>>>(pa, *cam, *til, *opt); break;
            }
        } else if (flags & GS3D_RENDER_DEFER_COLOUR) {
            switch (opt->sh_degree) {
                case 0: k_project<0, false, false><<<pgrid, 256, 0, stream>>>(pa, *cam, *til, *opt); break;
                case 1: k_project<1, false, false><<<pgrid, 256, 0, stream>>>(pa, *cam, *til, *opt); break;
                case 2: k_project<2, false, false><<<pgrid, 256, 0, stream>>>(pa, *cam, *til, *opt); break;
                default: k_project<3, false, false><<<pgrid, 256, 0, stream>>>(pa, *cam, *til, *opt); break;
            }
        } else {
            switch (opt->sh_degree) {
                case 0: k_project<0, false><<<pgrid, 256, 0, stream>>>(pa, *cam, *til, *opt); break;
                case 1: k_project<1, false><<<pgrid, 256, 0, stream>>>(pa, *cam, *til, *opt); break;
                case 2: k_project<2, false><<<pgrid, 256, 0, stream>>>(pa, *cam, *til, *opt); break;
                default: k_project<3, false><<<pgrid, 256, 0, stream>>>(pa, *cam, *til, *opt); break;
            }
        }
        GS3D_LAUNCHED("k_project");
    }
    if (!(flags & GS3D_RENDER_REFERENCE_ORDER) && nb_tiles <= tile_sort_max_tiles()) {
        // F4 - F7 as a tile-bucket sort (tile_sort.cu): same sorted arrays and tile ends
        const int4* ranges = reinterpret_cast<const int4*>(buf->intersected_tile_ranges);
        {
            ProfScope prof("tile_count", stream);
            GS3D_RETURN_IF(tile_sort_count(ws + L.sort, L.total - L.sort, counts, ranges, cap_n,
                                           til->nb_tiles_x, nb_tiles, buf->capacity_dup,
                                           buf->tiles_end_sdfgidx, stream));
        }
        if (!(flags & GS3D_RENDER_NO_HOST_SYNC)) {
            int32_t local[4];
            int32_t* dst = host_counts ? host_counts : local;
            GS3D_CUDA(cudaMemcpyAsync(dst, counts, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                      stream),
                      "copy counts");
            GS3D_CUDA(cudaStreamSynchronize(stream), "sync counts");
            if ((int64_t)dst[1] > buf->capacity_dup)
                return set_error("%d duplicated keys exceed capacity_dup = %lld", dst[1],
                                 (long long)buf->capacity_dup),
                       GS3D_ERR_CAPACITY;
        }
        {
            ProfScope prof("sort", stream);
            GS3D_RETURN_IF(tile_sort_order(ws + L.sort, counts, ranges, buf->depths, cap_n,
                                           til->nb_tiles_x, nb_tiles, buf->capacity_dup,
                                           buf->tiles_end_sdfgidx, buf->df2dgs_codes,
                                           buf->sdf2dgs_codes, buf->sdfgidx_to_fgidx, stream));
        }
        if (!(flags & GS3D_RENDER_DEFER_COLOUR)) {
            ProfScope prof("raster", stream);
            GS3D_RETURN_IF(launch_raster(*outputs, *cam, *til, *opt, *buf,
                                         !(flags & GS3D_RENDER_NO_CONTRIB_MASKS), stream));
        }
        if ((flags & GS3D_RENDER_NO_HOST_SYNC) && host_counts)
            GS3D_CUDA(cudaMemcpyAsync(host_counts, counts, 4 * sizeof(int32_t),
                                      cudaMemcpyDeviceToHost, stream),
                      "copy counts");
        return GS3D_OK;
    }
    // reference order: F4
    {
        ProfScope prof("dup_scan", stream);
        GS3D_RETURN_IF(inclusive_scan_i32(buf->nb_overlapped_tiles, buf->nb_overlapped_tiles_cs,
                                          cap_n, counts + 0, 0, counts + 1, sums, stream));
    }
    // F5
    {
        ProfScope prof("dup_keys", stream);
        k_dup_keys<<<grid_for(n, 256, 8), 256, 0, stream>>>(
            counts, buf->nb_overlapped_tiles, buf->nb_overlapped_tiles_cs,
            reinterpret_cast<const int4*>(buf->intersected_tile_ranges), buf->depths,
            til->nb_tiles_x, buf->capacity_dup, buf->df2dgs_codes, buf->dfgidx_to_fgidx, counts + 2);
        GS3D_LAUNCHED("k_dup_keys");
    }
    if (!(flags & GS3D_RENDER_NO_HOST_SYNC)) {
        int32_t local[4];
        int32_t* dst = host_counts ? host_counts : local;
        GS3D_CUDA(cudaMemcpyAsync(dst, counts, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost, stream),
                  "copy counts");
        GS3D_CUDA(cudaStreamSynchronize(stream), "sync counts");
        if ((int64_t)dst[1] > buf->capacity_dup)
            return set_error("%d duplicated keys exceed capacity_dup = %lld", dst[1],
                             (long long)buf->capacity_dup),
                   GS3D_ERR_CAPACITY;
    }
    // F6
    int highest = 33;
    for (int t = nb_tiles; t > 1; t >>= 1) ++highest;  // 33 + floor(log2(nb_tiles))
    {
        ProfScope prof("sort", stream);
        GS3D_RETURN_IF(radix_sort_pairs(ws + L.sort, L.total - L.sort, buf->df2dgs_codes,
                                        buf->sdf2dgs_codes, buf->dfgidx_to_fgidx,
                                        buf->sdfgidx_to_fgidx, buf->capacity_dup, counts + 1, 0,
                                        highest, stream));
    }
    // F7
    {
        ProfScope prof("tiles_end", stream);
        k_tiles_end<<<grid_for(buf->capacity_dup, 256, 8), 256, 0, stream>>>(
            counts, buf->capacity_dup, buf->sdf2dgs_codes, nb_tiles, buf->tiles_end_sdfgidx);
        GS3D_LAUNCHED("k_tiles_end");
    }
    // F8 / F9
    if (!(flags & GS3D_RENDER_DEFER_COLOUR)) {
        ProfScope prof("raster", stream);
        GS3D_RETURN_IF(launch_raster(*outputs, *cam, *til, *opt, *buf,
                                         !(flags & GS3D_RENDER_NO_CONTRIB_MASKS), stream));
    }
    if ((flags & GS3D_RENDER_NO_HOST_SYNC) && host_counts)
        GS3D_CUDA(cudaMemcpyAsync(host_counts, counts, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                  stream),
                  "copy counts");
    return GS3D_OK;
}

GS3D_API int gs3d_render_forward(const gs3d_render_outputs* outputs, const gs3d_gaussians* g,
                                 const gs3d_camera* cam, const gs3d_tiling* til,
                                 const gs3d_render_options* opt, gs3d_render_buffers* buf,
                                 int32_t* host_counts, uint32_t flags, gs3d_stream_t stream) {
    return render_forward_impl(outputs, g, nullptr, cam, til, opt, buf, host_counts, flags, stream);
}

GS3D_API int gs3d_render_forward_render_only(const gs3d_render_outputs* outputs,
                                             const gs3d_render_only_gaussians* ro,
                                             const gs3d_camera* cam, const gs3d_tiling* til,
                                             const gs3d_render_options* opt,
                                             gs3d_render_buffers* buf, int32_t* host_counts,
                                             uint32_t flags, gs3d_stream_t stream) {
    if (!ro) return invalid("NULL Gaussians");
    if (ro->n > 0 && !ro->covariances) return invalid("NULL covariances");
    gs3d_gaussians g{};
    g.n = ro->n;
    g.sh_degree = ro->sh_degree;
    g.means_opacity_features = ro->means_opacities;
    g.scaling_features = ro->covariances;   // not read: satisfies the shared argument checks
    g.rotation_features = ro->covariances;
    g.sh_coeffs = ro->sh_coeffs;
    return render_forward_impl(outputs, &g, ro->n > 0 ? ro->covariances : nullptr, cam, til, opt,
                               buf, host_counts, flags, stream);
}

GS3D_API int gs3d_render_forward_colour(const gs3d_render_outputs* outputs,
                                       const gs3d_gaussians* g, const gs3d_camera* cam,
                                       const gs3d_tiling* til, const gs3d_render_options* opt,
                                       gs3d_render_buffers* buf, uint32_t flags,
                                       gs3d_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    GS3D_RETURN_IF(check_common(g, cam, til, opt));
    if (!outputs || !buf || !buf->fgidx_to_gidx || !buf->device_counts ||
        !buf->means2d_opacities_inverse_covariances_colors)
        return invalid("NULL outputs or buffers");
    if (g->n > buf->capacity_n) return invalid("n = %d exceeds capacity_n = %lld", g->n, (long long)buf->capacity_n);
    ProjectArgs pa{};
    pa.mo4 = reinterpret_cast<const float4*>(g->means_opacity_features);
    pa.sh = g->sh_coeffs;
    pa.sh_stride = (g->sh_degree + 1) * (g->sh_degree + 1);
    pa.f2g = buf->fgidx_to_gidx;
    pa.counts = buf->device_counts;
    pa.f2d = buf->means2d_opacities_inverse_covariances_colors;
    const int pgrid = grid_for(g->n, 256, 8);
    {
        ProfScope prof("project", stream);
        switch (opt->sh_degree) {
            case 0: k_project_colour<0><<<pgrid, 256, 0, stream>>>(pa, *cam); break;
            case 1: k_project_colour<1><<<pgrid, 256, 0, stream>>>(pa, *cam); break;
            case 2: k_project_colour<2><<<pgrid, 256, 0, stream>>>(pa, *cam); break;
            default: k_project_colour<3><<<pgrid, 256, 0, stream>>>(pa, *cam); break;
        }
        GS3D_LAUNCHED("k_project_colour");
    }
    ProfScope prof("raster", stream);
    return launch_raster(*outputs, *cam, *til, *opt, *buf, !(flags & GS3D_RENDER_NO_CONTRIB_MASKS),
                         stream);
}

GS3D_API int gs3d_render_forward_given_colour(const gs3d_render_outputs* outputs,
                                             const gs3d_gaussians* g, const gs3d_camera* cam,
                                             const gs3d_tiling* til,
                                             const gs3d_render_options* opt,
                                             gs3d_render_buffers* buf, const float* colours,
                                             int64_t shard_rows, int32_t n_ranks,
                                             int32_t n_views, int32_t view, uint32_t flags,
                                             gs3d_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    GS3D_RETURN_IF(check_common(g, cam, til, opt));
    if (!outputs || !buf || !buf->fgidx_to_gidx || !buf->device_counts ||
        !buf->means2d_opacities_inverse_covariances_colors || !colours)
        return invalid("NULL outputs, buffers or colours");
    if (g->n > buf->capacity_n) return invalid("n = %d exceeds capacity_n = %lld", g->n, (long long)buf->capacity_n);
    if (shard_rows < 1 || n_ranks < 1 || n_views < 1 || view < 0 || view >= n_views)
        return invalid("colour layout S = %lld, N = %d, V = %d, view %d", (long long)shard_rows,
                       n_ranks, n_views, view);
    if ((reinterpret_cast<uintptr_t>(colours) & 15) != 0) return invalid("colours not 16-byte aligned");
    ProjectArgs pa{};
    pa.f2g = buf->fgidx_to_gidx;
    pa.counts = buf->device_counts;
    pa.f2d = buf->means2d_opacities_inverse_covariances_colors;
    {
        ProfScope prof("project", stream);
        k_fill_colours<<<grid_for(g->n, 256, 8), 256, 0, stream>>>(
            pa, reinterpret_cast<const float4*>(colours), shard_rows, n_ranks, n_views, view);
        GS3D_LAUNCHED("k_fill_colours");
    }
    ProfScope prof("raster", stream);
    return launch_raster(*outputs, *cam, *til, *opt, *buf, !(flags & GS3D_RENDER_NO_CONTRIB_MASKS),
                         stream);
}

GS3D_API int gs3d_shard_colours(const gs3d_gaussians* g, int32_t sh_degree,
                                const float* view_positions, int32_t n_views, int32_t g_begin,
                                int32_t g_end, float* colours, int64_t view_stride,
                                gs3d_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (!g || !view_positions || !colours) return invalid("NULL argument");
    if (sh_degree < 0 || sh_degree > 3 || sh_degree > g->sh_degree)
        return invalid("SH degree %d (storage %d)", sh_degree, g->sh_degree);
    if (g_begin < 0 || g_end < g_begin || g_end > g->n)
        return invalid("Gaussian range [%d, %d) of n = %d", g_begin, g_end, g->n);
    if (n_views < 1 || n_views > GS3D_MAX_FACTORED_VIEWS)
        return invalid("%d views (1 .. %d)", n_views, GS3D_MAX_FACTORED_VIEWS);
    if (view_stride < (int64_t)g_end - g_begin) return invalid("view stride %lld < range", (long long)view_stride);
    if ((reinterpret_cast<uintptr_t>(colours) & 15) != 0) return invalid("colours not 16-byte aligned");
    if (g_end == g_begin) return GS3D_OK;
    ProjectArgs pa{};
    pa.mo4 = reinterpret_cast<const float4*>(g->means_opacity_features);
    pa.sh = g->sh_coeffs;
    pa.sh_stride = (g->sh_degree + 1) * (g->sh_degree + 1);
    ColourViews cv{};
    for (int v = 0; v < n_views; ++v)
        for (int k = 0; k < 3; ++k) cv.p[v][k] = view_positions[3 * v + k];
    const int64_t cnt = (int64_t)g_end - g_begin;
    const unsigned grid = (unsigned)ceil_div(cnt, 128);
    float4* out = reinterpret_cast<float4*>(colours);
    ProfScope prof("shard_colours", stream);
    switch (sh_degree) {
        case 0: k_shard_colours<0><<<grid, 128, 0, stream>>>(pa, cv, n_views, g_begin, g_end, out, view_stride); break;
        case 1: k_shard_colours<1><<<grid, 128, 0, stream>>>(pa, cv, n_views, g_begin, g_end, out, view_stride); break;
        case 2: k_shard_colours<2><<<grid, 128, 0, stream>>>(pa, cv, n_views, g_begin, g_end, out, view_stride); break;
        default: k_shard_colours<3><<<grid, 128, 0, stream>>>(pa, cv, n_views, g_begin, g_end, out, view_stride); break;
    }
    GS3D_LAUNCHED("k_shard_colours");
    return GS3D_OK;
}

GS3D_API int gs3d_render_work_counts(const gs3d_camera* cam, const gs3d_tiling* til,
                                     const gs3d_render_options* opt,
                                     const gs3d_render_buffers* buf, uint64_t* counts_device,
                                     gs3d_stream_t stream) {
    if (!cam || !til || !opt || !buf || !counts_device) return invalid("NULL argument");
    if (til->tile_width <= 0 || til->tile_height <= 0 || til->tile_width * til->tile_height > 512 ||
        til->nb_tiles_x <= 0 || til->nb_tiles_y <= 0)
        return invalid("tiling %dx%d tiles of %dx%d", til->nb_tiles_x, til->nb_tiles_y,
                       til->tile_width, til->tile_height);
    if (!buf->sdfgidx_to_fgidx || !buf->tiles_end_sdfgidx || !buf->device_counts ||
        !buf->means2d_opacities_inverse_covariances_colors)
        return invalid("NULL render buffer array");
    return launch_raster_counts(*cam, *til, *opt, *buf,
                                reinterpret_cast<unsigned long long*>(counts_device),
                                reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
