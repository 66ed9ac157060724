/*
 * gs3d.h — C ABI of libgs3d.so, a B200-native (sm_100a) engine for the 3D Gaussian
 * Splatting render / gradient / optimizer / densification hot path of
 * ThreeDGaussianSplatting.jl.
 *
 * Every entry point is `extern "C"`, takes plain device pointers, sizes and POD structs,
 * returns an int status (GS3D_OK == 0, negative on error; details through
 * gs3d_last_error_string()) and is asynchronous on the cudaStream_t it is given, unless
 * stated otherwise.
 *
 * Array layouts are the reference's (Julia column-major, first index fastest); "k x n"
 * means k contiguous fp32 per Gaussian. Index values stored in arrays are 1-based
 * (0 = invalid), exactly as the reference stores them, so buffers can be shared with
 * CUDA.jl CuArrays unchanged.
 *
 * Reference citations are `path:line` inside LaurensDiels/ThreeDGaussianSplatting.jl.
 */
#ifndef GS3D_H
#define GS3D_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define GS3D_API __declspec(dllexport)
#else
#define GS3D_API __attribute__((visibility("default")))
#endif

typedef struct CUstream_st* gs3d_stream_t; /* ABI-compatible with cudaStream_t */

/* ---- status codes ------------------------------------------------------------------- */
#define GS3D_OK 0
#define GS3D_ERR_INVALID_ARGUMENT (-1)
#define GS3D_ERR_CUDA (-2)
#define GS3D_ERR_CAPACITY (-3)   /* duplicated-key count exceeds the caller's capacity   */
#define GS3D_ERR_WORKSPACE (-4)  /* workspace smaller than the *_workspace_size answer   */
#define GS3D_ERR_UNSUPPORTED (-5)

/* Device-side status bits written into render_buffers.device_counts[2]. */
#define GS3D_STATUS_DUP_OVERFLOW 1u

/* render flags */
#define GS3D_RENDER_NO_HOST_SYNC 1u /* never block: D is checked on the device only      */
#define GS3D_RENDER_REFERENCE_ORDER 2u /* F4-F7 as the reference stages them (see below)   */
#define GS3D_RENDER_NO_CONTRIB_MASKS 4u /* leave render_buffers.contrib_masks unwritten (a
                                       render that no backward follows)                   */
#define GS3D_RENDER_DEFER_COLOUR 8u /* stop before the colours and the blend (F1-F7 only, the
                                       SH coefficients not read); gs3d_render_forward_colour
                                       completes the render                              */

/* backward flags */
#define GS3D_BACKWARD_FIX_SH16 1u /* use coefficient 16 in the degree-3 direction Jacobian
                                     (the reference reads coefficient 15: sh.jl:249)     */
#define GS3D_BACKWARD_SKIP_SH_GRADS 2u /* leave sh_coeffs_grads unwritten: for an update by
                                     gs3d_adam_step_rebuild_sh, which recomputes them      */
#define GS3D_BACKWARD_ACCUMULATE_ROWS 4u /* the projection-backward entry points that write
                                     dense or geometry rows add to the rows (several views
                                     per step) instead of overwriting them; colour rows are
                                     per view and always written                          */
#define GS3D_BACKWARD_NO_COLOUR_DIRECTION 8u /* gs3d_backward_project_factored: leave the
                                     colour -> direction term out of the mean gradient and
                                     read no SH coefficient; the owner of the rows adds it
                                     (gs3d_factored_colour_direction_range)              */

/* ---- POD parameter structs ---------------------------------------------------------- */

/* PinholeCamera (cameras.jl:50-106). P is the 3x4 projection matrix K [R_w2c | t_w2c]
 * stored column-major (P[i + 3*j] = row i, column j), position is the optical centre. */
typedef struct gs3d_camera {
    int32_t width, height;
    float fx, fy, skew, cx, cy;
    float near_z, far_z;
    float P[12];
    float position[3];
} gs3d_camera;

/* RenderOptions (forward_structs.jl:579-719). Clip values are in continuous pixel
 * coordinates. clipping_mode: 0 = CovarianceBoundaryClamp, 1 = BoundaryFilter. */
typedef struct gs3d_render_options {
    float background[3];
    float antialiasing_min_factor;
    float min_alpha, max_alpha, min_transmittance;
    float dilation_x, dilation_y;
    float clip_x_min, clip_x_max, clip_y_min, clip_y_max;
    int32_t sh_degree;
    int32_t clipping_mode;
    int32_t use_antialiasing;
} gs3d_render_options;

/* Tiling (forward_structs.jl:340-424). */
typedef struct gs3d_tiling {
    int32_t tile_width, tile_height;
    int32_t nb_tiles_x, nb_tiles_y;
} gs3d_tiling;

/* TrainableGaussiansVector (gaussians.jl:30-52): SoA of AoS-k arrays. */
typedef struct gs3d_gaussians {
    int32_t n;
    int32_t sh_degree;              /* storage degree: sh_coeffs holds (d+1)^2 x 3 x n */
    float* means_opacity_features;  /* 4 x n : x, y, z, logit(opacity)                 */
    float* scaling_features;        /* 3 x n : log-scales                              */
    float* rotation_features;       /* 4 x n : unnormalised quaternion (r, x, y, z)    */
    float* sh_coeffs;               /* (d+1)^2 x 3 x n                                 */
} gs3d_gaussians;

/* RenderOnlyGaussiansVector (gaussians.jl:342-392): precomputed 3D covariances and opacities
 * after the sigmoid, for rendering only (no gradients). */
typedef struct gs3d_render_only_gaussians {
    int32_t n;
    int32_t sh_degree;              /* storage degree: sh_coeffs holds (d+1)^2 x 3 x n     */
    float* means_opacities;         /* 4 x n : x, y, z, opacity (16-byte aligned)          */
    float* covariances;             /* 6 x n : lower 3D covariance 11, 21, 31, 22, 32, 33  */
    float* sh_coeffs;               /* (d+1)^2 x 3 x n                                     */
} gs3d_render_only_gaussians;

/* RenderBuffers (forward_structs.jl:1541-1600) + Filtered2DGaussiansVector
 * (forward_structs.jl:762-786). All arrays are caller-owned. */
typedef struct gs3d_render_buffers {
    int64_t capacity_n;            /* >= n                                              */
    int64_t capacity_dup;          /* capacity of the four duplicated-key arrays        */
    uint8_t* keep_gaussians;       /* n   (Bool)                                        */
    int32_t* keep_gaussians_cs;    /* n   inclusive cumsum (may be NULL)                */
    int32_t* fgidx_to_gidx;        /* n   1-based                                       */
    float* depths;                 /* n                                                 */
    float* means2d_opacities_inverse_covariances_colors; /* 9 x n                       */
    int32_t* intersected_tile_ranges;                   /* 2 x 2 x n: xmin ymin xmax ymax */
    int32_t* nb_overlapped_tiles;      /* n                                             */
    int32_t* nb_overlapped_tiles_cs;   /* n   inclusive cumsum                          */
    int64_t* df2dgs_codes;         /* capacity_dup  tile << 32 | depth bits             */
    int32_t* dfgidx_to_fgidx;      /* capacity_dup                                      */
    int64_t* sdf2dgs_codes;        /* capacity_dup  sorted                              */
    int32_t* sdfgidx_to_fgidx;     /* capacity_dup  sorted                              */
    int32_t* tiles_end_sdfgidx;    /* nb_tiles                                          */
    int32_t* device_counts;        /* >= 4 int32: [0] F, [1] D, [2] status bits,
                                      [3] 1 when the render wrote contrib_masks          */
    void* workspace;               /* scan / sort scratch                               */
    size_t workspace_bytes;
    /* Optional (NULL: not used). Contribution masks the forward blend writes for the backward
     * blend: per 32 duplicated entries of a tile and per warp of the tile (32 pixels), one
     * 32-bit word whose bit j says that one of the warp's pixels blended entry j, or evaluated
     * it with alpha in [0.999 min_alpha, min_alpha), before it stopped. The backward then
     * visits only those entries. The forward writes them (and sets device_counts[3]) when
     * contrib_mask_words >= (D / 32 + #tiles + 1) * tile pixels / 32 and the tile has a
     * multiple of 32 pixels; otherwise the backward tests every entry itself, with the same
     * results. */
    uint32_t* contrib_masks;
    int64_t contrib_mask_words;
    /* Optional (NULL: tiles in row-major order). nb_tiles int32 that every forward blend fills,
     * once the tile ends are known, with the 0-based tile indices by descending number of
     * duplicated entries (8 buckets per octave, any order within a bucket); the forward and
     * backward blends then take tiles in this order, so that the longest tiles start first and
     * short ones fill the end of the launch. The results do not depend on it. */
    int32_t* tile_order;
} gs3d_render_buffers;

/* RenderOutputs (forward_structs.jl:1-65). Any pointer may be NULL except that backward
 * needs transmittance and last_contributing. rgb is 3 x h x w, the others h x w. */
typedef struct gs3d_render_outputs {
    float* rgb;
    float* transmittance;
    float* depth;
    int32_t* last_contributing_sdfgids;
} gs3d_render_outputs;

/* FilteredGaussiansGradientsVector (backward_structs.jl:1-29), indexed by fgidx. */
typedef struct gs3d_fgradients {
    int32_t sh_degree;               /* storage degree of sh_coeffs_grads               */
    float* mean2d_grads;             /* 2 x n */
    float* opacity_grads;            /* n     */
    float* licov2d_grads;            /* 3 x n */
    float* color_grads;              /* 3 x n */
    float* mean3d_grads;             /* 3 x n */
    float* opacity_feature_grads;    /* n     */
    float* scaling_features_grads;   /* 3 x n */
    float* rotation_features_grads;  /* 4 x n */
    float* sh_coeffs_grads;          /* (d+1)^2 x 3 x n */
} gs3d_fgradients;

/* GaussianAdamMomentsLearningRatesVector (optimizer.jl:9-29): moments interleaved
 * [m1, m2] per scalar. */
typedef struct gs3d_adam_moments {
    int32_t sh_degree;
    float* means_moments;              /* 2 x 3 x n */
    float* opacity_features_moments;   /* 2 x n     */
    float* scaling_features_moments;   /* 2 x 3 x n */
    float* rotation_features_moments;  /* 2 x 4 x n */
    float* sh_coeffs_moments;          /* 2 x (d+1)^2 x 3 x n */
} gs3d_adam_moments;

/* Adam hyper-parameters (optimizer.jl:831-833, training_structs.jl:43-85). */
typedef struct gs3d_adam_params {
    float lr_means, lr_opacity_features, lr_scaling_features, lr_rotation_features;
    float lr_sh_dc, lr_sh_rest;
    float beta1, beta2, epsilon;
    int32_t update_count;  /* before this step; the step uses t = update_count + 1 */
    int32_t sh_degree;     /* render-options degree of the step (Val(sh) in update!) */
} gs3d_adam_params;

/* AdaptiveDensityControlBuffers (training_structs.jl:259-290). */
typedef struct gs3d_adc_buffers {
    float* accumulated_mean2d_grad_norms_ndc; /* n */
    int32_t* rendering_contribution_counts;   /* n */
    float* max_scale_features;                /* n */
    uint8_t* should_prune;                    /* n */
    uint8_t* should_densify;                  /* n */
    uint8_t* should_clone;                    /* n */
    uint8_t* new_gaussian_counts;             /* n */
    int32_t* new_gaussian_counts_cs;          /* n */
    int32_t* ngidx_to_gidx;                   /* n' (capacity 2 n)                    */
    void* workspace;
    size_t workspace_bytes;
} gs3d_adc_buffers;

/* Thresholds of one densify/prune decision (training.jl:325-364). */
typedef struct gs3d_adc_params {
    float densification_mean2d_grad_norm_threshold_ndc;
    float densification_size_threshold;   /* already scaled by the scene radius */
    float pruning_min_opacity;
    float pruning_3d_max_scale;           /* already scaled by the scene radius */
    int32_t use_max_scale_pruning;        /* iteration > opacity_reset_interval */
} gs3d_adc_params;

/* ---- drop-in replacement of deps/cub_sort_pairs (cub_sort_pairs_wrapper.cu:31-62) --- */

/* Same signature as the reference's `determine_sort_pairs_temp_storage`
 * (cub_sort_pairs_wrapper.cu:49-62, bound by forward_core.jl:629-638). */
GS3D_API size_t determine_sort_pairs_temp_storage(
    const int64_t* keys_in, int64_t* keys_out,
    const int32_t* values_in, int32_t* values_out,
    int nb_items, int highest_key_bit);

/* Same signature as the reference's `sort_pairs` (cub_sort_pairs_wrapper.cu:31-43, bound
 * by forward_core.jl:646-659): stable LSD radix sort of int64 keys with int32 values over
 * bits [0, highest_key_bit). Runs on the legacy default stream, as the reference does. */
GS3D_API void sort_pairs(
    void* temp_storage, size_t temp_storage_bytes,
    const int64_t* keys_in, int64_t* keys_out,
    const int32_t* values_in, int32_t* values_out,
    int nb_items, int highest_key_bit);

/* Stream-ordered variant of sort_pairs that reports errors. */
GS3D_API int gs3d_sort_pairs_async(
    void* temp_storage, size_t temp_storage_bytes,
    const int64_t* keys_in, int64_t* keys_out,
    const int32_t* values_in, int32_t* values_out,
    int nb_items, int highest_key_bit, gs3d_stream_t stream);

/* No counterpart in the reference. gs3d_sort_pairs_async without temp storage: the scratch is a
 * static device array inside libgs3d.so (13 MiB per device), so the call allocates nothing,
 * for callers that cannot provide or allocate a temporary buffer. At most
 * GS3D_SORT_NO_ALLOC_MAX_ITEMS pairs (larger calls return GS3D_ERR_INVALID_ARGUMENT and
 * launch nothing). The scratch is shared by all calls on a device: calls whose work overlaps
 * on the device race; calls on one stream do not. Every call with nb_items > 0 looks the
 * scratch address up on the current device (nothing is cached, so a device reset between calls
 * is harmless); the first call on a device also loads the array there and must come before any
 * stream capture on that device. */
#define GS3D_SORT_NO_ALLOC_MAX_ITEMS (1 << 20)
GS3D_API int gs3d_sort_pairs_no_alloc(
    const int64_t* keys_in, int64_t* keys_out,
    const int32_t* values_in, int32_t* values_out,
    int nb_items, int highest_key_bit, gs3d_stream_t stream);

/* ---- render forward: render! GPU (forward_core.jl:196-314) -------------------------- */

/* Bytes of render_buffers.workspace needed for these capacities. */
GS3D_API int gs3d_render_forward_workspace_size(
    int64_t capacity_n, int64_t capacity_dup, int32_t nb_tiles, size_t* bytes);

/* Filter (F1), compact (F2), project (F3), count + scan duplicates (F4), write keys (F5),
 * sort (F6), tile ranges (F7), alpha-blend (F8) or fill the void image (F9).
 * By default F4-F7 run as a tile-bucket sort: per-tile counts and their scan give
 * tiles_end_sdfgidx, and each tile's entries are sorted by (depth bits, filtered index) in
 * shared memory, which yields sdf2dgs_codes, sdfgidx_to_fgidx and tiles_end_sdfgidx identical
 * to the reference's stable sort; df2dgs_codes is then scratch, and dfgidx_to_fgidx and
 * nb_overlapped_tiles_cs are not written. With GS3D_RENDER_REFERENCE_ORDER those three are
 * filled as the reference fills them (scan, keys in filtered order, stable radix sort).
 * The camera needs 0 <= near_z < far_z.
 * F and D are written to render_buffers.device_counts[0..1]; when host_counts is not NULL
 * they are also copied there (pinned memory; valid after the stream reaches this point).
 * Without GS3D_RENDER_NO_HOST_SYNC the call waits once for D and returns
 * GS3D_ERR_CAPACITY (host_counts filled, outputs undefined) when D > capacity_dup. */
GS3D_API int gs3d_render_forward(
    const gs3d_render_outputs* outputs, const gs3d_gaussians* gaussians,
    const gs3d_camera* camera, const gs3d_tiling* tiling,
    const gs3d_render_options* options, gs3d_render_buffers* buffers,
    int32_t* host_counts, uint32_t flags, gs3d_stream_t stream);

/* render! for a RenderOnlyGaussiansVector: gs3d_render_forward with the stored opacities and
 * the 2D covariances J V J^T of the stored 3D covariances V (gaussians.jl:1324-1327; T = J V,
 * then the lower entries of T J^T, each sum in index order); every other stage is shared. */
GS3D_API int gs3d_render_forward_render_only(
    const gs3d_render_outputs* outputs, const gs3d_render_only_gaussians* gaussians,
    const gs3d_camera* camera, const gs3d_tiling* tiling,
    const gs3d_render_options* options, gs3d_render_buffers* buffers,
    int32_t* host_counts, uint32_t flags, gs3d_stream_t stream);

/* Second half of a gs3d_render_forward called with GS3D_RENDER_DEFER_COLOUR (same arguments,
 * the same Gaussians): the colours of the filtered Gaussians (sh_coeffs_to_color, sh.jl:38-112;
 * the first half reads no SH coefficient) and the blend (F8 / F9). Together they equal one
 * gs3d_render_forward bit for bit. No counterpart in the reference: it lets a data-parallel
 * caller start a render while the SH coefficients of the previous update are still arriving.
 * Only GS3D_RENDER_NO_CONTRIB_MASKS is read from flags. */
GS3D_API int gs3d_render_forward_colour(
    const gs3d_render_outputs* outputs, const gs3d_gaussians* gaussians,
    const gs3d_camera* camera, const gs3d_tiling* tiling,
    const gs3d_render_options* options, gs3d_render_buffers* buffers, uint32_t flags,
    gs3d_stream_t stream);

/* Work counts of the last gs3d_render_forward with these buffers (sorted arrays, tile ends,
 * 2D records and device counts as it left them), as the reference's blend loop performs the
 * work (render_tiles_kernel!, forward_core.jl:928-968: every pixel examines its tile's entries
 * in sorted order until it stops): counts_device[0] = (pixel, Gaussian) evaluations, the
 * terminating one included; counts_device[1] = evaluations blended into the pixel, which are
 * also the (pixel, Gaussian) pairs the backward blend (backward_core.jl:96-293) differentiates.
 * counts_device is 2 uint64 in device memory, overwritten. For rooflines and tests; not on the
 * training path (it evaluates every pair without the rasteriser's culling). */
GS3D_API int gs3d_render_work_counts(
    const gs3d_camera* camera, const gs3d_tiling* tiling, const gs3d_render_options* options,
    const gs3d_render_buffers* buffers, uint64_t* counts_device, gs3d_stream_t stream);

/* ---- backward: backward! (backward_core.jl:37-72) ----------------------------------- */

/* Zeroes the 2D gradients (B1), runs the reverse blend with warp-reduced atomics (B2) and
 * the projection backward (B3, B4). rgb_image_grad is 3 x h x w. */
GS3D_API int gs3d_backward(
    const gs3d_fgradients* fgradients, const float* rgb_image_grad,
    const gs3d_render_outputs* outputs, const gs3d_gaussians* gaussians,
    const gs3d_camera* camera, const gs3d_tiling* tiling,
    const gs3d_render_options* options, const gs3d_render_buffers* buffers,
    uint32_t flags, gs3d_stream_t stream);

/* ---- optimizer: update! (optimizer.jl:964-1009) ------------------------------------- */

/* One sparse Adam step over the F filtered Gaussians (F read from device_counts[0]);
 * fgidx_to_gidx entries <= 0 are skipped (optimizer.jl:1099-1103). All 59 parameters of a
 * Gaussian are updated in one fused kernel. */
GS3D_API int gs3d_adam_step(
    const gs3d_gaussians* gaussians, const gs3d_adam_moments* moments,
    const gs3d_fgradients* fgradients, const int32_t* fgidx_to_gidx,
    const int32_t* device_counts, const gs3d_adam_params* params, gs3d_stream_t stream);

/* gs3d_adam_step with the SH gradients recomputed instead of read: for filtered Gaussian f the
 * gradient of coefficient k of channel c is live_c * color_grads[f][c] * basis_k(d), d the unit
 * direction from camera_position (HOST memory, 3 floats: the camera the backward ran for) to
 * the Gaussian's mean, live_c = (the projected colour of channel c, float 6 + c of row f of
 * projected, the render buffers' means2d_opacities_inverse_covariances_colors) >= 0: the
 * expression gs3d_backward evaluates (compute_sh_coeffs_grad!, backward_core.jl:936-964), so
 * the update equals gs3d_adam_step after gs3d_backward bit for bit as long as the Gaussians are
 * unchanged between the backward and this call (not across a densify step). The backward may
 * then run with GS3D_BACKWARD_SKIP_SH_GRADS. Needs SH storage degree 3 and 16-byte aligned
 * arrays. */
GS3D_API int gs3d_adam_step_rebuild_sh(
    const gs3d_gaussians* gaussians, const gs3d_adam_moments* moments,
    const gs3d_fgradients* fgradients, const int32_t* fgidx_to_gidx,
    const int32_t* device_counts, const float* projected, const float* camera_position,
    const gs3d_adam_params* params, gs3d_stream_t stream);

/* ---- multi-view data parallelism (no counterpart in the reference: it trains one view at a
 * time on one GPU, training.jl:173-244). A dense gradient row of 60 floats per Gaussian:
 * SH (3 x 16, channel-major; 16-byte aligned) at 0, mean(3) at 48, opacity feature(1) at 51,
 * scaling features(3) at 52, rotation features(4) at 55, touched(1) at 59. Rows from several
 * views/ranks are summed (NCCL), then gs3d_adam_step_dense applies the update! scalar rule to
 * every touched Gaussian; with one view it equals gs3d_adam_step. */
#define GS3D_DENSE_ROW 60

/* gs3d_backward with the 3D gradients written straight into dense rows (n rows, zeroed here,
 * touched flags set) instead of the F-compact 3D arrays of fgradients, which may be NULL; the
 * 2D arrays are filled as by gs3d_backward. */
GS3D_API int gs3d_backward_dense(
    const gs3d_fgradients* fgradients, const float* rgb_image_grad,
    const gs3d_render_outputs* outputs, const gs3d_gaussians* gaussians,
    const gs3d_camera* camera, const gs3d_tiling* tiling,
    const gs3d_render_options* options, const gs3d_render_buffers* buffers,
    uint32_t flags, float* dense, int32_t n, gs3d_stream_t stream);

/* gs3d_backward_dense in two phases, so that the rows of one range of Gaussians can be
 * exchanged while the next range is computed: gs3d_backward_raster fills the 2D arrays of
 * fgradients (B1, B2); gs3d_backward_project_dense then runs B3/B4 for the filtered Gaussians
 * whose 0-based index is in [g_begin, g_end), writing row gidx - g_begin of dense_rows (rows
 * are not zeroed here: the caller zeroes them, touched flags are set). */
GS3D_API int gs3d_backward_raster(
    const gs3d_fgradients* fgradients, const float* rgb_image_grad,
    const gs3d_render_outputs* outputs, const gs3d_gaussians* gaussians,
    const gs3d_camera* camera, const gs3d_tiling* tiling,
    const gs3d_render_options* options, const gs3d_render_buffers* buffers,
    uint32_t flags, gs3d_stream_t stream);
GS3D_API int gs3d_backward_project_dense(
    const gs3d_fgradients* fgradients, const gs3d_gaussians* gaussians,
    const gs3d_camera* camera, const gs3d_tiling* tiling,
    const gs3d_render_options* options, const gs3d_render_buffers* buffers,
    uint32_t flags, float* dense_rows, int32_t g_begin, int32_t g_end, gs3d_stream_t stream);

/* gs3d_adam_step_dense over the Gaussians [g_begin, g_end) only, whose rows start at dense[0]
 * (a rank's shard of reduce-scattered rows). */
GS3D_API int gs3d_adam_step_dense_range(
    const gs3d_gaussians* gaussians, const gs3d_adam_moments* moments, const float* dense,
    int32_t g_begin, int32_t g_end, const gs3d_adam_params* params, gs3d_stream_t stream);

/* Zero dense (n rows) and scatter the F-compact gradients of one view into it. */
GS3D_API int gs3d_scatter_dense_grads(
    const gs3d_fgradients* fgradients, const int32_t* fgidx_to_gidx,
    const int32_t* device_counts, int32_t sh_degree, float* dense, int32_t n,
    gs3d_stream_t stream);

GS3D_API int gs3d_adam_step_dense(
    const gs3d_gaussians* gaussians, const gs3d_adam_moments* moments, const float* dense,
    const gs3d_adam_params* params, gs3d_stream_t stream);

/* Factored rows: the dense row with its 48 SH gradients replaced by their factors. The SH
 * gradient of one view is the outer product of the 3 colour gradients (each zero where the
 * colour was clamped) with the 16 SH basis values of the view direction (compute_sh_coeffs_grad!,
 * backward_core.jl:936-964), so a view needs to send only its colour gradients; the owner of a
 * Gaussian rebuilds the sum over views from the cameras' positions. Geometry row: the dense row's
 * floats 48..59 (mean, opacity feature, scaling, rotation, touched), summed over views like dense
 * rows. Colour row (one per view, not summed): colour gradients 0..2 and flags at 3,
 * 1 + 2 live0 + 4 live1 + 8 live2 + 16 pos0 + 32 pos1 + 64 pos2 where the Gaussian is filtered
 * in that view (live: colour >= 0; pos: colour > 0), else 0. */
#define GS3D_GEOM_ROW 12
#define GS3D_COLOUR_ROW 4
#define GS3D_MAX_FACTORED_VIEWS 64

/* gs3d_backward_project_dense writing factored rows: geometry row and colour row
 * gidx - g_begin for the filtered Gaussians with index in [g_begin, g_end) (rows are not zeroed
 * here; colour_rows 16-byte aligned). */
GS3D_API int gs3d_backward_project_factored(
    const gs3d_fgradients* fgradients, const gs3d_gaussians* gaussians,
    const gs3d_camera* camera, const gs3d_tiling* tiling,
    const gs3d_render_options* options, const gs3d_render_buffers* buffers,
    uint32_t flags, float* geom_rows, float* colour_rows, int32_t g_begin, int32_t g_end,
    gs3d_stream_t stream);

/* gs3d_adam_step_dense_range from factored rows: geom_rows holds the summed geometry rows of
 * [g_begin, g_end); colour_rows the colour rows of n_views views (1 .. GS3D_MAX_FACTORED_VIEWS),
 * view v's row for Gaussian g at row v * view_stride + g - g_begin; view_positions (HOST memory,
 * 3 floats per view) the camera positions the views were rendered from. The SH gradient is
 * rebuilt as the sum over the views in order v = 0, 1, ... (with one view: the gradient
 * gs3d_backward writes, bit for bit). Needs SH storage degree 3 and 16-byte aligned arrays. */
GS3D_API int gs3d_adam_step_factored_range(
    const gs3d_gaussians* gaussians, const gs3d_adam_moments* moments, const float* geom_rows,
    const float* colour_rows, int32_t n_views, int64_t view_stride, const float* view_positions,
    int32_t g_begin, int32_t g_end, const gs3d_adam_params* params, gs3d_stream_t stream);

/* Sharded SH coefficients (no counterpart in the reference, which trains on one GPU): the rank
 * that owns Gaussians [g_begin, g_end) is the only one whose SH coefficients of that range are
 * current. It adds the colour -> direction term of the mean gradient that the other ranks left
 * out (GS3D_BACKWARD_NO_COLOUR_DIRECTION) before its update, and after the update computes the
 * colours the next step's views will blend, which then travel instead of the SH coefficients
 * (12 B per Gaussian and view instead of 192 B per Gaussian).
 *
 * gs3d_factored_colour_direction_range: for each Gaussian of the range whose geometry row is
 * touched and each view v (order 0, 1, ...) whose colour row (row v * view_stride + g - g_begin,
 * flags > 0) says it filtered the Gaussian, adds to the row's mean gradient the term
 * gs3d_backward_project_factored adds without the flag (compute from the Gaussian's current SH
 * coefficients and mean, so call it before the update of the range); view_positions (HOST
 * memory, 3 floats per view) the cameras the views were rendered from; sh_degree the render's
 * SH degree; flags: GS3D_BACKWARD_FIX_SH16. With one view the row equals the one
 * gs3d_backward_project_factored writes without the flag, bit for bit. */
GS3D_API int gs3d_factored_colour_direction_range(
    const gs3d_gaussians* gaussians, float* geom_rows, const float* colour_rows, int32_t n_views,
    int64_t view_stride, const float* view_positions, int32_t g_begin, int32_t g_end,
    int32_t sh_degree, uint32_t flags, gs3d_stream_t stream);

/* gs3d_shard_colours: the colours (sh_coeffs_to_color, sh.jl:38-112, clamped) of Gaussians
 * [g_begin, g_end) seen from n_views cameras (view_positions: HOST memory, 3 floats per view),
 * at SH degree sh_degree: float4 row v * view_stride + g - g_begin of `colours` (16-byte
 * aligned), w = 0. Each is the value the render's projection stores for that Gaussian and
 * camera, bit for bit. */
GS3D_API int gs3d_shard_colours(const gs3d_gaussians* gaussians, int32_t sh_degree,
                                const float* view_positions, int32_t n_views, int32_t g_begin,
                                int32_t g_end, float* colours, int64_t view_stride,
                                gs3d_stream_t stream);

/* gs3d_render_forward_colour with the colours given instead of computed from SH coefficients:
 * Gaussian g = c N S + q S + i (0 <= q < N = n_ranks, 0 <= i < S = shard_rows) takes float4 row
 * ((c N + q) V + view) S + i of `colours` (V = n_views; the layout in which rank q's
 * gs3d_shard_colours output for the views of every rank arrives by one all-to-all per chunk
 * c). `colours` must hold that row for every g < n. Given the colours gs3d_shard_colours
 * computes, the outputs equal gs3d_render_forward's bit for bit. */
GS3D_API int gs3d_render_forward_given_colour(
    const gs3d_render_outputs* outputs, const gs3d_gaussians* gaussians,
    const gs3d_camera* camera, const gs3d_tiling* tiling, const gs3d_render_options* options,
    gs3d_render_buffers* buffers, const float* colours, int64_t shard_rows, int32_t n_ranks,
    int32_t n_views, int32_t view, uint32_t flags, gs3d_stream_t stream);

/* ---- loss: training.jl:196-217 (L1 + weight * DSSIM, with gradient) ----------------- */

GS3D_API int gs3d_loss_workspace_size(int32_t width, int32_t height, size_t* bytes);

/* rendered and target are 3 x h x w. Writes the scalar loss to loss_device[0] (and
 * [1] = L1, [2] = DSSIM) and the gradient image. */
GS3D_API int gs3d_loss_l1_dssim(
    const float* rendered, const float* target, int32_t width, int32_t height,
    float dssim_weight, float* loss_device, float* rgb_image_grad,
    void* workspace, size_t workspace_bytes, gs3d_stream_t stream);

/* ---- adaptive density control: training.jl:313-580, gaussians.jl:1526-1694 ---------- */

/* update_adc_stats_kernel! (training.jl:472-497). */
GS3D_API int gs3d_adc_stats(
    const gs3d_adc_buffers* adc, const gs3d_fgradients* fgradients,
    const int32_t* fgidx_to_gidx, const int32_t* device_counts,
    int32_t width, int32_t height, gs3d_stream_t stream);

/* Bytes of adc_buffers.workspace (the scan of the new-Gaussian counts) for n Gaussians. */
GS3D_API int gs3d_adc_workspace_size(int32_t n, size_t* bytes);

/* Masks, counts and their scan (training.jl:325-389) and ngidx_to_gidx
 * (training.jl:557-580). Blocks once and returns n' through new_n. */
GS3D_API int gs3d_densify_prune_plan(
    const gs3d_adc_buffers* adc, const gs3d_gaussians* gaussians,
    const gs3d_adc_params* params, int32_t* new_n, gs3d_stream_t stream);

/* Fill the n' Gaussians and moments (gaussians.jl:1589-1694, optimizer.jl:1342-1378) into
 * caller-allocated outputs and retarget fgidx_to_gidx (training.jl:514-541). Split means
 * use a counter-based normal sampler keyed by (seed, old gidx). */
GS3D_API int gs3d_densify_apply(
    const gs3d_adc_buffers* adc, const gs3d_gaussians* old_gaussians,
    const gs3d_adam_moments* old_moments, const gs3d_gaussians* new_gaussians,
    const gs3d_adam_moments* new_moments, int32_t* fgidx_to_gidx,
    const int32_t* device_counts, float log_splitting_scale_factor, uint64_t seed,
    gs3d_stream_t stream);

/* Dense-row counterpart of the fgidx_to_gidx retarget for multi-view data parallelism:
 * dense_new (n' rows, GS3D_DENSE_ROW floats) gets the row of the original for the carried
 * Gaussian and the first clone, zero rows otherwise. Run after gs3d_densify_prune_plan. */
GS3D_API int gs3d_densify_remap_dense(
    const gs3d_adc_buffers* adc, int32_t n_old, const float* dense_old, float* dense_new,
    gs3d_stream_t stream);

/* reset_opacities! (gaussians.jl:1093-1101) + zero_opacity_features_adam_moments!
 * (optimizer.jl:754-756). */
GS3D_API int gs3d_opacity_reset(
    const gs3d_gaussians* gaussians, const gs3d_adam_moments* moments,
    float max_opacity, gs3d_stream_t stream);

/* ---- misc ---------------------------------------------------------------------------- */
GS3D_API const char* gs3d_last_error_string(void);
GS3D_API int gs3d_version(void);

/* Stage timers (no counterpart in the reference beyond its GUI render timer, gui.jl:358-373):
 * when enabled, every entry point records CUDA events on its stream around each stage
 * (keep_compact, project, dup_scan, dup_keys, sort, tiles_end, raster, zero_2d, bwd_raster,
 * bwd_project, adam, loss, adc_stats). Enabling (or disabling) clears earlier records.
 * gs3d_profile_report waits for the recorded events and writes "stage launches total_ms"
 * lines. Host-thread unsafe; for measurement runs. */
GS3D_API int gs3d_profile_enable(int enable);
GS3D_API int gs3d_profile_report(char* buf, size_t len);

#ifdef __cplusplus
}
#endif
#endif /* GS3D_H */
