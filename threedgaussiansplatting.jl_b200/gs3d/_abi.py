"""ctypes mirror of include/gs3d.h and the loader of libgs3d.so.

The library is the product: every compute call goes through it. If it is missing or cannot
be loaded, ``lib()`` raises; there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libgs3d.so"

GS3D_OK = 0
GS3D_ERR_INVALID_ARGUMENT = -1
GS3D_ERR_CUDA = -2
GS3D_ERR_CAPACITY = -3
GS3D_ERR_WORKSPACE = -4
GS3D_ERR_UNSUPPORTED = -5
GS3D_STATUS_DUP_OVERFLOW = 1
GS3D_RENDER_NO_HOST_SYNC = 1
GS3D_RENDER_REFERENCE_ORDER = 2
GS3D_RENDER_NO_CONTRIB_MASKS = 4
GS3D_RENDER_DEFER_COLOUR = 8
GS3D_BACKWARD_FIX_SH16 = 1
GS3D_BACKWARD_SKIP_SH_GRADS = 2
GS3D_BACKWARD_ACCUMULATE_ROWS = 4
GS3D_BACKWARD_NO_COLOUR_DIRECTION = 8
GS3D_DENSE_ROW = 60
GS3D_GEOM_ROW = 12
GS3D_COLOUR_ROW = 4
GS3D_MAX_FACTORED_VIEWS = 64

f32p = C.POINTER(C.c_float)
i32p = C.POINTER(C.c_int32)
i64p = C.POINTER(C.c_int64)
u8p = C.POINTER(C.c_uint8)


class Camera(C.Structure):
    _fields_ = [("width", C.c_int32), ("height", C.c_int32), ("fx", C.c_float), ("fy", C.c_float),
                ("skew", C.c_float), ("cx", C.c_float), ("cy", C.c_float), ("near_z", C.c_float),
                ("far_z", C.c_float), ("P", C.c_float * 12), ("position", C.c_float * 3)]


class RenderOptionsC(C.Structure):
    _fields_ = [("background", C.c_float * 3), ("antialiasing_min_factor", C.c_float),
                ("min_alpha", C.c_float), ("max_alpha", C.c_float),
                ("min_transmittance", C.c_float), ("dilation_x", C.c_float),
                ("dilation_y", C.c_float), ("clip_x_min", C.c_float), ("clip_x_max", C.c_float),
                ("clip_y_min", C.c_float), ("clip_y_max", C.c_float), ("sh_degree", C.c_int32),
                ("clipping_mode", C.c_int32), ("use_antialiasing", C.c_int32)]


class TilingC(C.Structure):
    _fields_ = [("tile_width", C.c_int32), ("tile_height", C.c_int32),
                ("nb_tiles_x", C.c_int32), ("nb_tiles_y", C.c_int32)]


class GaussiansC(C.Structure):
    _fields_ = [("n", C.c_int32), ("sh_degree", C.c_int32), ("means_opacity_features", C.c_void_p),
                ("scaling_features", C.c_void_p), ("rotation_features", C.c_void_p),
                ("sh_coeffs", C.c_void_p)]


class RenderOnlyGaussiansC(C.Structure):
    _fields_ = [("n", C.c_int32), ("sh_degree", C.c_int32), ("means_opacities", C.c_void_p),
                ("covariances", C.c_void_p), ("sh_coeffs", C.c_void_p)]


class RenderBuffersC(C.Structure):
    _fields_ = [("capacity_n", C.c_int64), ("capacity_dup", C.c_int64),
                ("keep_gaussians", C.c_void_p), ("keep_gaussians_cs", C.c_void_p),
                ("fgidx_to_gidx", C.c_void_p), ("depths", C.c_void_p),
                ("means2d_opacities_inverse_covariances_colors", C.c_void_p),
                ("intersected_tile_ranges", C.c_void_p), ("nb_overlapped_tiles", C.c_void_p),
                ("nb_overlapped_tiles_cs", C.c_void_p), ("df2dgs_codes", C.c_void_p),
                ("dfgidx_to_fgidx", C.c_void_p), ("sdf2dgs_codes", C.c_void_p),
                ("sdfgidx_to_fgidx", C.c_void_p), ("tiles_end_sdfgidx", C.c_void_p),
                ("device_counts", C.c_void_p), ("workspace", C.c_void_p),
                ("workspace_bytes", C.c_size_t), ("contrib_masks", C.c_void_p),
                ("contrib_mask_words", C.c_int64), ("tile_order", C.c_void_p)]


class RenderOutputsC(C.Structure):
    _fields_ = [("rgb", C.c_void_p), ("transmittance", C.c_void_p), ("depth", C.c_void_p),
                ("last_contributing_sdfgids", C.c_void_p)]


class FGradientsC(C.Structure):
    _fields_ = [("sh_degree", C.c_int32), ("mean2d_grads", C.c_void_p),
                ("opacity_grads", C.c_void_p), ("licov2d_grads", C.c_void_p),
                ("color_grads", C.c_void_p), ("mean3d_grads", C.c_void_p),
                ("opacity_feature_grads", C.c_void_p), ("scaling_features_grads", C.c_void_p),
                ("rotation_features_grads", C.c_void_p), ("sh_coeffs_grads", C.c_void_p)]


class AdamMomentsC(C.Structure):
    _fields_ = [("sh_degree", C.c_int32), ("means_moments", C.c_void_p),
                ("opacity_features_moments", C.c_void_p),
                ("scaling_features_moments", C.c_void_p),
                ("rotation_features_moments", C.c_void_p), ("sh_coeffs_moments", C.c_void_p)]


class AdamParamsC(C.Structure):
    _fields_ = [("lr_means", C.c_float), ("lr_opacity_features", C.c_float),
                ("lr_scaling_features", C.c_float), ("lr_rotation_features", C.c_float),
                ("lr_sh_dc", C.c_float), ("lr_sh_rest", C.c_float), ("beta1", C.c_float),
                ("beta2", C.c_float), ("epsilon", C.c_float), ("update_count", C.c_int32),
                ("sh_degree", C.c_int32)]


class AdcBuffersC(C.Structure):
    _fields_ = [("accumulated_mean2d_grad_norms_ndc", C.c_void_p),
                ("rendering_contribution_counts", C.c_void_p), ("max_scale_features", C.c_void_p),
                ("should_prune", C.c_void_p), ("should_densify", C.c_void_p),
                ("should_clone", C.c_void_p), ("new_gaussian_counts", C.c_void_p),
                ("new_gaussian_counts_cs", C.c_void_p), ("ngidx_to_gidx", C.c_void_p),
                ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t)]


class AdcParamsC(C.Structure):
    _fields_ = [("densification_mean2d_grad_norm_threshold_ndc", C.c_float),
                ("densification_size_threshold", C.c_float),
                ("pruning_min_opacity", C.c_float), ("pruning_3d_max_scale", C.c_float),
                ("use_max_scale_pruning", C.c_int32)]


P = C.POINTER
# name -> (restype, argtypes); every symbol include/gs3d.h declares
SIGNATURES = {
    "determine_sort_pairs_temp_storage": (C.c_size_t, [C.c_void_p, C.c_void_p, C.c_void_p,
                                                       C.c_void_p, C.c_int, C.c_int]),
    "sort_pairs": (None, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                          C.c_int, C.c_int]),
    "gs3d_sort_pairs_async": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "gs3d_sort_pairs_no_alloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_int, C.c_int, C.c_void_p]),
    "gs3d_render_forward_workspace_size": (C.c_int, [C.c_int64, C.c_int64, C.c_int32,
                                                     P(C.c_size_t)]),
    "gs3d_render_forward": (C.c_int, [P(RenderOutputsC), P(GaussiansC), P(Camera), P(TilingC),
                                      P(RenderOptionsC), P(RenderBuffersC), C.c_void_p,
                                      C.c_uint32, C.c_void_p]),
    "gs3d_render_forward_colour": (C.c_int, [P(RenderOutputsC), P(GaussiansC), P(Camera), P(TilingC),
                                             P(RenderOptionsC), P(RenderBuffersC), C.c_uint32,
                                             C.c_void_p]),
    "gs3d_render_forward_given_colour": (C.c_int, [P(RenderOutputsC), P(GaussiansC), P(Camera),
                                                   P(TilingC), P(RenderOptionsC), P(RenderBuffersC),
                                                   C.c_void_p, C.c_int64, C.c_int32, C.c_int32,
                                                   C.c_int32, C.c_uint32, C.c_void_p]),
    "gs3d_shard_colours": (C.c_int, [P(GaussiansC), C.c_int32, P(C.c_float), C.c_int32, C.c_int32,
                                     C.c_int32, C.c_void_p, C.c_int64, C.c_void_p]),
    "gs3d_factored_colour_direction_range": (C.c_int, [P(GaussiansC), C.c_void_p, C.c_void_p,
                                                       C.c_int32, C.c_int64, P(C.c_float),
                                                       C.c_int32, C.c_int32, C.c_int32, C.c_uint32,
                                                       C.c_void_p]),
    "gs3d_render_work_counts": (C.c_int, [P(Camera), P(TilingC), P(RenderOptionsC),
                                          P(RenderBuffersC), C.c_void_p, C.c_void_p]),
    "gs3d_render_forward_render_only": (C.c_int, [P(RenderOutputsC), P(RenderOnlyGaussiansC),
                                                  P(Camera), P(TilingC), P(RenderOptionsC),
                                                  P(RenderBuffersC), C.c_void_p, C.c_uint32,
                                                  C.c_void_p]),
    "gs3d_backward": (C.c_int, [P(FGradientsC), C.c_void_p, P(RenderOutputsC), P(GaussiansC),
                                P(Camera), P(TilingC), P(RenderOptionsC), P(RenderBuffersC),
                                C.c_uint32, C.c_void_p]),
    "gs3d_adam_step": (C.c_int, [P(GaussiansC), P(AdamMomentsC), P(FGradientsC), C.c_void_p,
                                 C.c_void_p, P(AdamParamsC), C.c_void_p]),
    "gs3d_scatter_dense_grads": (C.c_int, [P(FGradientsC), C.c_void_p, C.c_void_p, C.c_int32,
                                           C.c_void_p, C.c_int32, C.c_void_p]),
    "gs3d_adam_step_dense": (C.c_int, [P(GaussiansC), P(AdamMomentsC), C.c_void_p, P(AdamParamsC),
                                       C.c_void_p]),
    "gs3d_backward_dense": (C.c_int, [P(FGradientsC), C.c_void_p, P(RenderOutputsC), P(GaussiansC),
                                      P(Camera), P(TilingC), P(RenderOptionsC), P(RenderBuffersC),
                                      C.c_uint32, C.c_void_p, C.c_int32, C.c_void_p]),
    "gs3d_adam_step_dense_range": (C.c_int, [P(GaussiansC), P(AdamMomentsC), C.c_void_p, C.c_int32,
                                             C.c_int32, P(AdamParamsC), C.c_void_p]),
    "gs3d_backward_raster": (C.c_int, [P(FGradientsC), C.c_void_p, P(RenderOutputsC), P(GaussiansC),
                                       P(Camera), P(TilingC), P(RenderOptionsC), P(RenderBuffersC),
                                       C.c_uint32, C.c_void_p]),
    "gs3d_backward_project_dense": (C.c_int, [P(FGradientsC), P(GaussiansC), P(Camera), P(TilingC),
                                              P(RenderOptionsC), P(RenderBuffersC), C.c_uint32,
                                              C.c_void_p, C.c_int32, C.c_int32, C.c_void_p]),
    "gs3d_backward_project_factored": (C.c_int, [P(FGradientsC), P(GaussiansC), P(Camera),
                                                 P(TilingC), P(RenderOptionsC), P(RenderBuffersC),
                                                 C.c_uint32, C.c_void_p, C.c_void_p, C.c_int32,
                                                 C.c_int32, C.c_void_p]),
    "gs3d_adam_step_factored_range": (C.c_int, [P(GaussiansC), P(AdamMomentsC), C.c_void_p,
                                                C.c_void_p, C.c_int32, C.c_int64,
                                                P(C.c_float), C.c_int32, C.c_int32,
                                                P(AdamParamsC), C.c_void_p]),
    "gs3d_adam_step_rebuild_sh": (C.c_int, [P(GaussiansC), P(AdamMomentsC), P(FGradientsC),
                                            C.c_void_p, C.c_void_p, C.c_void_p, P(C.c_float),
                                            P(AdamParamsC), C.c_void_p]),
    "gs3d_loss_workspace_size": (C.c_int, [C.c_int32, C.c_int32, P(C.c_size_t)]),
    "gs3d_loss_l1_dssim": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_float,
                                     C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "gs3d_adc_stats": (C.c_int, [P(AdcBuffersC), P(FGradientsC), C.c_void_p, C.c_void_p,
                                 C.c_int32, C.c_int32, C.c_void_p]),
    "gs3d_adc_workspace_size": (C.c_int, [C.c_int32, P(C.c_size_t)]),
    "gs3d_densify_prune_plan": (C.c_int, [P(AdcBuffersC), P(GaussiansC), P(AdcParamsC),
                                          P(C.c_int32), C.c_void_p]),
    "gs3d_densify_apply": (C.c_int, [P(AdcBuffersC), P(GaussiansC), P(AdamMomentsC),
                                     P(GaussiansC), P(AdamMomentsC), C.c_void_p, C.c_void_p,
                                     C.c_float, C.c_uint64, C.c_void_p]),
    "gs3d_opacity_reset": (C.c_int, [P(GaussiansC), P(AdamMomentsC), C.c_float, C.c_void_p]),
    "gs3d_densify_remap_dense": (C.c_int, [P(AdcBuffersC), C.c_int32, C.c_void_p, C.c_void_p,
                                           C.c_void_p]),
    "gs3d_last_error_string": (C.c_char_p, []),
    "gs3d_version": (C.c_int, []),
    "gs3d_profile_enable": (C.c_int, [C.c_int]),
    "gs3d_profile_report": (C.c_int, [C.c_char_p, C.c_size_t]),
}


def profile_enable(on: bool = True) -> None:
    check(lib().gs3d_profile_enable(1 if on else 0))


def profile_report() -> dict[str, tuple[int, float]]:
    """{stage: (launches, total_ms)} of the records since profile_enable (waits for them)."""
    buf = C.create_string_buffer(1 << 16)
    check(lib().gs3d_profile_report(buf, len(buf)))
    out = {}
    for line in buf.value.decode().splitlines():
        name, n, ms = line.split()
        out[name] = (int(n), float(ms))
    return out

_LIB = None


class Gs3dError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"gs3d status {status}: {message}")
        self.status = status


def lib():
    """Load libgs3d.so (once). Raises if the library is missing: there is no fallback."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with gs3d.build.build()")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def check(status: int) -> None:
    if status != GS3D_OK:
        msg = lib().gs3d_last_error_string().decode(errors="replace")
        raise Gs3dError(status, msg)
