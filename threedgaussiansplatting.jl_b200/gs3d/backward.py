"""backward! (backward_core.jl:37-72) through libgs3d.so, and its gradient buffers
(FilteredGaussiansGradientsVector, backward_structs.jl:1-29), indexed by filtered index."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _abi
from .render import _stream_handle
from .structs import (GaussiansVector, PinholeCamera, RenderBuffers, RenderOptions,
                      RenderOutputs, Tiling, _ptr, check_sh_degree)


@dataclass
class FilteredGaussiansGradients:
    mean2d_grads: torch.Tensor             # (n, 2)
    opacity_grads: torch.Tensor            # (n,)
    licov2d_grads: torch.Tensor            # (n, 3)
    color_grads: torch.Tensor              # (n, 3)
    mean3d_grads: torch.Tensor             # (n, 3)
    opacity_feature_grads: torch.Tensor    # (n,)
    scaling_features_grads: torch.Tensor   # (n, 3)
    rotation_features_grads: torch.Tensor  # (n, 4)
    sh_coeffs_grads: torch.Tensor          # (n, 3, (d+1)^2)

    @classmethod
    def create(cls, capacity: int, sh_degree: int, device) -> "FilteredGaussiansGradients":
        n = max(capacity, 1)
        f = dict(dtype=torch.float32, device=device)
        order = (sh_degree + 1) ** 2
        return cls(torch.zeros((n, 2), **f), torch.zeros(n, **f), torch.zeros((n, 3), **f),
                   torch.zeros((n, 3), **f), torch.zeros((n, 3), **f), torch.zeros(n, **f),
                   torch.zeros((n, 3), **f), torch.zeros((n, 4), **f),
                   torch.zeros((n, 3, order), **f))

    @property
    def capacity(self) -> int:
        return self.mean2d_grads.shape[0]

    @property
    def sh_degree(self) -> int:
        return int(round(self.sh_coeffs_grads.shape[2] ** 0.5)) - 1

    def set_sh_degree(self, d: int) -> None:
        """set_sh_degree! for gradients (backward_structs.jl:342-354): grow the SH axis (new
        entries zero; the reference leaves them unset)."""
        check_sh_degree(d)
        old = self.sh_coeffs_grads
        new = torch.zeros((old.shape[0], 3, (d + 1) ** 2), dtype=old.dtype, device=old.device)
        k = min(old.shape[2], new.shape[2])
        new[:, :, :k] = old[:, :, :k]
        self.sh_coeffs_grads = new

    def resize(self, capacity: int) -> None:
        """set_nb_gaussians! for gradients (contents are not kept)."""
        fresh = FilteredGaussiansGradients.create(capacity, self.sh_degree,
                                                  self.mean2d_grads.device)
        self.__dict__.update(fresh.__dict__)

    def to_c(self) -> _abi.FGradientsC:
        f = _abi.FGradientsC()
        f.sh_degree = self.sh_degree
        f.mean2d_grads = _ptr(self.mean2d_grads)
        f.opacity_grads = _ptr(self.opacity_grads)
        f.licov2d_grads = _ptr(self.licov2d_grads)
        f.color_grads = _ptr(self.color_grads)
        f.mean3d_grads = _ptr(self.mean3d_grads)
        f.opacity_feature_grads = _ptr(self.opacity_feature_grads)
        f.scaling_features_grads = _ptr(self.scaling_features_grads)
        f.rotation_features_grads = _ptr(self.rotation_features_grads)
        f.sh_coeffs_grads = _ptr(self.sh_coeffs_grads)
        return f


def backward(fgradients: FilteredGaussiansGradients, rgb_image_grad: torch.Tensor,
             outputs: RenderOutputs, gaussians: GaussiansVector, camera: PinholeCamera,
             tiling: Tiling, options: RenderOptions, buffers: RenderBuffers,
             fix_sh16: bool = False, stream: torch.cuda.Stream | None = None,
             skip_sh_grads: bool = False):
    """Gradients of the loss w.r.t. the filtered Gaussians' parameters, from the gradient
    image `rgb_image_grad` ((w, h, 3), i.e. 3 x h x w). The forward render must have run with
    the same arguments. `fix_sh16` uses SH coefficient 16 in the last degree-3 term of the
    colour/direction Jacobian; the default reproduces the reference (coefficient 15).
    `skip_sh_grads` leaves the SH gradients unwritten (for AdamOptimizer.update_rebuild_sh)."""
    assert rgb_image_grad.is_contiguous() and rgb_image_grad.dtype == torch.float32
    if fgradients.capacity < buffers.capacity_n:
        raise ValueError("gradient buffers smaller than the render buffers")
    lib = _abi.lib()
    args = [fgradients.to_c(), outputs.to_c(), gaussians.to_c(), camera.to_c(), tiling.to_c(),
            options.to_c(), buffers.to_c()]
    flags = (_abi.GS3D_BACKWARD_FIX_SH16 if fix_sh16 else 0) | \
        (_abi.GS3D_BACKWARD_SKIP_SH_GRADS if skip_sh_grads else 0)
    _abi.check(lib.gs3d_backward(C.byref(args[0]), C.c_void_p(rgb_image_grad.data_ptr()),
                                 C.byref(args[1]), C.byref(args[2]), C.byref(args[3]),
                                 C.byref(args[4]), C.byref(args[5]), C.byref(args[6]), flags,
                                 C.c_void_p(_stream_handle(stream))))
    return fgradients


def backward_raster(fgradients: FilteredGaussiansGradients, rgb_image_grad: torch.Tensor,
                    outputs: RenderOutputs, gaussians: GaussiansVector, camera: PinholeCamera,
                    tiling: Tiling, options: RenderOptions, buffers: RenderBuffers,
                    fix_sh16: bool = False, stream: torch.cuda.Stream | None = None):
    """First phase of backward(): the 2D gradients only (B1, B2)."""
    assert rgb_image_grad.is_contiguous() and rgb_image_grad.dtype == torch.float32
    lib = _abi.lib()
    args = [fgradients.to_c(), outputs.to_c(), gaussians.to_c(), camera.to_c(), tiling.to_c(),
            options.to_c(), buffers.to_c()]
    flags = _abi.GS3D_BACKWARD_FIX_SH16 if fix_sh16 else 0
    _abi.check(lib.gs3d_backward_raster(C.byref(args[0]), C.c_void_p(rgb_image_grad.data_ptr()),
                                        C.byref(args[1]), C.byref(args[2]), C.byref(args[3]),
                                        C.byref(args[4]), C.byref(args[5]), C.byref(args[6]), flags,
                                        C.c_void_p(_stream_handle(stream))))
    return fgradients


def backward_project_dense(fgradients: FilteredGaussiansGradients, gaussians: GaussiansVector,
                           camera: PinholeCamera, tiling: Tiling, options: RenderOptions,
                           buffers: RenderBuffers, dense_rows: torch.Tensor, g_begin: int,
                           g_end: int, fix_sh16: bool = False,
                           stream: torch.cuda.Stream | None = None, accumulate: bool = False) -> None:
    """Second phase: 3D gradients of the filtered Gaussians with index in [g_begin, g_end)
    into row gidx - g_begin of `dense_rows` (a view starting at row g_begin; not zeroed here).
    `accumulate`: add to the rows (another view of the same step) instead of overwriting."""
    assert dense_rows.is_contiguous() and dense_rows.dtype == torch.float32
    lib = _abi.lib()
    args = [fgradients.to_c(), gaussians.to_c(), camera.to_c(), tiling.to_c(), options.to_c(),
            buffers.to_c()]
    flags = (_abi.GS3D_BACKWARD_FIX_SH16 if fix_sh16 else 0) | \
        (_abi.GS3D_BACKWARD_ACCUMULATE_ROWS if accumulate else 0)
    _abi.check(lib.gs3d_backward_project_dense(
        C.byref(args[0]), C.byref(args[1]), C.byref(args[2]), C.byref(args[3]), C.byref(args[4]),
        C.byref(args[5]), flags, C.c_void_p(dense_rows.data_ptr()), int(g_begin), int(g_end),
        C.c_void_p(_stream_handle(stream))))


def backward_dense(fgradients: FilteredGaussiansGradients, rgb_image_grad: torch.Tensor,
                   outputs: RenderOutputs, gaussians: GaussiansVector, camera: PinholeCamera,
                   tiling: Tiling, options: RenderOptions, buffers: RenderBuffers,
                   dense: torch.Tensor, fix_sh16: bool = False,
                   stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """backward() with the 3D gradients written into `dense` ((rows >= n, GS3D_DENSE_ROW)
    float32, zeroed here) at each Gaussian's row instead of the F-compact 3D arrays; the 2D
    gradients still go to `fgradients`."""
    assert rgb_image_grad.is_contiguous() and rgb_image_grad.dtype == torch.float32
    assert dense.is_contiguous() and dense.dtype == torch.float32 and dense.shape[1] == 60
    if fgradients.capacity < buffers.capacity_n:
        raise ValueError("gradient buffers smaller than the render buffers")
    lib = _abi.lib()
    args = [fgradients.to_c(), outputs.to_c(), gaussians.to_c(), camera.to_c(), tiling.to_c(),
            options.to_c(), buffers.to_c()]
    flags = _abi.GS3D_BACKWARD_FIX_SH16 if fix_sh16 else 0
    _abi.check(lib.gs3d_backward_dense(C.byref(args[0]), C.c_void_p(rgb_image_grad.data_ptr()),
                                       C.byref(args[1]), C.byref(args[2]), C.byref(args[3]),
                                       C.byref(args[4]), C.byref(args[5]), C.byref(args[6]), flags,
                                       C.c_void_p(dense.data_ptr()), dense.shape[0],
                                       C.c_void_p(_stream_handle(stream))))
    return dense


def backward_project_factored(fgradients: FilteredGaussiansGradients, gaussians: GaussiansVector,
                              camera: PinholeCamera, tiling: Tiling, options: RenderOptions,
                              buffers: RenderBuffers, geom_rows: torch.Tensor,
                              colour_rows: torch.Tensor, g_begin: int, g_end: int,
                              fix_sh16: bool = False,
                              stream: torch.cuda.Stream | None = None,
                              accumulate: bool = False, colour_direction: bool = True) -> None:
    """backward_project_dense() into factored rows: geometry row (12 floats) and colour row
    (3 colour gradients + flags) gidx - g_begin of views starting at row g_begin.
    `accumulate`: add to the geometry rows (another view of the same step); the colour rows are
    this view's own. `colour_direction=False`: leave the colour -> direction term of the mean
    gradient to the rows' owner (colour_direction_rows); the SH coefficients are not read."""
    for t in (geom_rows, colour_rows):
        assert t.is_contiguous() and t.dtype == torch.float32
    lib = _abi.lib()
    args = [fgradients.to_c(), gaussians.to_c(), camera.to_c(), tiling.to_c(), options.to_c(),
            buffers.to_c()]
    flags = (_abi.GS3D_BACKWARD_FIX_SH16 if fix_sh16 else 0) | \
        (_abi.GS3D_BACKWARD_ACCUMULATE_ROWS if accumulate else 0) | \
        (0 if colour_direction else _abi.GS3D_BACKWARD_NO_COLOUR_DIRECTION)
    _abi.check(lib.gs3d_backward_project_factored(
        C.byref(args[0]), C.byref(args[1]), C.byref(args[2]), C.byref(args[3]), C.byref(args[4]),
        C.byref(args[5]), flags, C.c_void_p(geom_rows.data_ptr()),
        C.c_void_p(colour_rows.data_ptr()), int(g_begin), int(g_end),
        C.c_void_p(_stream_handle(stream))))


def colour_direction_rows(gaussians: GaussiansVector, geom_rows: torch.Tensor,
                          colour_rows: torch.Tensor, n_views: int, view_stride: int, positions,
                          g_begin: int, g_end: int, sh_degree: int, fix_sh16: bool = False,
                          stream: torch.cuda.Stream | None = None) -> None:
    """Add to geometry rows [g_begin, g_end) the colour -> direction term of the mean gradient
    that backward_project_factored(colour_direction=False) left out, for each view whose colour
    row (row v * view_stride + g - g_begin) filtered the Gaussian
    (gs3d_factored_colour_direction_range). `positions`: (n_views, 3) camera positions (host)."""
    import numpy as np
    pos = np.ascontiguousarray(positions, dtype=np.float32)
    for t in (geom_rows, colour_rows):
        assert t.is_contiguous() and t.dtype == torch.float32
    flags = _abi.GS3D_BACKWARD_FIX_SH16 if fix_sh16 else 0
    _abi.check(_abi.lib().gs3d_factored_colour_direction_range(
        C.byref(gaussians.to_c()), C.c_void_p(geom_rows.data_ptr()),
        C.c_void_p(colour_rows.data_ptr()), int(n_views), int(view_stride),
        pos.ctypes.data_as(C.POINTER(C.c_float)), int(g_begin), int(g_end), int(sh_degree), flags,
        C.c_void_p(_stream_handle(stream))))
