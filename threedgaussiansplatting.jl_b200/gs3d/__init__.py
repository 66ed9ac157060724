"""gs3d — B200-native (sm_100a) 3D Gaussian Splatting hot path with the interface of
ThreeDGaussianSplatting.jl: render! / backward! / update! / training_step! and the
densify/prune calls, all computed by hand-written CUDA kernels in libgs3d.so.
"""
from . import _abi
from ._abi import Gs3dError, lib
from .structs import (CLAMP, FILTER, GaussiansVector, PinholeCamera, RenderBuffers,
                      RenderOnlyGaussiansVector, RenderOptions, RenderOutputs, Tiling,
                      default_tile_size, fov_deg_to_focal_length, fov_to_focal_length,
                      look_at_camera)
from .render import counts, render

__all__ = [
    "CLAMP", "FILTER", "GaussiansVector", "PinholeCamera", "RenderBuffers",
    "RenderOnlyGaussiansVector", "RenderOptions",
    "RenderOutputs", "Tiling", "default_tile_size", "fov_deg_to_focal_length",
    "fov_to_focal_length", "look_at_camera", "render", "counts", "lib", "Gs3dError",
]
