"""Sparse Adam of the reference (optimizer.jl): moments interleaved [m1, m2] per scalar
(GaussianAdamMomentsLearningRatesVector, optimizer.jl:9-29) and update! (optimizer.jl:964-1009)
through one fused kernel of libgs3d.so."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _abi
from .backward import FilteredGaussiansGradients
from .render import _stream_handle
from .structs import GaussiansVector, _ptr, check_sh_degree

DEFAULT_BETA1 = 0.9
DEFAULT_BETA2 = 0.999
DEFAULT_EPSILON = 1e-15


@dataclass
class AdamMoments:
    means_moments: torch.Tensor              # (n, 3, 2)
    opacity_features_moments: torch.Tensor   # (n, 2)
    scaling_features_moments: torch.Tensor   # (n, 3, 2)
    rotation_features_moments: torch.Tensor  # (n, 4, 2)
    sh_coeffs_moments: torch.Tensor          # (n, 3, (d+1)^2, 2)

    @classmethod
    def zeros(cls, n: int, sh_degree: int, device) -> "AdamMoments":
        f = dict(dtype=torch.float32, device=device)
        return cls(torch.zeros((n, 3, 2), **f), torch.zeros((n, 2), **f), torch.zeros((n, 3, 2), **f),
                   torch.zeros((n, 4, 2), **f), torch.zeros((n, 3, (sh_degree + 1) ** 2, 2), **f))

    @classmethod
    def empty(cls, n: int, sh_degree: int, device) -> "AdamMoments":
        """Uninitialised moments (for outputs a kernel writes in full)."""
        f = dict(dtype=torch.float32, device=device)
        return cls(torch.empty((n, 3, 2), **f), torch.empty((n, 2), **f), torch.empty((n, 3, 2), **f),
                   torch.empty((n, 4, 2), **f), torch.empty((n, 3, (sh_degree + 1) ** 2, 2), **f))

    @property
    def n(self) -> int:
        return self.means_moments.shape[0]

    @property
    def sh_degree(self) -> int:
        return int(round(self.sh_coeffs_moments.shape[2] ** 0.5)) - 1

    def tensors(self):
        return (self.means_moments, self.opacity_features_moments, self.scaling_features_moments,
                self.rotation_features_moments, self.sh_coeffs_moments)

    def set_sh_degree(self, d: int) -> None:
        """set_sh_degree! (optimizer.jl:737-746): grow the SH axis keeping old values."""
        check_sh_degree(d)
        old = self.sh_coeffs_moments
        new = torch.zeros((old.shape[0], 3, (d + 1) ** 2, 2), dtype=old.dtype, device=old.device)
        k = min(old.shape[2], new.shape[2])
        new[:, :, :k] = old[:, :, :k]
        self.sh_coeffs_moments = new

    def to_c(self) -> _abi.AdamMomentsC:
        m = _abi.AdamMomentsC()
        m.sh_degree = self.sh_degree
        m.means_moments = _ptr(self.means_moments)
        m.opacity_features_moments = _ptr(self.opacity_features_moments)
        m.scaling_features_moments = _ptr(self.scaling_features_moments)
        m.rotation_features_moments = _ptr(self.rotation_features_moments)
        m.sh_coeffs_moments = _ptr(self.sh_coeffs_moments)
        return m


@dataclass
class LearningRates:
    means: float
    opacity_features: float = 0.05
    scaling_features: float = 0.005
    rotation_features: float = 0.001
    sh_coeffs_dc: float = 0.0025
    sh_coeffs_rest: float = 0.0025 / 20


class AdamOptimizer:
    """MutableAdamOptimizer (optimizer.jl:783-870) over a GaussiansVector."""

    def __init__(self, gaussians: GaussiansVector, lrs: LearningRates, beta1=DEFAULT_BETA1,
                 beta2=DEFAULT_BETA2, epsilon=DEFAULT_EPSILON, update_count: int = 0):
        self.gaussians = gaussians
        self.moments = AdamMoments.zeros(gaussians.n, gaussians.sh_degree, gaussians.device)
        self.lrs = lrs
        self.beta1, self.beta2, self.epsilon = float(beta1), float(beta2), float(epsilon)
        self.update_count = int(update_count)

    def params_c(self, sh_degree: int) -> _abi.AdamParamsC:
        p = _abi.AdamParamsC()
        p.lr_means = self.lrs.means
        p.lr_opacity_features = self.lrs.opacity_features
        p.lr_scaling_features = self.lrs.scaling_features
        p.lr_rotation_features = self.lrs.rotation_features
        p.lr_sh_dc = self.lrs.sh_coeffs_dc
        p.lr_sh_rest = self.lrs.sh_coeffs_rest
        p.beta1, p.beta2, p.epsilon = self.beta1, self.beta2, self.epsilon
        p.update_count = self.update_count
        p.sh_degree = int(sh_degree)
        return p

    def update(self, fgradients: FilteredGaussiansGradients, fgidx_to_gidx: torch.Tensor,
               device_counts: torch.Tensor, sh_degree: int,
               stream: torch.cuda.Stream | None = None) -> GaussiansVector:
        """update!(opt, fgradients, Val(sh_degree)): one sparse Adam step over the filtered
        Gaussians (count device_counts[0]) and update_count += 1."""
        args = [self.gaussians.to_c(), self.moments.to_c(), fgradients.to_c(),
                self.params_c(sh_degree)]
        _abi.check(_abi.lib().gs3d_adam_step(
            C.byref(args[0]), C.byref(args[1]), C.byref(args[2]),
            C.c_void_p(fgidx_to_gidx.data_ptr()), C.c_void_p(device_counts.data_ptr()),
            C.byref(args[3]), C.c_void_p(_stream_handle(stream))))
        self.update_count += 1
        return self.gaussians

    def update_rebuild_sh(self, fgradients: FilteredGaussiansGradients, fgidx_to_gidx: torch.Tensor,
                          device_counts: torch.Tensor, projected: torch.Tensor, camera_position,
                          sh_degree: int, stream: torch.cuda.Stream | None = None) -> GaussiansVector:
        """update() with the SH gradients recomputed from the colour gradients, the projected
        colours (`projected`: the render buffers' (n, 9) projection rows) and the camera
        position the backward ran for (gs3d_adam_step_rebuild_sh): the same step, bit for bit,
        when the Gaussians did not change since the backward; needs SH storage degree 3."""
        import numpy as np
        pos = np.ascontiguousarray(np.asarray(camera_position, dtype=np.float32).reshape(3))
        args = [self.gaussians.to_c(), self.moments.to_c(), fgradients.to_c(),
                self.params_c(sh_degree)]
        _abi.check(_abi.lib().gs3d_adam_step_rebuild_sh(
            C.byref(args[0]), C.byref(args[1]), C.byref(args[2]),
            C.c_void_p(fgidx_to_gidx.data_ptr()), C.c_void_p(device_counts.data_ptr()),
            C.c_void_p(projected.data_ptr()), pos.ctypes.data_as(C.POINTER(C.c_float)),
            C.byref(args[3]), C.c_void_p(_stream_handle(stream))))
        self.update_count += 1
        return self.gaussians


def bias_corrections(beta1: float, beta2: float, update_count: int) -> tuple[float, float]:
    """1 - beta^t rounded to float32 (t = update_count + 1), as libgs3d computes them."""
    import numpy as np
    t = update_count + 1
    b1 = np.float32(1.0) - np.float32(float(np.float32(beta1)) ** t)
    b2 = np.float32(1.0) - np.float32(float(np.float32(beta2)) ** t)
    return float(b1), float(b2)
