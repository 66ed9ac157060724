"""Adaptive density control through libgs3d.so: AdaptiveDensityControlBuffers
(training_structs.jl:259-290) and the densify/prune calls of maybe_densify_and_prune!
(training.jl:313-444), adaptive_density_control! (gaussians.jl:1526-1573,
optimizer.jl:1304-1325), maybe_opacity_reset! (training.jl:272-280)."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _abi
from .backward import FilteredGaussiansGradients
from .optimizer import AdamMoments
from .render import _stream_handle
from .structs import GaussiansVector, _ptr


@dataclass
class AdcBuffers:
    accumulated_mean2d_grad_norms_ndc: torch.Tensor
    rendering_contribution_counts: torch.Tensor
    max_scale_features: torch.Tensor
    should_prune: torch.Tensor
    should_densify: torch.Tensor
    should_clone: torch.Tensor
    new_gaussian_counts: torch.Tensor
    new_gaussian_counts_cs: torch.Tensor
    ngidx_to_gidx: torch.Tensor
    workspace: torch.Tensor

    @classmethod
    def create(cls, n: int, device) -> "AdcBuffers":
        m = max(n, 1)
        dev = torch.device(device)
        nbytes = C.c_size_t(0)
        _abi.check(_abi.lib().gs3d_adc_workspace_size(m, C.byref(nbytes)))
        u8 = dict(dtype=torch.uint8, device=dev)
        return cls(torch.zeros(m, dtype=torch.float32, device=dev),
                   torch.zeros(m, dtype=torch.int32, device=dev),
                   torch.zeros(m, dtype=torch.float32, device=dev), torch.zeros(m, **u8),
                   torch.zeros(m, **u8), torch.zeros(m, **u8), torch.zeros(m, **u8),
                   torch.zeros(m, dtype=torch.int32, device=dev),
                   torch.zeros(2 * m, dtype=torch.int32, device=dev),
                   torch.empty(int(nbytes.value), **u8))

    @property
    def capacity(self) -> int:
        return self.accumulated_mean2d_grad_norms_ndc.shape[0]

    def set_nb_gaussians(self, n: int) -> None:
        """set_nb_gaussians! (training_structs.jl): reset the statistics for n Gaussians. The
        arrays are kept when they hold n (the other arrays are outputs the next plan writes in
        full), else replaced with 25% headroom for the growth of later densify steps."""
        if n <= self.capacity:
            self.accumulated_mean2d_grad_norms_ndc.zero_()
            self.rendering_contribution_counts.zero_()
            return
        fresh = AdcBuffers.create(n + n // 4, self.workspace.device)
        self.__dict__.update(fresh.__dict__)

    def to_c(self) -> _abi.AdcBuffersC:
        a = _abi.AdcBuffersC()
        for name in ("accumulated_mean2d_grad_norms_ndc", "rendering_contribution_counts",
                     "max_scale_features", "should_prune", "should_densify", "should_clone",
                     "new_gaussian_counts", "new_gaussian_counts_cs", "ngidx_to_gidx", "workspace"):
            setattr(a, name, _ptr(getattr(self, name)))
        a.workspace_bytes = self.workspace.numel()
        return a


def adc_stats(adc: AdcBuffers, fgradients: FilteredGaussiansGradients, fgidx_to_gidx: torch.Tensor,
              device_counts: torch.Tensor, width: int, height: int, stream=None) -> None:
    a, f = adc.to_c(), fgradients.to_c()
    _abi.check(_abi.lib().gs3d_adc_stats(C.byref(a), C.byref(f), C.c_void_p(fgidx_to_gidx.data_ptr()),
                                         C.c_void_p(device_counts.data_ptr()), width, height,
                                         C.c_void_p(_stream_handle(stream))))


def densify_prune_plan(adc: AdcBuffers, gaussians: GaussiansVector, densify_grad_threshold: float,
                       densify_size_threshold: float, prune_min_opacity: float,
                       prune_max_scale: float, use_max_scale_pruning: bool, stream=None) -> int:
    """Masks, counts, their scan and ngidx_to_gidx; returns the new Gaussian count n'."""
    p = _abi.AdcParamsC()
    p.densification_mean2d_grad_norm_threshold_ndc = densify_grad_threshold
    p.densification_size_threshold = densify_size_threshold
    p.pruning_min_opacity = prune_min_opacity
    p.pruning_3d_max_scale = prune_max_scale
    p.use_max_scale_pruning = int(use_max_scale_pruning)
    out = C.c_int32(0)
    a, g = adc.to_c(), gaussians.to_c()
    _abi.check(_abi.lib().gs3d_densify_prune_plan(C.byref(a), C.byref(g), C.byref(p), C.byref(out),
                                                  C.c_void_p(_stream_handle(stream))))
    return int(out.value)


def densify_apply(adc: AdcBuffers, gaussians: GaussiansVector, moments: AdamMoments, new_n: int,
                  splitting_scale_factor: float, seed: int, fgidx_to_gidx: torch.Tensor | None = None,
                  device_counts: torch.Tensor | None = None, stream=None):
    """Build the n' Gaussians and moments; retarget fgidx_to_gidx (F = device_counts[0]) in
    place when given. Returns (new GaussiansVector, new AdamMoments)."""
    dev = gaussians.device
    f = dict(dtype=torch.float32, device=dev)
    S = gaussians.sh_coeffs.shape[2]
    ng = GaussiansVector(torch.empty((new_n, 4), **f), torch.empty((new_n, 3), **f),
                         torch.empty((new_n, 4), **f), torch.empty((new_n, 3, S), **f))
    nm = AdamMoments.empty(new_n, moments.sh_degree, dev)  # k_adc_apply writes every moment
    a, og, om, ngc, nmc = adc.to_c(), gaussians.to_c(), moments.to_c(), ng.to_c(), nm.to_c()
    log_split = float(np.log(np.float32(splitting_scale_factor)))
    _abi.check(_abi.lib().gs3d_densify_apply(
        C.byref(a), C.byref(og), C.byref(om), C.byref(ngc), C.byref(nmc),
        C.c_void_p(fgidx_to_gidx.data_ptr()) if fgidx_to_gidx is not None else None,
        C.c_void_p(device_counts.data_ptr()) if device_counts is not None else None,
        log_split, int(seed) & 0xFFFFFFFFFFFFFFFF, C.c_void_p(_stream_handle(stream))))
    return ng, nm


def opacity_reset(gaussians: GaussiansVector, moments: AdamMoments, max_opacity: float, stream=None):
    g, m = gaussians.to_c(), moments.to_c()
    _abi.check(_abi.lib().gs3d_opacity_reset(C.byref(g), C.byref(m), float(max_opacity),
                                             C.c_void_p(_stream_handle(stream))))
