"""The training loss of training_step! (training.jl:196-217) through libgs3d.so:
L = (1 - w) L1 + w DSSIM with its gradient image. DSSIM follows Wang et al. (2004) (11-tap
Gaussian window, sigma 1.5, zero padding); the reference's FastCUDASSIM is not vendored, so
the SSIM term's parity with it is unpinned."""
from __future__ import annotations

import ctypes as C

import torch

from . import _abi
from .render import _stream_handle


class LossComputer:
    """Holds the workspace for one image size. __call__ writes the gradient image and returns
    the device tensor [loss, L1, DSSIM] (no host synchronisation)."""

    def __init__(self, width: int, height: int, device, dssim_weight: float = 0.2):
        self.width, self.height = int(width), int(height)
        self.weight = float(dssim_weight)
        nbytes = C.c_size_t(0)
        _abi.check(_abi.lib().gs3d_loss_workspace_size(self.width, self.height, C.byref(nbytes)))
        self.workspace = torch.empty(int(nbytes.value), dtype=torch.uint8, device=device)
        self.value = torch.zeros(4, dtype=torch.float32, device=device)

    def __call__(self, rendered: torch.Tensor, target: torch.Tensor, grad_out: torch.Tensor,
                 stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        for t in (rendered, target, grad_out):
            assert t.shape == (self.width, self.height, 3) and t.is_contiguous()
        _abi.check(_abi.lib().gs3d_loss_l1_dssim(
            C.c_void_p(rendered.data_ptr()), C.c_void_p(target.data_ptr()), self.width,
            self.height, self.weight, C.c_void_p(self.value.data_ptr()),
            C.c_void_p(grad_out.data_ptr()), C.c_void_p(self.workspace.data_ptr()),
            self.workspace.numel(), C.c_void_p(_stream_handle(stream))))
        return self.value
